"""The allocation-free Pairwise backward against the workspace one, through the C ABI.

tropnn_b200_pairwise_backward_noalloc serves callers that cannot allocate device memory
(a fixed, fully pre-partitioned memory budget, a foreign-language caller without a CUDA
allocator, a loop that cannot afford cudaMalloc's implicit synchronisation): it takes no
workspace and uses a fixed 8 MiB buffer inside the library instead. This file runs last
(pytest collects files in name order) and passes alone in a fresh process as well as after
the other tests: the first call on the device sets up the buffer's address, and two calls
in a row must both match tropnn_b200_pairwise_backward.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import tropnn_b200
from tests.golden_cases import rel_err
from tropnn_b200 import _native as nat

pytestmark = pytest.mark.gpu
FP32_TOL = 1e-5  # the value tolerance of every fp32 parity test in this suite


def _forward(layer: tropnn_b200.PairwiseLinear, seed: int, rows: int):
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, layer.in_features, generator=gen).cuda()
    g = torch.randn(rows, layer.out_features, generator=gen).cuda().contiguous()
    with torch.no_grad():
        layer(x)
    idx = layer._last_indices.reshape(rows, layer.tables).contiguous()
    u = layer._last_margins.reshape(rows, layer.tables, layer.comparisons).contiguous()
    return g, idx, u


def _outputs(layer: tropnn_b200.PairwiseLinear, rows: int):
    dev = torch.device("cuda")
    return (
        torch.full((rows, layer.in_features), float("nan"), device=dev),
        torch.full((layer.tables, layer.comparisons), float("nan"), device=dev),
        torch.full_like(layer.lut, float("nan")),
    )


def _backward(layer, rows, g, idx, u, *, noalloc: bool):
    lib = nat.load()
    gx, gthr, glut = _outputs(layer, rows)
    common = (
        g.data_ptr(), rows, layer.out_features, layer.output_scale, idx.data_ptr(), u.data_ptr(),
        layer.anchors.data_ptr(), layer.tables, layer.comparisons, layer.in_features, layer.lut.data_ptr(), nat.F32,
        1, nat.SURROGATES["fast_sigmoid_odd"], gx.data_ptr(), gthr.data_ptr(), nat.F32, glut.data_ptr(),
    )
    stream = torch.cuda.current_stream().cuda_stream
    if noalloc:
        status = lib.tropnn_b200_pairwise_backward_noalloc(*common, stream)
    else:
        ws_bytes = lib.tropnn_b200_pairwise_backward_workspace_size(rows, layer.tables, layer.comparisons,
                                                                     layer.in_features, 1)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
        status = lib.tropnn_b200_pairwise_backward(*common, ws.data_ptr(), ws_bytes, stream)
    nat.check(status, "pairwise backward")
    torch.cuda.synchronize()
    return gx.cpu().numpy(), gthr.cpu().numpy(), glut.detach().cpu().numpy()


def test_noalloc_backward_matches_workspace_backward_twice() -> None:
    # Config 2's layer: PairwiseLinear(256 -> 512, T16, C6), 4096 rows (well inside 8 MiB).
    layer = tropnn_b200.PairwiseLinear(256, 512, tables=16, comparisons=6, seed=0).cuda()
    rows = 4096
    for call, seed in enumerate((11, 12)):  # two calls in a row, different inputs
        g, idx, u = _forward(layer, seed, rows)
        want = _backward(layer, rows, g, idx, u, noalloc=False)
        got = _backward(layer, rows, g, idx, u, noalloc=True)
        for name, a, b in zip(("grad_latent", "grad_thresholds", "grad_lut"), got, want):
            assert np.isfinite(a).all(), (call, name)
            assert rel_err(a, b) <= FP32_TOL, (call, name)


def test_noalloc_backward_rejects_problems_beyond_its_buffer() -> None:
    lib = nat.load()
    rows, tables, comparisons, in_f = 65536, 256, 8, 4096
    need = lib.tropnn_b200_pairwise_backward_workspace_size(rows, tables, comparisons, in_f, 1)
    assert need > (8 << 20)
    status = lib.tropnn_b200_pairwise_backward_noalloc(
        None, rows, 16, 1.0, None, None, None, tables, comparisons, in_f, None, nat.F32, 1, 0,
        None, None, nat.F32, None, torch.cuda.current_stream().cuda_stream,
    )
    with pytest.raises(ValueError, match="fixed 8388608-byte buffer"):
        nat.check(status, "pairwise_backward_noalloc")
