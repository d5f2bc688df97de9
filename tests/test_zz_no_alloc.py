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
    use_min = int(layer.use_min_margin_ste)
    common = (
        g.data_ptr(), rows, layer.out_features, layer.output_scale, idx.data_ptr(), u.data_ptr(),
        layer.anchors.data_ptr(), layer.tables, layer.comparisons, layer.in_features, layer.lut.data_ptr(), nat.F32,
        use_min, nat.SURROGATES["fast_sigmoid_odd"], gx.data_ptr(), gthr.data_ptr(), nat.F32, glut.data_ptr(),
    )
    stream = torch.cuda.current_stream().cuda_stream
    if noalloc:
        status = lib.tropnn_b200_pairwise_backward_noalloc(*common, stream)
    else:
        ws_bytes = lib.tropnn_b200_pairwise_backward_workspace_size(rows, layer.tables, layer.comparisons,
                                                                     layer.in_features, use_min)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
        status = lib.tropnn_b200_pairwise_backward(*common, ws.data_ptr(), ws_bytes, stream)
    nat.check(status, "pairwise backward")
    torch.cuda.synchronize()
    return gx.cpu().numpy(), gthr.cpu().numpy(), glut.detach().cpu().numpy()


@pytest.mark.parametrize(
    ("in_f", "out_f", "tables", "comparisons", "use_min", "rows"),
    [
        # Config 2's layer, 4096 rows: the one-kernel LUT gradient and the min-margin STE.
        (256, 512, 16, 6, True, 4096),
        # More than 1024 columns and the full STE: the bucket_sort + segment_rowsum LUT
        # gradient, whose row permutation and bucket segments live in the fixed buffer, and
        # the per-comparison STE gradients (rows x tables x comparisons floats).
        (96, 1100, 12, 5, False, 2048),
    ],
)
def test_noalloc_backward_matches_workspace_backward_twice(in_f, out_f, tables, comparisons, use_min, rows) -> None:
    layer = tropnn_b200.PairwiseLinear(in_f, out_f, tables=tables, comparisons=comparisons, seed=0,
                                       use_min_margin_ste=use_min).cuda()
    need = nat.load().tropnn_b200_pairwise_backward_workspace_size(rows, tables, comparisons, in_f, int(use_min))
    assert 0 < need <= (8 << 20)
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


def test_noalloc_backward_rejects_bad_sizes() -> None:
    lib = nat.load()
    status = lib.tropnn_b200_pairwise_backward_noalloc(
        None, 16, 16, 1.0, None, None, None, 0, 4, 32, None, nat.F32, 1, 0,
        None, None, nat.F32, None, torch.cuda.current_stream().cuda_stream,
    )
    with pytest.raises(ValueError, match="bad sizes"):
        nat.check(status, "pairwise_backward_noalloc")
