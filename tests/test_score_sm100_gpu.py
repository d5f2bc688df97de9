"""The tensor-core (tcgen05) route scores against the fp32 SIMT route kernel.

With half-precision latent and parameters, tropnn_b200_trop_route runs the scores as a
tcgen05 GEMM with the top-2 in its epilogue. The same call with the latent upcast to f32
takes the SIMT fp32-FMA kernel. Both see exactly the same values (the upcast is exact and
every f16/bf16 product is exact in f32), so routes must agree wherever the top-2 margin
exceeds 1e-4 relative, and margins within 1e-5 relative (f32 summation order only).

With f32 parameters and a workspace the scores run in kind::tf32 with split operands
(3xTF32): routes must agree with the fp32 FMA kernel and the oracle wherever the gate pins
them, and margins within 1e-5 relative.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from tests.golden_cases import rel_err, route_gate
from tropnn_b200 import _native as nat

pytestmark = pytest.mark.gpu


def _route(z: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, *, workspace: bool = False) -> tuple[np.ndarray, ...]:
    """The route through the C ABI; ``workspace`` gives f32 calls room for the 3xTF32 path."""
    lib = nat.load()
    items, code_dim = z.shape
    heads, cells, _ = weight.shape
    dev = z.device
    w64 = torch.empty(items, heads, dtype=torch.int64, device=dev)
    win = torch.empty(items, heads, dtype=torch.uint8, device=dev)
    run = torch.empty(items, heads, dtype=torch.uint8, device=dev)
    m = torch.empty(items, heads, dtype=torch.float32, device=dev)
    ws_bytes = 0
    if workspace:
        ws_bytes = int(lib.tropnn_b200_trop_route_workspace_size(items, code_dim, heads, cells, nat.float_code(z.dtype),
                                                                 nat.float_code(weight.dtype)))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev) if ws_bytes else None
    status = lib.tropnn_b200_trop_route(
        z.data_ptr(), nat.float_code(z.dtype), items, code_dim, weight.data_ptr(), bias.data_ptr(),
        nat.float_code(bias.dtype), nat.float_code(weight.dtype), heads, cells, w64.data_ptr(), win.data_ptr(),
        run.data_ptr(), nat.U8, m.data_ptr(), nat.ptr(ws), ws_bytes, torch.cuda.current_stream().cuda_stream,
    )
    nat.check(status, "trop_route")
    torch.cuda.synchronize()
    return w64.cpu().numpy(), win.cpu().numpy(), run.cpu().numpy(), m.cpu().numpy()


def _case(items: int, heads: int, cells: int, code_dim: int, dtype: torch.dtype, seed: int = 0):
    gen = torch.Generator().manual_seed(seed)
    z = (torch.randn(items, code_dim, generator=gen)).to(dtype)
    weight = (torch.randn(heads, cells, code_dim, generator=gen) / code_dim**0.5).to(dtype)
    bias = (0.1 * torch.randn(heads, cells, generator=gen)).to(dtype)
    return z.cuda(), weight.cuda(), bias.cuda()


def _check(items: int, heads: int, cells: int, code_dim: int, dtype: torch.dtype) -> None:
    z, weight, bias = _case(items, heads, cells, code_dim, dtype)
    simt = _route(z.float(), weight, bias)  # f32 latent: SIMT fp32 path
    scores = oracle.trop_scores(z.float().cpu().numpy(), weight.float().cpu().numpy(), bias.float().cpu().numpy())
    win_gate, run_gate = route_gate(scores)
    assert win_gate.mean() > 0.99
    ref_w, ref_r, ref_m = oracle.top2_indices(scores)
    # Half latent, f32 bias: tensor-core path, the bias added in the epilogue; a workspace (which
    # this path does not use) changes nothing.
    for workspace in (False, True):
        tc = _route(z, weight, bias.float(), workspace=workspace)
        assert np.array_equal(tc[0], tc[1].astype(np.int64))
        assert np.array_equal(tc[1][win_gate], simt[1][win_gate])
        assert np.array_equal(tc[2][run_gate], simt[2][run_gate])
        assert rel_err(tc[3], simt[3]) <= 1e-5
        assert np.array_equal(tc[1][win_gate].astype(np.int64), ref_w[win_gate])
        assert np.array_equal(tc[2][run_gate].astype(np.int64), ref_r[run_gate])
        assert rel_err(tc[3], ref_m) <= 1e-5


@pytest.mark.parametrize("cells", [2, 4, 8, 16, 32, 64])
def test_cells(cells: int) -> None:
    _check(items=256, heads=max(4, 1024 // cells), cells=cells, code_dim=64, dtype=torch.float16)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_config5_layer_shape(dtype: torch.dtype) -> None:
    """Config 5's router: H1024, K16, D256 (16384 score columns), 640 rows."""
    _check(items=640, heads=1024, cells=16, code_dim=256, dtype=dtype)


@pytest.mark.parametrize(
    ("items", "heads", "cells", "code_dim"),
    [
        (300, 12, 16, 64),  # ragged rows (300 = 2*128 + 44) and a half-filled last score tile
        (129, 9, 16, 40),  # code_dim not a multiple of 64 (zero-filled k block), 9 heads
        (1000, 200, 8, 128),  # many tiles, several column splits
        (128, 8, 16, 384),  # 6 k blocks: one 128-row half per row block, 8-stage ring
        (200, 8, 16, 448),  # 7 k blocks: 7-stage ring
        (130, 16, 8, 512),  # largest code_dim (8 k blocks, 6-stage ring), 2 rows in the last block
        (20000, 128, 16, 128),  # ~8.5 units per CTA: z block reloads inside a CTA's range
        (12345, 96, 4, 256),  # odd row count, 3 tiles per row block, second half empty at the end
    ],
)
def test_ragged_shapes(items: int, heads: int, cells: int, code_dim: int) -> None:
    _check(items, heads, cells, code_dim, torch.float16)


def test_no_device_error_after_tensor_core_runs() -> None:
    import ctypes

    _check(items=512, heads=64, cells=16, code_dim=64, dtype=torch.float16)
    flag = ctypes.c_int(-1)
    nat.check(nat.load().tropnn_b200_device_error(ctypes.byref(flag)), "device_error")
    assert flag.value == 0


@pytest.mark.parametrize(
    ("items", "heads", "cells", "code_dim"),
    [
        (512, 256, 16, 64),  # config 3's router
        (8, 32, 4, 32),  # config 1's router (below 64 rows: the fp32 FMA kernel either way)
        (64, 32, 4, 32),  # the fewest rows the tf32 path takes
        (300, 12, 16, 64),  # ragged rows, a half-filled score tile
        (1000, 40, 8, 128),  # largest code_dim of the tf32 path (4 k blocks)
        (129, 9, 32, 36),  # code_dim not a multiple of 32 (zero-filled k block)
        (20000, 64, 2, 16),  # many units per CTA, two cells
    ],
)
def test_f32_tensor_core_route(items: int, heads: int, cells: int, code_dim: int) -> None:
    z, weight, bias = _case(items, heads, cells, code_dim, torch.float32, seed=3)
    tc = _route(z, weight, bias, workspace=True)  # 3xTF32 tensor cores
    simt = _route(z, weight, bias)  # no workspace: fp32 FMA kernel
    scores = oracle.trop_scores(z.cpu().numpy(), weight.cpu().numpy(), bias.cpu().numpy())
    win_gate, run_gate = route_gate(scores)
    ref_w, ref_r, ref_m = oracle.top2_indices(scores)
    assert np.array_equal(tc[0], tc[1].astype(np.int64))
    for got in (tc, simt):
        assert np.array_equal(got[1][win_gate].astype(np.int64), ref_w[win_gate])
        assert np.array_equal(got[2][run_gate].astype(np.int64), ref_r[run_gate])
        assert rel_err(got[3], ref_m) <= 1e-5


def test_f32_route_workspace_query() -> None:
    lib = nat.load()
    assert lib.tropnn_b200_trop_route_workspace_size(512, 64, 256, 16, nat.F32, nat.F32) >= 2 * 4 * (512 + 4096) * 64
    # Half precision: the tensor-core route needs no scratch.
    assert lib.tropnn_b200_trop_route_workspace_size(512, 64, 256, 16, nat.F16, nat.F16) == 0
    assert lib.tropnn_b200_trop_route_workspace_size(512, 64, 256, 16, nat.F32, nat.F16) == 0
