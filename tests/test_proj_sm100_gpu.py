"""The tensor-core projection z = half(half(x) P^T) (tropnn_b200_trop_proj, layers/tropical.py:96-99)
against an f64 reference of the same rounding steps: at most one unit in the last place of the
parameter dtype anywhere (the f32 accumulation order differs from the reference's, which can only
move a sum across a rounding boundary), on the unsplit and the split-contraction paths, ragged
row and input widths, every supported code_dim, f16 and bf16; split runs are deterministic.
The projection's backward (grad_x on the tensor-core linear map, grad_P on the tensor-core
weight-gradient kernel) against f64 products."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from tests.golden_cases import rel_err
from tropnn_b200 import _native as nat
from tropnn_b200.ops import proj_eligible, trop_project_b200

pytestmark = pytest.mark.gpu


def _ulp(a: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """Spacing of ``dtype`` at |a| (its smallest normal spacing below the normal range)."""
    mant = 10 if dtype == torch.float16 else 7
    tiny = torch.finfo(dtype).tiny
    e = torch.floor(torch.log2(a.abs().clamp_min(tiny)))
    return torch.exp2(e - mant)


@pytest.mark.parametrize(
    ("rows", "in_f", "dim", "dtype"),
    [
        (300, 4096, 256, torch.float16),  # 3 row blocks: 16 contraction slices
        (2048, 4096, 256, torch.float16),  # one GPU's shard of config 5 at 8 GPUs: 8 slices
        (20000, 512, 128, torch.float16),  # unsplit, ragged last row block
        (130, 200, 64, torch.bfloat16),  # input width not a multiple of 64
        (1000, 784, 192, torch.bfloat16),
    ],
)
def test_projection_matches_rounded_reference(rows: int, in_f: int, dim: int, dtype: torch.dtype) -> None:
    gen = torch.Generator().manual_seed(rows + in_f)
    x = torch.randn(rows, in_f, generator=gen)
    w = (torch.randn(dim, in_f, generator=gen) / in_f**0.5).to(dtype)
    xd, wd = x.cuda(), w.cuda()
    assert proj_eligible(xd, wd)
    z = trop_project_b200(xd, wd)
    torch.cuda.synchronize()
    assert z.dtype == dtype and z.shape == (rows, dim)
    ref = x.to(dtype).double() @ w.double().t()  # exact sums of the rounded operands
    z64 = z.cpu().double()
    err = (z64 - ref).abs()
    # One rounding unit of the output dtype, plus the f32 accumulation error of a long
    # contraction (absolute, ~1e-5 of the largest output: it dominates for sums that cancel
    # to near zero, where the dtype's unit is tiny).
    bound = _ulp(ref, dtype).double() + 3e-5 * float(ref.abs().max())
    assert bool((err <= bound).all()), float((err / bound).max())
    # Mostly the correctly rounded sum: only sums within the f32 error of a rounding boundary
    # may round the other way.
    assert float((z64 != ref.to(dtype).double()).double().mean()) < 0.05
    again = trop_project_b200(xd, wd)
    assert torch.equal(z, again)  # deterministic (the split path sums its slices in order)


def test_projection_backward() -> None:
    rows, in_f, dim = 640, 1024, 256
    gen = torch.Generator().manual_seed(3)
    x = torch.randn(rows, in_f, generator=gen)
    w = (torch.randn(dim, in_f, generator=gen) / in_f**0.5).half()
    g = torch.randn(rows, dim, generator=gen).half()
    xd = x.cuda().requires_grad_(True)
    wd = w.cuda().requires_grad_(True)
    z = trop_project_b200(xd, wd)
    z.backward(g.cuda())
    torch.cuda.synchronize()
    gx_ref = g.double() @ w.double()
    gw_ref = g.double().t() @ x.half().double()
    assert xd.grad.dtype == torch.float32
    assert rel_err(xd.grad.cpu().numpy(), gx_ref.numpy()) <= 1e-5
    assert wd.grad.dtype == torch.float16
    assert rel_err(wd.grad.float().cpu().numpy(), gw_ref.numpy()) <= 2e-3


def test_projection_rejects_unsupported_shapes() -> None:
    x = torch.randn(4, 100, device="cuda")
    assert not proj_eligible(x, torch.randn(256, 100, device="cuda").half())  # in % 8
    assert not proj_eligible(torch.randn(4, 96, device="cuda"), torch.randn(100, 96, device="cuda").half())
    lib = nat.load()
    status = lib.tropnn_b200_trop_proj(x.data_ptr(), 4, 100, x.data_ptr(), nat.F16, 256, x.data_ptr(), None, 0,
                                       torch.cuda.current_stream().cuda_stream)
    with pytest.raises(ValueError, match="in_features"):
        nat.check(status, "trop_proj")


def _wgrad(x: torch.Tensor, g: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """grad_P = g^T half(x) through the C ABI (g transposed first, as the layer does)."""
    lib = nat.load()
    rows, in_f = x.shape
    dim = g.shape[1]
    pdt = nat.float_code(dtype)
    stream = nat.stream_handle(x.device)
    g_t = torch.empty((dim, rows), device=x.device, dtype=dtype)
    nat.check(lib.tropnn_b200_transpose_to_half(g.data_ptr(), pdt, rows, dim, pdt, None, g_t.data_ptr(), stream),
              "transpose_to_half")
    out = torch.empty((dim, in_f), device=x.device, dtype=dtype)
    ws_bytes = int(lib.tropnn_b200_trop_proj_wgrad_workspace_size(rows, in_f, dim))
    ws = torch.empty(max(ws_bytes, 1), device=x.device, dtype=torch.uint8)
    nat.check(lib.tropnn_b200_trop_proj_wgrad(x.data_ptr(), rows, in_f, g_t.data_ptr(), pdt, dim, out.data_ptr(),
                                              ws.data_ptr(), ws_bytes, stream), "trop_proj_wgrad")
    return out


@pytest.mark.parametrize(
    ("rows", "in_f", "dim", "dtype"),
    [
        (16384, 4096, 256, torch.float16),  # config 5's train step: 4 sample slices per feature tile
        (2048, 4096, 256, torch.float16),  # one GPU's shard at 8 GPUs
        (200, 200, 64, torch.bfloat16),  # ragged samples (zero-filled k block) and features
        (8, 512, 128, torch.float16),  # one k block: unsplit, direct stores
        (1000, 784, 192, torch.bfloat16),
    ],
)
def test_projection_weight_gradient(rows: int, in_f: int, dim: int, dtype: torch.dtype) -> None:
    """grad_P against f64 sums of the rounded operands: one rounding unit plus the f32
    accumulation error; deterministic."""
    gen = torch.Generator().manual_seed(rows + dim)
    x = torch.randn(rows, in_f, generator=gen)
    g = torch.randn(rows, dim, generator=gen).to(dtype)
    xd, gd = x.cuda(), g.cuda()
    got = _wgrad(xd, gd, dtype)
    torch.cuda.synchronize()
    ref = g.double().t() @ x.to(dtype).double()
    err = (got.cpu().double() - ref).abs()
    bound = _ulp(ref, dtype).double() + 3e-5 * float(ref.abs().max())
    assert bool((err <= bound).all()), float((err / bound).max())
    assert torch.equal(got, _wgrad(xd, gd, dtype))
