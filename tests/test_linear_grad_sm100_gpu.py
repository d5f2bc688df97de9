"""The tensor-core gradients of the f32 output map (linear_dgrad, linear_wgrad, tf32_split)
against float64 products.

The reference's output map F.linear(hidden, W.float(), b.float()) (layers/tropical.py:140-146)
has f32 gradients grad_hidden = g W, grad_W = (g^T hidden).to(W.dtype), grad_b =
g.sum(0).to(b.dtype). On backend="b200" they run as tcgen05 tf32 GEMMs with split operands
(x = big + small): the f32 results within 2e-5 of the largest exact value at a 4096-long
contraction (the tensor-core accumulator truncates, ~1e-5 measured; torch's f32 FMA GEMM:
2.4e-6; the layer's half-precision tolerance: 2e-2), with f32 range (gradients of 1e-9 do
not underflow), and grad_W within one rounding of the parameter dtype.
"""

from __future__ import annotations

import pytest
import torch

from tests.golden_cases import rel_err
from tropnn_b200 import _native as nat
from tropnn_b200.ops import linear_f32out_b200

pytestmark = pytest.mark.gpu

F32_TOL = 2e-5
HALF_TOL = {torch.float16: 1e-3, torch.bfloat16: 8e-3}


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _operands(rows, out_features, in_features, dtype, scale=1.0, seed=0):
    gen = torch.Generator().manual_seed(seed)
    g = (torch.randn(rows, out_features, generator=gen) * scale).cuda()
    h = torch.randn(rows, in_features, generator=gen).cuda()
    w = (torch.randn(out_features, in_features, generator=gen) / in_features**0.5).to(dtype).cuda()
    return g, h, w


def _dgrad(g, w):
    rows, out_features = g.shape
    in_features = w.shape[1]
    w32 = w.float().contiguous()
    out = torch.full((rows, in_features), float("nan"), device="cuda")
    lib = nat.load()
    ws_bytes = int(lib.tropnn_b200_linear_dgrad_workspace_size(rows, out_features, in_features))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda") if ws_bytes else None
    nat.check(
        lib.tropnn_b200_linear_dgrad(g.data_ptr(), rows, out_features, w32.data_ptr(), in_features, out.data_ptr(),
                                     nat.ptr(ws), ws_bytes, _stream()),
        "linear_dgrad",
    )
    return out


def _wgrad(g, h, dtype):
    rows, out_features = g.shape
    in_features = h.shape[1]
    lib = nat.load()
    hb, hs = torch.empty_like(h), torch.empty_like(h)
    nat.check(lib.tropnn_b200_tf32_split(h.data_ptr(), h.numel(), hb.data_ptr(), hs.data_ptr(), _stream()), "tf32_split")
    gw = torch.full((out_features, in_features), float("nan"), device="cuda", dtype=dtype)
    gb = torch.full((out_features,), float("nan"), device="cuda")
    nat.check(
        lib.tropnn_b200_linear_wgrad(g.data_ptr(), rows, out_features, hb.data_ptr(), hs.data_ptr(), in_features,
                                     nat.float_code(dtype), gw.data_ptr(), gb.data_ptr(), _stream()),
        "linear_wgrad",
    )
    return gw, gb


SHAPES = [
    (1000, 4096, 256),  # config 5's output map on 1000 rows (8 row blocks; 32 W blocks x 4 slices)
    (300, 96, 64),  # ragged rows; one partial W block
    (129, 32, 32),  # one row in the last block; the narrowest widths
    (4096, 512, 192),  # N = 192
    (16, 4160, 128),  # fewer contraction blocks than cluster slices (empty slices); 33 W blocks
    (1, 64, 256),  # a single row
]


@pytest.mark.parametrize(("rows", "out_features", "in_features"), SHAPES)
def test_dgrad(rows, out_features, in_features):
    g, _, w = _operands(rows, out_features, in_features, torch.float16)
    out = _dgrad(g, w)
    torch.cuda.synchronize()
    ref = g.double() @ w.double()
    assert rel_err(out.cpu().numpy(), ref.cpu().numpy()) <= F32_TOL


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize(("rows", "out_features", "in_features"), SHAPES)
def test_wgrad(dtype, rows, out_features, in_features):
    g, h, _ = _operands(rows, out_features, in_features, dtype, seed=1)
    gw, gb = _wgrad(g, h, dtype)
    torch.cuda.synchronize()
    ref_w = g.double().t() @ h.double()
    assert rel_err(gw.double().cpu().numpy(), ref_w.cpu().numpy()) <= HALF_TOL[dtype]
    # The f32 result before rounding is within f32 accuracy: compare with the rounded exact.
    assert rel_err(gw.double().cpu().numpy(), ref_w.to(dtype).double().cpu().numpy()) <= HALF_TOL[dtype]
    assert rel_err(gb.cpu().numpy(), g.double().sum(0).cpu().numpy()) <= F32_TOL


def test_tiny_gradients_keep_f32_range():
    """Gradients of 1e-9 (below f16's smallest subnormal) keep full relative accuracy."""
    g, h, w = _operands(512, 256, 128, torch.float16, scale=1e-9, seed=2)
    out = _dgrad(g, w)
    gw, gb = _wgrad(g, h, torch.bfloat16)
    torch.cuda.synchronize()
    assert rel_err(out.cpu().numpy(), (g.double() @ w.double()).cpu().numpy()) <= F32_TOL
    assert rel_err(gb.cpu().numpy(), g.double().sum(0).cpu().numpy()) <= F32_TOL
    assert rel_err(gw.double().cpu().numpy(), (g.double().t() @ h.double()).cpu().numpy()) <= HALF_TOL[torch.bfloat16]


def test_wgrad_deterministic():
    g, h, _ = _operands(2048, 256, 256, torch.float16, seed=3)
    a_w, a_b = _wgrad(g, h, torch.float16)
    b_w, b_b = _wgrad(g, h, torch.float16)
    torch.cuda.synchronize()
    assert torch.equal(a_w, b_w) and torch.equal(a_b, b_b)


def test_tf32_split_is_exact():
    gen = torch.Generator().manual_seed(4)
    x = (torch.randn(1000, 64, generator=gen) * 1e3).cuda()
    big, small = torch.empty_like(x), torch.empty_like(x)
    nat.check(nat.load().tropnn_b200_tf32_split(x.data_ptr(), x.numel(), big.data_ptr(), small.data_ptr(), _stream()),
              "tf32_split")
    torch.cuda.synchronize()
    low = (1 << 13) - 1
    assert int((big.view(torch.int32) & low).abs().sum()) == 0
    assert int((small.view(torch.int32) & low).abs().sum()) == 0
    assert rel_err((big.double() + small.double()).cpu().numpy(), x.double().cpu().numpy()) <= 2**-22


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_autograd_matches_reference(dtype):
    """linear_f32out_b200's backward against the reference's f32 F.linear backward."""
    rows, out_features, in_features = 640, 1024, 256
    gen = torch.Generator().manual_seed(5)
    x = torch.randn(rows, in_features, generator=gen).cuda().requires_grad_(True)
    w = (torch.randn(out_features, in_features, generator=gen) / 16).to(dtype).cuda().requires_grad_(True)
    b = (0.1 * torch.randn(out_features, generator=gen)).to(dtype).cuda().requires_grad_(True)
    g = torch.randn(rows, out_features, generator=gen).cuda()
    linear_f32out_b200(x, w, b).backward(g)
    torch.cuda.synchronize()
    xd = x.detach().double()
    assert rel_err(x.grad.cpu().numpy(), (g.double() @ w.detach().double()).cpu().numpy()) <= F32_TOL
    assert w.grad.dtype == dtype and b.grad.dtype == dtype
    assert rel_err(w.grad.double().cpu().numpy(), (g.double().t() @ xd).cpu().numpy()) <= HALF_TOL[dtype]
    assert rel_err(b.grad.double().cpu().numpy(), g.double().sum(0).cpu().numpy()) <= HALF_TOL[dtype]
