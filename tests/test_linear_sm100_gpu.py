"""The tensor-core f32-output linear map (split_half + linear_f32out) against f32 torch.

The output map of a half-precision TropLinear multiplies the f32 hidden by the upcast
weight in f32 (layers/tropical.py:140-146). On backend="b200" the hidden is split into
[hi | lo] halves and multiplied on the tensor cores with f32 accumulation: within 5e-6
relative of the f32 product for f16 weights (hi + lo keeps ~22 bits) and 3e-5 for bf16
(~16 bits), far inside the 2e-2 tolerance of half-precision layers.
"""

from __future__ import annotations

import pytest
import torch

from tests.golden_cases import rel_err
from tropnn_b200 import _native as nat
from tropnn_b200.ops import linear_f32out_b200

pytestmark = pytest.mark.gpu

TOL = {torch.float16: 5e-6, torch.bfloat16: 3e-5}


def _case(rows, in_features, out_features, dtype, with_bias, seed=0):
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, in_features, generator=gen).cuda()
    w = (torch.randn(out_features, in_features, generator=gen) / in_features**0.5).to(dtype).cuda()
    b = (0.1 * torch.randn(out_features, generator=gen)).to(dtype).cuda() if with_bias else None
    return x, w, b


def _reference(x, w, b):
    out = x.double() @ w.double().t()
    if b is not None:
        out = out + b.double()
    return out


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize(
    ("rows", "in_features", "out_features", "with_bias"),
    [
        (1000, 256, 4096, True),  # config 5's output map, 8 row blocks
        (300, 64, 100, True),  # ragged rows, one partial output tile
        (129, 128, 260, False),  # one row in the last block, 2 tiles (second nearly empty)
        (4096, 192, 512, True),  # several row blocks per CTA
    ],
)
def test_against_f32(dtype, rows, in_features, out_features, with_bias):
    x, w, b = _case(rows, in_features, out_features, dtype, with_bias)
    out = linear_f32out_b200(x, w, b)
    torch.cuda.synchronize()
    assert out.dtype == torch.float32 and out.shape == (rows, out_features)
    assert rel_err(out.cpu().numpy(), _reference(x, w, b).cpu().numpy()) <= TOL[dtype]


def test_plain_half_gemm_one_slice():
    """slices = 1: a plain f16 x f16 -> f32 product."""
    x, w, b = _case(512, 128, 384, torch.float16, True, seed=1)
    xh = x.half().contiguous()
    out = torch.empty(512, 384, device="cuda")
    lib = nat.load()
    b32 = b.float().contiguous()
    nat.check(
        lib.tropnn_b200_linear_f32out(
            xh.data_ptr(), 512, 1, w.data_ptr(), 384, 128, nat.F16, b32.data_ptr(), out.data_ptr(),
            torch.cuda.current_stream().cuda_stream,
        ),
        "linear_f32out",
    )
    torch.cuda.synchronize()
    ref = xh.double() @ w.double().t() + b.double()
    assert rel_err(out.cpu().numpy(), ref.cpu().numpy()) <= 1e-6


def test_split_half_is_exact_to_two_terms():
    gen = torch.Generator().manual_seed(2)
    x = (torch.randn(64, 128, generator=gen) * 3).cuda()
    out = torch.empty(64, 256, dtype=torch.float16, device="cuda")
    nat.check(
        nat.load().tropnn_b200_split_half(
            x.data_ptr(), 64, 128, nat.F16, None, out.data_ptr(), torch.cuda.current_stream().cuda_stream
        ),
        "split_half",
    )
    torch.cuda.synchronize()
    hi, lo = out[:, :128].float(), out[:, 128:].float()
    assert torch.equal(out[:, :128], x.half())
    assert ((hi + lo - x).abs() <= x.abs() * 2.0**-21 + 1e-7).all()


def test_backward_matches_f32_autograd():
    x, w, b = _case(256, 128, 64, torch.float16, True, seed=4)
    w = w.clone().requires_grad_(True)
    b = b.clone().requires_grad_(True)
    xr = x.clone().requires_grad_(True)
    out = linear_f32out_b200(xr, w, b)
    g = torch.randn_like(out)
    out.backward(g)
    x2 = x.clone().requires_grad_(True)
    w2 = w.detach().clone().requires_grad_(True)
    b2 = b.detach().clone().requires_grad_(True)
    ref = torch.nn.functional.linear(x2, w2.float(), b2.float())
    ref.backward(g)
    assert rel_err(xr.grad.cpu().numpy(), x2.grad.cpu().numpy()) <= 1e-6
    assert w.grad.dtype == torch.float16 and b.grad.dtype == torch.float16
    assert rel_err(w.grad.float().cpu().numpy(), w2.grad.float().cpu().numpy()) <= 1e-3
    assert rel_err(b.grad.float().cpu().numpy(), b2.grad.float().cpu().numpy()) <= 1e-3
