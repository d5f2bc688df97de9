"""The f32 tensor-core product (tropnn_b200_gemm_tf32x3, 3xTF32) and the f32 linear map built on
it (ops.linear_f32_b200: forward and backward of F.linear in f32) against f64 products: within
the fp32 parity tolerance (1e-5 of the largest output) for the shapes of configs 1 and 3 and
ragged ones (k not a multiple of the 32-wide k block, m and n not multiples of 128, n not a
multiple of 4 with plain stores), with and without bias; the transpose and column-sum helpers
exactly."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from tests.golden_cases import rel_err
from tropnn_b200.ops import gemm_f32, linear_f32_b200, linear_f32_eligible, transpose_f32

pytestmark = pytest.mark.gpu
FP32_TOL = 1e-5


@pytest.mark.parametrize(
    ("m", "n", "k", "with_bias"),
    [
        (512, 64, 784, False),  # config 3 layer 1 projection
        (512, 128, 64, True),  # config 3 layer 1 output map
        (512, 10, 64, True),  # config 3 layer 2 output map (n % 4 != 0: plain stores)
        (8, 512, 32, True),  # config 1 output map (at most 32 rows: the f32 FMA kernel)
        (32, 300, 1000, False),  # the largest row count of the f32 FMA kernel, long contraction
        (1, 7, 8, True),  # one row
        (33, 64, 256, True),  # the fewest rows of the tensor-core kernel
        (300, 200, 100, True),  # ragged everywhere
        (4096, 4096, 256, False),  # many tiles
    ],
)
def test_gemm_matches_f64(m: int, n: int, k: int, with_bias: bool) -> None:
    gen = torch.Generator().manual_seed(m + n + k)
    a = torch.randn(m, k, generator=gen)
    b = torch.randn(n, k, generator=gen) / k**0.5
    bias = torch.randn(n, generator=gen) if with_bias else None
    c = gemm_f32(a.cuda(), b.cuda(), None if bias is None else bias.cuda())
    torch.cuda.synchronize()
    ref = a.double() @ b.double().t() + (0 if bias is None else bias.double())
    assert c.shape == (m, n)
    assert rel_err(c.cpu().numpy(), ref.numpy()) <= FP32_TOL


def test_transpose_and_padding() -> None:
    x = torch.randn(37, 45, device="cuda")
    t = transpose_f32(x)
    assert t.shape == (45, 40)
    assert torch.equal(t[:, :37], x.t()) and bool((t[:, 37:] == 0).all())


@pytest.mark.parametrize(("rows", "in_f", "out_f"), [(512, 784, 64), (512, 64, 10), (33, 128, 130)])
def test_linear_f32_forward_backward(rows: int, in_f: int, out_f: int) -> None:
    gen = torch.Generator().manual_seed(rows + out_f)
    x = torch.randn(rows, in_f, generator=gen)
    w = torch.randn(out_f, in_f, generator=gen) / in_f**0.5
    b = torch.randn(out_f, generator=gen)
    g = torch.randn(rows, out_f, generator=gen)
    xd, wd, bd = (t.cuda().requires_grad_(True) for t in (x, w, b))
    assert linear_f32_eligible(xd, wd)
    y = linear_f32_b200(xd, wd, bd)
    y.backward(g.cuda())
    torch.cuda.synchronize()
    x64, w64, g64 = x.double(), w.double(), g.double()
    assert rel_err(y.detach().cpu().numpy(), (x64 @ w64.t() + b.double()).numpy()) <= FP32_TOL
    assert rel_err(xd.grad.cpu().numpy(), (g64 @ w64).numpy()) <= FP32_TOL
    assert rel_err(wd.grad.cpu().numpy(), (g64.t() @ x64).numpy()) <= FP32_TOL
    assert np.array_equal(bd.grad.cpu().numpy(), g.sum(0).numpy()) or rel_err(bd.grad.cpu().numpy(), g64.sum(0).numpy()) <= 1e-6
