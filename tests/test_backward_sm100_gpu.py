"""The tensor-core min-face backward (trop_gm, trop_router_term, trop_param_grad) against the
oracle's coefficient-form backward (layers/tropical_exact.py:204-237).

Half-precision parameters with u8 routes, code_dim a multiple of 64 and a row count that is a
multiple of 8 take this path. The reference backward is evaluated in f32 on the same routes
(read back through the C ABI route call, which the forward uses), so the comparison isolates
arithmetic: the GEMMs round g (code gradient) and gm (router term, router gradient) to the
parameter dtype once, which keeps every gradient within 5e-3 (f16) / 2e-2 (bf16) relative,
inside the 2e-2 half-precision tolerance.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from tests.golden_cases import rel_err
from tropnn_b200 import _native as nat
from tropnn_b200.ops import trop_route_hidden_packed

pytestmark = pytest.mark.gpu

TOL = {torch.float16: 5e-3, torch.bfloat16: 2e-2}


def _routes(z, weight, bias):
    lib = nat.load()
    items, code_dim = z.shape
    heads, cells, _ = weight.shape
    win = torch.empty(items, heads, dtype=torch.uint8, device=z.device)
    run = torch.empty(items, heads, dtype=torch.uint8, device=z.device)
    m = torch.empty(items, heads, dtype=torch.float32, device=z.device)
    nat.check(
        lib.tropnn_b200_trop_route(
            z.data_ptr(), nat.float_code(z.dtype), items, code_dim, weight.data_ptr(), bias.float().data_ptr(), nat.F32,
            nat.float_code(weight.dtype), heads, cells, None, win.data_ptr(), run.data_ptr(), nat.U8, m.data_ptr(),
            None, 0, torch.cuda.current_stream().cuda_stream,
        ),
        "trop_route",
    )
    torch.cuda.synchronize()
    return win.long().cpu().numpy(), run.long().cpu().numpy(), m.cpu().numpy()


def _check(items, heads, cells, code_dim, dtype, training, seed=0, g_scale=1.0, check_params=True, z_dtype=None):
    gen = torch.Generator().manual_seed(seed)
    z = torch.randn(items, code_dim, generator=gen).to(z_dtype or dtype).cuda()
    weight = (torch.randn(heads, cells, code_dim, generator=gen) / code_dim**0.5).to(dtype).cuda()
    bias = (0.1 * torch.randn(heads, cells, generator=gen)).to(dtype).cuda()
    code = (0.5 * torch.randn(heads, cells, code_dim, generator=gen)).to(dtype).cuda()
    g = (torch.randn(items, code_dim, generator=gen) * g_scale).cuda()
    scale = heads**-0.5
    params = [t.clone().requires_grad_(True) for t in (weight, bias, code)]
    zl = z.clone().requires_grad_(True)
    hidden, _, _ = trop_route_hidden_packed(
        zl.view(1, items, code_dim), params[0], params[1], params[2], code_scale=scale, training=training, keep_margins=True
    )
    hidden.backward(g.view(1, items, code_dim))
    torch.cuda.synchronize()
    win, run, m = _routes(z, weight, bias)
    ref = oracle.trop_route_backward(
        g.cpu().numpy(), z.float().cpu().numpy(), weight.float().cpu().numpy(), code.float().cpu().numpy(), win, run, m,
        code_scale=scale, training=training,
    )
    tol = TOL[dtype]
    assert rel_err(zl.grad.float().cpu().numpy(), ref["grad_latent"]) <= tol
    if not check_params:
        return
    assert rel_err(params[2].grad.float().cpu().numpy(), ref["grad_code"]) <= tol
    if training:
        assert rel_err(params[0].grad.float().cpu().numpy(), ref["grad_router_weight"]) <= tol
        assert rel_err(params[1].grad.float().cpu().numpy(), ref["grad_router_bias"]) <= tol
    else:
        assert params[0].grad is None and params[1].grad is None


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("training", [True, False])
def test_config5_shape(dtype, training):
    """Config 5's layer (H1024, K16, D256) on a 512-row slice."""
    _check(512, 1024, 16, 256, dtype, training)


@pytest.mark.parametrize("cells", [2, 4, 8, 32])
def test_cells(cells):
    _check(256, max(8, 512 // cells), cells, 128, torch.float16, True)


@pytest.mark.parametrize(
    ("items", "heads", "cells", "code_dim"),
    [
        (136, 12, 16, 64),  # one full and one 8-row k block of rows; 192 cells (a partial tile)
        (1000, 200, 8, 192),  # many tiles, N=192
        (2048, 64, 16, 256),  # several row blocks per CTA in the gm / router-term GEMMs
    ],
)
def test_shapes(items, heads, cells, code_dim):
    _check(items, heads, cells, code_dim, torch.float16, True)


@pytest.mark.parametrize("g_scale", [1e-7, 1e5])
def test_gradient_range(g_scale):
    """Upstream gradients far below f16's normal range (1e-7: rounded to f16 as they are, g and gm
    would mostly flush to zero) and beyond its maximum (1e5: g itself would overflow): the
    power-of-two gradient scale keeps grad_latent (f32 here: an f32 latent) within the tolerance
    of O(1) gradients.
    The parameter gradients are f16 outputs, rounded like the reference's (whose f32 values are
    cast back to the parameter dtype), so at these scales they leave f16's range in both."""
    _check(512, 256, 16, 128, torch.float16, True, seed=3, g_scale=g_scale, check_params=False, z_dtype=torch.float32)


def test_small_gradients_parameter_grads():
    """Gradients of 1e-3 (gm ~1e-5: its f16 rounding alone would keep ~1e-2 relative): every
    gradient, the f16 parameter gradients included, within the tolerance."""
    _check(512, 256, 16, 128, torch.float16, True, seed=4, g_scale=1e-3, z_dtype=torch.float32)


def test_no_device_error():
    import ctypes

    _check(256, 64, 16, 128, torch.float16, True)
    flag = ctypes.c_int(-1)
    nat.check(nat.load().tropnn_b200_device_error(ctypes.byref(flag)), "device_error")
    assert flag.value == 0
