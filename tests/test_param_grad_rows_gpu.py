"""tropnn_b200_trop_param_grad_rows: the f32 TropLinear code, router and router-bias gradients
summed straight from the rows (tropical_exact.py:204-237 summed over the batch), against the
same sums in f64 on the CPU, at ragged shapes (rows not a multiple of the 128-row staging chunk,
code_dim not a multiple of the 32-column CTA chunk), 2 and 32 cells, eval (no runner-up term)
and partial requests. f32 accumulation in a different order: 1e-5 relative."""

from __future__ import annotations

import pytest
import torch

from tests.golden_cases import rel_err
from tropnn_b200 import _native as nat

pytestmark = pytest.mark.gpu


def _expected(g, z, win, run, cw, cr, const, gm, heads, cells):
    items, dim = g.shape
    gc = torch.zeros(heads, cells, dim, dtype=torch.float64)
    gw = torch.zeros(heads, cells, dim, dtype=torch.float64)
    gb = torch.zeros(heads, cells, dtype=torch.float64)
    g64, z64 = g.double(), z.double()
    for h in range(heads):
        w = win[:, h].long()
        coef = (cw[:, h] if cw is not None else torch.full((items,), const)).double()
        gc[h].index_add_(0, w, coef[:, None] * g64)
        if run is not None:
            r = run[:, h].long()
            gc[h].index_add_(0, r, cr[:, h].double()[:, None] * g64)
            m = gm[:, h].double()
            gw[h].index_add_(0, w, m[:, None] * z64)
            gw[h].index_add_(0, r, -m[:, None] * z64)
            gb[h].index_add_(0, w, m)
            gb[h].index_add_(0, r, -m)
    return gc, gw, gb


@pytest.mark.parametrize(
    ("items", "dim", "heads", "cells", "training", "want"),
    [
        (300, 40, 7, 16, True, "both"),  # ragged rows and columns
        (1, 64, 3, 2, True, "both"),  # one row, two cells
        (513, 96, 5, 32, True, "router"),  # 32 cells, router only
        (257, 33, 4, 8, False, "code"),  # eval: winners only, constant coefficient
        (2048, 64, 16, 16, True, "code"),
    ],
)
def test_param_grad_rows_matches_f64_sums(items, dim, heads, cells, training, want) -> None:
    gen = torch.Generator().manual_seed(items + dim)
    g = torch.randn(items, dim, generator=gen)
    z = torch.randn(items, dim, generator=gen)
    win = torch.randint(0, cells, (items, heads), generator=gen).to(torch.uint8)
    run = ((win.long() + torch.randint(1, cells, (items, heads), generator=gen)) % cells).to(torch.uint8)
    cw = torch.rand(items, heads, generator=gen)
    cr = torch.rand(items, heads, generator=gen)
    gm = torch.randn(items, heads, generator=gen)
    const = 0.37
    want_code = want in ("both", "code")
    want_router = training and want in ("both", "router")
    dev = torch.device("cuda")
    gd, zd, wd, rd, cwd, crd, gmd = (t.to(dev) for t in (g, z, win, run, cw, cr, gm))
    gc = torch.full((heads, cells, dim), float("nan"), device=dev) if want_code else None
    gw = torch.full((heads, cells, dim), float("nan"), device=dev) if want_router else None
    gb = torch.full((heads, cells), float("nan"), device=dev) if want_router else None
    lib = nat.load()
    nat.check(
        lib.tropnn_b200_trop_param_grad_rows(
            gd.data_ptr(), zd.data_ptr(), items, dim, nat.F32, heads, cells, wd.data_ptr(),
            rd.data_ptr() if training else None, nat.U8, cwd.data_ptr() if training else None,
            crd.data_ptr() if training else None, const, gmd.data_ptr() if training else None, nat.ptr(gc),
            nat.ptr(gw), nat.ptr(gb), nat.stream_handle(dev),
        ),
        "trop_param_grad_rows",
    )
    torch.cuda.synchronize()
    ec, ew, eb = _expected(g, z, win, run if training else None, cw if training else None, cr, const, gm, heads, cells)
    if want_code:
        assert rel_err(gc.cpu().numpy(), ec.float().numpy()) <= 1e-5
    if want_router:
        assert rel_err(gw.cpu().numpy(), ew.float().numpy()) <= 1e-5
        assert rel_err(gb.cpu().numpy(), eb.float().numpy()) <= 1e-5


def test_param_grad_rows_is_deterministic() -> None:
    gen = torch.Generator().manual_seed(5)
    items, dim, heads, cells = 1000, 64, 8, 16
    dev = torch.device("cuda")
    g, z = torch.randn(items, dim, generator=gen).to(dev), torch.randn(items, dim, generator=gen).to(dev)
    win = torch.randint(0, cells, (items, heads), generator=gen).to(torch.uint8).to(dev)
    run = ((win.long() + 1) % cells).to(torch.uint8)
    cw, cr, gm = (torch.randn(items, heads, generator=gen).to(dev) for _ in range(3))
    lib = nat.load()
    outs = []
    for _ in range(2):
        gc = torch.empty(heads, cells, dim, device=dev)
        gw = torch.empty(heads, cells, dim, device=dev)
        gb = torch.empty(heads, cells, device=dev)
        nat.check(lib.tropnn_b200_trop_param_grad_rows(
            g.data_ptr(), z.data_ptr(), items, dim, nat.F32, heads, cells, win.data_ptr(), run.data_ptr(), nat.U8,
            cw.data_ptr(), cr.data_ptr(), 1.0, gm.data_ptr(), gc.data_ptr(), gw.data_ptr(), gb.data_ptr(),
            nat.stream_handle(dev)), "trop_param_grad_rows")
        outs.append((gc, gw, gb))
    torch.cuda.synchronize()
    assert all(torch.equal(a, b) for a, b in zip(outs[0], outs[1]))


def test_param_grad_rows_rejects_unsupported() -> None:
    lib = nat.load()
    dev = torch.device("cuda")
    x = torch.zeros(4, 8, device=dev)
    routes = torch.zeros(4, 2, device=dev, dtype=torch.uint8)
    out = torch.zeros(2, 64, 8, device=dev)
    # 64 cells: beyond the kernel's 32.
    status = lib.tropnn_b200_trop_param_grad_rows(
        x.data_ptr(), x.data_ptr(), 4, 8, nat.F32, 2, 64, routes.data_ptr(), None, nat.U8, None, None, 1.0, None,
        out.data_ptr(), None, None, nat.stream_handle(dev))
    assert status != 0 and b"32 cells" in lib.tropnn_b200_last_error()
