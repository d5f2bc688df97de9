"""Config 5 at its real layer shapes on the GPU against the numpy oracle.

* PairwiseLinear(4096 -> 4096, tables=1024, comparisons=8) with an f16 LUT (2 GiB): forward
  indices bit-exact, output, grad_latent and grad_thresholds over all tables, and grad_lut
  through the above-1024-column path (bucket_sort + segment_rowsum) compared densely on every
  16th table (tables are independent) plus a check over all tables: every row adds its
  scaled gradient to exactly one bucket per table, so the bucket sums of grad_lut add up to
  tables * output_scale * sum_n g[n]. The oracle runs in row chunks (its [rows, tables, out]
  gathers are 128 MiB per 8 rows here).
* TropLinear(4096 -> 4096, heads=1024, cells=16, code_dim=256), f16 parameters, 512 rows,
  the whole layer (projection, tensor-core route scores and top-2, one-hot code sum, output
  map, and in training every gradient: projection, router weight and bias, code, output map).
  Rows are drawn from a seeded pool and kept where every head's route is pinned by the parity
  gate (winner, and in training the runner as well), so that the row-summed parameter
  gradients are comparable (a multiple of 8 rows: the tensor-core backward's granularity).

Tolerance: 2e-2 relative (f16 parameters), the parity rule for half-precision layers.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
import tropnn_b200
import tropnn_b200.ops
from oracle.tropnn_oracle import _round_to
from tests.golden_cases import rel_err, state_arrays
from tests.trop_check import check_trop_layer, pinned_batch

pytestmark = pytest.mark.gpu
HALF_TOL = 2e-2


# ------------------------------------------------------------------ PairwiseLinear


@pytest.fixture(scope="module")
def pairwise_cfg5():
    layer = tropnn_b200.PairwiseLinear(4096, 4096, tables=1024, comparisons=8, seed=0).half()
    lut32 = layer.lut.detach().float().numpy()  # f16 values, exact in f32; converted once
    anchors = layer.anchors.numpy().copy()
    thresholds = layer.thresholds.detach().float().numpy()
    return layer.cuda(), lut32, anchors, thresholds


def _pairwise_inputs(rows: int, seed: int) -> tuple[np.ndarray, np.ndarray]:
    gen = torch.Generator().manual_seed(seed)
    return torch.randn(rows, 4096, generator=gen).numpy(), torch.randn(rows, 4096, generator=gen).numpy()


def test_pairwise_config5_train_matches_oracle(pairwise_cfg5) -> None:
    layer, lut32, anchors, thresholds = pairwise_cfg5
    rows, chunk = 64, 8
    x, g = _pairwise_inputs(rows, seed=21)
    layer.train()
    layer.zero_grad(set_to_none=True)
    xt = torch.from_numpy(x).cuda().requires_grad_(True)
    y = layer(xt)
    y.backward(torch.from_numpy(g).cuda().view_as(y))
    torch.cuda.synchronize()
    got_y = y.detach().float().cpu().numpy().reshape(rows, -1)
    got_idx = layer._last_indices.cpu().numpy().reshape(rows, -1)

    want_y = np.empty_like(got_y)
    want_gx = np.empty((rows, 4096), dtype=np.float32)
    want_gthr = np.zeros((1024, 8), dtype=np.float64)
    indices = np.empty((rows, 1024), dtype=np.int64)
    for lo in range(0, rows, chunk):
        sl = slice(lo, lo + chunk)
        fwd = oracle.pairwise_forward(x[sl], anchors, thresholds, lut32, output_scale=layer.output_scale)
        want_y[sl] = fwd["out"]
        indices[sl] = fwd["indices"]
        bwd = oracle.pairwise_backward(
            g[sl], fwd["indices"], fwd["margins"], anchors, lut32, in_features=4096,
            output_scale=layer.output_scale, use_min_margin_ste=True, lut_grad=False,
        )
        want_gx[sl] = bwd["x"]
        want_gthr += bwd["thresholds"]
    assert np.array_equal(got_idx, indices)  # first-layer comparator routes: bit-exact
    assert rel_err(got_y, want_y) <= HALF_TOL
    assert rel_err(xt.grad.cpu().numpy(), want_gx) <= HALF_TOL
    assert rel_err(layer.thresholds.grad.float().cpu().numpy(), want_gthr) <= HALF_TOL

    # grad_lut: dense on every 16th table (the oracle's full [1024, 256, 4096] f32 gradient
    # would be 4 GiB), from the same rows and routes.
    grad_lut = layer.lut.grad
    assert grad_lut.dtype == torch.float16 and bool(torch.isfinite(grad_lut).all())
    sub = slice(0, 1024, 16)
    ref = oracle.pairwise_backward(
        g, indices[:, sub], None, anchors[sub], lut32[sub], in_features=4096, output_scale=layer.output_scale,
        use_min_margin_ste=True, ste=False,
    )["lut"]
    assert rel_err(grad_lut[sub].float().cpu().numpy(), ref) <= HALF_TOL
    # All tables: bucket sums per table equal output_scale * sum_n g (each row lands in one
    # bucket per table), and buckets no row selected stay exactly zero.
    col_sum = torch.from_numpy(g.astype(np.float64).sum(axis=0) * layer.output_scale).cuda()
    per_table = grad_lut.float().sum(dim=1).double()  # [1024, 4096]
    assert float((per_table - col_sum).abs().max() / col_sum.abs().max()) <= HALF_TOL
    hit = torch.zeros(1024, 256, dtype=torch.bool, device="cuda")
    hit[torch.arange(1024).repeat(rows), torch.from_numpy(indices.reshape(-1)).cuda()] = True
    assert float(grad_lut[~hit].abs().max()) == 0.0


def test_pairwise_config5_eval_matches_oracle(pairwise_cfg5) -> None:
    layer, lut32, anchors, thresholds = pairwise_cfg5
    rows = 32
    x, _ = _pairwise_inputs(rows, seed=22)
    layer.eval()
    with torch.no_grad():
        y = layer(torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    fwd = oracle.pairwise_forward(x, anchors, thresholds, lut32, output_scale=layer.output_scale)
    assert np.array_equal(layer._last_indices.cpu().numpy().reshape(rows, -1), fwd["indices"])
    assert np.array_equal(layer._last_margins.cpu().numpy().reshape(rows, 1024, 8), fwd["margins"])
    assert rel_err(y.float().cpu().numpy().reshape(rows, -1), fwd["out"]) <= HALF_TOL


# ------------------------------------------------------------------ TropLinear


@pytest.fixture(scope="module")
def trop_cfg5():
    layer = tropnn_b200.TropLinear(4096, 4096, heads=1024, cells=16, code_dim=256, seed=0).half()
    return layer, state_arrays(layer)


@pytest.mark.parametrize("train", [True, False])
def test_trop_config5_layer_matches_oracle(trop_cfg5, train: bool) -> None:
    """The projection against the oracle's rounded z (one f16 unit plus the f32 accumulation
    error: two summation orders may round a sum on a boundary differently), then the whole
    layer, forward and backward, on 512 pinned rows with the oracle routing on the layer's z
    (tests/trop_check.py)."""
    layer, st = trop_cfg5
    gen = torch.Generator().manual_seed(31 if train else 32)
    pool = torch.randn(3072, 4096, generator=gen).numpy()
    g = torch.randn(512, 4096, generator=gen).numpy()
    layer = layer.cuda()
    z_oracle = _round_to(_round_to(pool, "float16") @ st["proj.weight"].astype(np.float32).T, "float16")
    with torch.no_grad():
        z_pool = tropnn_b200.ops.trop_project_b200(torch.from_numpy(pool).cuda(), layer.proj.weight).float().cpu().numpy()
    ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(z_oracle), 2.0**-14))) - 10)
    bound = ulp + 3e-5 * float(np.abs(z_oracle).max())
    assert np.all(np.abs(z_pool - z_oracle) <= bound), "projection beyond one f16 unit of the oracle"
    x = pinned_batch(layer, pool, 512, train=train)
    check_trop_layer(layer, x, g, train=train, tol=HALF_TOL)
    layer.cpu()
