"""A TropLinear layer on the GPU against the numpy oracle on rows whose routes the parity
gate pins (test helper).

Route indices are compared wherever the parity gate pins them; values and gradients are
compared on a batch in which the gate pins every route (the winner, and in training also the
runner-up, whose code enters the min-face mix): near-tie routes are outside the parity
contract, and a flipped route moves a row-summed parameter gradient by far more than the
tolerance. The oracle routes on the layer's own z:

* f32 projection weights: the oracle's f32 z (the GPU's 3xTF32 product differs by ~1e-6
  relative, far inside the 1e-4 gate);
* half-precision projection weights: z as the layer computes it (ops.trop_project_b200 on the
  same rows), since two f32 summation orders may round a sum on a rounding boundary of the
  half dtype one unit apart, which moves a score by up to ~1e-4 relative. The projection
  itself is checked separately (tests/test_proj_sm100_gpu.py).

Rows are independent, and the projection's result for a row depends only on the row and the
batch size, so a batch in which some route is not pinned is repaired by replacing those rows
with further rows of the pool (same size, the other rows' z unchanged).
"""

from __future__ import annotations

import numpy as np
import torch

import oracle
import tropnn_b200
import tropnn_b200.ops
from tests.golden_cases import rel_err, route_gate, state_arrays


def _layer_z(layer: tropnn_b200.TropLinear, st: dict, x: np.ndarray, pdt: str) -> np.ndarray:
    if layer.proj.weight.dtype in (torch.float16, torch.bfloat16) and tropnn_b200.ops.proj_eligible(
        torch.empty(1, x.shape[1], device="cuda"), layer.proj.weight.cuda()
    ):
        with torch.no_grad():
            z = tropnn_b200.ops.trop_project_b200(torch.from_numpy(x).cuda(), layer.proj.weight.cuda())
        return z.float().cpu().numpy()
    return oracle.trop_linear_forward(x, st, code_scale=1.0, training=False, param_dtype=pdt)["z"]


def _pinned(st: dict, z: np.ndarray, train: bool) -> np.ndarray:
    win, run = route_gate(oracle.trop_scores(z, st["router_weight"], st["router_bias"]))
    return (run if train else win).all(axis=1)


def pinned_batch(layer: tropnn_b200.TropLinear, pool: np.ndarray, rows: int, *, train: bool) -> np.ndarray:
    """``rows`` rows of ``pool`` whose routes the gate pins at batch size ``rows``."""
    st = state_arrays(layer)
    pdt = str(layer.proj.weight.dtype).replace("torch.", "")
    pinned = _pinned(st, _layer_z(layer, st, pool, pdt), train)
    spare = [int(i) for i in np.nonzero(pinned)[0]]
    assert len(spare) >= rows, f"only {len(spare)} pinned rows in a pool of {pool.shape[0]}"
    chosen, spare = spare[:rows], spare[rows:]
    for _ in range(8):
        ok = _pinned(st, _layer_z(layer, st, pool[chosen], pdt), train)
        if ok.all():
            return pool[chosen]
        for i in np.nonzero(~ok)[0]:
            assert spare, "the pool ran out of pinned rows"
            chosen[i] = spare.pop(0)
    raise AssertionError("no pinned batch found")


def check_trop_routes(layer: tropnn_b200.TropLinear, x: np.ndarray, *, train: bool) -> None:
    """Winners of a whole batch (no row selection) against the oracle wherever the gate pins them."""
    st = state_arrays(layer)
    pdt = str(layer.proj.weight.dtype).replace("torch.", "")
    layer = layer.cuda().train(train)
    with torch.no_grad():
        layer(torch.from_numpy(x).cuda())
    z = _layer_z(layer, st, x, pdt)
    scores = oracle.trop_scores(z, st["router_weight"], st["router_bias"])
    win, _ = route_gate(scores)
    want = oracle.top2_indices(scores)[0]
    got = layer._last_indices.cpu().numpy().reshape(x.shape[0], -1)
    assert np.array_equal(got[win], want[win])


def check_trop_layer(layer: tropnn_b200.TropLinear, x: np.ndarray, g: np.ndarray, *, train: bool, tol: float) -> None:
    """Runs ``layer`` forward and backward on ``x`` (every route pinned, see pinned_batch) and
    compares routes, margins, output and every gradient with the oracle on the layer's z."""
    st = state_arrays(layer)
    pdt = str(layer.proj.weight.dtype).replace("torch.", "")
    layer = layer.cuda().train(train)
    layer.zero_grad(set_to_none=True)
    xt = torch.from_numpy(x).cuda().requires_grad_(True)
    y = layer(xt)
    y.backward(torch.from_numpy(g).cuda().view_as(y))
    torch.cuda.synchronize()
    n = x.shape[0]
    z = _layer_z(layer, st, x, pdt)
    route = oracle.trop_route_hidden(z, st["router_weight"], st["router_bias"], st["code"],
                                     code_scale=layer.code_scale, training=train)
    w_out = st["output_proj.weight"].astype(np.float32)
    fwd = {**route, "z": z, "y": (route["hidden"] @ w_out.T + st["output_proj.bias"].astype(np.float32)).astype(np.float32)}
    assert np.array_equal(layer._last_indices.cpu().numpy().reshape(n, -1), fwd["winner"])
    assert rel_err(layer._last_margins.cpu().numpy().reshape(n, -1), fwd["margins"]) <= max(tol, 1e-5)
    assert rel_err(y.detach().float().cpu().numpy().reshape(n, -1), fwd["y"]) <= tol
    ref = oracle.trop_linear_backward(g, x, st, fwd, code_scale=layer.code_scale, training=train, param_dtype=pdt)
    assert rel_err(xt.grad.cpu().numpy(), ref["x"]) <= tol
    params = dict(layer.named_parameters())
    for key in ("proj.weight", "code", "output_proj.weight", "output_proj.bias"):
        p = params[key]
        assert p.grad is not None and p.grad.dtype == p.dtype, key
        assert rel_err(p.grad.float().cpu().numpy(), ref[key]) <= tol, key
    if train:
        for key in ("router_weight", "router_bias"):
            assert rel_err(params[key].grad.float().cpu().numpy(), ref[key]) <= tol, key
    else:
        assert params["router_weight"].grad is None and params["router_bias"].grad is None
