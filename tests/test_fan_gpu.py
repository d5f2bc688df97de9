"""TropFanLinear (layers/fan.py:21-330) on the b200 kernels against the reference's golden
vectors and against the numpy oracle at classifier width.

The layer is TropLinear's path with the sites and lifting as the router and the generated
value table as the code: routes are compared where the parity gate pins them, values and every
gradient (sites through both the scores and the values, value_scale or value_coeff /
value_basis, lifting, proj, output map, x) within 1e-5 relative for f32 parameters and 2e-2 for
f16. At width, batches are pinned as the TropLinear checks do (every winner, and in training
every runner-up, clear of the 1e-4 margin gate) and the oracle routes on the layer's own z.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
import tropnn_b200
import tropnn_b200.ops
from tests.golden_cases import build_layer, case_names, load_case, rel_err, route_gate, state_arrays, tolerance
from tests.gpu_runner import run_b200

pytestmark = pytest.mark.gpu
FP32_TOL = 1e-5
PARAMS = ("proj.weight", "sites", "lifting", "value_scale", "value_coeff", "value_basis", "output_proj.weight",
          "output_proj.bias")


def _gate(st: dict, z: np.ndarray, train: bool) -> np.ndarray:
    win, run = route_gate(oracle.trop_scores(z, st["sites"], st["lifting"]))
    return run if train else win


def _oracle_z(layer: tropnn_b200.TropFanLinear, st: dict, x: np.ndarray) -> np.ndarray:
    """The layer's own z: f16 projections as the projection kernel rounds them, f32 ones as the
    oracle computes them (3xTF32 differs by ~1e-6 relative, inside the gate)."""
    if layer.proj.weight.dtype == torch.float16:
        with torch.no_grad():
            return tropnn_b200.ops.trop_project_b200(torch.from_numpy(x).cuda(), layer.proj.weight.cuda()).float().cpu().numpy()
    pdt = str(layer.proj.weight.dtype).replace("torch.", "")
    return oracle.trop_fan_forward(x, st, code_scale=1.0, training=False, fan_value_mode=layer.fan_value_mode,
                                   param_dtype=pdt)["z"]


def _pinned_batch(layer: tropnn_b200.TropFanLinear, pool: np.ndarray, rows: int, train: bool) -> np.ndarray:
    st = state_arrays(layer)
    ok = _gate(st, _oracle_z(layer, st, pool), train).all(axis=1)
    spare = [int(i) for i in np.nonzero(ok)[0]]
    assert len(spare) >= rows, f"only {len(spare)} pinned rows"
    chosen, spare = spare[:rows], spare[rows:]
    for _ in range(8):
        good = _gate(st, _oracle_z(layer, st, pool[chosen]), train).all(axis=1)
        if good.all():
            return pool[chosen]
        for i in np.nonzero(~good)[0]:
            chosen[i] = spare.pop(0)
    raise AssertionError("no pinned batch found")


@pytest.mark.parametrize("name", case_names("fan"))
def test_fan_matches_reference_golden(name: str) -> None:
    arrays, meta = load_case(name)
    layer = build_layer(arrays, meta)
    st = state_arrays(layer)
    got = run_b200(layer, arrays, meta)
    tol = tolerance(meta)
    assert rel_err(got["y"], arrays["y"]) <= tol
    x = arrays["x"].reshape(-1, arrays["x"].shape[-1]).astype(np.float32)
    z = oracle.trop_fan_forward(x, st, code_scale=meta["code_scale"], training=False,
                                fan_value_mode=meta["fan_value_mode"])["z"]
    win = _gate(st, z, False)
    assert np.array_equal(got["last_indices"].reshape(win.shape)[win], arrays["last_indices"].reshape(win.shape)[win])
    assert rel_err(got["last_margins"], arrays["last_margins"]) <= max(tol, 1e-5)
    if meta["train"]:
        assert rel_err(got["grad.x"], arrays["grad.x"]) <= tol
        for key in PARAMS:
            if f"has_grad.{key}" not in arrays:
                continue
            assert bool(got[f"has_grad.{key}"]) == bool(arrays[f"has_grad.{key}"]), key
            if bool(arrays[f"has_grad.{key}"]):
                assert rel_err(got[f"grad.{key}"], arrays[f"grad.{key}"].astype(np.float32)) <= tol, key


@pytest.mark.parametrize(
    ("mode", "half", "train"),
    [("site", False, True), ("basis", False, True), ("site", False, False), ("site", True, True), ("basis", True, False)],
)
def test_fan_at_classifier_width_matches_oracle(mode: str, half: bool, train: bool) -> None:
    layer = tropnn_b200.TropFanLinear(784, 128, heads=256, cells=16, code_dim=64, seed=5, fan_value_mode=mode)
    if half:
        layer = layer.half()
    layer = layer.cuda().train(train)
    gen = np.random.default_rng(11)
    pool = gen.standard_normal((2048, 784)).astype(np.float32)
    x = _pinned_batch(layer, pool, 512, train)
    g = gen.standard_normal((512, 128)).astype(np.float32)
    st = state_arrays(layer)
    tol = 2e-2 if half else FP32_TOL
    layer.zero_grad(set_to_none=True)
    xt = torch.from_numpy(x).cuda().requires_grad_(True)
    y = layer(xt)
    y.backward(torch.from_numpy(g).cuda().view_as(y))
    torch.cuda.synchronize()
    z = _oracle_z(layer, st, x)
    values = oracle.fan_generated_values(st, fan_value_mode=mode)
    if half:
        values = values.astype(np.float16).astype(np.float32)  # the kernels take the table in the router's dtype
    route = oracle.trop_route_hidden(z, st["sites"], st["lifting"], values, code_scale=layer.code_scale, training=train)
    w_out = st["output_proj.weight"].astype(np.float32)
    fwd = {**route, "z": z, "values": values,
           "y": (route["hidden"] @ w_out.T + st["output_proj.bias"].astype(np.float32)).astype(np.float32)}
    n = x.shape[0]
    assert np.array_equal(layer._last_indices.cpu().numpy().reshape(n, -1), fwd["winner"])
    assert rel_err(y.detach().float().cpu().numpy().reshape(n, -1), fwd["y"]) <= tol
    pdt = str(layer.proj.weight.dtype).replace("torch.", "")
    ref = oracle.trop_fan_backward(g, x, st, fwd, code_scale=layer.code_scale, training=train, fan_value_mode=mode,
                                   param_dtype=pdt)
    assert rel_err(xt.grad.cpu().numpy(), ref["x"]) <= tol
    for name, p in layer.named_parameters():
        if ref[name] is None:
            # Eval: the routes carry no gradient to the lifting (nor to basis-mode sites).
            assert p.grad is None, name
            continue
        assert p.grad is not None, name
        assert rel_err(p.grad.float().cpu().numpy(), ref[name]) <= tol, name


def test_fan_tied_recovery_raises() -> None:
    layer = tropnn_b200.TropFanLinear(16, 8, heads=4, cells=4, code_dim=8, fan_recovery_mode="tied").cuda()
    with pytest.raises(RuntimeError, match="tied"):
        layer(torch.randn(3, 16, device="cuda"))
