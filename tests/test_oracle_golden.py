"""Pins the numpy oracle to the reference: golden vectors recorded from the reference's
torch path, and the reference's own known-answer tests."""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from tests.golden_cases import build_layer, case_names, load_case, rel_err, route_gate, state_arrays, tolerance
from tests.oracle_runner import run_oracle


@pytest.mark.parametrize("name", case_names())
def test_oracle_matches_reference_golden(name: str) -> None:
    arrays, meta = load_case(name)
    layer = build_layer(arrays, meta)  # also checks the seeded init against the reference
    state = state_arrays(layer)
    got = run_oracle(arrays, meta, state)
    tol = tolerance(meta)
    assert rel_err(got["y"], arrays["y"]) <= tol
    if "last_indices" in arrays:
        if meta["kind"] in ("trop", "fan"):
            win, _ = route_gate(got["_scores"])
            ref = arrays["last_indices"].reshape(win.shape)
            assert np.array_equal(got["last_indices"].reshape(win.shape)[win], ref[win])
        else:
            # First-layer pairwise indices are bit-exact: (x_a - x_b) - theta in f32.
            assert np.array_equal(got["last_indices"], arrays["last_indices"])
            assert np.array_equal(got["last_margins"], arrays["last_margins"])
    if meta["train"]:
        assert rel_err(got["grad.x"], arrays["grad.x"]) <= tol
        for key in [k for k in arrays if k.startswith("grad.") and k != "grad.x"]:
            if key.startswith("grad.anchors") or not bool(arrays[f"has_{key}"]):
                continue
            assert rel_err(got[key], arrays[key].astype(np.float32)) <= tol, key


# --- reference known-answer tests (restated on the oracle) ---------------------------


def test_top2_kat() -> None:
    """tests/test_routing.py:21-28."""
    scores = np.array([[[1.0, 3.0, 2.0], [5.0, -1.0, 4.5]]], dtype=np.float32)
    winner, runner, margins = oracle.top2_indices(scores)
    assert winner.tolist() == [[1, 0]]
    assert runner.tolist() == [[2, 2]]
    np.testing.assert_allclose(margins, [[1.0, 0.5]])


def test_minface_kat() -> None:
    """tests/test_routing.py:31-38."""
    mixed = oracle.minface_mix(np.array([[[10.0, 2.0]]], np.float32), np.array([[[14.0, 6.0]]], np.float32), np.array([[1.0]], np.float32))
    np.testing.assert_allclose(mixed, [[[11.0, 3.0]]])


def test_packing_dtypes_kat() -> None:
    """tests/test_routing.py:13-18."""
    assert oracle.packed_route_index_dtype(8) == np.uint8
    assert oracle.packed_route_index_dtype(1000) == np.int16
    assert oracle.packed_route_index_dtype(40000) == np.int64


def _unit_trop_params(router: list[float]) -> dict[str, np.ndarray]:
    return {
        "proj.weight": np.ones((1, 1), np.float32),
        "router_weight": np.array(router, np.float32).reshape(1, 3, 1),
        "router_bias": np.zeros((1, 3), np.float32),
        "code": np.array([10.0, 20.0, 30.0], np.float32).reshape(1, 3, 1),
        "output_proj.weight": np.ones((1, 1), np.float32),
        "output_proj.bias": np.zeros(1, np.float32),
    }


def test_trop_eval_winner_only_kat() -> None:
    """tests/test_tropical_core.py:19-32: eval outputs 12 and 28."""
    params = _unit_trop_params([1.0, 0.0, -1.0])
    y1 = oracle.trop_linear_forward(np.array([[2.0]], np.float32), params, code_scale=1.0, training=False)["y"]
    y2 = oracle.trop_linear_forward(np.array([[-2.0]], np.float32), params, code_scale=1.0, training=False)["y"]
    np.testing.assert_allclose(y1.squeeze(), 12.0)
    np.testing.assert_allclose(y2.squeeze(), 28.0)


def test_trop_train_minface_kat() -> None:
    """tests/test_tropical_core.py:35-49: 1 + 10 + (0.5/1.1)(20-10)."""
    params = _unit_trop_params([1.0, 0.9, -1.0])
    y = oracle.trop_linear_forward(np.array([[1.0]], np.float32), params, code_scale=1.0, training=True)["y"]
    np.testing.assert_allclose(y.squeeze(), 1.0 + 10.0 + (0.5 / 1.1) * 10.0, atol=1e-6)


def test_surrogate_sign_kat() -> None:
    """tests/test_pairwise.py:9-15."""
    grad = oracle.surrogate_gradient(np.array([-2.0, 0.0, 2.0], np.float32), "fast_sigmoid_odd")
    assert grad[0] > 0 and grad[1] == 0 and grad[2] < 0


def test_zig_route_kat() -> None:
    """kernels/src/tropical.zig:352-379: hidden = (7, 21, 14, 13) with code_scale 0.5."""
    latent = np.array([[2.0, 1.0], [-1.0, 3.0]], np.float32)
    weight = np.array([1, 0, 0, 1, -1, 0, 0, -1], np.float32).reshape(2, 2, 2)
    code = np.array([10, 0, 0, 20, 30, 0, 0, 40], np.float32).reshape(2, 2, 2)
    out = oracle.trop_route_hidden(latent, weight, np.zeros((2, 2), np.float32), code, code_scale=0.5, training=False)
    np.testing.assert_allclose(out["hidden"].reshape(-1), [7.0, 21.0, 14.0, 13.0], atol=1e-6)


def test_zig_comparison_hash_kat() -> None:
    """kernels/src/lut.zig:320-325: x=(3,1,-1), anchors (0,1),(1,2), offsets (1.5,3) -> index 1."""
    idx, _ = oracle.pairwise_indices(
        np.array([[3.0, 1.0, -1.0]], np.float32), np.array([[[0, 1], [1, 2]]]), np.array([[1.5, 3.0]], np.float32)
    )
    assert int(idx[0, 0]) == 1
