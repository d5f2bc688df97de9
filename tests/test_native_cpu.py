"""The C++ restatement of the reference's Zig CPU inference kernels (oracle/native_cpu.cpp):
pinned by the Zig files' own known-answer tests, then checked against the reference's golden
eval outputs and the numpy oracle. CPU only."""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from oracle import native
from tests.golden_cases import build_layer, case_names, load_case, rel_err, state_arrays


@pytest.fixture(scope="module", autouse=True)
def _library() -> None:
    native.build()


@pytest.mark.parametrize("threads", [1, 4])
def test_zig_route_known_answer(threads: int) -> None:
    """kernels/src/tropical.zig:352-379 ("f32 tropical route selects best cells")."""
    latent = np.array([[2.0, 1.0], [-1.0, 3.0]], np.float32)
    weight = np.array([[[1.0, 0.0], [0.0, 1.0]], [[-1.0, 0.0], [0.0, -1.0]]], np.float32)
    bias = np.zeros((2, 2), np.float32)
    code = np.array([[[10.0, 0.0], [0.0, 20.0]], [[30.0, 0.0], [0.0, 40.0]]], np.float32)
    hidden = native.trop_route_hidden(latent, weight, bias, code, code_scale=0.5, threads=threads)
    assert np.allclose(hidden, [[7.0, 21.0], [14.0, 13.0]], atol=1e-6, rtol=0)
    hidden16 = native.trop_route_hidden(latent, weight.astype(np.float16), bias.astype(np.float16),
                                        code.astype(np.float16), code_scale=0.5, threads=threads)
    assert np.array_equal(hidden16, hidden)


def test_zig_comparison_hash_known_answer() -> None:
    """kernels/src/lut.zig:320-325 ("comparison hash uses thresholds"): index 1, read back through
    a one-column LUT whose rows hold their own index."""
    x = np.array([[3.0, 1.0, -1.0]], np.float32)
    anchors = np.array([[[0, 1], [1, 2]]], np.int64)
    offsets = np.array([[1.5, 3.0]], np.float32)
    lut = np.arange(4, dtype=np.float32).reshape(1, 4, 1)
    assert native.lut_forward(x, anchors, offsets, lut)[0, 0] == 1.0


def _eval_cases(kind: str) -> list[str]:
    """Eval fixtures of the default path (exact_fused="eval" cases take the reassociated torch path
    in the reference whatever the backend, layers/tropical.py:92)."""
    return [n for n in case_names(kind)
            if not load_case(n)[1]["train"] and load_case(n)[1]["kwargs"].get("exact_fused") != "eval"]


@pytest.mark.parametrize("name", _eval_cases("trop"))
def test_trop_eval_matches_reference_golden(name: str) -> None:
    arrays, meta = load_case(name)
    layer = build_layer(arrays, meta)
    params = state_arrays(layer)
    x = arrays["x"].reshape(-1, arrays["x"].shape[-1])
    y = native.trop_linear_eval(x, params, code_scale=meta["code_scale"], threads=4)
    expect = arrays["y"].reshape(y.shape)
    tol = 2e-2 if meta["half"] else 1e-5
    assert rel_err(y, expect) <= tol
    fwd = oracle.trop_linear_forward(x, params, code_scale=meta["code_scale"], training=False)
    assert rel_err(y, fwd["y"]) <= tol
    hidden = native.trop_route_hidden(fwd["z"], params["router_weight"], params["router_bias"], params["code"],
                                      code_scale=meta["code_scale"])
    assert rel_err(hidden, fwd["hidden"]) <= 1e-5


@pytest.mark.parametrize("name", _eval_cases("pairwise"))
def test_pairwise_eval_matches_reference_golden(name: str) -> None:
    arrays, meta = load_case(name)
    layer = build_layer(arrays, meta)
    params = state_arrays(layer)
    x = arrays["x"].reshape(-1, arrays["x"].shape[-1])
    y = native.pairwise_eval(x, params, output_scale=meta["output_scale"], threads=4)
    expect = arrays["y"].reshape(y.shape)
    assert rel_err(y, expect) <= (2e-2 if meta["half"] else 1e-5)
    fwd = oracle.pairwise_forward(x, params["anchors"], params["thresholds"], params["lut"],
                                  output_scale=meta["output_scale"])
    assert rel_err(y, fwd["out"]) <= 1e-5


@pytest.mark.parametrize(("cells", "dim", "f16"), [(4, 32, False), (16, 64, True), (3, 40, False), (7, 19, True)])
def test_trop_hidden_against_oracle_and_threads(cells: int, dim: int, f16: bool) -> None:
    """Random shapes, both score orders (2-4 cells and the generic path) and ragged widths: the
    native hidden against the numpy oracle, and bit-identical for 1 and 8 threads."""
    rng = np.random.default_rng(cells * 100 + dim)
    heads, n = 24, 700
    dt = np.float16 if f16 else np.float32
    w = rng.standard_normal((heads, cells, dim)).astype(dt)
    b = (0.1 * rng.standard_normal((heads, cells))).astype(dt)
    c = rng.standard_normal((heads, cells, dim)).astype(dt)
    z = rng.standard_normal((n, dim)).astype(np.float32)
    one = native.trop_route_hidden(z, w, b, c, code_scale=0.25, threads=1)
    many = native.trop_route_hidden(z, w, b, c, code_scale=0.25, threads=8)
    assert np.array_equal(one, many)
    ref = oracle.trop_route_hidden(z, w.astype(np.float32), b.astype(np.float32), c.astype(np.float32),
                                   code_scale=0.25, training=False)
    # Rows whose top-2 scores are within rounding of each other may pick either cell; compare
    # the rows whose margins are clear.
    clear = (ref["margins"] > 1e-4).all(axis=1)
    assert clear.mean() > 0.9
    assert rel_err(one[clear], ref["hidden"][clear]) <= 1e-5


@pytest.mark.parametrize(("tables", "comparisons", "f16"), [(16, 6, False), (32, 8, True), (5, 3, False)])
def test_lut_forward_against_oracle_and_threads(tables: int, comparisons: int, f16: bool) -> None:
    rng = np.random.default_rng(tables + comparisons)
    n, inn, out = 500, 64, 96
    x = rng.standard_normal((n, inn)).astype(np.float32)
    anchors = rng.integers(0, inn, (tables, comparisons, 2)).astype(np.int64)
    thr = (0.1 * rng.standard_normal((tables, comparisons))).astype(np.float32)
    lut = rng.standard_normal((tables, 1 << comparisons, out)).astype(np.float16 if f16 else np.float32)
    one = native.lut_forward(x, anchors, thr, lut, threads=1)
    many = native.lut_forward(x, anchors, thr, lut, threads=8)
    assert np.array_equal(one, many)
    ref = oracle.pairwise_forward(x, anchors, thr, lut.astype(np.float32), output_scale=1.0)["out"]
    assert rel_err(one, ref) <= 1e-5


def test_bad_arguments_raise() -> None:
    x = np.zeros((2, 4), np.float32)
    lut = np.zeros((1, 2, 3), np.float32)
    with pytest.raises(ValueError):
        native.lut_forward(x, np.array([[[0, 4]]], np.int64), np.zeros((1, 1), np.float32), lut)
    with pytest.raises(ValueError):
        native.trop_route_hidden(x, np.zeros((2, 2, 3), np.float32), np.zeros((2, 2), np.float32),
                                 np.zeros((2, 2, 3), np.float32), code_scale=1.0)
