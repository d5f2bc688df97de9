"""CPU oracle of tropnn's routed-layer hot path — TEST INFRASTRUCTURE ONLY.

A plain-numpy restatement of the reference's default torch path (``backend="torch"``,
``exact_fused="off"``) for TropLinear and PairwiseLinear, forward and backward. Only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its ``cpu_baseline`` leg and
``--impl reference`` arm) may import it, and only as the checker / the timed CPU
baseline: the product path (``tropnn_b200``) never calls it.

Parity pin: every function below is checked against golden vectors produced by the
reference itself (``tests/golden/make_golden.py`` imports the reference package and
records its outputs and autograd gradients) and against the reference's own
known-answer tests (tests/test_routing.py, tests/test_tropical_core.py,
tests/test_pairwise.py, kernels/src/tropical.zig:352-379, kernels/src/lut.zig:320-325).
See ``tests/test_oracle_golden.py``.

Arithmetic is float32 with the reference's operation order where it matters
(``(x_a - x_b) - theta``; ``w + U (r - w)``; ``latent + sum * code_scale``); matrix
products use numpy's float32 BLAS, so sums differ from torch's by reassociation only.
Ties in the top-2 keep the lowest cell index (the reference's torch.topk on CPU does not
pin tie order, so tied routes are outside the parity contract).
"""

from __future__ import annotations

import numpy as np

F32 = np.float32

__all__ = [
    "fan_generated_values",
    "fast_sigmoid_odd_surrogate",
    "izhikevich_surrogate",
    "minface_mix",
    "packed_route_index_dtype",
    "pairwise_backward",
    "pairwise_forward",
    "pairwise_indices",
    "surrogate_gradient",
    "top2_indices",
    "trop_fan_backward",
    "trop_fan_forward",
    "trop_linear_backward",
    "trop_linear_exact_eval",
    "trop_linear_forward",
    "trop_route_backward",
    "trop_route_hidden",
    "trop_scores",
]


# ---------------------------------------------------------------------------
# routing helpers (layers/routing.py, layers/surrogate.py)
# ---------------------------------------------------------------------------


def packed_route_index_dtype(cells: int) -> np.dtype:
    """layers/routing.py:18-23."""
    if cells <= 256:
        return np.dtype(np.uint8)
    if cells <= 32767:
        return np.dtype(np.int16)
    return np.dtype(np.int64)


def top2_indices(scores: np.ndarray) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """layers/routing.py:7-10: winner, runner-up and margin over the last axis."""
    order = np.argsort(-scores, axis=-1, kind="stable")
    winner = order[..., 0]
    runner = order[..., 1]
    s1 = np.take_along_axis(scores, winner[..., None], axis=-1)[..., 0]
    s2 = np.take_along_axis(scores, runner[..., None], axis=-1)[..., 0]
    return winner.astype(np.int64), runner.astype(np.int64), (s1 - s2).astype(F32)


def minface_mix(winner_values: np.ndarray, runner_values: np.ndarray, margins: np.ndarray) -> np.ndarray:
    """layers/routing.py:13-15: w + (0.5 / (1 + |m|)) (r - w)."""
    alpha = (F32(0.5) / (F32(1.0) + np.abs(margins))).astype(F32)
    return (winner_values + alpha[..., None] * (runner_values - winner_values)).astype(F32)


def fast_sigmoid_odd_surrogate(u: np.ndarray) -> np.ndarray:
    """layers/surrogate.py:16-17: -0.5 sign(u) / (1 + |u|)^2."""
    return (F32(-0.5) * np.sign(u).astype(F32) / np.square(F32(1.0) + np.abs(u))).astype(F32)


def izhikevich_surrogate(u: np.ndarray) -> np.ndarray:
    """layers/surrogate.py:9-13."""
    sig = (F32(1.0) / (F32(1.0) + np.exp(-np.abs(u).astype(F32)))).astype(F32)
    sign = np.where(u > 0, F32(-1.0), F32(1.0)).astype(F32)
    return (sign * F32(2.0) * sig * (F32(1.0) - sig)).astype(F32)


def surrogate_gradient(u: np.ndarray, surrogate: str = "fast_sigmoid_odd") -> np.ndarray:
    """layers/surrogate.py:20-25."""
    if surrogate == "fast_sigmoid_odd":
        return fast_sigmoid_odd_surrogate(u)
    if surrogate == "izhikevich":
        return izhikevich_surrogate(u)
    raise ValueError(f"unsupported surrogate {surrogate!r}")


# ---------------------------------------------------------------------------
# TropLinear
# ---------------------------------------------------------------------------


def _f32(a: np.ndarray) -> np.ndarray:
    return np.asarray(a, dtype=F32)


def trop_scores(z: np.ndarray, router_weight: np.ndarray, router_bias: np.ndarray) -> np.ndarray:
    """backend.py:45-46: s[n,h,k] = <z[n], W[h,k]> + b[h,k] for z [N, D]."""
    heads, cells, code_dim = router_weight.shape
    flat = _f32(router_weight).reshape(heads * cells, code_dim)
    scores = (_f32(z) @ flat.T).reshape(z.shape[0], heads, cells)
    return (scores + _f32(router_bias)[None]).astype(F32)


def trop_route_hidden(
    z: np.ndarray,
    router_weight: np.ndarray,
    router_bias: np.ndarray,
    code: np.ndarray,
    *,
    code_scale: float,
    training: bool,
) -> dict[str, np.ndarray]:
    """layers/tropical.py:207-221 (+ :131-138): scores, top-2 and the selected-code sum.

    ``z`` is [N, D] float32; parameters are upcast to float32 as the reference does
    (``.to(compute_dtype)``). Returns hidden [N, D], winner/runner [N, H] int64,
    margins [N, H].
    """
    z = _f32(z)
    code32 = _f32(code)
    heads = code32.shape[0]
    scores = trop_scores(z, router_weight, router_bias)
    winner, runner, margins = top2_indices(scores)
    head_ix = np.arange(heads)[None, :]
    winner_values = code32[head_ix, winner]  # [N, H, D]
    if training:
        runner_values = code32[head_ix, runner]
        values = minface_mix(winner_values, runner_values, margins)
    else:
        values = winner_values
    hidden = (z + values.sum(axis=1, dtype=F32) * F32(code_scale)).astype(F32)
    return {"hidden": hidden, "winner": winner, "runner": runner, "margins": margins, "scores": scores}


def trop_route_backward(
    grad_hidden: np.ndarray,
    z: np.ndarray,
    router_weight: np.ndarray,
    code: np.ndarray,
    winner: np.ndarray,
    runner: np.ndarray,
    margins: np.ndarray,
    *,
    code_scale: float,
    training: bool,
) -> dict[str, np.ndarray | None]:
    """Min-face backward in coefficient form, layers/tropical_exact.py:204-237.

    Equal (up to reassociation) to autograd through the torch path of
    layers/tropical.py:207-221. Router gradients are None in eval mode, where the
    output does not depend on the margins.
    """
    g = _f32(grad_hidden)
    z = _f32(z)
    W = _f32(router_weight)
    c = _f32(code)
    n, heads = winner.shape
    cells = W.shape[1]
    rows = np.arange(n)[:, None]
    head_ix = np.arange(heads)[None, :]
    coeff = np.zeros((n, heads, cells), dtype=F32)
    if training:
        alpha = (F32(0.5) / (F32(1.0) + np.abs(margins))).astype(F32)
        np.add.at(coeff, (rows, head_ix, winner), F32(1.0) - alpha)
        np.add.at(coeff, (rows, head_ix, runner), alpha)
    else:
        np.add.at(coeff, (rows, head_ix, winner), F32(1.0))
    grad_code = (np.einsum("nhc,nr->hcr", coeff, g, dtype=F32) * F32(code_scale)).astype(F32)
    grad_z = g.copy()
    grad_w = grad_b = None
    if training:
        delta = c[head_ix, runner] - c[head_ix, winner]  # [N, H, D]
        dalpha = (F32(-0.5) * np.sign(margins).astype(F32) / np.square(F32(1.0) + np.abs(margins))).astype(F32)
        grad_margin = ((g[:, None, :] * delta).sum(axis=-1, dtype=F32) * F32(code_scale) * dalpha).astype(F32)
        route = np.zeros((n, heads, cells), dtype=F32)
        np.add.at(route, (rows, head_ix, winner), grad_margin)
        np.add.at(route, (rows, head_ix, runner), -grad_margin)
        grad_w = np.einsum("nhc,nr->hcr", route, z, dtype=F32).astype(F32)
        grad_b = route.sum(axis=0, dtype=F32)
        grad_z = (grad_z + np.einsum("nhc,hcr->nr", route, W, dtype=F32)).astype(F32)
    return {"grad_latent": grad_z, "grad_router_weight": grad_w, "grad_router_bias": grad_b, "grad_code": grad_code}


def _round_bf16(a: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 -> float32, round-to-nearest-even on the upper 16 bits."""
    bits = np.ascontiguousarray(a, dtype=F32).view(np.uint32).astype(np.uint64)
    bits = ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16) << 16
    return bits.astype(np.uint32).view(F32)


def _round_to(a: np.ndarray, param_dtype: str) -> np.ndarray:
    if param_dtype == "bfloat16":
        return _round_bf16(a)
    if param_dtype == "float16":
        return np.asarray(a, dtype=np.float16).astype(F32)
    return _f32(a)


def _param_dtype(params: dict[str, np.ndarray], override: str | None) -> str:
    return override if override is not None else str(np.asarray(params["proj.weight"]).dtype)


def trop_linear_forward(
    x: np.ndarray, params: dict[str, np.ndarray], *, code_scale: float, training: bool, param_dtype: str | None = None
) -> dict[str, np.ndarray]:
    """TropLinear.forward (layers/tropical.py:89-99, :140-146 via base.py:64-84).

    ``x`` [N, in] float32; ``params`` holds the state_dict arrays (float32/float16, or
    float32 arrays of bfloat16 values with ``param_dtype="bfloat16"``). The projection
    casts x to the projection's dtype and rounds z to it (tropical.py:99), then
    everything runs in float32.
    """
    pdt = _param_dtype(params, param_dtype)
    x32 = _round_to(x, pdt)
    z = _round_to(x32 @ _f32(params["proj.weight"]).T, pdt)
    route = trop_route_hidden(
        z, params["router_weight"], params["router_bias"], params["code"], code_scale=code_scale, training=training
    )
    y = (route["hidden"] @ _f32(params["output_proj.weight"]).T + _f32(params["output_proj.bias"])).astype(F32)
    return {"y": y, "z": z, **route}


def trop_linear_exact_eval(x: np.ndarray, params: dict[str, np.ndarray], *, code_scale: float) -> dict[str, np.ndarray]:
    """TropLinear eval with ``exact_fused="eval"`` (layers/tropical_exact.py:257-358, selected at
    layers/tropical.py:92 in eval under no_grad): the reassociated form with effective weights,
    every product in float32 (parameters upcast to the compute dtype, x not rounded to them):
    router_eff = W P [H,K,in], value_eff = c Wout^T [H,K,out], base = Wout P [out,in];
    scores = x router_eff^T + b, top-2; y = x base^T + b_out + code_scale * sum_h value_eff[h, w]."""
    w = _f32(params["router_weight"])
    heads, cells, dim = w.shape
    proj = _f32(params["proj.weight"])
    w_out = _f32(params["output_proj.weight"])
    router_eff = (w.reshape(heads * cells, dim) @ proj).astype(F32)
    value_eff = (_f32(params["code"]).reshape(heads * cells, dim) @ w_out.T).astype(F32).reshape(heads, cells, -1)
    base = (w_out @ proj).astype(F32)
    x32 = _f32(x)
    n = x32.shape[0]
    scores = ((x32 @ router_eff.T).reshape(n, heads, cells) + _f32(params["router_bias"])[None]).astype(F32)
    winner, runner, margins = top2_indices(scores)
    out = (x32 @ base.T + _f32(params["output_proj.bias"])).astype(F32)
    value_sum = value_eff[np.arange(heads)[None, :], winner].sum(axis=1, dtype=F32)
    y = (out + value_sum * F32(code_scale)).astype(F32)
    return {"y": y, "winner": winner, "runner": runner, "margins": margins, "scores": scores}


def trop_linear_backward(
    grad_y: np.ndarray,
    x: np.ndarray,
    params: dict[str, np.ndarray],
    fwd: dict[str, np.ndarray],
    *,
    code_scale: float,
    training: bool,
    param_dtype: str | None = None,
) -> dict[str, np.ndarray | None]:
    """Autograd of trop_linear_forward: output map, route backward, projection."""
    gy = _f32(grad_y)
    w_out = _f32(params["output_proj.weight"])
    grad_hidden = gy @ w_out
    route = trop_route_backward(
        grad_hidden,
        fwd["z"],
        params["router_weight"],
        params["code"],
        fwd["winner"],
        fwd["runner"],
        fwd["margins"],
        code_scale=code_scale,
        training=training,
    )
    gz = route["grad_latent"]
    x32 = _round_to(x, _param_dtype(params, param_dtype))
    return {
        "x": (gz @ _f32(params["proj.weight"])).astype(F32),
        "proj.weight": (gz.T @ x32).astype(F32),
        "router_weight": route["grad_router_weight"],
        "router_bias": route["grad_router_bias"],
        "code": route["grad_code"],
        "output_proj.weight": (gy.T @ fwd["hidden"]).astype(F32),
        "output_proj.bias": gy.sum(axis=0, dtype=F32),
    }


# ---------------------------------------------------------------------------
# TropFanLinear
# ---------------------------------------------------------------------------


def fan_generated_values(params: dict[str, np.ndarray], *, fan_value_mode: str) -> np.ndarray:
    """TropFanLinear.generated_values (layers/fan.py:159-171) in float32: "site" mode is
    F.normalize(sites, dim=-1, eps=1e-12) * value_scale[..., None]; "basis" mode is
    einsum("hkr,rd->hkd", value_coeff, value_basis)."""
    if fan_value_mode == "site":
        sites = _f32(params["sites"])
        norm = np.sqrt(np.square(sites).sum(axis=-1, keepdims=True, dtype=F32)).astype(F32)
        unit = (sites / np.maximum(norm, F32(1e-12))).astype(F32)
        return (unit * _f32(params["value_scale"])[..., None]).astype(F32)
    return np.einsum("hkr,rd->hkd", _f32(params["value_coeff"]), _f32(params["value_basis"]), dtype=F32).astype(F32)


def trop_fan_forward(
    x: np.ndarray,
    params: dict[str, np.ndarray],
    *,
    code_scale: float,
    training: bool,
    fan_value_mode: str,
    param_dtype: str | None = None,
) -> dict[str, np.ndarray]:
    """TropFanLinear.forward (layers/fan.py:96-99, :201-222, :276-330 via base.py:64-84): the
    projection as TropLinear's, scores against the sites with the lifting as bias, the top-2,
    the (min-face mixed in training) generated values of the routed cells summed onto the
    latent, and the output map."""
    pdt = _param_dtype(params, param_dtype)
    x32 = _round_to(x, pdt)
    z = _round_to(x32 @ _f32(params["proj.weight"]).T, pdt)
    values = fan_generated_values(params, fan_value_mode=fan_value_mode)
    route = trop_route_hidden(z, params["sites"], params["lifting"], values, code_scale=code_scale, training=training)
    y = (route["hidden"] @ _f32(params["output_proj.weight"]).T + _f32(params["output_proj.bias"])).astype(F32)
    return {"y": y, "z": z, "values": values, **route}


def trop_fan_backward(
    grad_y: np.ndarray,
    x: np.ndarray,
    params: dict[str, np.ndarray],
    fwd: dict[str, np.ndarray],
    *,
    code_scale: float,
    training: bool,
    fan_value_mode: str,
    param_dtype: str | None = None,
) -> dict[str, np.ndarray | None]:
    """Autograd of trop_fan_forward: TropLinear's backward with the sites as router weights
    and the value table as code, then the value gradient carried into the value parameters
    (site mode: the normalisation's Jacobian (g - u (u.g)) / max(|s|, eps) and value_scale's
    sum(g . u); basis mode: the two einsum factors)."""
    gy = _f32(grad_y)
    w_out = _f32(params["output_proj.weight"])
    grad_hidden = gy @ w_out
    route = trop_route_backward(
        grad_hidden,
        fwd["z"],
        params["sites"],
        fwd["values"],
        fwd["winner"],
        fwd["runner"],
        fwd["margins"],
        code_scale=code_scale,
        training=training,
    )
    gz = route["grad_latent"]
    gv = route["grad_code"]
    x32 = _round_to(x, _param_dtype(params, param_dtype))
    out: dict[str, np.ndarray | None] = {
        "x": (gz @ _f32(params["proj.weight"])).astype(F32),
        "proj.weight": (gz.T @ x32).astype(F32),
        "lifting": route["grad_router_bias"],
        "output_proj.weight": (gy.T @ fwd["hidden"]).astype(F32),
        "output_proj.bias": gy.sum(axis=0, dtype=F32),
    }
    grad_sites = route["grad_router_weight"]
    if fan_value_mode == "site":
        sites = _f32(params["sites"])
        norm = np.sqrt(np.square(sites).sum(axis=-1, keepdims=True, dtype=F32)).astype(F32)
        denom = np.maximum(norm, F32(1e-12))
        unit = (sites / denom).astype(F32)
        scale = _f32(params["value_scale"])[..., None]
        out["value_scale"] = (gv * unit).sum(axis=-1, dtype=F32)
        g_unit = (gv * scale).astype(F32)
        radial = (g_unit * unit).sum(axis=-1, keepdims=True, dtype=F32)
        from_values = np.where(norm > F32(1e-12), (g_unit - unit * radial) / denom, g_unit / denom).astype(F32)
    else:
        coeff = _f32(params["value_coeff"])
        basis = _f32(params["value_basis"])
        out["value_coeff"] = np.einsum("hkd,rd->hkr", gv, basis, dtype=F32).astype(F32)
        out["value_basis"] = np.einsum("hkr,hkd->rd", coeff, gv, dtype=F32).astype(F32)
        from_values = None
    if from_values is not None:
        grad_sites = from_values if grad_sites is None else (grad_sites + from_values).astype(F32)
    out["sites"] = grad_sites
    return out


# ---------------------------------------------------------------------------
# PairwiseLinear
# ---------------------------------------------------------------------------


def pairwise_indices(x: np.ndarray, anchors: np.ndarray, thresholds: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """layers/pairwise.py:127-135: u = (x_a - x_b) - theta, idx = sum_r [u > 0] 2^r."""
    x = _f32(x)
    xa = x[:, anchors[:, :, 0]]  # [N, T, C]
    xb = x[:, anchors[:, :, 1]]
    u = ((xa - xb) - _f32(thresholds)[None]).astype(F32)
    powers = (1 << np.arange(anchors.shape[1], dtype=np.int64))
    idx = ((u > 0).astype(np.int64) * powers).sum(axis=-1)
    return idx, u


def pairwise_forward(
    x: np.ndarray, anchors: np.ndarray, thresholds: np.ndarray, lut: np.ndarray, *, output_scale: float
) -> dict[str, np.ndarray]:
    """layers/pairwise.py:99-135, 243-248 and base.py:76-77 (forward value; the STE term is 0)."""
    idx, u = pairwise_indices(x, anchors, thresholds)
    lut32 = _f32(lut)
    tables = lut32.shape[0]
    selected = lut32[np.arange(tables)[None, :], idx]  # [N, T, out]
    out = selected.sum(axis=1, dtype=F32)
    if output_scale != 1.0:
        out = (out * F32(output_scale)).astype(F32)
    return {"out": out, "indices": idx, "margins": u}


def pairwise_backward(
    grad_out: np.ndarray,
    indices: np.ndarray,
    margins: np.ndarray,
    anchors: np.ndarray,
    lut: np.ndarray,
    *,
    in_features: int,
    output_scale: float,
    use_min_margin_ste: bool,
    surrogate: str = "fast_sigmoid_odd",
    ste: bool = True,
    lut_grad: bool = True,
) -> dict[str, np.ndarray | None]:
    """Autograd of PairwiseLinear's torch path (layers/pairwise.py:137-200, 243-248).

    grad_lut[t, idx] += g (the STE term's forward factor is 0, so it adds nothing);
    with ``ste``: min mode r* = argmin |u| (first on ties), nb = idx ^ 2^r*,
    gu = <g, lut[t,nb] - lut[t,idx]> S(u_r*), grad_x[a] += gu, grad_x[b] -= gu,
    grad_theta[t,r*] -= gu; full mode does every r. ``lut_grad=False`` skips the LUT
    gradient (``"lut"`` is None), so that large layers can be checked row chunk by row chunk.
    """
    g = (_f32(grad_out) * F32(output_scale)).astype(F32) if output_scale != 1.0 else _f32(grad_out)
    lut32 = _f32(lut)
    tables, table_size, out_features = lut32.shape
    n = g.shape[0]
    grad_lut = np.zeros_like(lut32) if lut_grad else None
    for t in range(tables if lut_grad else 0):
        # index_select backward: the rows of g summed per selected LUT row (a stable
        # sort groups each bucket's rows in ascending row order, then one reduceat).
        idx_t = indices[:, t]
        order = np.argsort(idx_t, kind="stable")
        sorted_idx = idx_t[order]
        if sorted_idx.size == 0:
            continue
        starts = np.flatnonzero(np.r_[True, sorted_idx[1:] != sorted_idx[:-1]])
        grad_lut[t, sorted_idx[starts]] = np.add.reduceat(g[order], starts, axis=0)
    result: dict[str, np.ndarray | None] = {"lut": grad_lut, "x": None, "thresholds": None}
    if not ste:
        return result
    comparisons = anchors.shape[1]
    table_ix = np.arange(tables)[None, :]
    current = lut32[table_ix, indices]  # [N, T, out]
    grad_margins = np.zeros((n, tables, comparisons), dtype=F32)
    if use_min_margin_ste:
        rmin = np.argmin(np.abs(margins), axis=-1)  # first index on ties, like torch.argmin
        umin = np.take_along_axis(margins, rmin[..., None], axis=-1)[..., 0]
        neighbor = lut32[table_ix, indices ^ (1 << rmin)]
        dot = (g[:, None, :] * (neighbor - current)).sum(axis=-1, dtype=F32)
        gu = (dot * surrogate_gradient(umin, surrogate)).astype(F32)
        np.put_along_axis(grad_margins, rmin[..., None], gu[..., None], axis=-1)
    else:
        for r in range(comparisons):
            neighbor = lut32[table_ix, indices ^ (1 << r)]
            dot = (g[:, None, :] * (neighbor - current)).sum(axis=-1, dtype=F32)
            grad_margins[:, :, r] = dot * surrogate_gradient(margins[:, :, r], surrogate)
    grad_x = np.zeros((n, in_features), dtype=F32)
    flat_a = anchors[:, :, 0].reshape(-1)
    flat_b = anchors[:, :, 1].reshape(-1)
    gm_flat = grad_margins.reshape(n, -1)
    for col in range(gm_flat.shape[1]):
        grad_x[:, flat_a[col]] += gm_flat[:, col]
        grad_x[:, flat_b[col]] -= gm_flat[:, col]
    result["x"] = grad_x
    result["thresholds"] = (-grad_margins.sum(axis=0, dtype=F32)).astype(F32)
    return result
