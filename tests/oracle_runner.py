"""Runs the numpy oracle on a golden case, returning results keyed like the fixture (test helper)."""

from __future__ import annotations

import numpy as np

import oracle


def _flat_x(x: np.ndarray) -> tuple[np.ndarray, tuple[int, int]]:
    if x.ndim == 2:
        return x, (x.shape[0], 1)
    return x.reshape(-1, x.shape[-1]), (x.shape[0], x.shape[1])


def run_oracle(arrays: dict[str, np.ndarray], meta: dict, state: dict[str, np.ndarray]) -> dict[str, np.ndarray]:
    x, (b, s) = _flat_x(arrays["x"].astype(np.float32))
    train = meta["train"]
    out: dict[str, np.ndarray] = {}
    if meta["kind"] == "trop":
        if meta["kwargs"].get("exact_fused") == "eval" and not train:
            fwd = oracle.trop_linear_exact_eval(x, state, code_scale=meta["code_scale"])
        else:
            fwd = oracle.trop_linear_forward(x, state, code_scale=meta["code_scale"], training=train)
        out["y"] = fwd["y"].reshape(b, s, -1)
        out["last_indices"] = fwd["winner"].reshape(b, s, -1)
        out["last_margins"] = fwd["margins"].reshape(b, s, -1)
        out["_scores"] = fwd["scores"]
        if train:
            gy = arrays["grad_out"].reshape(b * s, -1).astype(np.float32)
            grads = oracle.trop_linear_backward(gy, x, state, fwd, code_scale=meta["code_scale"], training=True)
            out["grad.x"] = grads["x"].reshape(arrays["x"].shape)
            for key in ("proj.weight", "router_weight", "router_bias", "code", "output_proj.weight", "output_proj.bias"):
                out[f"grad.{key}"] = grads[key]
        return out
    if meta["kind"] == "fan":
        mode = meta["fan_value_mode"]
        fwd = oracle.trop_fan_forward(x, state, code_scale=meta["code_scale"], training=train, fan_value_mode=mode)
        out["y"] = fwd["y"].reshape(b, s, -1)
        out["last_indices"] = fwd["winner"].reshape(b, s, -1)
        out["last_margins"] = fwd["margins"].reshape(b, s, -1)
        out["_scores"] = fwd["scores"]
        if train:
            gy = arrays["grad_out"].reshape(b * s, -1).astype(np.float32)
            grads = oracle.trop_fan_backward(gy, x, state, fwd, code_scale=meta["code_scale"], training=True, fan_value_mode=mode)
            out["grad.x"] = grads["x"].reshape(arrays["x"].shape)
            for key in grads:
                if key != "x":
                    out[f"grad.{key}"] = grads[key]
        return out
    kw = meta["kwargs"]
    fwd = oracle.pairwise_forward(x, state["anchors"], state["thresholds"], state["lut"], output_scale=meta["output_scale"])
    out["y"] = fwd["out"].reshape(b, s, -1)
    out["last_indices"] = fwd["indices"].reshape(b, s, -1)
    out["last_margins"] = fwd["margins"].reshape(b, s, *fwd["margins"].shape[1:])
    if train:
        gy = arrays["grad_out"].reshape(b * s, -1).astype(np.float32)
        grads = oracle.pairwise_backward(
            gy,
            fwd["indices"],
            fwd["margins"],
            state["anchors"],
            state["lut"],
            in_features=meta["in_features"],
            output_scale=meta["output_scale"],
            use_min_margin_ste=kw.get("use_min_margin_ste", True),
            surrogate=kw.get("surrogate", "fast_sigmoid_odd"),
        )
        out["grad.x"] = grads["x"].reshape(arrays["x"].shape)
        out["grad.lut"] = grads["lut"]
        out["grad.thresholds"] = grads["thresholds"]
    return out
