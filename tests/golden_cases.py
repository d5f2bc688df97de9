"""Loading of the golden fixtures and rebuilding of their layers (test helper).

Each fixture (tests/golden/*.npz, written by tests/golden/make_golden.py from the
reference package) stores the sha256 of the reference layer's state_dict. ``build_layer``
rebuilds the layer with this package's own seeded constructors and checks those hashes,
so every fixture also pins the initialisation parity.
"""

from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np
import torch

import tropnn_b200

GOLDEN = Path(__file__).resolve().parent / "golden"


def case_names(kind: str | None = None) -> list[str]:
    manifest = json.loads((GOLDEN / "manifest.json").read_text())
    return sorted(name for name, meta in manifest.items() if kind is None or meta["kind"] == kind)


def load_case(name: str) -> tuple[dict[str, np.ndarray], dict]:
    with np.load(GOLDEN / f"{name}.npz") as data:
        arrays = {k: data[k] for k in data.files}
    meta = json.loads(str(arrays.pop("meta")))
    return arrays, meta


def sha256(t: torch.Tensor) -> str:
    return hashlib.sha256(t.detach().cpu().contiguous().numpy().tobytes()).hexdigest()


def build_layer(arrays: dict[str, np.ndarray], meta: dict) -> torch.nn.Module:
    """Rebuilds the fixture's layer on CPU and checks its state against the reference's hashes."""
    kw = dict(meta["kwargs"])
    if meta["kind"] == "trop":
        layer = tropnn_b200.TropLinear(
            meta["in_features"],
            meta["out_features"],
            heads=meta["heads"],
            cells=meta["cells"],
            code_dim=meta["code_dim"],
            seed=meta["seed"],
            **kw,
        )
        if meta.get("router_bias") is not None:
            with torch.no_grad():
                layer.router_bias.copy_(torch.tensor(meta["router_bias"]).expand_as(layer.router_bias))
    elif meta["kind"] == "fan":
        layer = tropnn_b200.TropFanLinear(
            meta["in_features"],
            meta["out_features"],
            heads=meta["heads"],
            cells=meta["cells"],
            code_dim=meta["code_dim"],
            seed=meta["seed"],
            **kw,
        )
        if meta.get("lifting") is not None:
            with torch.no_grad():
                layer.lifting.copy_(torch.tensor(meta["lifting"]).expand_as(layer.lifting))
    else:
        layer = tropnn_b200.PairwiseLinear(
            meta["in_features"],
            meta["out_features"],
            tables=meta["tables"],
            comparisons=meta["comparisons"],
            seed=meta["seed"],
            **kw,
        )
    if meta["half"]:
        layer = layer.half()
    for key, value in layer.state_dict().items():
        expected = str(arrays[f"sha256.{key}"])
        if sha256(value) != expected:
            raise AssertionError(f"seeded init differs from the reference for {key}")
    return layer


def state_arrays(layer: torch.nn.Module) -> dict[str, np.ndarray]:
    """state_dict as numpy; bfloat16 tensors become float32 arrays of the same values."""
    return {
        k: (v.detach().cpu().float() if v.dtype == torch.bfloat16 else v.detach().cpu()).numpy()
        for k, v in layer.state_dict().items()
    }


def rel_err(actual, expected) -> float:
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    assert a.shape == e.shape, (a.shape, e.shape)
    if e.size == 0:
        return 0.0
    scale = max(float(np.abs(e).max()), 1e-30)
    return float(np.abs(a - e).max()) / scale


def route_gate(scores: np.ndarray, rel: float = 1e-4) -> tuple[np.ndarray, np.ndarray]:
    """Masks of (row, head) routes whose winner / runner are pinned by the margin rule:
    winner where s1 - s2 > rel * max(|s1|, |s2|), runner additionally where s2 - s3 > ..."""
    top = -np.sort(-scores, axis=-1)
    s1, s2 = top[..., 0], top[..., 1]
    win = (s1 - s2) > rel * np.maximum(np.maximum(np.abs(s1), np.abs(s2)), 1e-30)
    if scores.shape[-1] == 2:
        return win, win  # with two cells the winner fixes the runner-up
    s3 = top[..., 2]
    run = win & ((s2 - s3) > rel * np.maximum(np.maximum(np.abs(s2), np.abs(s3)), 1e-30))
    return win, run


def tolerance(meta: dict) -> float:
    """Value tolerance of the parity rule: 1e-5 relative in fp32, 2e-2 with f16 params."""
    return 2e-2 if meta["half"] else 1e-5
