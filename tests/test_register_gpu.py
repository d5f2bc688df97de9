"""The reference package's own TropLinear / TropFanLinear / PairwiseLinear, switched to backend="b200" by
``tropnn_b200.register``, on the GPU against every golden case the reference recorded: same
outputs, route debug cache and gradients as the reference's torch path within the parity
tolerances, and bit-identical to this package's own layers (one code path)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from tests.golden_cases import build_layer, case_names, load_case, rel_err, sha256, tolerance
from tests.gpu_runner import run_b200
from tests.reference_pkg import import_reference

pytestmark = pytest.mark.gpu
FP32_TOL = 1e-5


def _reference_layer(tropnn, meta: dict) -> torch.nn.Module:
    kw = dict(meta["kwargs"])
    if meta["kind"] == "trop":
        layer = tropnn.TropLinear(meta["in_features"], meta["out_features"], heads=meta["heads"], cells=meta["cells"],
                                  code_dim=meta["code_dim"], seed=meta["seed"], backend="b200", **kw)
        if meta.get("router_bias") is not None:
            with torch.no_grad():
                layer.router_bias.copy_(torch.tensor(meta["router_bias"]).expand_as(layer.router_bias))
    elif meta["kind"] == "fan":
        layer = tropnn.TropFanLinear(meta["in_features"], meta["out_features"], heads=meta["heads"], cells=meta["cells"],
                                     code_dim=meta["code_dim"], seed=meta["seed"], backend="b200", **kw)
        if meta.get("lifting") is not None:
            with torch.no_grad():
                layer.lifting.copy_(torch.tensor(meta["lifting"]).expand_as(layer.lifting))
    else:
        layer = tropnn.PairwiseLinear(meta["in_features"], meta["out_features"], tables=meta["tables"],
                                      comparisons=meta["comparisons"], seed=meta["seed"], backend="b200", **kw)
    return layer.half() if meta["half"] else layer


@pytest.mark.parametrize("name", case_names())
def test_registered_reference_layer_matches_golden(name: str) -> None:
    tropnn = import_reference()
    arrays, meta = load_case(name)
    ref_layer = _reference_layer(tropnn, meta)
    for key, value in ref_layer.state_dict().items():
        assert sha256(value) == str(arrays[f"sha256.{key}"]), key
    got = run_b200(ref_layer, arrays, meta)
    own = run_b200(build_layer(arrays, meta), arrays, meta)
    exact_eval = meta["kwargs"].get("exact_fused") == "eval" and not meta["train"]
    tol = FP32_TOL if exact_eval else tolerance(meta)
    assert rel_err(got["y"], arrays["y"]) <= tol
    # One implementation behind both front doors: identical results.
    assert set(got) == set(own)
    for key in got:
        assert np.array_equal(got[key], own[key], equal_nan=True), key
    if meta["train"]:
        assert rel_err(got["grad.x"], arrays["grad.x"]) <= tol
