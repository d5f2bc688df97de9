"""``tropnn_b200.register`` on the reference package's own classes (host side, no GPU): a
reference ``TropLinear`` / ``TropFanLinear`` / ``PairwiseLinear`` built with ``backend="b200"`` has the reference's
parameters (bit-identical to this package's layers for the same seed), rejects CPU input
instead of falling back, and every other backend keeps its reference behaviour."""

from __future__ import annotations

import pytest
import torch

import tropnn_b200
from tests.reference_pkg import import_reference


def _same_state(a: torch.nn.Module, b: torch.nn.Module) -> None:
    sa, sb = a.state_dict(), b.state_dict()
    assert list(sa) == list(sb)
    for k in sa:
        assert sa[k].dtype == sb[k].dtype and torch.equal(sa[k], sb[k]), k


def test_registered_trop_matches_own_layer() -> None:
    tropnn = import_reference()
    ref = tropnn.TropLinear(48, 40, heads=8, cells=4, code_dim=16, seed=3, backend="b200")
    own = tropnn_b200.TropLinear(48, 40, heads=8, cells=4, code_dim=16, seed=3)
    assert isinstance(ref, tropnn.TropLinear) and ref.backend == "b200"
    _same_state(ref, own)
    with pytest.raises(ValueError, match="CUDA"):
        ref(torch.randn(2, 48))


@pytest.mark.parametrize("mode", ["site", "basis"])
def test_registered_fan_matches_own_layer(mode: str) -> None:
    tropnn = import_reference()
    ref = tropnn.TropFanLinear(48, 40, heads=8, cells=4, code_dim=16, seed=4, backend="b200", fan_value_mode=mode,
                               fan_basis_rank=5)
    own = tropnn_b200.TropFanLinear(48, 40, heads=8, cells=4, code_dim=16, seed=4, fan_value_mode=mode, fan_basis_rank=5)
    assert ref.backend == "b200"
    _same_state(ref, own)
    torch.testing.assert_close(ref.generated_values(), own.generated_values(), rtol=0, atol=0)
    with pytest.raises(ValueError, match="CUDA"):
        ref(torch.randn(2, 48))


def test_registered_pairwise_matches_own_layer() -> None:
    tropnn = import_reference()
    ref = tropnn.PairwiseLinear(40, 24, tables=6, comparisons=5, seed=2, backend="b200")
    own = tropnn_b200.PairwiseLinear(40, 24, tables=6, comparisons=5, seed=2)
    assert ref.backend == "b200"
    _same_state(ref, own)
    with pytest.raises(ValueError, match="CUDA"):
        ref(torch.randn(2, 40))


def test_register_is_idempotent_and_keeps_other_backends() -> None:
    tropnn = import_reference()
    tropnn_b200.register(tropnn)  # second call: no double wrapping
    layer = tropnn.TropLinear(12, 6, heads=3, cells=4, code_dim=5, seed=1)
    assert layer.backend == "torch"
    y = layer(torch.randn(4, 12))  # the reference's own CPU path still runs
    assert y.shape == (4, 1, 6)
    pair = tropnn.PairwiseLinear(12, 6, tables=3, comparisons=3, seed=1, backend="torch")
    assert pair(torch.randn(4, 12)).shape == (4, 1, 6)


def test_op_wrappers_take_the_reference_keywords() -> None:
    """target= and score_route_max_bytes= of the reference's op wrappers are accepted; a
    non-CUDA target is refused before anything runs."""
    trop = tropnn_b200.TropLinear(6, 4, heads=3, cells=4, code_dim=5)
    pair = tropnn_b200.PairwiseLinear(6, 4, tables=3, comparisons=3)
    with pytest.raises(ValueError, match="target"):
        tropnn_b200.trop_route_hidden_b200(
            torch.randn(1, 2, 5), trop.router_weight, trop.router_bias, trop.code, code_scale=1.0, target="llvm"
        )
    with pytest.raises(ValueError, match="score_route_max_bytes"):
        tropnn_b200.trop_route_hidden_b200(
            torch.randn(1, 2, 5), trop.router_weight, trop.router_bias, trop.code, code_scale=1.0,
            score_route_max_bytes=-1,
        )
    with pytest.raises(ValueError, match="target"):
        tropnn_b200.pairwise_b200(
            torch.randn(1, 2, 6), pair.anchors, pair.thresholds, pair.lut, use_min_margin_ste=True, target="metal"
        )
    # A CUDA target and a valid cap pass the keyword checks and reach the device check.
    with pytest.raises(ValueError, match="CUDA"):
        tropnn_b200.trop_route_hidden_b200(
            torch.randn(1, 2, 5), trop.router_weight, trop.router_bias, trop.code, code_scale=1.0,
            target="cuda", score_route_max_bytes=1 << 20,
        )
    with pytest.raises(ValueError, match="CUDA"):
        tropnn_b200.pairwise_b200(
            torch.randn(1, 2, 6), pair.anchors, pair.thresholds, pair.lut, use_min_margin_ste=True, target="cuda"
        )
