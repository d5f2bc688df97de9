"""Host-side behaviour of the drop-in layers that needs no GPU: constructor validation,
state_dict layout, seeded init, and loud failure instead of a CPU fallback."""

from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np
import pytest
import torch

import tropnn_b200
from tropnn_b200 import PairwiseLinear, TropLinear

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_trop_state_dict_layout_matches_reference() -> None:
    layer = TropLinear(256, 512, heads=32, cells=4, code_dim=32, seed=0)
    shapes = {k: (tuple(v.shape), v.dtype) for k, v in layer.state_dict().items()}
    assert list(shapes) == ["router_weight", "router_bias", "code", "proj.weight", "output_proj.weight", "output_proj.bias"]
    assert shapes["router_weight"] == ((32, 4, 32), torch.float32)
    assert shapes["router_bias"] == ((32, 4), torch.float32)
    assert shapes["proj.weight"] == ((32, 256), torch.float32)
    assert shapes["output_proj.weight"] == ((512, 32), torch.float32)
    assert layer.code_scale == pytest.approx(1 / 32**0.5)


def test_pairwise_state_dict_layout_matches_reference() -> None:
    layer = PairwiseLinear(256, 512, tables=16, comparisons=6, seed=0)
    shapes = {k: (tuple(v.shape), v.dtype) for k, v in layer.state_dict().items()}
    assert list(shapes) == ["thresholds", "lut", "anchors", "powers"]
    assert shapes["lut"] == ((16, 64, 512), torch.float32)
    assert shapes["anchors"] == ((16, 6, 2), torch.int64)
    assert shapes["powers"] == ((6,), torch.int64)
    assert bool((layer.anchors[..., 0] != layer.anchors[..., 1]).all())
    assert layer.output_scale == pytest.approx(0.25)


def test_config5_trop_init_matches_reference_hashes() -> None:
    expected = json.loads((GOLDEN / "cfg5_trop_init_sha256.json").read_text())
    layer = TropLinear(4096, 4096, heads=1024, cells=16, code_dim=256, seed=0).half()
    got = {k: hashlib.sha256(v.contiguous().numpy().tobytes()).hexdigest() for k, v in layer.state_dict().items()}
    assert got == expected


def test_reference_state_dict_loads() -> None:
    a = TropLinear(6, 4, heads=3, cells=4, code_dim=5, seed=1)
    b = TropLinear(6, 4, heads=3, cells=4, code_dim=5, seed=2)
    b.load_state_dict(a.state_dict())
    for k, v in a.state_dict().items():
        assert torch.equal(v, b.state_dict()[k])


@pytest.mark.parametrize("backend", ["torch", "tilelang", "triton", "auto", "zig"])
def test_other_backends_are_rejected(backend: str) -> None:
    with pytest.raises(ValueError, match="b200"):
        TropLinear(6, 4, heads=3, cells=4, code_dim=5, backend=backend)
    with pytest.raises(ValueError, match="b200"):
        PairwiseLinear(6, 4, tables=3, comparisons=3, backend=backend)


def test_constructor_validation_mirrors_reference() -> None:
    with pytest.raises(ValueError, match="heads"):
        TropLinear(6, 4, heads=0)
    with pytest.raises(ValueError, match="cells"):
        TropLinear(6, 4, cells=1)
    with pytest.raises(ValueError, match="exact_fused"):
        TropLinear(6, 4, exact_fused="bogus")
    with pytest.raises(ValueError, match="in_features"):
        PairwiseLinear(0, 4)
    with pytest.raises(ValueError, match="surrogate"):
        PairwiseLinear(6, 4, surrogate="nope")
    with pytest.raises(ValueError, match="comparisons"):
        PairwiseLinear(6, 4, comparisons=13)


def test_cpu_input_raises_instead_of_falling_back() -> None:
    trop = TropLinear(6, 4, heads=3, cells=4, code_dim=5)
    pair = PairwiseLinear(6, 4, tables=3, comparisons=3)
    with pytest.raises(ValueError, match="CUDA"):
        trop(torch.randn(2, 6))
    with pytest.raises(ValueError, match="CUDA"):
        pair(torch.randn(2, 6))
    with pytest.raises(ValueError, match="CUDA"):
        tropnn_b200.pairwise_b200(
            torch.randn(1, 2, 6), pair.anchors, pair.thresholds, pair.lut, use_min_margin_ste=True
        )
    with pytest.raises(ValueError, match="CUDA"):
        tropnn_b200.trop_route_hidden_b200(
            torch.randn(1, 2, 5), trop.router_weight, trop.router_bias, trop.code, code_scale=1.0
        )


def test_packed_route_index_dtype_mirrors_reference() -> None:
    assert tropnn_b200.packed_route_index_dtype(8) == torch.uint8
    assert tropnn_b200.packed_route_index_dtype(256) == torch.uint8
    assert tropnn_b200.packed_route_index_dtype(1000) == torch.int16
    assert tropnn_b200.packed_route_index_dtype(40000) == torch.int64


def test_missing_library_fails_loudly(tmp_path: Path) -> None:
    from tropnn_b200 import _native as nat

    with pytest.raises(nat.B200Unavailable, match="not found"):
        nat.load(tmp_path / "missing.so")


def test_exact_eval_effective_weights_and_cache() -> None:
    """The exact eval path's effective weights (layers/tropical_exact.py:257-291) against numpy,
    built once per parameter version and rebuilt after an in-place update (host logic; the
    kernels that consume them are checked in tests/test_tropical_gpu.py)."""
    from tropnn_b200.layers import _exact_eval_params

    layer = tropnn_b200.TropLinear(12, 7, heads=3, cells=4, code_dim=5, seed=1, exact_fused="eval")
    cpu = torch.device("cpu")
    router_eff, bias, value_eff, base = _exact_eval_params(layer, cpu)
    w = layer.router_weight.detach().numpy().reshape(12, 5).copy()
    p = layer.proj.weight.detach().numpy().copy()  # copies: the parameter changes in place below
    w_out = layer.output_proj.weight.detach().numpy().copy()
    assert np.allclose(router_eff.numpy().reshape(12, 12), w @ p, atol=1e-6)
    assert np.allclose(value_eff.numpy().reshape(12, 7), layer.code.detach().numpy().reshape(12, 5) @ w_out.T, atol=1e-6)
    assert np.allclose(base.numpy(), w_out @ p, atol=1e-6)
    assert torch.equal(bias, layer.router_bias.detach())
    assert _exact_eval_params(layer, cpu)[0] is router_eff  # cached
    with torch.no_grad():
        layer.proj.weight.mul_(0.5)
    again = _exact_eval_params(layer, cpu)
    assert again[0] is not router_eff
    assert np.allclose(again[3].numpy(), w_out @ (0.5 * p), atol=1e-6)
