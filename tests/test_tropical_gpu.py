"""TropLinear backend="b200" on the GPU against the reference's golden vectors and the numpy
oracle. Route indices are compared where the top-2 margin exceeds 1e-4 relative (the
parity gate); values within 1e-5 relative in fp32, 2e-2 with f16/bf16 parameters, on
batches whose routes the gate pins (tests/trop_check.py)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
import tropnn_b200
from tests.golden_cases import build_layer, case_names, load_case, rel_err, route_gate, state_arrays, tolerance
from tests.gpu_runner import run_b200
from tests.trop_check import check_trop_layer, check_trop_routes, pinned_batch

pytestmark = pytest.mark.gpu
FP32_TOL = 1e-5


def _exact_eval(meta: dict) -> bool:
    return meta["kwargs"].get("exact_fused") == "eval" and not meta["train"]


def _gate_from_state(x: np.ndarray, st: dict, exact: bool = False) -> tuple[np.ndarray, np.ndarray]:
    if exact:
        ref = oracle.trop_linear_exact_eval(x, st, code_scale=1.0)
    else:
        ref = oracle.trop_linear_forward(x, st, code_scale=1.0, training=False)
    return route_gate(ref["scores"])


@pytest.mark.parametrize("name", case_names("trop"))
def test_trop_matches_reference_golden(name: str) -> None:
    arrays, meta = load_case(name)
    layer = build_layer(arrays, meta)
    st = state_arrays(layer)
    got = run_b200(layer, arrays, meta)
    # The exact eval path computes in f32 whatever the parameter dtype (so does the reference's).
    tol = FP32_TOL if _exact_eval(meta) else tolerance(meta)
    assert rel_err(got["y"], arrays["y"]) <= tol
    x = arrays["x"].reshape(-1, arrays["x"].shape[-1]).astype(np.float32)
    win, _ = _gate_from_state(x, st, exact=_exact_eval(meta))
    if "last_indices" in arrays:
        assert np.array_equal(got["last_indices"].reshape(win.shape)[win], arrays["last_indices"].reshape(win.shape)[win])
        assert rel_err(got["last_margins"], arrays["last_margins"]) <= max(tol, 1e-5)
    else:
        assert "last_indices" not in got  # cache_route_debug=False
    if meta["train"]:
        assert rel_err(got["grad.x"], arrays["grad.x"]) <= tol
        for key in ("proj.weight", "router_weight", "router_bias", "code", "output_proj.weight", "output_proj.bias"):
            assert bool(got[f"has_grad.{key}"]) == bool(arrays[f"has_grad.{key}"]), key
            assert rel_err(got[f"grad.{key}"], arrays[f"grad.{key}"].astype(np.float32)) <= tol, key


def _inputs(n: int, in_f: int, out_f: int, seed: int = 1, uniform: bool = False) -> tuple[np.ndarray, np.ndarray]:
    gen = torch.Generator().manual_seed(seed)
    x = torch.rand(n, in_f, generator=gen) if uniform else torch.randn(n, in_f, generator=gen)
    return x.numpy(), torch.randn(n, out_f, generator=gen).numpy()


def _run(layer: tropnn_b200.TropLinear, x: np.ndarray, g: np.ndarray, *, train: bool) -> dict:
    layer = layer.cuda().train(train)
    xt = torch.from_numpy(x).cuda().requires_grad_(True)
    y = layer(xt)
    y.backward(torch.from_numpy(g).cuda().view_as(y))
    torch.cuda.synchronize()
    out = {"y": y.detach().float().cpu().numpy().reshape(x.shape[0], -1), "grad.x": xt.grad.cpu().numpy()}
    out["winner"] = layer._last_indices.cpu().numpy().reshape(x.shape[0], -1)
    out["margins"] = layer._last_margins.cpu().numpy().reshape(x.shape[0], -1)
    for name, p in layer.named_parameters():
        out[f"grad.{name}"] = None if p.grad is None else p.grad.float().cpu().numpy()
    return out


def _check_against_oracle(layer: tropnn_b200.TropLinear, x: np.ndarray, g: np.ndarray, *, train: bool, tol: float) -> None:
    """Routes of the whole pool ``x`` under the gate, then routes, values and every gradient on
    a batch of half the pool (rounded to a multiple of 8) whose routes the gate pins."""
    check_trop_routes(layer, x, train=train)
    rows = max(1, x.shape[0] // 2 // 8 * 8) if x.shape[0] >= 16 else max(1, x.shape[0] // 2)
    xb = pinned_batch(layer, x, rows, train=train)
    check_trop_layer(layer, xb, g[:rows], train=train, tol=tol)


@pytest.mark.parametrize("train", [True, False])
def test_config3_layer1_batch512(train: bool) -> None:
    """Config 3 layer 1: TropLinear(784->128, H256, K16, D64), U[0,1] inputs, batch 512 (from a
    pool of 1024 rows)."""
    layer = tropnn_b200.TropLinear(784, 128, heads=256, cells=16, code_dim=64, seed=0)
    x, g = _inputs(1024, 784, 128, uniform=True)
    _check_against_oracle(layer, x, g, train=train, tol=FP32_TOL)


@pytest.mark.parametrize(
    ("in_f", "out_f", "heads", "cells", "code_dim", "n"),
    [
        (256, 512, 32, 4, 32, 8),  # config 1
        (5, 3, 1, 2, 1, 7),  # minimum heads/cells/code_dim
        (40, 20, 6, 300, 12, 64),  # int16 route packing (cells > 256)
        (33, 17, 9, 256, 7, 130),  # u8 packing at its maximum, ragged code_dim
        (64, 48, 16, 9, 256, 300),  # code_dim 256 (largest on the SIMT path)
    ],
)
def test_shapes_and_edges(in_f: int, out_f: int, heads: int, cells: int, code_dim: int, n: int) -> None:
    layer = tropnn_b200.TropLinear(in_f, out_f, heads=heads, cells=cells, code_dim=code_dim, seed=4)
    x, g = _inputs(2 * n, in_f, out_f, seed=2)
    _check_against_oracle(layer, x, g, train=True, tol=FP32_TOL)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_half_precision_parameters(dtype: torch.dtype) -> None:
    """Config-5 style: half parameters, f32 input, f32 accumulation."""
    layer = tropnn_b200.TropLinear(256, 256, heads=64, cells=16, code_dim=64, seed=0)
    with torch.no_grad():
        layer.router_bias.copy_(torch.linspace(-2.0, 2.0, 16).expand_as(layer.router_bias))
    layer = layer.to(dtype)
    x, g = _inputs(512, 256, 256, seed=3)
    _check_against_oracle(layer, x, g, train=True, tol=2e-2)
    assert layer.code.grad.dtype == dtype and layer.router_weight.grad.dtype == dtype


def test_eval_and_train_kats_on_gpu() -> None:
    """tests/test_tropical_core.py:19-49 on the b200 kernels."""
    layer = tropnn_b200.TropLinear(1, 1, heads=1, cells=3, code_dim=1, seed=0, use_output_scaling=False)
    with torch.no_grad():
        layer.proj.weight.fill_(1.0)
        layer.router_weight[0, :, 0] = torch.tensor([1.0, 0.0, -1.0])
        layer.router_bias.zero_()
        layer.code[0, :, 0] = torch.tensor([10.0, 20.0, 30.0])
        layer.output_proj.weight.fill_(1.0)
        layer.output_proj.bias.zero_()
    layer = layer.cuda().eval()
    assert float(layer(torch.tensor([[2.0]], device="cuda")).squeeze()) == pytest.approx(12.0)
    assert float(layer(torch.tensor([[-2.0]], device="cuda")).squeeze()) == pytest.approx(28.0)
    with torch.no_grad():
        layer.router_weight[0, :, 0] = torch.tensor([1.0, 0.9, -1.0], device="cuda")
    layer.train()
    y = float(layer(torch.tensor([[1.0]], device="cuda")).squeeze())
    assert y == pytest.approx(1.0 + 10.0 + (0.5 / 1.1) * 10.0, abs=1e-6)


def test_output_shapes_and_debug_cache() -> None:
    layer = tropnn_b200.TropLinear(5, 3, heads=4, cells=3, code_dim=4, seed=0).cuda()
    y2 = layer(torch.randn(7, 5, device="cuda"))
    assert y2.shape == (7, 1, 3)
    assert layer._last_indices.shape == (7, 1, 4) and layer._last_indices.dtype == torch.int64
    y3 = layer(torch.randn(7, 2, 5, device="cuda"))
    assert y3.shape == (7, 2, 3)
    quiet = tropnn_b200.TropLinear(5, 3, heads=4, cells=3, code_dim=4, seed=0, cache_route_debug=False).cuda()
    quiet(torch.randn(2, 5, device="cuda"))
    assert quiet._last_indices is None and quiet._last_margins is None


def test_index_forcing_backward_through_c_abi() -> None:
    """Feeds the oracle's routes to tropnn_b200_trop_backward (one C call) to isolate the
    backward arithmetic from the forward's routing."""
    from tropnn_b200 import _native as nat

    layer = tropnn_b200.TropLinear(48, 32, heads=16, cells=8, code_dim=24, seed=6)
    n, D, H, K = 200, 24, 16, 8
    x, _ = _inputs(n, 48, 32, seed=9)
    st = state_arrays(layer)
    fwd = oracle.trop_linear_forward(x, st, code_scale=layer.code_scale, training=True)
    gen = torch.Generator().manual_seed(5)
    gh = torch.randn(n, D, generator=gen).numpy()
    ref = oracle.trop_route_backward(
        gh, fwd["z"], st["router_weight"], st["code"], fwd["winner"], fwd["runner"], fwd["margins"],
        code_scale=layer.code_scale, training=True,
    )
    dev = torch.device("cuda")
    t = {k: torch.from_numpy(np.ascontiguousarray(v)).to(dev) for k, v in
         dict(g=gh, z=fwd["z"], W=st["router_weight"], c=st["code"], m=fwd["margins"]).items()}
    win = torch.from_numpy(fwd["winner"]).to(dev, torch.uint8).contiguous()
    run = torch.from_numpy(fwd["runner"]).to(dev, torch.uint8).contiguous()
    lib = nat.load()
    ws_bytes = lib.tropnn_b200_trop_backward_workspace_size(n, H, K, 1)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    gz = torch.empty(n, D, device=dev)
    gW = torch.empty(H, K, D, device=dev)
    gb = torch.empty(H, K, device=dev)
    gc = torch.empty(H, K, D, device=dev)
    status = lib.tropnn_b200_trop_backward(
        t["g"].data_ptr(), t["z"].data_ptr(), n, D, t["W"].data_ptr(), t["c"].data_ptr(), nat.F32, H, K,
        win.data_ptr(), run.data_ptr(), nat.U8, t["m"].data_ptr(), layer.code_scale, 1, gz.data_ptr(),
        gW.data_ptr(), gb.data_ptr(), gc.data_ptr(), ws.data_ptr(), ws_bytes, torch.cuda.current_stream().cuda_stream,
    )
    nat.check(status, "trop_backward")
    torch.cuda.synchronize()
    assert rel_err(gz.cpu().numpy(), ref["grad_latent"]) <= FP32_TOL
    assert rel_err(gW.cpu().numpy(), ref["grad_router_weight"]) <= FP32_TOL
    assert rel_err(gb.cpu().numpy(), ref["grad_router_bias"]) <= FP32_TOL
    assert rel_err(gc.cpu().numpy(), ref["grad_code"]) <= FP32_TOL


def test_backward_is_deterministic() -> None:
    layer = tropnn_b200.TropLinear(784, 128, heads=256, cells=16, code_dim=64, seed=0)
    x, g = _inputs(512, 784, 128, uniform=True)
    a = _run(layer, x, g, train=True)
    layer.zero_grad(set_to_none=True)
    b = _run(layer, x, g, train=True)
    for key in ("grad.router_weight", "grad.router_bias", "grad.code", "grad.x"):
        assert np.array_equal(a[key], b[key]), key


def test_invalid_arguments_raise() -> None:
    layer = tropnn_b200.TropLinear(6, 4, heads=3, cells=4, code_dim=5).cuda()
    with pytest.raises(TypeError):
        layer(torch.randn(2, 6, device="cuda", dtype=torch.float64))
    z = torch.randn(1, 2, 5, device="cuda")
    with pytest.raises(ValueError):
        tropnn_b200.trop_route_hidden_b200(z, layer.router_weight, layer.router_bias[:2], layer.code, code_scale=1.0)
    with pytest.raises(ValueError):
        tropnn_b200.trop_route_hidden_b200(z[..., :4], layer.router_weight, layer.router_bias, layer.code, code_scale=1.0)


@pytest.mark.parametrize(
    ("in_f", "out_f", "heads", "cells", "code_dim", "n", "half"),
    [
        (256, 512, 32, 4, 32, 4096, False),  # config 1's layer at a wide batch
        (784, 128, 256, 16, 64, 512, False),  # config 3 layer 1
        (256, 256, 64, 16, 64, 300, True),  # f16 parameters: the exact path still computes in f32
        (1536, 40, 8, 3, 24, 65, False),  # the widest input the exact path routes on; 3 cells
    ],
)
def test_exact_eval_path_matches_oracle(in_f, out_f, heads, cells, code_dim, n, half) -> None:
    """exact_fused="eval" in eval under no_grad (layers/tropical.py:92): the reassociated path of
    layers/tropical_exact.py:297-358 against its oracle restatement. Winners bit-exact where the
    top-2 margin clears the parity gate; outputs of the rows whose every head clears it within
    1e-5 relative."""
    layer = tropnn_b200.TropLinear(in_f, out_f, heads=heads, cells=cells, code_dim=code_dim, seed=5,
                                   exact_fused="eval")
    if half:
        layer = layer.half()
    layer = layer.cuda().eval()
    gen = torch.Generator().manual_seed(9)
    x = torch.randn(n, in_f, generator=gen)
    with torch.no_grad():
        y = layer(x.cuda())
    assert getattr(layer, "_b200_exact_eval_cache", None) is not None  # the exact path ran
    st = state_arrays(layer)
    ref = oracle.trop_linear_exact_eval(x.numpy(), st, code_scale=layer.code_scale)
    win, _ = route_gate(ref["scores"])
    got_w = layer._last_indices.cpu().numpy().reshape(n, heads)
    assert np.array_equal(got_w[win], ref["winner"][win])
    assert rel_err(layer._last_margins.cpu().numpy().reshape(n, heads), ref["margins"]) <= 1e-5
    rows = win.all(axis=1) & (got_w == ref["winner"]).all(axis=1)
    assert rows.mean() > 0.5
    assert rel_err(y.float().cpu().numpy().reshape(n, -1)[rows], ref["y"][rows]) <= FP32_TOL


def test_exact_eval_dispatch_and_cache() -> None:
    """The exact path runs only in eval under no_grad and for inputs of at most 1536 features;
    its effective weights are rebuilt when a parameter changes in place."""
    layer = tropnn_b200.TropLinear(64, 48, heads=8, cells=4, code_dim=16, seed=2, exact_fused="eval").cuda()
    x = torch.randn(33, 64, device="cuda")
    layer.train()
    with torch.no_grad():
        layer(x)
    assert getattr(layer, "_b200_exact_eval_cache", None) is None  # training: the default path
    layer.eval()
    layer(x)
    assert getattr(layer, "_b200_exact_eval_cache", None) is None  # grad enabled: the default path
    with torch.no_grad():
        y0 = layer(x)
        key0 = layer._b200_exact_eval_cache[0]
        layer.code.mul_(2.0)
        y1 = layer(x)
    assert layer._b200_exact_eval_cache[0] != key0
    st = state_arrays(layer)
    ref = oracle.trop_linear_exact_eval(x.cpu().numpy(), st, code_scale=layer.code_scale)
    assert rel_err(y1.cpu().numpy().reshape(33, -1), ref["y"]) <= FP32_TOL
    assert not torch.equal(y0, y1)
    wide = tropnn_b200.TropLinear(2048, 16, heads=4, cells=4, code_dim=16, seed=3, exact_fused="eval").cuda().eval()
    with torch.no_grad():
        wide(torch.randn(5, 2048, device="cuda"))
    assert getattr(wide, "_b200_exact_eval_cache", None) is None  # wider than the route kernel's row stage
