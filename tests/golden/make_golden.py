"""Generates the golden fixtures in this directory by running the reference tropnn package.

Run in a checkout where the reference package is importable (default: a read-only
source tree at $TROPNN_REFERENCE, imported as ``tropnn`` through a temporary symlink):

    TROPNN_REFERENCE=/path/to/tropnn python tests/golden/make_golden.py [--only NAME ...]

(``--only`` rewrites just the named fixtures; every case still draws its inputs, in order,
from the one seeded generator, so each fixture's inputs do not depend on the selection.)

Each case records, from the reference's torch path on CPU (``backend="torch"``; TropLinear,
TropFanLinear and PairwiseLinear;
``exact_fused="off"``, or ``"eval"`` where a case's kwargs ask for the reassociated eval path of
layers/tropical_exact.py:297-358): the seeded state_dict, the seeded inputs, the forward outputs,
the route debug cache (``_last_indices`` / ``_last_margins``) and, for training cases,
every gradient of ``(y * grad_out).sum()`` (an upstream gradient ``grad_out``). The
fixtures are the parity anchor of the numpy oracle and of the CUDA kernels; nothing at
test or bench time reads the reference itself.
"""

from __future__ import annotations

import hashlib
import json
import os
import sys
import tempfile
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _import_reference():
    src = Path(os.environ.get("TROPNN_REFERENCE", "/root/reference")).resolve()
    if not (src / "layers" / "tropical.py").exists():
        raise SystemExit(f"reference tropnn sources not found at {src}")
    tmp = Path(tempfile.mkdtemp(prefix="tropnn_ref_"))
    (tmp / "tropnn").symlink_to(src)
    sys.path.insert(0, str(tmp))
    sys.dont_write_bytecode = True
    import tropnn  # noqa: PLC0415

    return tropnn


def _arr(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().numpy().copy()


def _sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.detach().cpu().contiguous().numpy().tobytes()).hexdigest()


def _state(module: torch.nn.Module) -> dict[str, np.ndarray]:
    """sha256 of every state_dict tensor; the tensors themselves only for tiny layers
    (the tests rebuild larger ones from the seed and check the hashes)."""
    state = module.state_dict()
    out = {f"sha256.{k}": np.array(_sha(v)) for k, v in state.items()}
    if sum(v.numel() * v.element_size() for v in state.values()) <= 64 * 1024:
        out.update({f"state.{k}": _arr(v) for k, v in state.items()})
    return out


def _grads(module: torch.nn.Module) -> dict[str, np.ndarray]:
    out = {}
    for name, p in module.named_parameters():
        out[f"grad.{name}"] = _arr(p.grad) if p.grad is not None else np.zeros(0, dtype=np.float32)
        out[f"has_grad.{name}"] = np.array(p.grad is not None)
    return out


def _run_case(layer: torch.nn.Module, x: torch.Tensor, *, train: bool, grad_out: torch.Tensor | None) -> dict[str, np.ndarray]:
    rec: dict[str, np.ndarray] = {}
    rec.update(_state(layer))
    rec["x"] = _arr(x)
    layer.train(train)
    if train:
        xg = x.clone().requires_grad_(True)
        y = layer(xg)
        assert grad_out is not None
        (y * grad_out).sum().backward()
        rec["grad.x"] = _arr(xg.grad)
        rec["grad_out"] = _arr(grad_out)
        rec.update(_grads(layer))
    else:
        with torch.no_grad():
            y = layer(x)
    rec["y"] = _arr(y)
    if layer._last_indices is not None:
        rec["last_indices"] = _arr(layer._last_indices)
        rec["last_margins"] = _arr(layer._last_margins)
    return rec


def _save(name: str, rec: dict[str, np.ndarray], meta: dict) -> None:
    rec = dict(rec)
    rec["meta"] = np.array(json.dumps(meta))
    np.savez_compressed(HERE / f"{name}.npz", **rec)


def _bias_separate(layer, values: torch.Tensor) -> None:
    with torch.no_grad():
        layer.router_bias.copy_(values.expand_as(layer.router_bias))


def main(only: set[str] | None = None) -> None:
    tropnn = _import_reference()
    TropLinear, PairwiseLinear, TropFanLinear = tropnn.TropLinear, tropnn.PairwiseLinear, tropnn.TropFanLinear
    gen = torch.Generator().manual_seed(1)
    manifest = {}

    def trop(name, in_f, out_f, *, heads, cells, code_dim, batch, steps=None, train, seed=0, half=False, bias=None, uniform=False, **kw):
        layer = TropLinear(in_f, out_f, heads=heads, cells=cells, code_dim=code_dim, seed=seed, **kw)
        if bias is not None:
            _bias_separate(layer, bias)
        if half:
            layer = layer.half()
        shape = (batch, in_f) if steps is None else (batch, steps, in_f)
        x = torch.rand(shape, generator=gen) if uniform else torch.randn(shape, generator=gen)
        y_shape = (batch, 1 if steps is None else steps, out_f)
        g = torch.randn(y_shape, generator=gen) if train else None
        rec = _run_case(layer, x, train=train, grad_out=g)
        meta = dict(kind="trop", in_features=in_f, out_features=out_f, heads=heads, cells=cells, code_dim=code_dim,
                    seed=seed, train=train, half=half, code_scale=layer.code_scale, kwargs=kw,
                    router_bias=None if bias is None else [float(v) for v in bias])
        if only is None or name in only:
            _save(name, rec, meta)
        manifest[name] = meta

    def pair(name, in_f, out_f, *, tables, comparisons, batch, steps=None, train, seed=0, half=False, uniform=False, **kw):
        layer = PairwiseLinear(in_f, out_f, tables=tables, comparisons=comparisons, seed=seed, **kw)
        if half:
            layer = layer.half()
        shape = (batch, in_f) if steps is None else (batch, steps, in_f)
        x = torch.rand(shape, generator=gen) if uniform else torch.randn(shape, generator=gen)
        y_shape = (batch, 1 if steps is None else steps, out_f)
        g = torch.randn(y_shape, generator=gen) if train else None
        rec = _run_case(layer, x, train=train, grad_out=g)
        meta = dict(kind="pairwise", in_features=in_f, out_features=out_f, tables=tables, comparisons=comparisons,
                    seed=seed, train=train, half=half, output_scale=layer.output_scale, kwargs=kw)
        if only is None or name in only:
            _save(name, rec, meta)
        manifest[name] = meta

    def fan(name, in_f, out_f, *, heads, cells, code_dim, batch, steps=None, train, seed=0, half=False, lifting=None, **kw):
        layer = TropFanLinear(in_f, out_f, heads=heads, cells=cells, code_dim=code_dim, seed=seed, **kw)
        if lifting is not None:
            with torch.no_grad():
                layer.lifting.copy_(lifting.expand_as(layer.lifting))
        if half:
            layer = layer.half()
        shape = (batch, in_f) if steps is None else (batch, steps, in_f)
        x = torch.randn(shape, generator=gen)
        y_shape = (batch, 1 if steps is None else steps, out_f)
        g = torch.randn(y_shape, generator=gen) if train else None
        rec = _run_case(layer, x, train=train, grad_out=g)
        meta = dict(kind="fan", in_features=in_f, out_features=out_f, heads=heads, cells=cells, code_dim=code_dim,
                    seed=seed, train=train, half=half, code_scale=layer.code_scale, kwargs=kw,
                    fan_value_mode=layer.fan_value_mode, lifting=None if lifting is None else [float(v) for v in lifting])
        if only is None or name in only:
            _save(name, rec, meta)
        manifest[name] = meta

    # config 1: TropLinear(256->512, H32, K4, D32) eval forward, batch 8, seed 0.
    trop("cfg1_trop_eval_b8", 256, 512, heads=32, cells=4, code_dim=32, batch=8, train=False)
    trop("cfg1_trop_train_b8", 256, 512, heads=32, cells=4, code_dim=32, batch=8, train=True)
    # config 2: PairwiseLinear(256->512, T16, C6) forward + STE backward, batch 8 (and 64).
    pair("cfg2_pair_train_b8", 256, 512, tables=16, comparisons=6, batch=8, train=True)
    pair("cfg2_pair_eval_b8", 256, 512, tables=16, comparisons=6, batch=8, train=False)
    pair("cfg2_pair_full_ste_b8", 256, 512, tables=16, comparisons=6, batch=8, train=True, use_min_margin_ste=False)
    # config 3: the two TropLinear layers of the 784->128->10 classifier (seed + idx).
    trop("cfg3_trop_l1_train_b16", 784, 128, heads=256, cells=16, code_dim=64, batch=16, train=True, seed=0, uniform=True)
    trop("cfg3_trop_l2_train_b16", 128, 10, heads=256, cells=16, code_dim=64, batch=16, train=True, seed=1)
    # config 4: the two PairwiseLinear layers of the 784->128->10 classifier.
    pair("cfg4_pair_l1_train_b16", 784, 128, tables=136, comparisons=6, batch=16, train=True, seed=0, uniform=True)
    pair("cfg4_pair_l2_train_b16", 128, 10, tables=136, comparisons=6, batch=16, train=True, seed=1)
    # config 5 at reduced width (f16 parameters, f32 input).
    trop("cfg5s_trop_half_eval_b32", 256, 256, heads=64, cells=16, code_dim=64, batch=32, train=False, half=True)
    trop("cfg5s_trop_half_train_b32", 256, 256, heads=64, cells=16, code_dim=64, batch=32, train=True, half=True)
    pair("cfg5s_pair_half_eval_b32", 256, 128, tables=32, comparisons=8, batch=32, train=False, half=True)
    pair("cfg5s_pair_half_train_b32", 256, 128, tables=32, comparisons=8, batch=32, train=True, half=True)
    # Reference-test shapes (tests/test_backend_parity.py:348-392, tests/test_tropical_core.py:124-214).
    pair("small_pair_min_b4", 8, 5, tables=3, comparisons=3, batch=4, train=True, seed=1)
    pair("small_pair_full_b4", 8, 5, tables=3, comparisons=3, batch=4, train=True, seed=1, use_min_margin_ste=False)
    pair("small_pair_izh_b4", 8, 5, tables=3, comparisons=3, batch=4, train=True, seed=2, surrogate="izhikevich")
    trop("small_trop_bias_train", 6, 4, heads=3, cells=4, code_dim=5, batch=5, steps=2, train=True, seed=2,
         bias=torch.tensor([-3.0, -1.0, 1.0, 3.0]))
    trop("small_trop_cells8_train", 6, 4, heads=5, cells=8, code_dim=5, batch=5, steps=2, train=True, seed=7,
         bias=torch.linspace(-4.0, 3.0, steps=8), cache_route_debug=False)
    trop("small_trop_eval_3d", 6, 4, heads=3, cells=4, code_dim=5, batch=5, steps=2, train=False, seed=1)
    trop("small_trop_cells300_train", 16, 8, heads=3, cells=300, code_dim=8, batch=6, train=True, seed=3)
    # exact_fused="eval": the reassociated eval path (layers/tropical_exact.py:297-358; run under
    # no_grad, as its dispatch at layers/tropical.py:92 requires).
    trop("cfg1_trop_exact_eval_b8", 256, 512, heads=32, cells=4, code_dim=32, batch=8, train=False, exact_fused="eval")
    trop("small_trop_exact_eval_3d", 6, 4, heads=3, cells=4, code_dim=5, batch=5, steps=2, train=False, seed=4,
         exact_fused="eval")
    trop("cfg5s_trop_half_exact_eval_b32", 256, 256, heads=64, cells=16, code_dim=64, batch=32, train=False, half=True,
         exact_fused="eval")

    # TropFanLinear (layers/fan.py:21-330): site and basis value modes, train and eval, f32 and f16.
    fan("small_fan_site_train", 6, 4, heads=3, cells=4, code_dim=5, batch=5, steps=2, train=True, seed=2,
        lifting=torch.tensor([-3.0, -1.0, 1.0, 3.0]))
    fan("small_fan_basis_train", 6, 4, heads=3, cells=4, code_dim=5, batch=5, steps=2, train=True, seed=3,
        lifting=torch.tensor([-3.0, -1.0, 1.0, 3.0]), fan_value_mode="basis", fan_basis_rank=3)
    fan("cfg1s_fan_site_eval_b8", 256, 512, heads=32, cells=4, code_dim=32, batch=8, train=False)
    fan("mid_fan_basis_train_b16", 256, 128, heads=64, cells=16, code_dim=64, batch=16, train=True, seed=1,
        fan_value_mode="basis", fan_basis_rank=16)
    fan("mid_fan_site_half_train_b32", 256, 256, heads=64, cells=16, code_dim=64, batch=32, train=True, half=True)

    # Full-size seeded init of config 5's TropLinear: sha256 of every state_dict tensor.
    big = TropLinear(4096, 4096, heads=1024, cells=16, code_dim=256, seed=0).half()
    hashes = {k: hashlib.sha256(v.detach().contiguous().numpy().tobytes()).hexdigest() for k, v in big.state_dict().items()}
    (HERE / "cfg5_trop_init_sha256.json").write_text(json.dumps(hashes, indent=1, sort_keys=True) + "\n")
    (HERE / "manifest.json").write_text(json.dumps(manifest, indent=1, sort_keys=True) + "\n")
    print(f"wrote {len(manifest)} cases to {HERE}")


if __name__ == "__main__":
    import argparse

    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--only", nargs="*", default=None, help="fixture names to (re)write; default all")
    args = parser.parse_args()
    main(set(args.only) if args.only is not None else None)
