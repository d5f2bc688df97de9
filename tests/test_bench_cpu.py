"""CPU pieces of bench.py's classifier step (configs 3 and 4): the numpy Adam update and
cross-entropy gradient against torch's own on CPU, and the CPU oracle step end to end."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import bench


def test_adam_update_matches_torch() -> None:
    rng = np.random.default_rng(3)
    p0 = rng.standard_normal((7, 5)).astype(np.float32)
    grads = [rng.standard_normal((7, 5)).astype(np.float32) for _ in range(4)]
    tp = torch.nn.Parameter(torch.from_numpy(p0.copy()))
    opt = torch.optim.Adam([tp], lr=1e-3)
    p, m, v = p0.copy(), np.zeros_like(p0), np.zeros_like(p0)
    for t, g in enumerate(grads, start=1):
        tp.grad = torch.from_numpy(g.copy())
        opt.step()
        bench._adam_update(p, g, m, v, t)
    assert np.allclose(p, tp.detach().numpy(), rtol=0, atol=1e-6)


def test_classifier_oracle_step_runs_and_moves_parameters() -> None:
    """One numpy classifier step on a small sample: every parameter of both layers moves, and the
    cross-entropy gradient it starts from matches torch's."""
    for name in ("trop_cfg3_clf", "pair_cfg4_clf"):
        w = bench.WORKLOADS[name]
        state = bench._classifier_state(w)
        before = [{k: lay["params"][k].copy() for k in lay["names"]} for lay in state["layers"]]
        rng = np.random.default_rng(0)
        x = rng.random((16, w.in_features), dtype=np.float32)
        labels = rng.integers(0, w.out_features, 16)
        bench._oracle_classifier_step(w, state, x, labels)
        for lay, old in zip(state["layers"], before):
            for k in lay["names"]:
                assert not np.array_equal(lay["params"][k], old[k]), (name, k)
    logits = torch.randn(6, 10, requires_grad=True)
    labels = torch.randint(0, 10, (6,))
    torch.nn.functional.cross_entropy(logits, labels).backward()
    lg = logits.detach().numpy()
    e = np.exp(lg - lg.max(axis=1, keepdims=True))
    grad = e / e.sum(axis=1, keepdims=True)
    grad[np.arange(6), labels.numpy()] -= 1.0
    assert np.allclose(grad / 6, logits.grad.numpy(), atol=1e-7)


def test_reference_arm_line_keeps_the_contract(monkeypatch) -> None:
    """bench.py --impl reference on config 1: one JSON object with the base keys, impl, a
    cpu_baseline describing the run (here the C++ Zig-kernel port) and an e2e with no copies;
    ranks other than 0 print nothing."""
    import argparse

    args = argparse.Namespace(steps=1, warmup=1, cpu_impl="auto")
    w = bench.WORKLOADS["trop_cfg1"]
    monkeypatch.setenv("RANK", "1")
    monkeypatch.setenv("WORLD_SIZE", "2")
    assert bench.run_reference(args, w) is None
    monkeypatch.setenv("RANK", "0")
    monkeypatch.setenv("WORLD_SIZE", "1")
    line = bench.run_reference(args, w)
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference" and line["value"] > 0 and line["steps"] == 1
    assert line["cpu_baseline"]["kind"] == "port" and "Zig" in line["cpu_baseline"]["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_cpu_path_choice_and_e2e_buffers(monkeypatch) -> None:
    W = bench.WORKLOADS
    monkeypatch.setattr(torch.Tensor, "pin_memory", lambda self: self)  # no driver here: shapes only
    assert bench.cpu_impl_for(W["pairwise_cfg2"], "auto") == "torch"  # training: the torch path only
    assert bench.cpu_impl_for(W["trop_cfg5_eval"], "auto") == "torch"  # BLAS scores beat the Zig dots there
    assert bench.cpu_impl_for(W["trop_cfg1"], "auto") == "zig"
    with pytest.raises(SystemExit):
        bench.cpu_impl_for(W["pairwise_cfg2"], "zig")
    x = torch.empty(W["pairwise_cfg2"].rows_per_gpu, 256)
    bufs = bench._result_buffers(W["pairwise_cfg2"], x)
    assert [tuple(b.shape) for b in bufs] == [(4096, 1, 512), (4096, 256)]
    assert [tuple(b.shape) for b in bench._result_buffers(W["trop_cfg3_clf"], torch.empty(512, 784))] == [(1,)]
    assert bench._input_grad(W["pairwise_cfg2"]) and not bench._input_grad(W["trop_cfg3_clf"])
    assert not bench._input_grad(W["trop_cfg1"])
