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
    # Training and config 5: the reference's torch path, itself when installed, else its port.
    torch_path = "reference" if bench.reference_package_root() is not None else "torch"
    assert bench.cpu_impl_for(W["pairwise_cfg2"], "auto") == torch_path
    assert bench.cpu_impl_for(W["trop_cfg5_eval"], "auto") == torch_path  # BLAS scores beat the Zig dots there
    assert bench.cpu_impl_for(W["trop_cfg1"], "auto") == "zig"
    with pytest.raises(SystemExit):
        bench.cpu_impl_for(W["pairwise_cfg2"], "zig")
    x = torch.empty(W["pairwise_cfg2"].rows_per_gpu, 256)
    bufs = bench._result_buffers(W["pairwise_cfg2"], x)
    assert [tuple(b.shape) for b in bufs] == [(4096, 1, 512), (4096, 256)]
    assert [tuple(b.shape) for b in bench._result_buffers(W["trop_cfg3_clf"], torch.empty(512, 784))] == [(1,)]
    assert bench._input_grad(W["pairwise_cfg2"]) and not bench._input_grad(W["trop_cfg3_clf"])
    assert not bench._input_grad(W["trop_cfg1"])


def test_workload_scaling_splits_the_global_batch() -> None:
    W = bench.WORKLOADS
    assert W["trop_cfg5_train"].scaling == "strong"
    assert [W["trop_cfg5_train"].rows_on_rank(n) for n in (1, 2, 4, 8)] == [16384, 8192, 4096, 2048]
    assert W["trop_cfg5_train"].global_rows(8) == 16384
    assert W["pairwise_cfg2"].rows_on_rank(4) == 4096 and W["pairwise_cfg2"].global_rows(4) == 4 * 4096


def test_reference_arm_times_the_reference_package_itself(monkeypatch) -> None:
    """With the reference installed, --impl reference times its own torch path (kind
    "reference"), here on a tiny config 2 sample."""
    import argparse
    import dataclasses

    if bench.reference_package_root() is None:
        pytest.skip("the reference package is not installed under baseline/_ref")
    monkeypatch.setenv("RANK", "0")
    monkeypatch.setenv("WORLD_SIZE", "1")
    w = dataclasses.replace(bench.WORKLOADS["pairwise_cfg2"], ref_sample_rows=16)
    line = bench.run_reference(argparse.Namespace(steps=2, warmup=1, cpu_impl="auto"), w)
    assert line["impl"] == "reference" and line["value"] > 0
    assert line["cpu_baseline"]["kind"] == "reference" and "torch threads" in line["cpu_baseline"]["sample"]
    assert line["config"]["rows_per_step_sample"] == 16
