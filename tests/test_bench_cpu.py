"""CPU pieces of bench.py's classifier step (configs 3 and 4): the numpy Adam update and
cross-entropy gradient against torch's own on CPU, and the CPU oracle step end to end."""

from __future__ import annotations

import numpy as np
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
