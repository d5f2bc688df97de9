"""Batch-row data parallelism on two gloo ranks (CPU): sharding plus the gradient all-reduce
of tropnn_b200.distributed give the full-batch gradient of a mean loss on every rank.

The per-shard gradients come from the numpy oracle of the PairwiseLinear backward (the CUDA
kernels compute the same quantity on the GPU), so this checks the host logic of the N>1 path
without a GPU.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from tropnn_b200.distributed import allreduce_gradients, row_range, shard_rows


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_row_range_partitions_rows() -> None:
    for rows in (0, 1, 7, 4096, 4099):
        for world in (1, 2, 3, 8):
            spans = [row_range(rows, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == rows
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        row_range(10, 2, 2)


def _problem():
    gen = torch.Generator().manual_seed(3)
    tables, comparisons, in_f, out_f, rows = 6, 4, 32, 24, 64
    anchors = torch.stack([torch.randperm(in_f, generator=gen)[: 2 * comparisons].view(comparisons, 2) for _ in range(tables)])
    thresholds = 0.1 * torch.randn(tables, comparisons, generator=gen)
    lut = 0.02 * torch.randn(tables, 1 << comparisons, out_f, generator=gen)
    x = torch.randn(rows, in_f, generator=gen)
    g = torch.randn(rows, out_f, generator=gen) / rows  # gradient of a mean loss
    return anchors.numpy(), thresholds.numpy(), lut.numpy(), x.numpy(), g.numpy()


def _grads(anchors, thresholds, lut, x, g):
    fwd = oracle.pairwise_forward(x, anchors, thresholds, lut, output_scale=0.5)
    bwd = oracle.pairwise_backward(
        g, fwd["indices"], fwd["margins"], anchors, lut, in_features=x.shape[1], output_scale=0.5, use_min_margin_ste=True
    )
    return bwd["lut"], bwd["thresholds"]


def _rank(rank: int, world: int, port: int, queue) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        anchors, thresholds, lut, x, g = _problem()
        xs = shard_rows(torch.from_numpy(x), rank, world).numpy()
        gs = shard_rows(torch.from_numpy(g), rank, world).numpy()
        glut, gthr = _grads(anchors, thresholds, lut, xs, gs)
        p_lut = torch.nn.Parameter(torch.zeros(lut.shape))
        p_thr = torch.nn.Parameter(torch.zeros(thresholds.shape))
        # Each rank's gradient is of the mean over its own shard; the all-reduce average
        # then equals the gradient of the global mean (equal shard sizes).
        p_lut.grad = torch.from_numpy(glut * world)
        p_thr.grad = torch.from_numpy(gthr * world)
        calls = allreduce_gradients([p_lut, p_thr], bucket_bytes=4096)
        queue.put((rank, p_lut.grad.numpy(), p_thr.grad.numpy(), calls))
    finally:
        dist.destroy_process_group()


def test_two_rank_allreduce_equals_full_batch_gradient() -> None:
    world = 2
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = [queue.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    anchors, thresholds, lut, x, g = _problem()
    full_lut, full_thr = _grads(anchors, thresholds, lut, x, g)
    for _, glut, gthr, calls in results:
        np.testing.assert_allclose(glut, full_lut, rtol=1e-5, atol=1e-7)
        np.testing.assert_allclose(gthr, full_thr, rtol=1e-5, atol=1e-7)
        assert calls >= 2  # the LUT gradient (24 KiB) is reduced in 4 KiB slices
    np.testing.assert_array_equal(results[0][1], results[1][1])


def _overlap_rank(rank: int, world: int, port: int, queue) -> None:
    from tropnn_b200 import distributed as tdist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        a = torch.nn.Parameter(torch.zeros(5))
        b = torch.nn.Parameter(torch.zeros(3))
        a.grad = torch.full((5,), float(rank + 1))
        b.grad = torch.full((3,), float(10 * (rank + 1)))
        # Outside the context the in-backward hooks do nothing.
        tdist.reduce_gradient_now(b.grad)
        untouched = b.grad.clone()
        with tdist.overlapped_gradient_sync():
            tdist.reduce_gradient_now(b.grad)  # as the Pairwise backward does for thresholds
        calls = allreduce_gradients([a, b])  # must skip b (already averaged), reduce a
        calls_again = allreduce_gradients([a, b])  # the mark is consumed: b is reduced now
        # A gradient averaged inside its own kernel (the fused LUT-gradient path) is marked the
        # same way and skipped once.
        c = torch.nn.Parameter(torch.zeros(4))
        c.grad = torch.full((4,), float(rank + 7))
        tdist.mark_reduced(c.grad)
        calls_marked = allreduce_gradients([c])
        queue.put((rank, untouched.numpy(), a.grad.numpy(), b.grad.numpy(), calls, calls_again, c.grad.numpy(),
                   calls_marked))
    finally:
        dist.destroy_process_group()


def test_overlapped_sync_marks_and_skips() -> None:
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    procs = [ctx.Process(target=_overlap_rank, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = [queue.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, untouched, ga, gb, calls, calls_again, gc, calls_marked in results:
        assert np.array_equal(untouched, np.full(3, 10.0 * (rank + 1)))
        assert np.allclose(ga, np.full(5, 1.5))  # mean of 1 and 2, reduced once
        assert np.allclose(gb, np.full(3, 15.0))  # mean of 10 and 20 (second pass: mean of equal values)
        assert calls == 1 and calls_again == 1
        assert calls_marked == 0 and np.array_equal(gc, np.full(4, float(rank + 7)))


def test_fused_lut_context_sets_and_restores() -> None:
    """fused_lut_allreduce publishes its peer set to the backward (fused_lut_peer) and restores
    the previous one on exit, nested contexts included."""
    from tropnn_b200 import distributed as tdist

    assert tdist.fused_lut_peer() is None
    outer, inner = object(), object()
    with tdist.fused_lut_allreduce(outer):
        assert tdist.fused_lut_peer() is outer
        with tdist.fused_lut_allreduce(inner):
            assert tdist.fused_lut_peer() is inner
        assert tdist.fused_lut_peer() is outer
    assert tdist.fused_lut_peer() is None
