"""NVLink peer-memory gradient all-reduce (tropnn_b200.distributed.PeerAllReduce) on 2, 3, 4
and 8 GPUs (one-shot on two ranks, two-shot above): sums and averages of several f32 tensors
match the exact result on every rank, results are bit-identical across ranks, repeated calls
and CUDA-graph replays stay in step, and NCCL-free calls leave the device error word clear.
Each world size is skipped on a machine with fewer GPUs."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank: int, world: int, port: int, queue) -> None:
    import ctypes
    import datetime

    import torch.distributed as dist

    from tropnn_b200 import _native as nat
    from tropnn_b200.distributed import PeerAllReduce

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    device = torch.device("cuda", rank)
    torch.cuda.set_device(device)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=device, timeout=datetime.timedelta(seconds=60))
    peer = None
    try:
        peer = PeerAllReduce(600_000)
        gen = torch.Generator().manual_seed(100 + rank)
        sizes = [524_288, 96, 1, 70_001]
        host = [torch.randn(n, generator=gen) for n in sizes]
        expected_sum = None
        gathered = [None] * world
        dist.all_gather_object(gathered, [h.double() for h in host])
        expected_sum = [sum(g[i] for g in gathered) for i in range(len(sizes))]
        # Eager sum.
        t = [h.to(device) for h in host]
        peer.all_reduce_(t, average=False)
        torch.cuda.synchronize()
        err_sum = max(float((a.cpu().double() - e).abs().max() / e.abs().max()) for a, e in zip(t, expected_sum))
        # Eager average, called twice (epochs advance).
        t2 = [h.to(device) for h in host]
        peer.all_reduce_(t2, average=True)
        t3 = [h.to(device) for h in host]
        peer.all_reduce_(t3, average=True)
        torch.cuda.synchronize()
        err_avg = max(float((a.cpu().double() - e / world).abs().max() / (e / world).abs().max()) for a, e in zip(t3, expected_sum))
        same = all(torch.equal(a, b) for a, b in zip(t2, t3))
        # Captured in a CUDA graph and replayed: every replay reduces the fresh input.
        buf = [h.to(device) for h in host]
        side = torch.cuda.Stream(device)
        side.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(side):
            peer.all_reduce_(buf, average=True)
        torch.cuda.current_stream(device).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            peer.all_reduce_(buf, average=True)
        replay_errs = []
        for _ in range(3):
            for b, h in zip(buf, host):
                b.copy_(h.to(device))
            graph.replay()
            torch.cuda.synchronize()
            replay_errs.append(
                max(float((a.cpu().double() - e / world).abs().max() / (e / world).abs().max()) for a, e in zip(buf, expected_sum))
            )
        del graph
        # The LUT gradient with the average fused into its kernel equals the plain kernel
        # followed by the peer all-reduce (both sum the ranks' local sums in rank order).
        lib = nat.load()
        stream = torch.cuda.current_stream(device).cuda_stream
        T, C, out_f, n = 16, 6, 512, 1000
        lut_gen = torch.Generator().manual_seed(7 + rank)
        g = torch.randn(n, out_f, generator=lut_gen).to(device)
        idx = torch.randint(0, 1 << C, (n, T), generator=lut_gen).to(device)
        plain = torch.empty(T, 1 << C, out_f, device=device)
        nat.check(lib.tropnn_b200_pairwise_lut_grad(g.data_ptr(), n, out_f, idx.data_ptr(), T, C, 0.5, plain.data_ptr(),
                                                    nat.F32, stream), "lut_grad")
        peer.all_reduce_([plain.view(-1)], average=True)
        lut_peer = PeerAllReduce(PeerAllReduce.lut_capacity(T, C, out_f))
        fused_results = []
        for _ in range(3):  # repeated calls advance the slot counters in step
            fused = torch.full_like(plain, float("nan"))
            buffers, w_, r_, cap = lut_peer.raw()
            nat.check(lib.tropnn_b200_pairwise_lut_grad_allreduce(
                g.data_ptr(), n, out_f, idx.data_ptr(), T, C, 0.5, fused.data_ptr(), nat.F32, buffers, w_, r_, cap, 1,
                stream), "lut_grad_allreduce")
            fused_results.append(fused)
        torch.cuda.synchronize()
        fused_same = all(torch.equal(f, plain) for f in fused_results)
        lut_peer.close()
        checksum = sum(float(x.double().sum()) for x in t3) + float(plain.double().sum())
        flag = ctypes.c_int(-1)
        nat.check(nat.load().tropnn_b200_device_error(ctypes.byref(flag)), "device_error")
        queue.put((rank, err_sum, err_avg, same and fused_same, replay_errs, checksum, flag.value))
    finally:
        if peer is not None:
            peer.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3, 4, 8])
def test_peer_allreduce(world: int) -> None:
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    port = _free_port()
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = sorted(queue.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    checksums = set()
    for rank, err_sum, err_avg, same, replay_errs, checksum, flag in results:
        assert err_sum <= 1e-6 and err_avg <= 1e-6, (rank, err_sum, err_avg)
        assert same
        assert max(replay_errs) <= 1e-6
        assert flag == 0
        checksums.add(checksum)
    assert len(checksums) == 1  # bit-identical results on every rank
