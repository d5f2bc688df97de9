"""One-process-per-GPU data parallelism for the b200 layers.

The reference is single-device (no collective anywhere). Rows of a routed layer are
independent in forward and backward, so the layers scale by batch-row sharding: rank r
of W takes rows [r*N/W, (r+1)*N/W), keeps a full parameter replica, and after the
backward the parameter gradients are summed across ranks (NCCL all-reduce over
NVLink/NVSwitch for ``backend="nccl"``, gloo on CPU for tests) and divided by W, so
every rank holds the gradient of the global-batch mean loss.

Gradients are packed into flat buckets per dtype (``bucket_bytes`` each) so that a
layer with many small tensors costs a few collectives, while a large LUT gradient is
reduced in slices that can overlap with other work on the communication stream.
"""

from __future__ import annotations

import contextlib
import ctypes
import threading
from collections.abc import Iterable, Iterator, Sequence

import torch
import torch.distributed as dist
from torch import Tensor

__all__ = [
    "PeerAllReduce",
    "allreduce_gradients",
    "fused_lut_allreduce",
    "overlapped_gradient_sync",
    "row_range",
    "shard_rows",
]

DEFAULT_BUCKET_BYTES = 64 * 1024 * 1024


def row_range(rows: int, rank: int, world_size: int) -> tuple[int, int]:
    """Contiguous [start, stop) of ``rows`` owned by ``rank`` (balanced to within one row)."""
    if world_size < 1 or not 0 <= rank < world_size:
        raise ValueError(f"bad rank {rank} for world size {world_size}")
    base, extra = divmod(rows, world_size)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard_rows(t: Tensor, rank: int, world_size: int) -> Tensor:
    """This rank's row shard of ``t`` (rows along dim 0)."""
    start, stop = row_range(t.shape[0], rank, world_size)
    return t[start:stop]


_REDUCED_ATTR = "_tropnn_b200_reduced"


class _OverlapState:
    """Process-wide switch read by the b200 backward (the autograd engine runs backward on
    its own thread, so a thread-local would not be seen there)."""

    def __init__(self) -> None:
        self.active = False
        self.group: dist.ProcessGroup | None = None
        self.peer: PeerAllReduce | None = None
        self.lock = threading.Lock()
        self.streams: dict[torch.device, torch.cuda.Stream] = {}
        self.lut_peer: PeerAllReduce | None = None


_overlap = _OverlapState()


@contextlib.contextmanager
def fused_lut_allreduce(peer: "PeerAllReduce") -> Iterator[None]:
    """Within this context the b200 PairwiseLinear backward computes its LUT gradient with the
    all-reduce over ``peer``'s NVLink buffers fused into the same kernel
    (tropnn_b200_pairwise_lut_grad_allreduce: each block is pushed to every rank as soon as it
    is summed), averaging across ``peer``'s group, and marks it reduced so that
    ``allreduce_gradients`` skips it. ``peer`` must be a set of its own (sized with
    ``PeerAllReduce.lut_capacity``); layers it cannot take fall back to the regular path."""
    with _overlap.lock:
        prev = _overlap.lut_peer
        _overlap.lut_peer = peer
    try:
        yield
    finally:
        with _overlap.lock:
            _overlap.lut_peer = prev


def fused_lut_peer() -> "PeerAllReduce | None":
    """The peer set of an active ``fused_lut_allreduce`` context (None outside it)."""
    return _overlap.lut_peer


def mark_reduced(grad: Tensor) -> None:
    """Marks ``grad`` as already averaged across the group (``allreduce_gradients`` skips it once)."""
    setattr(grad, _REDUCED_ATTR, True)


@contextlib.contextmanager
def overlapped_gradient_sync(
    group: dist.ProcessGroup | None = None, *, peer: "PeerAllReduce | None" = None
) -> Iterator[None]:
    """Within this context the b200 PairwiseLinear backward averages its parameter gradients
    across ``group`` itself: the LUT gradient's all-reduce is enqueued on a side stream as soon
    as the LUT gradient is written and overlaps the straight-through kernels that follow; the
    (small) threshold gradient is reduced after them. With ``peer`` (built on the same group),
    gradients it accepts go through the NVLink peer-memory kernel, the rest through the
    group's backend. Gradients reduced this way are marked, and ``allreduce_gradients`` skips
    them. Assumes one backward per parameter per step."""
    with _overlap.lock:
        prev = (_overlap.active, _overlap.group, _overlap.peer)
        _overlap.active, _overlap.group, _overlap.peer = True, group, peer
    try:
        yield
    finally:
        with _overlap.lock:
            _overlap.active, _overlap.group, _overlap.peer = prev


def _overlap_enabled() -> bool:
    return _overlap.active and dist.is_available() and dist.is_initialized() and dist.get_world_size(_overlap.group) > 1


def _average_op(group: dist.ProcessGroup | None) -> tuple[dist.ReduceOp, bool]:
    """(op, divide afterwards): NCCL averages inside the collective, other backends sum."""
    if dist.get_backend(group) == "nccl":
        return dist.ReduceOp.AVG, False
    return dist.ReduceOp.SUM, True


def begin_gradient_reduce(grad: Tensor) -> torch.cuda.Stream | None:
    """Starts averaging ``grad`` across the overlap group on a side stream (no-op outside
    ``overlapped_gradient_sync``). Returns the stream to hand to ``end_gradient_reduce``."""
    if not _overlap_enabled():
        return None
    device = grad.device
    side = _overlap.streams.get(device)
    if side is None:
        side = _overlap.streams.setdefault(device, torch.cuda.Stream(device))
    current = torch.cuda.current_stream(device)
    side.wait_stream(current)
    with torch.cuda.stream(side):
        _average_in_place(grad)
    if not torch.cuda.is_current_stream_capturing():
        grad.record_stream(side)  # eager: keep the block alive until the side stream is done
    setattr(grad, _REDUCED_ATTR, True)
    return side


def end_gradient_reduce(side: torch.cuda.Stream | None, device: torch.device) -> None:
    """Makes the current stream wait for a reduction started by ``begin_gradient_reduce``."""
    if side is not None:
        torch.cuda.current_stream(device).wait_stream(side)


def reduce_gradient_now(grad: Tensor) -> None:
    """Averages ``grad`` across the overlap group on the current stream (no-op outside
    ``overlapped_gradient_sync``). Call it after ``end_gradient_reduce`` of any pending
    reduction: reductions through one ``PeerAllReduce`` must not run concurrently."""
    if not _overlap_enabled():
        return
    _average_in_place(grad)
    setattr(grad, _REDUCED_ATTR, True)


def _average_in_place(grad: Tensor) -> None:
    """Averages ``grad`` across the overlap group on the current stream."""
    peer = _overlap.peer
    if peer is not None and peer.accepts([grad]):
        peer.all_reduce_([grad], average=True)
        return
    op, divide = _average_op(_overlap.group)
    dist.all_reduce(grad, op=op, group=_overlap.group)
    if divide:
        grad.div_(dist.get_world_size(_overlap.group))


class PeerAllReduce:
    """All-reduce of f32 gradients over NVLink peer memory for one process group on one
    node (tropnn_b200_peer_allreduce_f32): every rank allocates one peer buffer (16
    receive areas of ``capacity`` floats), the ranks exchange its CUDA IPC handle, and each
    call is one kernel per rank: on two ranks it pushes its tensors into every rank's buffer
    and sums the received copies after one flag barrier; on more it reduce-scatters and
    all-gathers by pushes around two flag barriers. For
    the few-MiB gradients of the benchmark layers it replaces NCCL's latency-bound
    protocol (~22 us for 2 MiB on two B200s). Collective: every rank must construct it
    and call it in the same order; call ``close`` on every rank before
    ``destroy_process_group``.
    """

    def __init__(self, capacity: int, *, group: dist.ProcessGroup | None = None) -> None:
        from . import _native as nat

        self._nat = nat
        self._lib = nat.load()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > self.max_ranks():
            raise ValueError(f"PeerAllReduce supports at most {self.max_ranks()} ranks, got {self.world}")
        self.capacity = max(64, (int(capacity) + 63) // 64 * 64)
        local = ctypes.c_void_p()
        handle = (ctypes.c_ubyte * 64)()
        nat.check(self._lib.tropnn_b200_peer_buffer_create(self.capacity, ctypes.byref(local), handle), "peer_buffer_create")
        self._local = local.value
        handles: list[bytes | None] = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        pointers: list[int] = []
        self._opened: list[int] = []
        for peer, h in enumerate(handles):
            if peer == self.rank:
                pointers.append(self._local)
                continue
            ptr = ctypes.c_void_p()
            raw = (ctypes.c_ubyte * 64).from_buffer_copy(h)
            nat.check(self._lib.tropnn_b200_peer_buffer_open(raw, ctypes.byref(ptr)), "peer_buffer_open")
            pointers.append(ptr.value)
            self._opened.append(ptr.value)
        self._buffers = (ctypes.c_void_p * self.world)(*pointers)
        dist.barrier(group=group)

    @staticmethod
    def max_ranks() -> int:
        return 8

    @staticmethod
    def lut_capacity(tables: int, comparisons: int, out_features: int) -> int:
        """Floats a set needs for the fused LUT-gradient all-reduce of a PairwiseLinear layer
        (-1 when the fused kernel does not take the shape)."""
        from . import _native as nat

        return int(nat.load().tropnn_b200_pairwise_lut_grad_peer_floats(tables, comparisons, out_features))

    def raw(self) -> tuple[ctypes.Array, int, int, int]:
        """(buffer pointer array, world, rank, capacity) for the library's fused kernels."""
        return self._buffers, self.world, self.rank, self.capacity

    def accepts(self, tensors: Sequence[Tensor]) -> bool:
        """Whether one call can reduce ``tensors`` (f32, contiguous, on this GPU, fitting)."""
        return (
            0 < len(tensors) <= 8
            and all(t.is_cuda and t.dtype == torch.float32 and t.is_contiguous() for t in tensors)
            and sum(t.numel() for t in tensors) <= self.capacity
        )

    def all_reduce_(self, tensors: Sequence[Tensor], *, average: bool = True) -> None:
        """Sums (averages) ``tensors`` in place across the group; stream-ordered on the
        current stream (capturable in a CUDA graph)."""
        if not self.accepts(tensors):
            raise ValueError("PeerAllReduce.all_reduce_: needs 1-8 contiguous f32 CUDA tensors within the capacity")
        n = len(tensors)
        segments = (ctypes.c_void_p * n)(*[t.data_ptr() for t in tensors])
        counts = (ctypes.c_int64 * n)(*[t.numel() for t in tensors])
        stream = self._nat.stream_handle(tensors[0].device)
        self._nat.check(
            self._lib.tropnn_b200_peer_allreduce_f32(
                self._buffers, self.world, self.rank, self.capacity, segments, counts, n, int(average), stream
            ),
            "peer_allreduce",
        )

    def close(self) -> None:
        """Unmaps the peers' buffers and frees this rank's (collective)."""
        if self._local is None:
            return
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        for ptr in self._opened:
            self._nat.check(self._lib.tropnn_b200_peer_buffer_close(ctypes.c_void_p(ptr)), "peer_buffer_close")
        self._opened = []
        dist.barrier(group=self.group)
        self._nat.check(self._lib.tropnn_b200_peer_buffer_destroy(ctypes.c_void_p(self._local)), "peer_buffer_destroy")
        self._local = None


def _buckets(grads: list[Tensor], bucket_bytes: int) -> list[list[Tensor]]:
    by_dtype: dict[torch.dtype, list[Tensor]] = {}
    for g in grads:
        by_dtype.setdefault(g.dtype, []).append(g)
    out: list[list[Tensor]] = []
    for group in by_dtype.values():
        current: list[Tensor] = []
        size = 0
        for g in group:
            nbytes = g.numel() * g.element_size()
            if current and size + nbytes > bucket_bytes:
                out.append(current)
                current, size = [], 0
            current.append(g)
            size += nbytes
        if current:
            out.append(current)
    return out


def allreduce_gradients(
    params: Iterable[torch.nn.Parameter] | torch.nn.Module,
    *,
    group: dist.ProcessGroup | None = None,
    average: bool = True,
    bucket_bytes: int = DEFAULT_BUCKET_BYTES,
    peer: PeerAllReduce | None = None,
) -> int:
    """Sums (and by default averages) ``.grad`` of ``params`` across the process group.

    Parameters without a gradient are skipped on every rank alike (the set must match
    across ranks, as it does for replicas stepping the same layers). With ``peer`` and
    gradients it accepts, one NVLink peer-memory all-reduce does all of them; otherwise
    NCCL (or the group's backend) reduces dtype buckets, a single tensor larger than
    ``bucket_bytes`` in slices of that size. Returns the number of collectives issued.
    """
    if isinstance(params, torch.nn.Module):
        params = params.parameters()
    grads = []
    for p in params:
        if p.grad is None:
            continue
        if getattr(p.grad, _REDUCED_ATTR, False):
            # Already averaged inside the backward (overlapped_gradient_sync).
            setattr(p.grad, _REDUCED_ATTR, False)
            continue
        grads.append(p.grad)
    if not grads:
        return 0
    world = dist.get_world_size(group)
    if world == 1:
        return 0
    if peer is not None and peer.accepts(grads):
        peer.all_reduce_(grads, average=average)
        return 1
    # NCCL averages inside the collective (ncclAvg); other backends sum, then divide.
    fused_avg = average and dist.get_backend(group) == "nccl"
    op = dist.ReduceOp.AVG if fused_avg else dist.ReduceOp.SUM
    divide = average and not fused_avg
    calls = 0
    for bucket in _buckets(grads, bucket_bytes):
        if len(bucket) == 1:
            flat = bucket[0].view(-1)
            step = max(1, bucket_bytes // flat.element_size())
            for start in range(0, flat.numel(), step):
                piece = flat[start : start + step]
                dist.all_reduce(piece, op=op, group=group)
                calls += 1
                if divide:
                    piece.div_(world)
            continue
        flat = torch.cat([g.reshape(-1) for g in bucket])
        dist.all_reduce(flat, op=op, group=group)
        calls += 1
        if divide:
            flat.div_(world)
        offset = 0
        for g in bucket:
            n = g.numel()
            g.copy_(flat[offset : offset + n].view_as(g))
            offset += n
    return calls
