"""Per-launch CUDA-event tracing of the b200 kernels.

Inside ``with launch_trace() as tr:`` every native entry point called by the b200 ops is
bracketed by a pair of CUDA events recorded on the stream the kernel is launched on
(the current torch stream). The trace is process-wide, because autograd runs the CUDA
backward on its own thread. Under CUDA-graph capture the events are recorded as
external event nodes, so every replay re-records them and the durations are pure
device time (no host gaps); call ``tr.harvest()`` after each replay has synchronised.
Outside a trace the ops record nothing.
"""

from __future__ import annotations

import contextlib
import threading
from dataclasses import dataclass, field

import torch


@dataclass
class _Record:
    name: str
    start: torch.cuda.Event
    end: torch.cuda.Event


@dataclass
class LaunchTrace:
    records: list[_Record] = field(default_factory=list)
    totals_ms: dict[str, float] = field(default_factory=dict)
    counts: dict[str, int] = field(default_factory=dict)
    _lock: threading.Lock = field(default_factory=threading.Lock)

    def begin(self, name: str) -> _Record:
        external = torch.cuda.is_current_stream_capturing()
        rec = _Record(
            name,
            torch.cuda.Event(enable_timing=True, external=external),
            torch.cuda.Event(enable_timing=True, external=external),
        )
        rec.start.record()
        return rec

    def end(self, rec: _Record) -> None:
        rec.end.record()
        with self._lock:
            self.records.append(rec)

    def harvest(self) -> None:
        """Adds the durations of the currently recorded events to the totals (synchronises).
        Eager traces call it once at the end; graph traces after every replay."""
        torch.cuda.synchronize()
        with self._lock:
            for rec in self.records:
                self.totals_ms[rec.name] = self.totals_ms.get(rec.name, 0.0) + rec.start.elapsed_time(rec.end)
                self.counts[rec.name] = self.counts.get(rec.name, 0) + 1

    def clear_records(self) -> None:
        with self._lock:
            self.records.clear()

    @property
    def launches(self) -> int:
        return sum(self.counts.values())

    def summary(self) -> dict[str, dict[str, float]]:
        """{name: {"launches": n, "total_ms": t, "mean_ms": t / n}} over harvested launches."""
        return {
            name: {"launches": self.counts[name], "total_ms": total, "mean_ms": total / self.counts[name]}
            for name, total in self.totals_ms.items()
        }


_lock = threading.Lock()
_active: LaunchTrace | None = None


def current() -> LaunchTrace | None:
    return _active


@contextlib.contextmanager
def launch_trace():
    global _active
    trace = LaunchTrace()
    with _lock:
        previous, _active = _active, trace
    try:
        yield trace
    finally:
        with _lock:
            _active = previous
