"""Per-launch CUDA-event tracing of the b200 kernels.

Inside ``with launch_trace() as tr:`` every native entry point called by the b200 ops is
bracketed by a pair of CUDA events recorded on the stream the kernel is launched on
(the current torch stream). ``tr.summary()`` then gives, per kernel entry point, the
launch count and the mean device duration. Outside a trace the ops record nothing.
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

    def begin(self, name: str) -> _Record:
        rec = _Record(name, torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        rec.start.record()
        return rec

    def end(self, rec: _Record) -> None:
        rec.end.record()
        self.records.append(rec)

    @property
    def launches(self) -> int:
        return len(self.records)

    def summary(self) -> dict[str, dict[str, float]]:
        """{name: {"launches": n, "total_ms": t, "mean_ms": t/n}} (synchronises)."""
        torch.cuda.synchronize()
        out: dict[str, dict[str, float]] = {}
        for rec in self.records:
            item = out.setdefault(rec.name, {"launches": 0, "total_ms": 0.0})
            item["launches"] += 1
            item["total_ms"] += rec.start.elapsed_time(rec.end)
        for item in out.values():
            item["mean_ms"] = item["total_ms"] / item["launches"]
        return out


_state = threading.local()


def current() -> LaunchTrace | None:
    return getattr(_state, "trace", None)


@contextlib.contextmanager
def launch_trace():
    previous = current()
    trace = LaunchTrace()
    _state.trace = trace
    try:
        yield trace
    finally:
        _state.trace = previous
