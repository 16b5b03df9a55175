"""Per-kernel CUDA-event timing for benchmarks.

When a ``KernelTimer`` is active, the conv and attention operators record
a pair of CUDA events around their launch on the launching stream, together
with the launch's algorithmic FLOPs.  Events are created with
``external=True`` so the records become event nodes when the step is
captured in a CUDA graph; after a replay, ``summary()`` reads the durations
of that replay.
"""

from __future__ import annotations

import contextlib
from dataclasses import dataclass, field

import torch

_ACTIVE: "KernelTimer | None" = None


@dataclass
class _Record:
    kind: str
    flops: float
    start: torch.cuda.Event
    end: torch.cuda.Event


@dataclass
class KernelTimer:
    records: list[_Record] = field(default_factory=list)

    @contextlib.contextmanager
    def time(self, kind: str, flops: float):
        start = torch.cuda.Event(enable_timing=True, external=True)
        end = torch.cuda.Event(enable_timing=True, external=True)
        start.record()
        try:
            yield
        finally:
            end.record()
            self.records.append(_Record(kind, flops, start, end))

    def summary(self) -> dict[str, dict[str, float]]:
        """Per kind: launches, total milliseconds, FLOPs (of the last replay)."""
        out: dict[str, dict[str, float]] = {}
        for r in self.records:
            d = out.setdefault(r.kind, {"launches": 0, "ms": 0.0, "flops": 0.0})
            d["launches"] += 1
            d["ms"] += r.start.elapsed_time(r.end)
            d["flops"] += r.flops
        return out


def active() -> KernelTimer | None:
    return _ACTIVE


@contextlib.contextmanager
def timing(timer: KernelTimer):
    """Activate ``timer`` for operators called inside the block."""
    global _ACTIVE
    previous = _ACTIVE
    _ACTIVE = timer
    try:
        yield timer
    finally:
        _ACTIVE = previous


@contextlib.contextmanager
def maybe_time(kind: str, flops: float):
    timer = _ACTIVE
    if timer is None:
        yield
    else:
        with timer.time(kind, flops):
            yield
