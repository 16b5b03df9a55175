"""Per-kernel timing for benchmarks.

When a ``KernelTimer`` is active, operators record the duration of each
launch together with its algorithmic FLOPs, in one of two ways:

* conv launches, with ``device_clock=True``: the kernel itself writes the
  device clock (%globaltimer) when its first CTA passes its dependency wait
  and when its last CTA (or the split-K reduce) finishes, into a slot of a
  device table (``ldb_conv_desc.clock``).  Nothing is added to the stream,
  so the timed graph keeps its programmatic-launch overlap.
* every other launch: a pair of CUDA events around it on the launching
  stream.  Events are created with ``external=True`` so the records become
  event nodes when the step is captured in a CUDA graph (they add gaps).

After a replay (``reset()`` before it when device clocks are used),
``summary()`` reads the durations of that replay.
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
    label: str = ""


@dataclass
class _ClockRecord:
    kind: str
    flops: float
    slot: int
    label: str = ""


@dataclass
class KernelTimer:
    records: list[_Record] = field(default_factory=list)
    device_clock: bool = False
    capacity: int = 4096
    clock_records: list[_ClockRecord] = field(default_factory=list)
    _table: torch.Tensor | None = None

    def clock_pointer(self, kind: str, flops: float, device: torch.device, label: str = "") -> int:
        """Address of a fresh (start, end) slot of the device clock table."""
        if self._table is None:
            self._table = torch.zeros((self.capacity, 2), dtype=torch.int64, device=device)
            self.reset()
        slot = len(self.clock_records)
        if slot >= self.capacity:
            raise RuntimeError("device clock table is full")
        self.clock_records.append(_ClockRecord(kind, flops, slot, label))
        return self._table[slot].data_ptr()

    def arm(self, device: torch.device) -> None:
        """Allocate the device clock table now (before a graph capture) and reset it."""
        if self._table is None:
            self._table = torch.zeros((self.capacity, 2), dtype=torch.int64, device=device)
        self.reset()

    def reset(self) -> None:
        """Re-arm the device clock table (start high, end 0) on the current stream."""
        if self._table is not None:
            self._table[:, 0].fill_(2 ** 62)
            self._table[:, 1].zero_()

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

    def launches(self) -> list[tuple[str, str, float, float]]:
        """(kind, label, FLOPs, milliseconds) of every recorded launch of the last replay, in order."""
        out = [(r.kind, r.label, r.flops, r.start.elapsed_time(r.end)) for r in self.records]
        if self.clock_records:
            table = self._table.cpu()
            for r in self.clock_records:
                start, end = (int(v) for v in table[r.slot])
                out.append((r.kind, r.label, r.flops, max(0, end - start) / 1e6))
        return out

    def summary(self) -> dict[str, dict[str, float]]:
        """Per kind: launches, total milliseconds, FLOPs (of the last replay)."""
        out: dict[str, dict[str, float]] = {}
        for r in self.records:
            d = out.setdefault(r.kind, {"launches": 0, "ms": 0.0, "flops": 0.0})
            d["launches"] += 1
            d["ms"] += r.start.elapsed_time(r.end)
            d["flops"] += r.flops
        if self.clock_records:
            table = self._table.cpu()
            for r in self.clock_records:
                start, end = (int(v) for v in table[r.slot])
                d = out.setdefault(r.kind, {"launches": 0, "ms": 0.0, "flops": 0.0})
                d["launches"] += 1
                d["ms"] += max(0, end - start) / 1e6
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


def device_clock(kind: str, flops: float, device: torch.device, label: str = "") -> int | None:
    """Clock-slot address for a launch that records its own device clock, or None."""
    timer = _ACTIVE
    if timer is None or not timer.device_clock:
        return None
    return timer.clock_pointer(kind, flops, device, label)


@contextlib.contextmanager
def maybe_time(kind: str, flops: float, *, device_clocked: bool = False):
    timer = _ACTIVE
    if timer is None or device_clocked:
        yield
    else:
        with timer.time(kind, flops):
            yield
