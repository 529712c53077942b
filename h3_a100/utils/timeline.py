"""Device timeline of a cycle from CUDA events on every stream (no profiler needed).

The reference's profiling path is ``nsys profile --trace=cuda,nvtx,osrt,nccl``
around the launcher (``scripts/profile_nsys.sh:13-19``) and its policy is to
report compute, collective, H2D and D2H time as separate interval unions
because they overlap (``docs/EXPERIMENT_PLAN.md:68-70``).  Nsight Systems is
not part of this image, and a profiler would also change the timing; this
module records the same four lanes itself:

* ``span(lane, name, stream)`` brackets work with two CUDA events on the
  stream that runs it (the DiT forwards and backwards and the optimizer steps
  on the compute stream, the frozen-weight gathers on the communication
  stream, the boundary copies on the copy stream);
* ``collect()`` resolves every event against one zero event recorded on the
  compute stream when the cycle started (``elapsed_time`` works across the
  streams of one device) and returns the intervals;
* ``unions()`` merges each lane's intervals and reports busy time per lane,
  the time two lanes were busy together, and the compute-idle time during
  which a transfer lane was busy (the exposed transfer time);
* ``write_chrome_trace(path)`` writes the intervals in the Chrome trace-event
  format (load in chrome://tracing or Perfetto), one track per lane.

Recording costs two events per span; it is off unless ``H3_TIMELINE`` names
an output directory (the trainer then writes one trace per rank and cycle).
"""

from __future__ import annotations

import contextlib
import json
import os
from collections import defaultdict
from collections.abc import Iterator

import torch

LANES = ("compute", "comm", "d2h", "h2d")


def merge(intervals: list[tuple[float, float]]) -> list[tuple[float, float]]:
    """Union of [start, end) intervals as a sorted disjoint list."""
    out: list[list[float]] = []
    for a, b in sorted(intervals):
        if b <= a:
            continue
        if out and a <= out[-1][1]:
            out[-1][1] = max(out[-1][1], b)
        else:
            out.append([a, b])
    return [(a, b) for a, b in out]


def total(intervals: list[tuple[float, float]]) -> float:
    return sum(b - a for a, b in intervals)


def intersect(x: list[tuple[float, float]], y: list[tuple[float, float]]) -> list[tuple[float, float]]:
    """Intersection of two disjoint sorted interval lists."""
    out, i, j = [], 0, 0
    while i < len(x) and j < len(y):
        a, b = max(x[i][0], y[j][0]), min(x[i][1], y[j][1])
        if a < b:
            out.append((a, b))
        if x[i][1] < y[j][1]:
            i += 1
        else:
            j += 1
    return out


class StreamTimeline:
    def __init__(self, enabled: bool | None = None, out_dir: str | None = None) -> None:
        out_dir = out_dir if out_dir is not None else os.environ.get("H3_TIMELINE")
        self.out_dir = out_dir
        self.enabled = bool(out_dir) if enabled is None else bool(enabled)
        self.enabled = self.enabled and torch.cuda.is_available()
        self._zero = None
        self._spans: list[tuple[str, str, object, object]] = []

    def start_cycle(self) -> None:
        if not self.enabled:
            return
        self._spans.clear()
        self._zero = torch.cuda.Event(enable_timing=True)
        self._zero.record(torch.cuda.current_stream())

    def _event(self, stream) -> object:
        ev = torch.cuda.Event(enable_timing=True)
        ev.record(stream)
        return ev

    @contextlib.contextmanager
    def span(self, lane: str, name: str, stream=None) -> Iterator[None]:
        if not self.enabled or self._zero is None:
            yield
            return
        stream = stream or torch.cuda.current_stream()
        begin = self._event(stream)
        try:
            yield
        finally:
            self._spans.append((lane, name, begin, self._event(stream)))

    def add(self, lane: str, name: str, begin, end) -> None:
        """Register an interval bracketed by two already-recorded events."""
        if self.enabled and self._zero is not None and begin is not None and end is not None:
            self._spans.append((lane, name, begin, end))

    def event(self, stream=None):
        """A timing event recorded now on ``stream`` (None when the timeline is off)."""
        if not self.enabled or self._zero is None:
            return None
        return self._event(stream or torch.cuda.current_stream())

    def collect(self) -> list[dict]:
        if not self.enabled or self._zero is None:
            return []
        torch.cuda.synchronize()
        zero = self._zero
        rows = [{"lane": lane, "name": name, "t0": zero.elapsed_time(a), "t1": zero.elapsed_time(b)}
                for lane, name, a, b in self._spans]
        self._spans.clear()
        self._zero = None
        return rows

    @staticmethod
    def unions(rows: list[dict]) -> dict:
        """Busy milliseconds per lane, pairwise overlap with compute, and exposed transfer time."""
        by_lane: dict[str, list[tuple[float, float]]] = defaultdict(list)
        for r in rows:
            by_lane[r["lane"]].append((r["t0"], r["t1"]))
        merged = {lane: merge(iv) for lane, iv in by_lane.items()}
        compute = merged.get("compute", [])
        span = (min((a for iv in merged.values() for a, _ in iv), default=0.0),
                max((b for iv in merged.values() for _, b in iv), default=0.0))
        out = {"span_ms": round(span[1] - span[0], 3), "busy_ms": {}, "overlap_with_compute_ms": {},
               "exposed_ms": {}}
        for lane, iv in merged.items():
            busy = total(iv)
            out["busy_ms"][lane] = round(busy, 3)
            if lane != "compute":
                both = total(intersect(iv, compute))
                out["overlap_with_compute_ms"][lane] = round(both, 3)
                out["exposed_ms"][lane] = round(busy - both, 3)
        return out

    @staticmethod
    def write_chrome_trace(rows: list[dict], path: str, pid: int = 0) -> None:
        tids = {lane: i for i, lane in enumerate(LANES)}
        events = [{"name": r["name"], "cat": r["lane"], "ph": "X", "pid": pid,
                   "tid": tids.setdefault(r["lane"], len(tids)), "ts": r["t0"] * 1e3,
                   "dur": max(0.0, r["t1"] - r["t0"]) * 1e3} for r in rows]
        events += [{"name": "thread_name", "ph": "M", "pid": pid, "tid": tid, "args": {"name": lane}}
                   for lane, tid in tids.items()]
        os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
        with open(path, "w") as fh:
            json.dump({"traceEvents": events, "displayTimeUnit": "ms"}, fh)
