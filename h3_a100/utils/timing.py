"""Device timers: CUDA events on the compute stream, reduced as max over ranks.

The reference timed its headline with rank-0 log timestamps; the metric here
is device time between two events bracketing the work, after a barrier and a
synchronize on both sides, taken as the maximum over ranks.
"""

from __future__ import annotations

import time
from collections import defaultdict

import torch

from ..parallel import distributed as pdist


class PhaseTimer:
    """Accumulates per-phase device milliseconds with CUDA events (wall time on CPU)."""

    def __init__(self, enabled: bool = True) -> None:
        self.enabled = enabled
        self.cuda = torch.cuda.is_available()
        self._open: dict[str, object] = {}
        self._events: dict[str, list] = defaultdict(list)
        self.totals_ms: dict[str, float] = defaultdict(float)

    def start(self, name: str) -> None:
        if not self.enabled:
            return
        if self.cuda:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self._open[name] = ev
        else:
            self._open[name] = time.perf_counter()

    def stop(self, name: str) -> None:
        if not self.enabled or name not in self._open:
            return
        begin = self._open.pop(name)
        if self.cuda:
            end = torch.cuda.Event(enable_timing=True)
            end.record()
            self._events[name].append((begin, end))
        else:
            self.totals_ms[name] += (time.perf_counter() - begin) * 1e3

    def collect(self) -> dict[str, float]:
        """Resolve pending events (synchronizes) and return totals."""
        if self.cuda:
            torch.cuda.synchronize()
            for name, pairs in self._events.items():
                self.totals_ms[name] += sum(b.elapsed_time(e) for b, e in pairs)
            self._events.clear()
        return dict(self.totals_ms)

    def reset(self) -> None:
        self._open.clear()
        self._events.clear()
        self.totals_ms.clear()


def max_over_ranks(values: dict[str, float]) -> dict[str, float]:
    return {k: pdist.all_reduce_max(v) for k, v in sorted(values.items())}
