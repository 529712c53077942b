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

    def take(self) -> dict[str, float]:
        """Totals since the last ``take`` (resolves pending events), then reset."""
        out = self.collect()
        self.reset()
        return out


def max_over_ranks(values: dict[str, float]) -> dict[str, float]:
    return {k: pdist.all_reduce_max(v) for k, v in sorted(values.items())}


class StallLedger:
    """Device time a stream spends blocked on another stream's event, by kind.

    ``wait(kind, event)`` makes the current stream wait on ``event`` and, on
    CUDA, brackets the wait with two timing events on the waiting stream: the
    first completes when the stream's earlier work is done, the second when
    the awaited event has fired, so their distance is exactly the time the
    stream sat idle waiting (zero when the awaited work finished first).  For
    the communication stream's all-gathers this is the *exposed*
    (non-overlapped) collective time the scaling report asks for.
    """

    def __init__(self) -> None:
        self.cuda = torch.cuda.is_available()
        self._pairs: dict[str, list] = defaultdict(list)
        self.counts: dict[str, int] = defaultdict(int)

    def wait(self, kind: str, event, stream=None) -> None:
        if event is None:
            return
        stream = stream or torch.cuda.current_stream()
        if not self.cuda:
            stream.wait_event(event)
            return
        before = torch.cuda.Event(enable_timing=True)
        after = torch.cuda.Event(enable_timing=True)
        before.record(stream)
        stream.wait_event(event)
        after.record(stream)
        self._pairs[kind].append((before, after))
        self.counts[kind] += 1

    def collect(self) -> dict[str, float]:
        """Milliseconds stalled per kind since the last collect (synchronizes)."""
        if self.cuda and self._pairs:
            torch.cuda.synchronize()
        out = {kind: float(sum(b.elapsed_time(a) for b, a in pairs)) for kind, pairs in self._pairs.items()}
        self._pairs.clear()
        return out
