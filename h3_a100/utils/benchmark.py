"""Benchmark helpers: GPU clock sampling during the timed region.

``ClockSampler`` runs ``nvidia-smi --query-gpu=... -lms 200`` in the
background while the timed region runs and summarises the SM clock (median
under load, max) and the clock-event reasons that were active, so a number
taken under thermal/hardware slowdown or a leftover clock lock can be
recognised.  It only reads GPU state; it never changes a setting.
"""

from __future__ import annotations

import csv
import io
import os
import shutil
import statistics
import subprocess
import tempfile

QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
REASON_COLUMNS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")


class ClockSampler:
    def __init__(self, gpu_indices: list[int] | None = None, period_ms: int = 200) -> None:
        self.gpu_indices = gpu_indices
        self.period_ms = period_ms
        self._proc = None
        self._file = None

    def start(self) -> None:
        exe = shutil.which("nvidia-smi")
        if exe is None:
            return
        self._file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self._proc = subprocess.Popen(
            [exe, f"--query-gpu={QUERY}", "--format=csv,noheader,nounits", f"-lms={self.period_ms}"],
            stdout=self._file, stderr=subprocess.DEVNULL)

    def stop(self) -> dict:
        if self._proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self._proc.terminate()
        try:
            self._proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self._proc.kill()
        self._file.flush()
        self._file.seek(0)
        text = self._file.read()
        self._file.close()
        os.unlink(self._file.name)
        return summarise(text, self.gpu_indices)


def _num(value: str):
    try:
        return float(value.strip())
    except ValueError:
        return None


def summarise(text: str, gpu_indices: list[int] | None) -> dict:
    rows = [r for r in csv.reader(io.StringIO(text)) if len(r) >= 9]
    clocks, maxes, reasons = [], [], set()
    for r in rows:
        idx = _num(r[0])
        if gpu_indices is not None and idx is not None and int(idx) not in gpu_indices:
            continue
        sm, smax, power = _num(r[1]), _num(r[2]), _num(r[3])
        if smax:
            maxes.append(smax)
        if sm is not None and power is not None and power > 200:   # "under load"
            clocks.append(sm)
        for name, value in zip(REASON_COLUMNS, r[5:9]):
            if value.strip().lower() == "active":
                reasons.add(name)
    return {
        "sm_mhz": statistics.median(clocks) if clocks else None,
        "sm_max_mhz": max(maxes) if maxes else None,
        "reasons": sorted(reasons),
        "samples": len(rows),
        "samples_under_load": len(clocks),
    }
