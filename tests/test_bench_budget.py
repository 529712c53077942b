"""bench.py's wall budget and its reference-arm contract (CPU).

A matched cycle takes minutes, so ``bench.py`` plans how many timed cycles fit
in its budget after the mandatory warm-up; the whole process must stay under
the caller's limit (1,800 s for the 1-GPU bench, 870 s per world size for the
scaling run) and still report at least one timed cycle.
"""

from __future__ import annotations

import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def test_plan_keeps_at_least_one_cycle_and_never_more_than_requested():
    assert bench.plan_timed_cycles(20, 820.0, 900.0, 150.0) == 1      # out of budget: still one cycle
    assert bench.plan_timed_cycles(1, 820.0, 100.0, 10.0) == 1        # never more than asked for
    assert bench.plan_timed_cycles(0, 820.0, 100.0, 10.0) == 0        # nothing asked, nothing run
    assert bench.plan_timed_cycles(20, 820.0, 100.0, 0.0) == 20


@pytest.mark.parametrize("setup_s,cycle_s,limit_s", [(40.0, 137.2, 870.0), (90.0, 145.3, 870.0),
                                                     (40.0, 137.2, 1800.0), (120.0, 150.0, 870.0)])
def test_driver_command_fits_its_limit(setup_s, cycle_s, limit_s):
    """--steps 20 --warmup 5 at the headline cycle time: 3 warm-up cycles, then
    the planned timed cycles, end (with the teardown reserve) inside both the
    default budget and the caller's limit."""
    budget = bench.DEFAULT_BUDGET_S
    warm = bench.MIN_WARMUP
    elapsed = setup_s + warm * cycle_s
    steps = bench.plan_timed_cycles(20, budget, elapsed, cycle_s * bench.CYCLE_SAFETY)
    assert steps >= 1
    end = elapsed + steps * cycle_s + bench.TEARDOWN_RESERVE_S
    assert end <= budget + 1e-6 or steps == 1
    assert end <= limit_s


def test_reference_arm_prints_one_line_and_exits_zero(tmp_path):
    proc = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference"],
                          capture_output=True, text=True, timeout=600, cwd=tmp_path)
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = [ln for ln in proc.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert line["impl"] == "reference" and "unavailable" in line
