"""Interval arithmetic of the event timeline and its Chrome-trace output (CPU)."""

import json

from h3_a100.utils.timeline import StreamTimeline, intersect, merge, total


def test_merge_and_intersect():
    assert merge([(5, 7), (0, 2), (1, 3), (6, 9), (9, 9)]) == [(0, 3), (5, 9)]
    assert intersect([(0, 3), (5, 9)], [(2, 6), (8, 12)]) == [(2, 3), (5, 6), (8, 9)]
    assert total([(0, 3), (5, 9)]) == 7


def test_unions_report_exposed_transfer_time():
    rows = [{"lane": "compute", "name": "fwd", "t0": 0.0, "t1": 10.0},
            {"lane": "compute", "name": "bwd", "t0": 5.0, "t1": 12.0},
            {"lane": "comm", "name": "all_gather", "t0": 8.0, "t1": 15.0},
            {"lane": "h2d", "name": "boundary_h2d", "t0": 20.0, "t1": 22.0}]
    u = StreamTimeline.unions(rows)
    assert u["busy_ms"] == {"compute": 12.0, "comm": 7.0, "h2d": 2.0}
    assert u["overlap_with_compute_ms"] == {"comm": 4.0, "h2d": 0.0}
    assert u["exposed_ms"] == {"comm": 3.0, "h2d": 2.0}
    assert u["span_ms"] == 22.0


def test_chrome_trace_has_one_track_per_lane(tmp_path):
    rows = [{"lane": "compute", "name": "fwd", "t0": 0.0, "t1": 1.5},
            {"lane": "d2h", "name": "boundary_d2h", "t0": 0.5, "t1": 0.75}]
    path = tmp_path / "t.json"
    StreamTimeline.write_chrome_trace(rows, str(path), pid=3)
    trace = json.loads(path.read_text())["traceEvents"]
    spans = [e for e in trace if e["ph"] == "X"]
    assert [(e["name"], e["pid"], e["ts"], e["dur"]) for e in spans] == [("fwd", 3, 0.0, 1500.0),
                                                                           ("boundary_d2h", 3, 500.0, 250.0)]
    names = {e["args"]["name"] for e in trace if e["ph"] == "M"}
    assert {"compute", "d2h"} <= names


def test_disabled_timeline_records_nothing():
    tl = StreamTimeline(enabled=False)
    tl.start_cycle()
    with tl.span("compute", "x"):
        pass
    assert tl.event() is None and tl.collect() == []
