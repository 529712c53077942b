"""Preflight report on a machine without a GPU (the B200 checks are skipped,
the config-derived sizes and the host-RAM check still run)."""

from __future__ import annotations

import json
import os

from h3_a100 import preflight

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_preflight_reports_config_sizes(tmp_path, monkeypatch):
    monkeypatch.setenv("LOCAL_WORLD_SIZE", "8")
    out = tmp_path / "report.json"
    code = preflight.main(["--config", os.path.join(ROOT, "configs", "h3_dmd_b200_world8.yaml"),
                           "--json", str(out)])
    report = json.loads(out.read_text())
    cfg = report["checks"]["config"]
    assert cfg["tokens"] == 37730
    assert cfg["boundary_bytes"] == 405_672_960
    assert abs(cfg["pinned_boundary_gib_per_node"] - 8 * 50 * 405_672_960 / 1024**3) < 0.2
    assert report["checks"]["host_ram_gib"] > 0
    # no extension or GPU is an error only where the kernels are expected to run
    assert code in (0, 1)
    assert isinstance(report["errors"], list) and isinstance(report["warnings"], list)
