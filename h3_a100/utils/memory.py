"""CUDA memory logging and opt-in residency attribution.

``log_cuda_memory`` mirrors the reference's per-stage allocated / reserved /
peak lines (``h3_a100/trainer_loop.py:318-327``); ``ResidencyLogger`` mirrors
``H3_MEMORY_ATTRIBUTION`` (``:329-405``): allocator stats, free/total device
memory, parameter bytes by class, optimizer-state bytes, AdaLN cache bytes and
boundary counters, emitted at named stages without synchronizing.

``BlockResidencyProbe`` is the per-block attribution of
``H3_MEMORY_ATTRIBUTION_BLOCKS`` (``h3_a100/trainer.py:246-267``): the DiT
calls it around every joint block (``H3DiT.block_probe``), and it logs the
allocated bytes before and after the block and the change, tagged with the
block index and whether the block ran with grad (original forward) or inside
a backward replay.
"""

from __future__ import annotations

import os

import torch

from ..config import env_flag
from .log import logger


def log_cuda_memory(stage: str) -> dict[str, float]:
    if not torch.cuda.is_available():
        return {}
    gib = 1024**3
    out = {
        "allocated_gib": torch.cuda.memory_allocated() / gib,
        "reserved_gib": torch.cuda.memory_reserved() / gib,
        "peak_gib": torch.cuda.max_memory_allocated() / gib,
    }
    logger.info("[h3-a100][memory] stage={} allocated_gib={:.2f} reserved_gib={:.2f} peak_gib={:.2f}",
                stage, out["allocated_gib"], out["reserved_gib"], out["peak_gib"])
    return out


class ResidencyLogger:
    def __init__(self, trainer) -> None:
        self.trainer = trainer
        self.enabled = env_flag("H3_MEMORY_ATTRIBUTION", False) and torch.cuda.is_available()
        self.path = os.environ.get("H3_MEMORY_ATTRIBUTION_FILE")

    def __call__(self, stage: str) -> None:
        if not self.enabled:
            return
        t = self.trainer
        stats = torch.cuda.memory_stats()
        free, total = torch.cuda.mem_get_info()
        cache = t.model.adaln_cache().stats().bytes if t.model is not None else 0
        params = t.model.memory_report() if t.model is not None else {}
        opt = {role: o.state_bytes() for role, o in getattr(t, "optimizers", {}).items()}
        boundary = {}
        reg = getattr(t, "boundary_staging", None)
        if reg is not None:
            boundary = {k: int(reg.stats.get(k, 0)) for k in (
                "cpu_copy_count", "restore_count", "offloaded_logical_bytes", "offloaded_storage_bytes")}
        logger.info("[h3-a100][residency] stage={} allocated={} reserved={} active={} inactive_split={} free={} "
                    "total={} params={} opt={} adaln_cache={} boundary={}", stage, torch.cuda.memory_allocated(),
                    torch.cuda.memory_reserved(), int(stats.get("active_bytes.all.current", 0)),
                    int(stats.get("inactive_split_bytes.all.current", 0)), free, total, params, opt, cache, boundary)


class BlockResidencyProbe:
    """Per-block allocated-memory attribution (opt-in, ``H3_MEMORY_ATTRIBUTION_BLOCKS=1``)."""

    def __init__(self) -> None:
        self.enabled = env_flag("H3_MEMORY_ATTRIBUTION_BLOCKS", False) and torch.cuda.is_available()
        self._before: dict[int, int] = {}
        self.records: list[dict] = []

    def __call__(self, index: int, where: str) -> None:
        if not self.enabled:
            return
        now = torch.cuda.memory_allocated()
        if where == "before":
            self._before[index] = now
            return
        before = self._before.pop(index, now)
        record = {"block": index, "grad": torch.is_grad_enabled(), "allocated_before": before,
                  "allocated_after": now, "delta": now - before,
                  "peak": torch.cuda.max_memory_allocated()}
        self.records.append(record)
        logger.info("[h3-a100][residency-block] block={} grad={} before={} after={} delta={} peak={}",
                    index, record["grad"], before, now, record["delta"], record["peak"])
