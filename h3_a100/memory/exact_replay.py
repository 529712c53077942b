"""Exact AdaLN replay audit, run by the checkpoint itself.

Contract kept from the reference (``h3_a100/exact_adaln_replay.py:50-223``):
a grad-enabled block checkpoint may only be created under a complete AdaLN
key, and each execution of the block, the original one and the backward
replay, must read its modulation from that key's cached table exactly once
and never miss (never fall back to the projection).  Per cycle that is
300 checkpoints / 600 executions / 600 hits / 0 misses for 1 Student + 5 Fake
grad forwards of 50 blocks; the stat names are the reference's, since the
cycle receipt is expressed in them.

Mechanism here: the block call carries its key (``call.key``) and the number
of modulation reads one execution makes (``call.fetches``: 1 for a block, the
block count for a checkpoint segment).  ``BlockCheckpointing`` calls
``note_checkpoint`` when it creates a checkpoint and routes every execution
through ``execute``, which hands the call a counting fetch and checks the
counts when the execution returns.  Nothing ambient is captured or restored.
"""

from __future__ import annotations

from typing import Any

import torch

STAT_KEYS = (
    "checkpoint_wrap_count",
    "scoped_execution_count",
    "cache_hit_count",
    "cache_miss_count",
    "captured_key_missing_count",
    "captured_key_incomplete_count",
    "unexpected_hit_delta_count",
)


def expected_cycle_counts(blocks: int, grad_forwards: int = 6, segment_size: int = 1) -> dict[str, int]:
    """Audit counters of one matched cycle (``grad_forwards`` grad DiT forwards)."""
    wraps = grad_forwards * -(-int(blocks) // int(segment_size))
    expected = dict.fromkeys(STAT_KEYS, 0)
    expected.update(checkpoint_wrap_count=wraps, scoped_execution_count=2 * wraps,
                    cache_hit_count=2 * grad_forwards * int(blocks))
    return expected


def cycle_delta(stats: dict[str, int], start: dict[str, int]) -> dict[str, int]:
    return {key: int(stats[key]) - int(start.get(key, 0)) for key in STAT_KEYS}


class ReplayAudit:
    policy = "exact_adaln_checkpoint_replay_scope"

    def __init__(self, cache) -> None:
        self.cache = cache
        self.stats = dict.fromkeys(STAT_KEYS, 0)

    def note_checkpoint(self, call: Any) -> None:
        """A grad checkpoint is being created for ``call``: its key must be cached for every block."""
        key = getattr(call, "key", None)
        if key is None:
            self.stats["captured_key_missing_count"] += 1
            raise RuntimeError("exact AdaLN replay: a block checkpoint was created without an AdaLN key; "
                               "the projection bank is never used as a fallback")
        if not self.cache.complete(key):
            self.stats["captured_key_incomplete_count"] += 1
            raise RuntimeError(f"exact AdaLN replay: key {key!r} has no complete modulation table "
                               "when the checkpoint is created")
        self.stats["checkpoint_wrap_count"] += 1

    def execute(self, call: Any, hidden: torch.Tensor) -> torch.Tensor:
        """Run one execution of ``call`` with counted modulation reads, then check the counts."""
        counts = [0, 0]   # hits, misses
        cache = self.cache

        def fetch(key, block):
            value = cache.fetch(key, block)
            counts[value is None] += 1
            return value

        self.stats["scoped_execution_count"] += 1
        try:
            out = call(hidden, fetch=fetch)
        finally:
            self.stats["cache_hit_count"] += counts[0]
            self.stats["cache_miss_count"] += counts[1]
        hits, misses = counts
        expected = int(getattr(call, "fetches", 1))
        if misses:
            raise RuntimeError(f"exact AdaLN replay miss for key {getattr(call, 'key', None)!r} ({misses} misses)")
        if hits != expected:
            self.stats["unexpected_hit_delta_count"] += 1
            raise RuntimeError(f"exact AdaLN replay expected {expected} modulation read(s) per execution, "
                               f"got {hits} for key {getattr(call, 'key', None)!r}")
        return out

    def receipt(self) -> dict[str, Any]:
        return {"policy": self.policy, "stats": dict(self.stats)}
