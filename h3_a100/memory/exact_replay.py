"""Exact AdaLN replay audit around the checkpoint function.

Same contract as the reference (``h3_a100/exact_adaln_replay.py:50-223``):
the outermost checkpoint wrapper captures the active AdaLN key when a block's
checkpoint is created (it must exist and be complete for every block), enters
that key around the original execution *and* the backward replay, and
requires each execution to take exactly one cache hit and no miss.  Per cycle
the trainer checks 300 wraps / 600 scoped executions / 600 hits / 0 misses
(1 Student + 5 Fake grad forwards x 50 blocks).

Chain installed by the trainer:
``exact AdaLN scope -> boundary staging -> native checkpoint``.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Callable

from ..models.adaln import AdaLNCacheController

EXPECTED_CYCLE_COUNTS = {
    "checkpoint_wrap_count": 300,
    "scoped_execution_count": 600,
    "cache_hit_count": 600,
    "cache_miss_count": 0,
    "captured_key_missing_count": 0,
    "captured_key_incomplete_count": 0,
    "unexpected_hit_delta_count": 0,
}


def expected_cycle_counts(blocks: int, grad_forwards: int = 6) -> dict[str, int]:
    wraps = blocks * grad_forwards
    return {**EXPECTED_CYCLE_COUNTS, "checkpoint_wrap_count": wraps,
            "scoped_execution_count": 2 * wraps, "cache_hit_count": 2 * wraps}


@dataclass
class ExactAdaLNReplayRegistration:
    transformer: Any
    controller: AdaLNCacheController
    original_checkpoint: Callable[..., Any]
    stats: dict[str, int]
    closed: bool = False

    def receipt(self) -> dict[str, Any]:
        return {"policy": "exact_adaln_checkpoint_replay_scope", "stats": dict(self.stats), "closed": self.closed}

    def remove(self) -> None:
        if not self.closed:
            self.transformer._gradient_checkpointing_func = self.original_checkpoint
            self.closed = True


def install_exact_adaln_checkpoint_replay_scope(
    transformer: Any, controller: AdaLNCacheController, *, expected_block_count: int = 50
) -> ExactAdaLNReplayRegistration:
    original = getattr(transformer, "_gradient_checkpointing_func", None)
    if not callable(original):
        raise RuntimeError("transformer has no callable checkpoint function")
    if not bool(getattr(transformer, "gradient_checkpointing", False)):
        raise RuntimeError("exact AdaLN replay scope requires gradient checkpointing")
    stats = {key: 0 for key in EXPECTED_CYCLE_COUNTS}

    def wrapped(function: Callable[..., Any], *args: Any, **kwargs: Any) -> Any:
        active = controller.current_scope()
        key = active.key
        if key is None:
            stats["captured_key_missing_count"] += 1
            raise RuntimeError(
                "Exact AdaLN checkpoint replay has no active cache key; "
                "refusing to fall back to the AdaLN projection bank."
            )
        if not controller.has_complete_key(key, expected_block_count):
            stats["captured_key_incomplete_count"] += 1
            raise RuntimeError(f"Exact AdaLN cache key {key!r} is incomplete before checkpoint creation")
        persistent = bool(active.persistent)
        stats["checkpoint_wrap_count"] += 1

        def scoped(*fn_args: Any, **fn_kwargs: Any) -> Any:
            before = controller.stats()
            stats["scoped_execution_count"] += 1
            try:
                with controller.scope(key, persistent=persistent):
                    return function(*fn_args, **fn_kwargs)
            finally:
                after = controller.stats()
                hits, misses = after.hits - before.hits, after.misses - before.misses
                stats["cache_hit_count"] += hits
                stats["cache_miss_count"] += misses
                if misses != 0:
                    raise RuntimeError(f"Exact AdaLN replay cache miss for key={key!r}; miss_delta={misses}")
                if hits != 1:
                    stats["unexpected_hit_delta_count"] += 1
                    raise RuntimeError(f"Exact AdaLN replay expected one cache hit per block, got {hits} for key={key!r}")

        return original(scoped, *args, **kwargs)

    transformer._gradient_checkpointing_func = wrapped
    return ExactAdaLNReplayRegistration(transformer, controller, original, stats)


def cycle_delta(stats: dict[str, int], start: dict[str, int]) -> dict[str, int]:
    return {key: int(stats[key]) - int(start.get(key, 0)) for key in EXPECTED_CYCLE_COUNTS}
