"""Multi-block checkpoint segments (diagnostic selective checkpointing).

Parity with the reference's ``_H3CheckpointSegment`` /
``configure_activation_checkpoint_segments`` (``h3_a100/model.py:40-75,
235-269``): ``segment_size`` consecutive blocks form one checkpoint call, so
one boundary is saved per segment instead of per block.  The production
boundary-staging policy requires ``segment_size == 1`` (the trainer rejects
the combination, as the reference does at ``h3_a100/trainer.py:123-128``).

Blocks here carry their replay context in the call object, so a segment is a
plain composition of block calls; nothing ambient must be restored at replay.
"""

from __future__ import annotations

from typing import Any, Callable


class SegmentCall:
    """One checkpointed callable that runs several block calls in order."""

    def __init__(self, calls: list[Callable[[Any], Any]], start: int) -> None:
        if not calls:
            raise ValueError("an activation-checkpoint segment cannot be empty")
        self.calls = list(calls)
        self.start = int(start)

    def __call__(self, hidden):
        for call in self.calls:
            hidden = call(hidden)
        return hidden


def group_calls(calls: list[Callable[[Any], Any]], segment_size: int) -> list[SegmentCall]:
    segment_size = int(segment_size)
    if segment_size < 1:
        raise ValueError(f"activation checkpoint segment_size must be >= 1, got {segment_size}")
    return [SegmentCall(calls[i:i + segment_size], i) for i in range(0, len(calls), segment_size)]
