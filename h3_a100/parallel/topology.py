"""Replicate x shard placement arithmetic.

Same contract as the reference's ``resolve_hybrid_topology``
(``h3_a100/distributed.py:24-52``): ``shard_size`` must divide the world,
ranks are laid out shard-fastest, and the data-parallel world stays the whole
world (placement never changes the batch).
"""

from __future__ import annotations

import dataclasses


@dataclasses.dataclass(frozen=True)
class HybridTopology:
    world_size: int
    shard_size: int
    replicate_size: int
    replicate_rank: int
    shard_rank: int

    @property
    def shard_group_ranks(self) -> list[int]:
        base = self.replicate_rank * self.shard_size
        return list(range(base, base + self.shard_size))

    @property
    def replicate_group_ranks(self) -> list[int]:
        return [r * self.shard_size + self.shard_rank for r in range(self.replicate_size)]


def resolve_hybrid_topology(world_size: int, rank: int, shard_size: int) -> HybridTopology:
    world_size, rank, shard_size = int(world_size), int(rank), int(shard_size)
    if world_size < 1:
        raise ValueError(f"world_size must be positive, got {world_size}.")
    if not 0 <= rank < world_size:
        raise ValueError(f"rank={rank} is outside world_size={world_size}.")
    if shard_size < 1 or world_size % shard_size:
        raise ValueError(f"shard_size={shard_size} must be positive and divide world_size={world_size}.")
    return HybridTopology(
        world_size=world_size,
        shard_size=shard_size,
        replicate_size=world_size // shard_size,
        replicate_rank=rank // shard_size,
        shard_rank=rank % shard_size,
    )
