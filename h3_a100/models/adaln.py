"""AdaLN modulation tables: the projection bank and an exact per-key cache.

What the reference does (``h3_a100/adaln_cache.py:51-268``,
``h3_a100/model.py:346-365``): every block's frozen ~260 M-parameter AdaLN
projection is moved into one bank so each projection can be its own sharded
unit, and block modulations are precomputed once per exact timestep table
and replayed: ``("rollout", i)`` keys persist for the whole run,
``("score", n)`` keys are dynamic, bounded, and dropped after use.  Stats
(hits / misses / stores / evictions / key kinds / bytes) are logged per cycle.

How this package does it:

* **The DiT owns the bank from construction** (``H3DiT.adaln_bank``); blocks
  never hold a projection, so nothing is moved or replaced after the fact.
* **One table per key.**  ``ModulationCache.build`` runs the time embedding
  once and writes every block's ``[R, 6, H]`` modulation into one
  ``[blocks, R, 6, H]`` fp32 tensor; a block reads row ``index`` of it.
* **Keys are explicit.**  Every consumer (block call, checkpoint replay,
  backward) names the key it needs; there is no ambient scope to restore.
  ``hold(key)`` pins a dynamic table while a forward/backward that reads it
  is in flight, so eviction can never pull it from under a replay.
* **Eviction** drops the oldest unheld dynamic table once more than
  ``max_dynamic_keys`` exist, never the one just built (the trainer also
  drops each score key explicitly right after its last use).

The cache is exact only while the time MLP and the bank are frozen;
``ModulationCache.attach`` refuses trainable ones.
"""

from __future__ import annotations

import contextlib
import dataclasses
from collections.abc import Callable, Hashable, Iterator
from typing import Any

import torch
from torch import nn

CacheKey = Hashable


@dataclasses.dataclass(frozen=True)
class CacheStats:
    hits: int
    misses: int
    stores: int
    evictions: int
    persistent_keys: int
    dynamic_keys: int
    bytes: int


class AdaLNBank(nn.Module):
    """All per-block AdaLN projections of one DiT (each one sharded unit)."""

    def __init__(self, projections: list[nn.Module]) -> None:
        super().__init__()
        if not projections:
            raise ValueError("an AdaLN bank needs at least one projection")
        self.projections = nn.ModuleList(projections)

    def __len__(self) -> int:
        return len(self.projections)

    def __getitem__(self, index: int) -> nn.Module:
        return self.projections[index]


@dataclasses.dataclass(eq=False)
class _Table:
    values: torch.Tensor          # [blocks, R, 6, H] fp32
    persistent: bool
    serial: int                   # creation order, for eviction
    holds: int = 0

    @property
    def nbytes(self) -> int:
        return self.values.numel() * self.values.element_size()


def frozen_or_raise(module: nn.Module, what: str) -> None:
    trainable = [n for n, p in module.named_parameters() if p.requires_grad]
    if trainable:
        raise RuntimeError(f"{what} must be frozen for exact AdaLN caching "
                           f"({len(trainable)} trainable tensors, e.g. {trainable[:3]})")


class ModulationCache:
    """Exact modulation tables, one per timestep key, read by (key, block)."""

    def __init__(self, num_blocks: int, *, enabled: bool = True, max_dynamic_keys: int = 2) -> None:
        if int(max_dynamic_keys) < 0:
            raise ValueError(f"max_dynamic_keys must be >= 0, got {max_dynamic_keys}")
        self.num_blocks = int(num_blocks)
        self.enabled = bool(enabled)
        self.max_dynamic_keys = int(max_dynamic_keys)
        self._tables: dict[CacheKey, _Table] = {}
        self._serial = 0
        self.hits = self.misses = self.stores = self.evictions = 0

    @classmethod
    def attach(cls, bank: AdaLNBank, time_embedder: nn.Module | None, *, enabled: bool = True,
               max_dynamic_keys: int = 2) -> "ModulationCache":
        frozen_or_raise(bank, "the AdaLN projection bank")
        if time_embedder is not None:
            frozen_or_raise(time_embedder, "the timestep embedder")
        return cls(len(bank), enabled=enabled, max_dynamic_keys=max_dynamic_keys)

    # ------------------------------------------------------------ building
    @torch.no_grad()
    def build(self, key: CacheKey, *, persistent: bool, temb: Callable[[], torch.Tensor],
              project: Callable[[int, torch.Tensor], torch.Tensor]) -> torch.Tensor:
        """Materialise every block's modulation for ``key`` (no-op when complete).

        ``temb()`` produces the time embedding (called only on a miss);
        ``project(i, temb)`` returns block ``i``'s ``[R, 6, H]`` modulation.
        Each computed block counts as one miss and one store.
        """
        table = self._tables.get(key)
        if table is not None:
            return table.values
        t = temb()
        first = project(0, t).float()
        values = torch.empty((self.num_blocks,) + tuple(first.shape), dtype=torch.float32, device=first.device)
        values[0] = first
        for index in range(1, self.num_blocks):
            values[index] = project(index, t)
        self.misses += self.num_blocks
        self.stores += self.num_blocks
        self._serial += 1
        self._tables[key] = _Table(values, bool(persistent), self._serial)
        self._evict(keep=key)
        return values

    def insert(self, key: CacheKey, values: torch.Tensor, *, persistent: bool) -> None:
        """Register a ready ``[blocks, R, 6, H]`` table (tests and restores)."""
        if values.shape[0] != self.num_blocks:
            raise ValueError(f"table has {values.shape[0]} blocks, cache expects {self.num_blocks}")
        self.stores += self.num_blocks
        self._serial += 1
        self._tables[key] = _Table(values.float(), bool(persistent), self._serial)
        self._evict(keep=key)

    # ------------------------------------------------------------ reading
    def fetch(self, key: CacheKey, block: int) -> torch.Tensor | None:
        """Counted read of block ``block``'s modulation; ``None`` (a miss) if absent."""
        table = self._tables.get(key)
        if table is None or not 0 <= block < self.num_blocks:
            self.misses += 1
            return None
        self.hits += 1
        return table.values[block]

    def complete(self, key: CacheKey) -> bool:
        return key in self._tables

    def persistent(self, key: CacheKey) -> bool:
        table = self._tables.get(key)
        return table is not None and table.persistent

    @contextlib.contextmanager
    def hold(self, key: CacheKey) -> Iterator[None]:
        """Keep ``key``'s table resident (no eviction) for the duration."""
        table = self._tables.get(key)
        if table is not None:
            table.holds += 1
        try:
            yield
        finally:
            if table is not None:
                table.holds -= 1

    # ------------------------------------------------------------ dropping
    def release(self, key: CacheKey) -> None:
        """Drop a dynamic table; persistent tables stay for the run."""
        table = self._tables.get(key)
        if table is not None and not table.persistent:
            del self._tables[key]

    def clear(self) -> None:
        self._tables.clear()

    def _evict(self, keep: CacheKey) -> None:
        """Drop the oldest unheld dynamic tables beyond the bound (never ``keep``, the newest).

        While held tables fill the bound the cache may exceed it; the next
        build after they are released brings it back.
        """
        dynamic = sorted((t.serial, k) for k, t in self._tables.items() if not t.persistent)
        excess = len(dynamic) - self.max_dynamic_keys
        for _, key in dynamic:
            if excess <= 0:
                break
            if key != keep and self._tables[key].holds == 0:
                del self._tables[key]
                self.evictions += 1
                excess -= 1

    # ------------------------------------------------------------ reporting
    def stats(self) -> CacheStats:
        persistent = sum(t.persistent for t in self._tables.values())
        return CacheStats(hits=self.hits, misses=self.misses, stores=self.stores, evictions=self.evictions,
                          persistent_keys=persistent, dynamic_keys=len(self._tables) - persistent,
                          bytes=sum(t.nbytes for t in self._tables.values()))

    def describe(self) -> dict[str, Any]:
        return dataclasses.asdict(self.stats())
