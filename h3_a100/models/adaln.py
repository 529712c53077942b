"""AdaLN projection bank and the exact, key-scoped modulation cache.

Behaviour matches the reference (``h3_a100/adaln_cache.py:51-268``): every
block's frozen ``adaln_proj`` moves into one bank (so each projection can be a
separately sharded unit) and the block keeps a parameter-free handle; outputs
are cached per (key, block) where a key names one exact timestep table.

* ``("rollout", i)`` keys are persistent and never evicted.
* ``("score", n)`` keys are dynamic, LRU-bounded by ``max_dynamic_keys`` and
  dropped by the trainer after the Fake/Teacher pair that uses them.
* Stats count hits, misses, stores, evictions, key kinds and bytes.

The cache is exact only while the time MLP and the bank are frozen; the
installer refuses trainable ones.  Unlike the reference, the DiT in this
package also passes the key explicitly into the checkpoint replay (see
``h3_a100.memory.exact_replay``), so replay never depends on ambient context.
"""

from __future__ import annotations

import contextlib
import contextvars
import dataclasses
import weakref
from collections import OrderedDict
from collections.abc import Hashable, Iterator, Sequence
from typing import Any

import torch
from torch import nn

CacheKey = Hashable
Modulation = tuple[torch.Tensor, ...]


@dataclasses.dataclass(frozen=True)
class CacheStats:
    hits: int
    misses: int
    stores: int
    evictions: int
    persistent_keys: int
    dynamic_keys: int
    bytes: int


@dataclasses.dataclass(frozen=True)
class Scope:
    key: CacheKey | None
    persistent: bool


class AdaLNCacheController:
    """Cache of per-block modulations, addressed by (scope key, block index)."""

    def __init__(self, *, enabled: bool = True, max_dynamic_keys: int = 2) -> None:
        if max_dynamic_keys < 0:
            raise ValueError(f"max_dynamic_keys must be non-negative, got {max_dynamic_keys}")
        self.enabled = bool(enabled)
        self.max_dynamic_keys = int(max_dynamic_keys)
        self._entries: OrderedDict[CacheKey, dict[int, Modulation]] = OrderedDict()
        self._persistent: set[CacheKey] = set()
        self._scope_var: contextvars.ContextVar[Scope] = contextvars.ContextVar(
            "h3_adaln_scope", default=Scope(None, False)
        )
        self._last = Scope(None, False)
        self._hits = self._misses = self._stores = self._evictions = 0

    # -- scoping -----------------------------------------------------------
    @contextlib.contextmanager
    def scope(self, key: CacheKey | None, *, persistent: bool = False) -> Iterator[None]:
        entry = Scope(key, bool(persistent))
        token = self._scope_var.set(entry)
        self._last = entry
        if key is not None and persistent:
            self._persistent.add(key)
        try:
            yield
        finally:
            self._scope_var.reset(token)

    def current_scope(self) -> Scope:
        return self._scope_var.get()

    def last_scope(self) -> Scope:
        return self._last

    # -- lookups -----------------------------------------------------------
    def lookup(self, key: CacheKey, block_index: int) -> Modulation | None:
        """Counted lookup of an existing entry; None (and a miss) if absent."""
        blocks = self._entries.get(key)
        if blocks is not None and block_index in blocks:
            self._entries.move_to_end(key)
            self._hits += 1
            return blocks[block_index]
        self._misses += 1
        return None

    def get_or_compute(self, block_index: int, temb: torch.Tensor, projection: Any) -> Modulation:
        scope = self._scope_var.get()
        if not self.enabled or scope.key is None:
            out = projection(temb)
            return (out,) if torch.is_tensor(out) else tuple(out)
        blocks = self._entries.get(scope.key)
        if blocks is not None and block_index in blocks:
            self._entries.move_to_end(scope.key)
            self._hits += 1
            return blocks[block_index]
        self._misses += 1
        with torch.no_grad():
            out = projection(temb.detach())
        modulation = (out.detach(),) if torch.is_tensor(out) else tuple(t.detach() for t in out)
        self.store(scope.key, block_index, modulation, persistent=scope.persistent)
        return modulation

    def store(self, key: CacheKey, block_index: int, modulation: Modulation, *, persistent: bool) -> None:
        blocks = self._entries.get(key)
        if blocks is None:
            blocks = {}
            self._entries[key] = blocks
        blocks[block_index] = modulation
        self._stores += 1
        if persistent:
            self._persistent.add(key)
        self._entries.move_to_end(key)
        self._evict_dynamic_keys()

    def has_complete_key(self, key: CacheKey, num_blocks: int) -> bool:
        blocks = self._entries.get(key)
        return blocks is not None and len(blocks) == int(num_blocks)

    def is_persistent(self, key: CacheKey) -> bool:
        return key in self._persistent

    def drop(self, key: CacheKey) -> None:
        if key not in self._persistent:
            self._entries.pop(key, None)

    def clear_dynamic(self) -> None:
        for key in [k for k in self._entries if k not in self._persistent]:
            del self._entries[key]

    def clear(self) -> None:
        self._entries.clear()
        self._persistent.clear()

    def stats(self) -> CacheStats:
        total = 0
        dynamic = 0
        for key, blocks in self._entries.items():
            dynamic += key not in self._persistent
            for modulation in blocks.values():
                total += sum(t.numel() * t.element_size() for t in modulation)
        return CacheStats(
            hits=self._hits,
            misses=self._misses,
            stores=self._stores,
            evictions=self._evictions,
            persistent_keys=len(self._persistent),
            dynamic_keys=dynamic,
            bytes=total,
        )

    def _evict_dynamic_keys(self) -> None:
        dynamic = [k for k in self._entries if k not in self._persistent]
        while len(dynamic) > self.max_dynamic_keys:
            self._entries.pop(dynamic.pop(0), None)
            self._evictions += 1


class AdaLNProjectionBank(nn.Module):
    """Owner of all per-block AdaLN projections (one sharded unit each)."""

    def __init__(self, projections: Sequence[nn.Module]) -> None:
        super().__init__()
        if not projections:
            raise ValueError("AdaLN bank cannot be empty")
        self.projections = nn.ModuleList(list(projections))


class AdaLNProjectionHandle(nn.Module):
    """Parameter-free stand-in for a block's projection; forwards to the cache."""

    def __init__(self, bank: AdaLNProjectionBank, controller: AdaLNCacheController, block_index: int) -> None:
        super().__init__()
        object.__setattr__(self, "_bank_ref", weakref.ref(bank))
        object.__setattr__(self, "_controller_ref", weakref.ref(controller))
        self.block_index = int(block_index)

    def forward(self, temb: torch.Tensor) -> Modulation:
        bank, controller = self._bank_ref(), self._controller_ref()
        if bank is None or controller is None:
            raise RuntimeError("AdaLN bank/controller was released")
        return controller.get_or_compute(self.block_index, temb, bank.projections[self.block_index])


def _blocks_of(transformer: nn.Module) -> list[nn.Module]:
    blocks = getattr(transformer, "transformer_blocks", None)
    if blocks is None:
        blocks = getattr(transformer, "blocks", None)
    if blocks is None:
        raise AttributeError("transformer has neither transformer_blocks nor blocks")
    return list(blocks)


def _assert_frozen(module: nn.Module, what: str) -> None:
    trainable = [name for name, p in module.named_parameters() if p.requires_grad]
    if trainable:
        raise RuntimeError(
            f"{what} must be frozen before enabling exact AdaLN caching; "
            f"found {len(trainable)} trainable parameters: {', '.join(trainable[:6])}"
        )


def install_adaln_cache(
    transformer: nn.Module, *, enabled: bool = True, max_dynamic_keys: int = 2
) -> AdaLNCacheController:
    """Move every ``block.adaln_proj`` into a bank and install cache handles (idempotent)."""
    existing = getattr(transformer, "_h3_adaln_controller", None)
    if existing is not None:
        return existing
    blocks = _blocks_of(transformer)
    projections = []
    for index, block in enumerate(blocks):
        projection = getattr(block, "adaln_proj", None)
        if projection is None:
            raise AttributeError(f"block {index} has no adaln_proj module")
        projections.append(projection)
    bank = AdaLNProjectionBank(projections)
    controller = AdaLNCacheController(enabled=enabled, max_dynamic_keys=max_dynamic_keys)
    transformer.add_module("adaln_bank", bank)
    object.__setattr__(transformer, "_h3_adaln_controller", controller)
    for index, block in enumerate(blocks):
        block.adaln_proj = AdaLNProjectionHandle(bank, controller, index)
    _assert_frozen(bank, "AdaLN bank")
    time_embedder = getattr(transformer, "time_embedder", None)
    if time_embedder is not None:
        _assert_frozen(time_embedder, "timestep embedder")
    return controller


def adaln_bank(transformer: nn.Module) -> AdaLNProjectionBank | None:
    bank = getattr(transformer, "adaln_bank", None)
    return bank if isinstance(bank, AdaLNProjectionBank) else None


def adaln_controller(transformer: nn.Module) -> AdaLNCacheController | None:
    controller = getattr(transformer, "_h3_adaln_controller", None)
    return controller if isinstance(controller, AdaLNCacheController) else None
