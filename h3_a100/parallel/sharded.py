"""Sharded frozen parameters: the FULL_SHARD runtime of this package.

The reference shards with torch FSDP2 using four unit groups
(``h3_a100/model.py:410-438``): the time embedder, each of the 50 AdaLN
projections, each refiner/transformer block (``reshard_after_forward`` =
``block_reshard``), and the root (not resharded).  Here the base is frozen
and the LoRA adapters live in per-role flat buffers (``h3_a100.models.lora``),
so a unit only has to hold frozen weights:

* each unit flattens its parameters into one buffer, padded so every rank's
  shard is a whole number of 128-byte lines, and keeps only its shard;
* ``gather()`` materialises the full weights (views into one gathered
  buffer) and ``release()`` drops them again when the unit reshards;
* gathering unit *i* starts the gather of the unit that runs next (forward
  order, or reverse order in backward), on a side stream, so the transfer
  overlaps the current unit's compute;
* AdaLN projection units are *row-sharded* instead: each rank multiplies the
  time embedding by its own rows and only the tiny outputs are gathered
  (``ShardedProjection``), so a 520 MB projection never crosses NVLink.

The transport is a ``Communicator`` (``h3_a100.parallel.comm``): NCCL as the
baseline, the native peer-memory kernels as the product path.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import nn

ALIGN_BYTES = 128


@dataclass(frozen=True)
class ParamSpec:
    name: str
    shape: tuple[int, ...]
    offset: int
    numel: int


class ShardedUnit:
    """One unit of frozen parameters flattened, padded and sharded."""

    def __init__(self, name: str, module: nn.Module, param_names: list[str], comm, *,
                 reshard_after_forward: bool = True) -> None:
        self.name = name
        self.module = module
        self.comm = comm
        self.world, self.rank = comm.world_size, comm.rank
        self.reshard_after_forward = bool(reshard_after_forward)
        params = [getattr(module, n) for n in param_names]
        dtype = params[0].dtype
        device = params[0].device
        self.dtype, self.device = dtype, device
        specs, offset = [], 0
        for n, p in zip(param_names, params):
            specs.append(ParamSpec(n, tuple(p.shape), offset, p.numel()))
            offset += p.numel()
        elem = torch.empty((), dtype=dtype).element_size()
        quantum = self.world * max(1, ALIGN_BYTES // elem)
        self.numel = offset
        self.padded = (offset + quantum - 1) // quantum * quantum
        self.shard_numel = self.padded // self.world
        self.specs = specs
        if self.world == 1:
            full = torch.empty(self.padded, dtype=dtype, device=device)
            for spec, p in zip(specs, params):
                full[spec.offset:spec.offset + spec.numel].copy_(p.detach().reshape(-1))
            self.shard = full
        else:
            self.shard = comm.alloc_shard(self.shard_numel, dtype)
            lo, hi = self.rank * self.shard_numel, (self.rank + 1) * self.shard_numel
            for spec, p in zip(specs, params):
                a, b = max(lo, spec.offset), min(hi, spec.offset + spec.numel)
                if a < b:
                    self.shard[a - lo:b - lo].copy_(p.detach().reshape(-1)[a - spec.offset:b - spec.offset])
        # The module's own parameters now alias the unit (world 1) or are freed.
        for spec, n in zip(specs, param_names):
            if self.world == 1:
                getattr(module, n).data = self.shard[spec.offset:spec.offset + spec.numel].view(spec.shape)
            else:
                getattr(module, n).data = torch.empty(0, dtype=dtype, device=device)
        self._full: torch.Tensor | None = self.shard if self.world == 1 else None
        self._pending = None
        self.next_unit: ShardedUnit | None = None
        self.prev_unit: ShardedUnit | None = None
        self.gather_count = 0

    def start_gather(self) -> None:
        if self._full is not None or self._pending is not None or self.world == 1:
            return
        self._pending = self.comm.all_gather_async(self.shard, self.padded)

    def _wait(self) -> torch.Tensor:
        if self._full is None:
            if self._pending is None:
                self.start_gather()
            self._full = self.comm.wait(self._pending)
            self._pending = None
            self.gather_count += 1
        return self._full

    def gather(self, backward: bool = False) -> dict[str, torch.Tensor]:
        full = self._wait()
        if self.world > 1:
            ahead = self.prev_unit if backward else self.next_unit
            if ahead is not None:
                ahead.start_gather()
        return {s.name: full[s.offset:s.offset + s.numel].view(s.shape) for s in self.specs}

    def release(self) -> None:
        if self.world > 1 and self.reshard_after_forward:
            if self._full is not None:
                self.comm.recycle(self._full)
            self._full = None

    def local_bytes(self) -> int:
        return self.shard.numel() * self.shard.element_size()


class ShardedProjection:
    """Row-sharded AdaLN projection: local rows x temb, then gather the outputs.

    ``weight [N, K]`` rows are split evenly (N padded to a multiple of the
    world); each rank keeps ``N/world`` rows.  ``forward(temb)`` returns the
    full ``SiLU(temb) @ W^T + b`` as [R, N] fp32 on every rank.
    """

    def __init__(self, module: nn.Module, comm, kernels) -> None:
        self.comm, self.kernels = comm, kernels
        w, b = module.weight, module.bias
        self.n, self.k = w.shape
        world, rank = comm.world_size, comm.rank
        self.rows = (self.n + world - 1) // world
        lo, hi = rank * self.rows, min(self.n, (rank + 1) * self.rows)
        self.weight = torch.zeros(self.rows, self.k, dtype=w.dtype, device=w.device)
        self.bias = torch.zeros(self.rows, dtype=b.dtype, device=b.device)
        if lo < hi:
            self.weight[:hi - lo].copy_(w.detach()[lo:hi])
            self.bias[:hi - lo].copy_(b.detach()[lo:hi])
        module.weight.data = torch.empty(0, dtype=w.dtype, device=w.device)
        module.bias.data = torch.empty(0, dtype=b.dtype, device=b.device)

    def __call__(self, temb: torch.Tensor) -> torch.Tensor:
        if hasattr(self.comm, "adaln_project") and temb.shape[0] <= 2:
            # Fused GEMV + all-gather: every rank stores its rows into every rank's
            # output buffer.  Two buffers alternate so a fast rank never overwrites
            # an output a slow rank has not copied yet.
            bufs = getattr(self.comm, "_adaln_out_buffers", None)
            need = 2 * self.comm.world_size * self.rows
            if bufs is None or bufs[0].numel() < need:
                bufs = [self.comm.alloc_symmetric(need, torch.float32) for _ in range(2)]
                self.comm._adaln_out_buffers = bufs
                self.comm._adaln_calls = 0
            buf = bufs[self.comm._adaln_calls % 2]
            self.comm._adaln_calls += 1
            r = temb.shape[0]
            out = buf[: r * self.comm.world_size * self.rows].view(r, -1)
            self.comm.adaln_project(temb, self.weight, self.bias, out)
            return out[:, :self.n].clone()
        local = self.kernels.adaln_project(temb, self.weight, self.bias)   # [R, rows] fp32
        full = self.comm.all_gather_rows(local.contiguous())                # [R, world*rows]
        return full[:, :self.n]

    def local_bytes(self) -> int:
        return self.weight.numel() * self.weight.element_size()


def link_order(units: list[ShardedUnit]) -> None:
    for a, b in zip(units, units[1:]):
        a.next_unit, b.prev_unit = b, a
