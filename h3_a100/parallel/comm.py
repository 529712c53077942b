"""Collective transports used by the sharded runtime and the optimizer.

``TorchComm`` is the baseline: ``torch.distributed`` (NCCL on GPU, gloo on
CPU), each collective issued on a dedicated communication stream so it
overlaps compute, with events (never host syncs) ordering it against the
compute stream.  ``h3_a100.parallel.p2p.PeerComm`` implements the same
interface with hand-written kernels over peer memory.
"""

from __future__ import annotations

from collections import defaultdict

import torch
import torch.distributed as dist


class _Pending:
    __slots__ = ("out", "event", "work")

    def __init__(self, out, event, work=None):
        self.out, self.event, self.work = out, event, work


class TorchComm:
    name = "nccl"

    def __init__(self, group=None, device: torch.device | None = None) -> None:
        self.group = group
        self.initialized = dist.is_available() and dist.is_initialized()
        self.world_size = dist.get_world_size(group) if self.initialized else 1
        self.rank = dist.get_rank(group) if self.initialized else 0
        self.device = device or torch.device("cpu")
        self.cuda = self.device.type == "cuda"
        self.backend = dist.get_backend(group) if self.initialized else "none"
        self._stream = torch.cuda.Stream(device=self.device) if self.cuda else None
        self._free: dict[int, list[tuple[torch.Tensor, object]]] = defaultdict(list)
        self.bytes_gathered = 0
        self.bytes_reduced = 0
        # Optional ``StallLedger``: when set, every wait of the compute stream
        # on a prefetched gather is timed as exposed all-gather time.
        self.ledger = None
        # Optional ``StreamTimeline``: gathers are recorded on the "comm" lane.
        self.timeline = None

    # ---------------- buffers ----------------
    def alloc_shard(self, numel: int, dtype: torch.dtype) -> torch.Tensor:
        return torch.empty(int(numel), dtype=dtype, device=self.device)

    def alloc_symmetric(self, numel: int, dtype: torch.dtype) -> torch.Tensor:
        """Plain (non-peer-mapped) zeroed buffer; the peer transport overrides this."""
        return torch.zeros(int(numel), dtype=dtype, device=self.device)

    def _buffer(self, numel: int, dtype: torch.dtype) -> torch.Tensor:
        free = self._free[numel]
        for i, (buf, event) in enumerate(free):
            if buf.dtype == dtype:
                del free[i]
                if event is not None:
                    self._stream.wait_event(event)
                return buf
        return torch.empty(numel, dtype=dtype, device=self.device)

    def recycle(self, buf: torch.Tensor) -> None:
        event = None
        if self.cuda:
            event = torch.cuda.Event()
            event.record(torch.cuda.current_stream(self.device))
        self._free[buf.numel()].append((buf, event))

    # ---------------- all-gather of a flat shard ----------------
    def all_gather_async(self, shard: torch.Tensor, total: int) -> _Pending:
        if not self.cuda:
            out = torch.empty(total, dtype=shard.dtype, device=shard.device)
            self._all_gather_flat(out, shard)
            return _Pending(out, None)
        self._stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self._stream):
            out = self._buffer(total, shard.dtype)
            t0 = self.timeline.event(self._stream) if self.timeline is not None else None
            self._all_gather_flat(out, shard)
            if t0 is not None:
                self.timeline.add("comm", "all_gather", t0, self.timeline.event(self._stream))
            event = torch.cuda.Event()
            event.record(self._stream)
        self.bytes_gathered += out.numel() * out.element_size()
        return _Pending(out, event)

    def _all_gather_flat(self, out: torch.Tensor, shard: torch.Tensor) -> None:
        if self.world_size == 1:
            out.copy_(shard)
        elif self.backend == "nccl":
            dist.all_gather_into_tensor(out, shard, group=self.group)
        else:
            dist.all_gather(list(out.view(self.world_size, -1).unbind(0)), shard, group=self.group)

    def wait(self, pending: _Pending) -> torch.Tensor:
        if pending.event is not None:
            stream = torch.cuda.current_stream(self.device)
            if self.ledger is not None:
                self.ledger.wait("all_gather", pending.event, stream)
            else:
                stream.wait_event(pending.event)
            pending.out.record_stream(stream)
        return pending.out

    # ---------------- small collectives ----------------
    def all_gather_rows(self, local: torch.Tensor) -> torch.Tensor:
        """[R, n] per rank -> [R, world*n] (rank-major columns)."""
        if self.world_size == 1:
            return local
        stacked = torch.empty((self.world_size,) + tuple(local.shape), dtype=local.dtype, device=local.device)
        if self.backend == "nccl":
            dist.all_gather_into_tensor(stacked.view(-1), local.reshape(-1), group=self.group)
        else:
            dist.all_gather(list(stacked.unbind(0)), local, group=self.group)
        return stacked.permute(1, 0, 2).reshape(local.shape[0], -1)

    def all_reduce_(self, tensor: torch.Tensor, op: str = "avg") -> torch.Tensor:
        if self.world_size == 1:
            return tensor
        self.bytes_reduced += tensor.numel() * tensor.element_size()
        if op == "avg" and self.backend == "nccl":
            dist.all_reduce(tensor, op=dist.ReduceOp.AVG, group=self.group)
        else:
            dist.all_reduce(tensor, op=dist.ReduceOp.SUM, group=self.group)
            if op == "avg":
                tensor.div_(self.world_size)
        return tensor

    def all_reduce_async_(self, tensor: torch.Tensor, op: str = "avg"):
        """Reduce on the comm stream; returns an event the compute stream must wait on."""
        if self.world_size == 1:
            return None
        if not self.cuda:
            self.all_reduce_(tensor, op)
            return None
        self._stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self._stream):
            self.all_reduce_(tensor, op)
            event = torch.cuda.Event()
            event.record(self._stream)
        return event

    def wait_event(self, event) -> None:
        if event is not None:
            torch.cuda.current_stream(self.device).wait_event(event)

    def reduce_scatter_(self, out: torch.Tensor, full: torch.Tensor, op: str = "avg") -> torch.Tensor:
        if self.world_size == 1:
            out.copy_(full)
            return out
        if self.backend == "nccl":
            dist.reduce_scatter_tensor(out, full, op=dist.ReduceOp.AVG if op == "avg" else dist.ReduceOp.SUM,
                                       group=self.group)
        else:
            chunks = list(full.view(self.world_size, -1).clone().unbind(0))
            dist.reduce_scatter(out, chunks, group=self.group)
            if op == "avg":
                out.div_(self.world_size)
        return out

    def all_gather_into_(self, out: torch.Tensor, shard: torch.Tensor) -> torch.Tensor:
        self._all_gather_flat(out, shard)
        return out
