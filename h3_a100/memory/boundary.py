"""Checkpoint-boundary staging to pinned host memory.

Policy and counters follow the reference's ``checkpoint_boundary_cpu``
(``h3_a100/checkpoint_boundary_offload.py:27-336``): every grad-enabled
checkpoint call stages exactly one tensor, its first argument (the block's
input hidden states), to host memory and brings it back when the block is
replayed in backward.  A forward pre/post hook pair on the transformer counts
grad forwards per role and requires ``expected_block_count`` checkpoint calls
per grad forward; stats keys and fail-closed errors are the reference's.

What differs is the data path.  The reference copies synchronously
(``copy_(non_blocking=False)``, ``:117,133``).  Here:

* the device->host copy runs on a dedicated copy stream after an event on
  the compute stream, into a slab from a pinned pool that is allocated once
  and reused every cycle (``PinnedSlabPool``);
* unpacking a boundary starts the host->device copy of the *next* boundary
  that backward will need (blocks replay in reverse order), so each upload
  overlaps the previous block's recompute + backward;
* the compute stream waits on per-copy events, never on the host.
"""

from __future__ import annotations

import json
import threading
import time
from collections import defaultdict
from contextlib import contextmanager
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Callable, Iterator

import torch

PRODUCTION_BLOCK_COUNT = 50
POLICY_NAME = "checkpoint_boundary_cpu"

STAT_KEYS = (
    "transformer_forward_count",
    "grad_transformer_forward_count",
    "checkpoint_call_count",
    "grad_checkpoint_call_count",
    "cpu_copy_count",
    "pack_count",
    "unpack_count",
    "duplicate_pack_count",
    "policy_filter_keep_count",
    "non_strided_keep_count",
    "zero_stride_keep_count",
    "offloaded_logical_bytes",
    "offloaded_storage_bytes",
    "student_grad_forward_count",
    "fake_grad_forward_count",
    "other_grad_forward_count",
    "prefetch_count",
)


def _nbytes(t: torch.Tensor) -> int:
    return int(t.numel() * t.element_size())


def _signature(t: torch.Tensor):
    return tuple(int(s) for s in t.shape), str(t.dtype), _nbytes(t)


def _alias(t: torch.Tensor):
    return (int(t.untyped_storage().data_ptr()), int(t.storage_offset()),
            tuple(t.shape), tuple(t.stride()), str(t.dtype))


def _pinned_empty(numel: int, dtype: torch.dtype) -> torch.Tensor:
    """Exact-size pinned buffer (the native allocator; torch's rounds up to a power of two)."""
    try:
        from .. import _C
    except ImportError:
        return torch.empty(numel, dtype=dtype, pin_memory=True)
    return _C.pinned_empty(numel, dtype)


def host_available_bytes() -> int:
    """MemAvailable from /proc/meminfo (0 when unreadable)."""
    try:
        with open("/proc/meminfo") as fh:
            for line in fh:
                if line.startswith("MemAvailable:"):
                    return int(line.split()[1]) * 1024
    except OSError:
        pass
    return 0


def choose_staging_target(requested: str, bytes_per_rank: int, local_ranks: int, device: torch.device) -> str:
    """Resolve ``auto`` to ``host`` or ``device``.

    ``host`` is the reference's policy (pinned host slabs).  ``device`` keeps
    the slabs in HBM: the same copies and counters, but the boundaries never
    leave the GPU.  ``auto`` picks ``host`` while every local rank's slabs fit
    in half of the node's available RAM, else ``device`` (an 8-rank node with
    20 GB of boundaries per rank would otherwise pin most of host memory).
    """
    requested = str(requested)
    if requested not in {"auto", "host", "device"}:
        raise ValueError(f"boundary staging target must be auto|host|device, got {requested!r}")
    if requested != "auto":
        return requested
    if device.type != "cuda":
        return "host"
    avail = host_available_bytes()
    return "host" if avail and bytes_per_rank * local_ranks <= avail // 2 else "device"


class PinnedSlabPool:
    """Reusable staging buffers keyed by (bytes, dtype).

    ``target="host"``: host slabs, pinned when requested.  ``target="device"``:
    slabs in the GPU's own memory (``device`` must then be a CUDA device).
    """

    def __init__(self, pin_memory: bool, target: str = "host", device: torch.device | None = None) -> None:
        self.target = str(target)
        self.device = device
        if self.target == "device" and (device is None or device.type != "cuda"):
            raise ValueError("device staging needs a CUDA device")
        self.pin_memory = bool(pin_memory) and torch.cuda.is_available() and self.target == "host"
        self._free: dict[tuple[int, torch.dtype], list[torch.Tensor]] = defaultdict(list)
        self.allocated_bytes = 0
        self._pending: list[tuple[torch.Tensor, Any]] = []
        self._lock = threading.Lock()

    def _sweep(self) -> None:
        still = []
        for slab, event in self._pending:
            if event is None or event.query():
                self._free[(slab.numel(), slab.dtype)].append(slab)
            else:
                still.append((slab, event))
        self._pending = still

    def acquire(self, numel: int, dtype: torch.dtype) -> torch.Tensor:
        key = (int(numel), dtype)
        with self._lock:
            self._sweep()
            if self._free[key]:
                return self._free[key].pop()
        if self.target == "device":
            slab = torch.empty(int(numel), dtype=dtype, device=self.device)
        elif self.pin_memory:
            slab = _pinned_empty(int(numel), dtype)
        else:
            slab = torch.empty(int(numel), dtype=dtype)
        self.allocated_bytes += slab.numel() * slab.element_size()
        return slab

    def release(self, slab: torch.Tensor, after_event=None) -> None:
        """Return a slab; with ``after_event`` it is reused only once that copy finished."""
        with self._lock:
            if after_event is None:
                self._free[(slab.numel(), slab.dtype)].append(slab)
            else:
                self._pending.append((slab, after_event))

    def reserve(self, count: int, numel: int, dtype: torch.dtype) -> None:
        """Pre-allocate ``count`` slabs (pinned allocation is slow; do it at setup)."""
        slabs = [self.acquire(numel, dtype) for _ in range(count)]
        for slab in slabs:
            self.release(slab)


@dataclass(eq=False)
class _Keep:
    tensor: torch.Tensor


@dataclass(eq=False)
class _Staged:
    slab: torch.Tensor
    shape: tuple
    stride: tuple
    dtype: torch.dtype
    device: torch.device
    d2h_done: Any = None           # torch.cuda.Event on the copy stream
    upload: torch.Tensor | None = None
    h2d_done: Any = None
    remaining_unpacks: int = 1


class BoundaryStager:
    """Moves boundaries host<->device on a side stream with one-ahead prefetch."""

    def __init__(self, pool: PinnedSlabPool, stats: dict[str, int]) -> None:
        self.pool = pool
        self.stats = stats
        self._stack: list[_Staged] = []
        self._stream = None

    def _copy_stream(self, device: torch.device):
        if device.type != "cuda":
            return None
        if self._stream is None:
            self._stream = torch.cuda.Stream(device=device)
        return self._stream

    def stage_out(self, tensor: torch.Tensor) -> _Staged:
        src = tensor.detach()
        if not src.is_contiguous():
            src = src.contiguous()
        slab = self.pool.acquire(src.numel(), src.dtype)
        staged = _Staged(slab, tuple(tensor.shape), tuple(tensor.stride()), tensor.dtype, tensor.device)
        stream = self._copy_stream(tensor.device)
        if stream is None:
            slab.copy_(src.reshape(-1))
        else:
            stream.wait_stream(torch.cuda.current_stream(tensor.device))
            with torch.cuda.stream(stream):
                slab.copy_(src.reshape(-1), non_blocking=True)
                staged.d2h_done = torch.cuda.Event()
                staged.d2h_done.record(stream)
            src.record_stream(stream)
        self._stack.append(staged)
        return staged

    def _start_upload(self, staged: _Staged) -> None:
        if staged.upload is not None:
            return
        stream = self._copy_stream(staged.device)
        self.stats["prefetch_count"] += 1
        if stream is None:
            staged.upload = staged.slab.clone()
            return
        with torch.cuda.stream(stream):
            # Allocate from the copy stream's pool.  A block taken from the
            # compute stream's pool may have been freed by kernels that are
            # still queued there; writing it from this stream without waiting
            # for them would corrupt their data.  The consumer stream is
            # recorded on the tensor when it is handed out (stage_in).
            staged.upload = torch.empty(staged.slab.numel(), dtype=staged.dtype, device=staged.device)
            if staged.d2h_done is not None:
                stream.wait_event(staged.d2h_done)
            staged.upload.copy_(staged.slab, non_blocking=True)
            staged.h2d_done = torch.cuda.Event()
            staged.h2d_done.record(stream)

    def stage_in(self, staged: _Staged) -> torch.Tensor:
        self._start_upload(staged)
        if staged.h2d_done is not None:
            consumer = torch.cuda.current_stream(staged.device)
            consumer.wait_event(staged.h2d_done)
            staged.upload.record_stream(consumer)
        out = torch.as_strided(staged.upload, staged.shape, staged.stride)
        index = next((i for i, item in enumerate(self._stack) if item is staged), None)
        if index is not None:
            del self._stack[index]
            if index > 0:
                # Backward replays blocks in reverse: the previous boundary is next.
                self._start_upload(self._stack[index - 1])
        staged.remaining_unpacks -= 1
        if staged.remaining_unpacks < 0:
            raise RuntimeError("checkpoint-boundary tensor unpacked too many times")
        if staged.remaining_unpacks == 0:
            self._recycle(staged)
        return out

    def _recycle(self, staged: _Staged) -> None:
        # The slab may be refilled only after its upload finished; the pool
        # checks the event without blocking the host.
        self.pool.release(staged.slab, after_event=staged.h2d_done)

    def live(self) -> int:
        return len(self._stack)


class _BoundaryScope:
    """saved-tensor hooks for one checkpoint call, matching only the boundary signature."""

    def __init__(self, *, target: torch.Tensor, stager: BoundaryStager, require_cuda: bool,
                 stats: dict[str, int]) -> None:
        if target.layout != torch.strided:
            raise RuntimeError("checkpoint boundary input must be strided")
        if any(s > 1 and st == 0 for s, st in zip(target.shape, target.stride())):
            raise RuntimeError("checkpoint boundary input cannot be a zero-stride view")
        if require_cuda and not target.is_cuda:
            raise RuntimeError(f"checkpoint boundary input must be CUDA, got {target.device}")
        self.signature = _signature(target)
        self.stager = stager
        self.stats = stats
        self._by_alias: dict[Any, _Staged] = {}
        self.copies = 0

    def _pack(self, tensor: torch.Tensor):
        self.stats["pack_count"] += 1
        if _signature(tensor) != self.signature:
            self.stats["policy_filter_keep_count"] += 1
            return _Keep(tensor)
        if tensor.layout != torch.strided:
            self.stats["non_strided_keep_count"] += 1
            return _Keep(tensor)
        if any(s > 1 and st == 0 for s, st in zip(tensor.shape, tensor.stride())):
            self.stats["zero_stride_keep_count"] += 1
            return _Keep(tensor)
        alias = _alias(tensor)
        existing = self._by_alias.get(alias)
        if existing is not None:
            existing.remaining_unpacks += 1
            self.stats["duplicate_pack_count"] += 1
            return existing
        staged = self.stager.stage_out(tensor)
        self._by_alias[alias] = staged
        self.copies += 1
        self.stats["cpu_copy_count"] += 1
        self.stats["offloaded_logical_bytes"] += _nbytes(tensor)
        self.stats["offloaded_storage_bytes"] += staged.slab.numel() * staged.slab.element_size()
        return staged

    def _unpack(self, packed):
        self.stats["unpack_count"] += 1
        if isinstance(packed, _Keep):
            return packed.tensor
        if not isinstance(packed, _Staged):
            raise TypeError(f"unexpected checkpoint-boundary saved object: {type(packed)!r}")
        return self.stager.stage_in(packed)

    @contextmanager
    def context(self) -> Iterator[None]:
        with torch.autograd.graph.saved_tensors_hooks(self._pack, self._unpack):
            yield
        if self.copies != 1:
            raise RuntimeError(
                f"checkpoint-boundary staging expected exactly one boundary copy, observed {self.copies}"
            )
        self._by_alias.clear()


@dataclass
class CheckpointBoundaryOffloadRegistration:
    transformer: torch.nn.Module
    original_checkpoint: Callable[..., Any]
    pre_hook: Any
    post_hook: Any
    role_getter: Callable[[], str]
    event_path: Path | None
    expected_block_count: int
    pin_memory: bool
    stats: dict[str, int]
    stager: BoundaryStager | None = None
    closed: bool = False
    extra: dict = field(default_factory=dict)

    def receipt(self) -> dict[str, Any]:
        return {
            "policy": POLICY_NAME,
            "expected_block_count": self.expected_block_count,
            "pin_memory": self.pin_memory,
            "event_path": None if self.event_path is None else str(self.event_path),
            "stats": dict(self.stats),
            "closed": self.closed,
        }

    def remove(self) -> None:
        if self.closed:
            return
        self.pre_hook.remove()
        self.post_hook.remove()
        self.transformer._gradient_checkpointing_func = self.original_checkpoint
        self.closed = True


def install_checkpoint_boundary_cpu_offload(
    transformer: torch.nn.Module,
    *,
    role_getter: Callable[[], str],
    event_path: Path | None = None,
    pin_memory: bool = True,
    expected_block_count: int = PRODUCTION_BLOCK_COUNT,
    require_cuda: bool = True,
    pool: PinnedSlabPool | None = None,
) -> CheckpointBoundaryOffloadRegistration:
    """Wrap ``transformer._gradient_checkpointing_func`` with boundary staging."""
    blocks = getattr(transformer, "transformer_blocks", None)
    if blocks is None or len(blocks) != int(expected_block_count):
        raise RuntimeError(
            "checkpoint-boundary CPU staging requires native per-block layout: "
            f"expected {expected_block_count} transformer blocks, got {0 if blocks is None else len(blocks)}"
        )
    if not bool(getattr(transformer, "gradient_checkpointing", False)):
        raise RuntimeError("checkpoint-boundary CPU staging requires gradient checkpointing")
    original = getattr(transformer, "_gradient_checkpointing_func", None)
    if not callable(original):
        raise RuntimeError("transformer has no callable gradient checkpoint function")
    path = None if event_path is None else Path(event_path)
    if path is not None:
        path.parent.mkdir(parents=True, exist_ok=True)
        if path.exists():
            raise FileExistsError(f"refusing to overwrite checkpoint-boundary events: {path}")

    stats = dict.fromkeys(STAT_KEYS, 0)
    stager = BoundaryStager(pool or PinnedSlabPool(pin_memory), stats)
    state: dict[str, Any] = {"calls": 0, "grad": False, "role": "unknown"}
    lock = threading.Lock()

    def write_event(payload: dict[str, Any]) -> None:
        if path is None:
            return
        with lock, path.open("a", encoding="utf-8") as fh:
            fh.write(json.dumps({"time_unix": time.time(), **payload}, sort_keys=True) + "\n")

    def wrapped(function: Callable[..., Any], *args: Any, **kwargs: Any) -> Any:
        index = int(state["calls"])
        state["calls"] = index + 1
        stats["checkpoint_call_count"] += 1
        if not torch.is_grad_enabled():
            return original(function, *args, **kwargs)
        if index >= int(expected_block_count):
            raise RuntimeError(f"checkpoint call count exceeded expected {expected_block_count}: index={index}")
        if not args or not torch.is_tensor(args[0]):
            raise RuntimeError(f"checkpoint block {index} has no tensor boundary input")
        stats["grad_checkpoint_call_count"] += 1
        boundary = args[0]
        scope = _BoundaryScope(target=boundary, stager=stager, require_cuda=require_cuda, stats=stats)
        before = int(stats["cpu_copy_count"])
        with scope.context():
            result = original(function, *args, **kwargs)
        write_event({
            "event": "checkpoint_boundary_saved",
            "block_index": index,
            "role": state["role"],
            "shape": list(boundary.shape),
            "dtype": str(boundary.dtype),
            "logical_bytes": _nbytes(boundary),
            "new_cpu_copies": int(stats["cpu_copy_count"]) - before,
        })
        return result

    def pre_hook(_module, _inputs) -> None:
        state["calls"] = 0
        state["grad"] = bool(torch.is_grad_enabled())
        state["role"] = str(role_getter())
        stats["transformer_forward_count"] += 1

    def post_hook(_module, _inputs, _output) -> None:
        if not state["grad"]:
            return
        calls = int(state["calls"])
        if calls != int(expected_block_count):
            raise RuntimeError(f"native checkpoint call count mismatch: {calls} != {expected_block_count}")
        stats["grad_transformer_forward_count"] += 1
        role = str(state["role"])
        key = {"student": "student_grad_forward_count", "fake": "fake_grad_forward_count"}.get(
            role, "other_grad_forward_count")
        stats[key] += 1
        write_event({"event": "grad_transformer_forward_complete", "role": role,
                     "checkpoint_calls": calls, "cpu_copies_total": int(stats["cpu_copy_count"])})

    pre = transformer.register_forward_pre_hook(pre_hook)
    post = transformer.register_forward_hook(post_hook, always_call=True)
    transformer._gradient_checkpointing_func = wrapped
    return CheckpointBoundaryOffloadRegistration(
        transformer=transformer,
        original_checkpoint=original,
        pre_hook=pre,
        post_hook=post,
        role_getter=role_getter,
        event_path=path,
        expected_block_count=int(expected_block_count),
        pin_memory=bool(pin_memory),
        stats=stats,
        stager=stager,
    )
