"""Thresholded saved-tensor offload (diagnostic, off by default).

Behaviour of the reference's ``SelectiveSavedTensorOffload``
(``h3_a100/activation_offload.py:54-193``): during the original grad forward,
every saved tensor whose storage is at least ``min_offload_bytes`` (and that
is not a parameter or buffer of ``model``) is copied to host memory; after
``begin_backward()`` tensors saved by checkpoint recomputation stay on the
device, so the policy cannot recurse into replay intermediates.  The
reference showed this does not cure its OOM; it is kept for A/B diagnosis and
is mutually exclusive with boundary staging.
"""

from __future__ import annotations

import contextlib
from dataclasses import dataclass
from typing import Iterator

import torch

STAT_KEYS = (
    "pack_count", "unpack_count", "offload_count", "offloaded_storage_bytes", "offloaded_logical_bytes",
    "keep_parameter_or_buffer_count", "keep_non_cuda_count", "keep_non_strided_count",
    "keep_zero_stride_count", "keep_below_threshold_count", "replay_pack_count", "replay_unpack_count",
)


def _storage_key(t: torch.Tensor):
    try:
        st = t.untyped_storage()
        return str(t.device), int(st.data_ptr()), int(st.nbytes())
    except Exception:  # noqa: BLE001 - storage-less tensors never match
        return str(t.device), 0, 0


def _storage_bytes(t: torch.Tensor) -> int:
    try:
        return int(t.untyped_storage().nbytes())
    except Exception:  # noqa: BLE001
        return int(t.numel() * t.element_size())


@dataclass(eq=False)
class _Keep:
    tensor: torch.Tensor


@dataclass(eq=False)
class _OnHost:
    host: torch.Tensor
    device: torch.device


class SelectiveSavedTensorOffload:
    def __init__(self, model: torch.nn.Module, *, logical_component: str, min_offload_bytes: int,
                 pin_memory: bool = True, offload_cpu_tensors: bool = False) -> None:
        if int(min_offload_bytes) < 0:
            raise ValueError("min_offload_bytes must be non-negative")
        self.model = model
        self.logical_component = str(logical_component)
        self.min_offload_bytes = int(min_offload_bytes)
        self.pin_memory = bool(pin_memory) and torch.cuda.is_available()
        # CPU tests exercise the mechanism on CPU tensors.
        self.offload_cpu_tensors = bool(offload_cpu_tensors)
        self.phase = "forward"
        self._excluded: set = set()
        self._handles: list[_OnHost] = []
        self.stats = dict.fromkeys(STAT_KEYS, 0)

    def _refresh_excluded(self) -> None:
        self._excluded = {_storage_key(t) for t in list(self.model.parameters()) + list(self.model.buffers())}

    def _pack(self, t: torch.Tensor):
        self.stats["pack_count"] += 1
        if self.phase != "forward":
            self.stats["replay_pack_count"] += 1
            return _Keep(t)
        if t.device.type != "cuda" and not self.offload_cpu_tensors:
            self.stats["keep_non_cuda_count"] += 1
            return _Keep(t)
        if _storage_key(t) in self._excluded:
            self.stats["keep_parameter_or_buffer_count"] += 1
            return _Keep(t)
        if t.layout != torch.strided:
            self.stats["keep_non_strided_count"] += 1
            return _Keep(t)
        if any(s > 1 and st == 0 for s, st in zip(t.shape, t.stride())):
            self.stats["keep_zero_stride_count"] += 1
            return _Keep(t)
        if _storage_bytes(t) < self.min_offload_bytes:
            self.stats["keep_below_threshold_count"] += 1
            return _Keep(t)
        src = t.detach()
        host = torch.empty_strided(tuple(src.shape), tuple(src.stride()), dtype=src.dtype, device="cpu",
                                   pin_memory=self.pin_memory)
        host.copy_(src)
        handle = _OnHost(host, t.device)
        self._handles.append(handle)
        self.stats["offload_count"] += 1
        self.stats["offloaded_storage_bytes"] += int(host.untyped_storage().nbytes())
        self.stats["offloaded_logical_bytes"] += int(t.numel() * t.element_size())
        return handle

    def _unpack(self, handle):
        self.stats["unpack_count"] += 1
        if isinstance(handle, _Keep):
            if self.phase != "forward":
                self.stats["replay_unpack_count"] += 1
            return handle.tensor
        if not isinstance(handle, _OnHost):
            raise TypeError(f"unexpected saved-tensor handle {type(handle)!r}")
        return handle.host.to(handle.device)

    def begin_backward(self) -> None:
        if self.phase != "forward":
            raise RuntimeError(f"saved-tensor offload phase is already {self.phase!r}")
        self.phase = "replay"

    @contextlib.contextmanager
    def context(self) -> Iterator["SelectiveSavedTensorOffload"]:
        self._refresh_excluded()
        try:
            with torch.autograd.graph.saved_tensors_hooks(self._pack, self._unpack):
                yield self
        finally:
            self._handles.clear()


@contextlib.contextmanager
def maybe_saved_tensor_offload(model: torch.nn.Module, *, enabled: bool, logical_component: str,
                               min_offload_bytes: int, pin_memory: bool = True,
                               offload_cpu_tensors: bool = False) -> Iterator[SelectiveSavedTensorOffload | None]:
    if not enabled:
        yield None
        return
    scope = SelectiveSavedTensorOffload(model, logical_component=logical_component,
                                        min_offload_bytes=min_offload_bytes, pin_memory=pin_memory,
                                        offload_cpu_tensors=offload_cpu_tensors)
    with scope.context():
        yield scope
