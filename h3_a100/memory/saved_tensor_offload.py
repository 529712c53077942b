"""Thresholded saved-tensor offload (diagnostic, off by default).

Behaviour kept from the reference's legacy policy
(``h3_a100/activation_offload.py:54-193``): during an original grad forward,
every tensor autograd saves whose storage is at least ``min_bytes`` and that
is not a parameter or buffer of the model is moved to host memory; once
backward starts (``begin_backward``), tensors saved by checkpoint replay stay
on the device, so the policy never recurses into replay intermediates.  The
reference measured that this does not cure its out-of-memory failure; it is
kept for A/B diagnosis and is mutually exclusive with boundary staging.

Design here: ``ThresholdOffload`` asks one question per saved tensor, "why
does this one stay?" (``_keep_reason``), and tallies the answers in a
counter; tensors that stay are handed back to autograd unchanged, offloaded
ones become a ``_HostCopy``.  Copies are stream-ordered on the current stream
(device->host on save, host->device on use), so no host synchronisation is
needed.
"""

from __future__ import annotations

import contextlib
from collections import Counter
from collections.abc import Iterator

import torch


class _HostCopy:
    __slots__ = ("host", "device")

    def __init__(self, host: torch.Tensor, device: torch.device) -> None:
        self.host, self.device = host, device


def _storage_id(t: torch.Tensor) -> tuple:
    try:
        st = t.untyped_storage()
        return t.device.type, t.device.index, int(st.data_ptr())
    except (RuntimeError, NotImplementedError):
        return t.device.type, t.device.index, -1


def _storage_nbytes(t: torch.Tensor) -> int:
    try:
        return int(t.untyped_storage().nbytes())
    except (RuntimeError, NotImplementedError):
        return int(t.numel() * t.element_size())


class ThresholdOffload:
    """saved_tensors_hooks policy: large, non-parameter tensors of the original forward go to host."""

    def __init__(self, model: torch.nn.Module, *, min_bytes: int, label: str = "", pin_memory: bool = True,
                 include_cpu: bool = False) -> None:
        if int(min_bytes) < 0:
            raise ValueError("min_bytes must be non-negative")
        self.model = model
        self.label = str(label)
        self.min_bytes = int(min_bytes)
        self.pin_memory = bool(pin_memory) and torch.cuda.is_available()
        self.include_cpu = bool(include_cpu)      # CPU tests exercise the mechanism on CPU tensors
        self.replaying = False
        self.counts: Counter[str] = Counter()
        self._frozen: set[tuple] = set()

    def _keep_reason(self, t: torch.Tensor) -> str | None:
        if self.replaying:
            return "replay"
        if t.device.type != "cuda" and not self.include_cpu:
            return "not_cuda"
        if t.layout != torch.strided:
            return "not_strided"
        if t.numel() > 1 and 0 in t.stride():
            return "broadcast_view"
        if _storage_id(t) in self._frozen:
            return "parameter_or_buffer"
        if _storage_nbytes(t) < self.min_bytes:
            return "below_threshold"
        return None

    def _pack(self, t: torch.Tensor):
        self.counts["saved"] += 1
        reason = self._keep_reason(t)
        if reason is not None:
            self.counts[f"kept_{reason}"] += 1
            return t
        src = t.detach()
        host = torch.empty_strided(tuple(src.shape), tuple(src.stride()), dtype=src.dtype, device="cpu",
                                   pin_memory=self.pin_memory)
        host.copy_(src, non_blocking=self.pin_memory)
        self.counts["offloaded"] += 1
        self.counts["offloaded_bytes"] += _storage_nbytes(host)
        return _HostCopy(host, t.device)

    def _unpack(self, obj):
        self.counts["used"] += 1
        if isinstance(obj, _HostCopy):
            return obj.host.to(obj.device, non_blocking=self.pin_memory)
        return obj

    def begin_backward(self) -> None:
        """From now on (checkpoint replay), saved tensors stay on the device."""
        if self.replaying:
            raise RuntimeError("saved-tensor offload is already in its backward phase")
        self.replaying = True

    @contextlib.contextmanager
    def active(self) -> Iterator["ThresholdOffload"]:
        self._frozen = {_storage_id(t) for t in (*self.model.parameters(), *self.model.buffers())}
        with torch.autograd.graph.saved_tensors_hooks(self._pack, self._unpack):
            yield self


@contextlib.contextmanager
def offload_scope(model: torch.nn.Module, *, enabled: bool, label: str, min_bytes: int, pin_memory: bool = True,
                  include_cpu: bool = False) -> Iterator[ThresholdOffload | None]:
    """``ThresholdOffload`` active for the duration, or ``None`` when the policy is off."""
    if not enabled:
        yield None
        return
    policy = ThresholdOffload(model, min_bytes=min_bytes, label=label, pin_memory=pin_memory,
                              include_cpu=include_cpu)
    with policy.active():
        yield policy
