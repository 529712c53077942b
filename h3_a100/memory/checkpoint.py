"""Per-block activation checkpointing of the DiT, with its policies attached explicitly.

The reference wraps the Diffusers transformer's ``_gradient_checkpointing_func``
twice (boundary staging, then the exact AdaLN replay scope) around torch's
non-reentrant checkpoint, and recovers role and AdaLN key from ambient
context in forward hooks (``h3_a100/checkpoint_boundary_offload.py:187-336``,
``h3_a100/exact_adaln_replay.py:50-142``).  Here the model is ours, so the
checkpoint itself owns both policies:

* ``BlockCheckpointing.run(call, hidden)`` is the checkpoint.  Its autograd
  node keeps exactly one tensor, the block input ``hidden``: either directly,
  or through ``BoundaryStaging.save`` (copied out to a staging slab and
  brought back by ``restore`` when backward replays the block).  Nothing else
  is saved; the block is recomputed in backward.
* The block call carries its own replay context (role's LoRA views, AdaLN
  key, RoPE table) and fetches its modulation through the function it is
  handed.  With a ``ReplayAudit`` attached, every execution (the original and
  the replay) goes through ``ReplayAudit.execute``, which hands the call a
  counting fetch and fails closed on a miss or a wrong number of reads.
* ``BlockCheckpointing.forward(role, grad)`` brackets one DiT forward: it
  counts forwards per role, checks that a grad forward made one checkpoint
  call per block (or per segment) and tells the staging policy.
* ``segment_size > 1`` groups consecutive block calls into one checkpointed
  segment (the reference's diagnostic SAC, ``h3_a100/model.py:40-75,235-269``):
  one saved boundary per segment.  It cannot be combined with boundary
  staging (``h3_a100/trainer.py:123-128``); the trainer rejects that.

``native_checkpoint(fn, hidden)`` is the same checkpoint without policies,
and ``torch_checkpoint`` the library baseline for A/B runs.
"""

from __future__ import annotations

import contextlib
import functools
from collections.abc import Iterator
from typing import Any, Callable

import torch
from torch.utils.checkpoint import checkpoint as _torch_checkpoint


class SegmentCall:
    """Consecutive block calls checkpointed as one unit (one saved boundary)."""

    def __init__(self, calls: list[Any], start: int) -> None:
        if not calls:
            raise ValueError("an activation-checkpoint segment cannot be empty")
        keys = {getattr(c, "key", None) for c in calls}
        if len(keys) != 1:
            raise ValueError("the block calls of one segment must share one AdaLN key")
        self.calls = list(calls)
        self.start = int(start)
        self.key = keys.pop()
        self.fetches = sum(int(getattr(c, "fetches", 1)) for c in calls)

    def __call__(self, hidden: torch.Tensor, fetch=None) -> torch.Tensor:
        for call in self.calls:
            hidden = call(hidden, fetch=fetch)
        return hidden


def group_calls(calls: list[Any], segment_size: int) -> list[Any]:
    """Block calls in segments of ``segment_size`` (size 1 keeps the calls themselves)."""
    segment_size = int(segment_size)
    if segment_size < 1:
        raise ValueError(f"activation checkpoint segment_size must be >= 1, got {segment_size}")
    if segment_size == 1:
        return list(calls)
    return [SegmentCall(calls[i:i + segment_size], i) for i in range(0, len(calls), segment_size)]


class _Checkpointed(torch.autograd.Function):
    """Runs ``call`` without keeping activations; backward recomputes it from the saved input."""

    @staticmethod
    def forward(ctx, plan, call, hidden):
        ctx.plan, ctx.call = plan, call
        if plan.staging is not None:
            ctx.boundary = plan.staging.save(hidden)
        else:
            ctx.boundary = None
            ctx.save_for_backward(hidden)
        return plan.execute(call, hidden)

    @staticmethod
    def backward(ctx, grad_out):
        plan = ctx.plan
        if ctx.boundary is not None:
            hidden = plan.staging.restore(ctx.boundary)
        else:
            (hidden,) = ctx.saved_tensors
        replay_input = hidden.detach().requires_grad_(True)
        with torch.enable_grad():
            out = plan.execute(ctx.call, replay_input)
        torch.autograd.backward(out, grad_out)
        ctx.call = ctx.boundary = None
        return None, None, replay_input.grad


class BlockCheckpointing:
    """Checkpoint plan of one DiT: segment size plus the optional staging and replay policies."""

    def __init__(self, num_blocks: int, *, segment_size: int = 1) -> None:
        if int(segment_size) < 1:
            raise ValueError(f"activation checkpoint segment_size must be >= 1, got {segment_size}")
        self.num_blocks = int(num_blocks)
        self.segment_size = int(segment_size)
        self.staging = None      # h3_a100.memory.boundary.BoundaryStaging
        self.replay = None       # h3_a100.memory.exact_replay.ReplayAudit
        self._calls = 0
        self.grad_forwards = 0

    @property
    def calls_per_grad_forward(self) -> int:
        return -(-self.num_blocks // self.segment_size)

    def attach_staging(self, staging) -> None:
        if self.segment_size != 1:
            raise ValueError("boundary staging needs one checkpoint per block (segment_size 1)")
        self.staging = staging

    def attach_replay(self, audit) -> None:
        self.replay = audit

    def segments(self, calls: list[Any]) -> list[Any]:
        return group_calls(calls, self.segment_size)

    @contextlib.contextmanager
    def forward(self, role: str, grad: bool) -> Iterator[None]:
        """One DiT forward of ``role``; a grad forward must checkpoint every block once."""
        self._calls = 0
        if self.staging is not None:
            self.staging.begin_forward(role, grad)
        yield
        if grad:
            if self._calls != self.calls_per_grad_forward:
                raise RuntimeError(f"grad forward of {role} made {self._calls} checkpoint calls, expected "
                                   f"{self.calls_per_grad_forward} ({self.num_blocks} blocks, "
                                   f"segment {self.segment_size})")
            self.grad_forwards += 1
        if self.staging is not None:
            self.staging.end_forward(role, grad, self._calls)

    def run(self, call, hidden: torch.Tensor) -> torch.Tensor:
        """Checkpoint one block call (or segment) on ``hidden``."""
        self._calls += 1
        grad = torch.is_grad_enabled()
        if self.staging is not None:
            self.staging.note_call(grad)
        if not grad:
            return self.execute(call, hidden)
        if self.replay is not None:
            self.replay.note_checkpoint(call)
        if not hidden.requires_grad:
            # LoRA gradients appear inside the replay: the node must exist even
            # when the block input itself needs no gradient.
            hidden = hidden.detach().requires_grad_(True)
        return _Checkpointed.apply(self, call, hidden)

    def execute(self, call, hidden: torch.Tensor) -> torch.Tensor:
        if self.replay is not None:
            return self.replay.execute(call, hidden)
        return call(hidden)


class _PlainCall:
    __slots__ = ("fn", "args")
    key = None
    fetches = 0

    def __init__(self, fn: Callable[..., torch.Tensor], args: tuple) -> None:
        self.fn, self.args = fn, args

    def __call__(self, hidden, fetch=None):
        return self.fn(hidden, *self.args)


_PLAIN = BlockCheckpointing(1)


def native_checkpoint(function: Callable[..., torch.Tensor], hidden: torch.Tensor, *args) -> torch.Tensor:
    """Checkpoint ``function(hidden, *args)`` saving only ``hidden`` (no staging, no audit)."""
    if not torch.is_grad_enabled():
        return function(hidden, *args)
    if not hidden.requires_grad:
        hidden = hidden.detach().requires_grad_(True)
    return _Checkpointed.apply(_PLAIN, _PlainCall(function, args), hidden)


torch_checkpoint = functools.partial(_torch_checkpoint, use_reentrant=False)
