"""Native per-block activation checkpointing.

``native_checkpoint(function, hidden)`` runs ``function`` without saving any
activation and saves only ``hidden`` (through ``ctx.save_for_backward``, so a
saved-tensor hook such as the boundary staging policy sees exactly one tensor
per call).  Backward recomputes ``function`` with grad enabled and
backpropagates through it.  This replaces the torch non-reentrant checkpoint
the reference wraps (``h3_a100/checkpoint_boundary_offload.py:187-336``): the
blocks here carry their replay context (role, AdaLN key, modulation) in the
callable itself, so nothing ambient has to survive until backward.

``torch_checkpoint`` is the library baseline (non-reentrant
``torch.utils.checkpoint``) for A/B runs.
"""

from __future__ import annotations

import functools

import torch
from torch.utils.checkpoint import checkpoint as _torch_checkpoint


class _NativeCheckpoint(torch.autograd.Function):
    @staticmethod
    def forward(ctx, function, hidden, *args):
        ctx.function = function
        ctx.args = args
        ctx.save_for_backward(hidden)
        return function(hidden, *args)

    @staticmethod
    def backward(ctx, grad_out):
        (hidden,) = ctx.saved_tensors
        replay_input = hidden.detach().requires_grad_(True)
        with torch.enable_grad():
            out = ctx.function(replay_input, *ctx.args)
        torch.autograd.backward(out, grad_out)
        ctx.function = None
        return (None, replay_input.grad) + (None,) * len(ctx.args)


def native_checkpoint(function, hidden: torch.Tensor, *args):
    if not torch.is_grad_enabled():
        return function(hidden, *args)
    if not hidden.requires_grad:
        # LoRA gradients are produced inside the replay; the node must exist
        # even when the boundary itself needs no gradient.
        hidden = hidden.detach().requires_grad_(True)
    return _NativeCheckpoint.apply(function, hidden, *args)


torch_checkpoint = functools.partial(_torch_checkpoint, use_reentrant=False)
