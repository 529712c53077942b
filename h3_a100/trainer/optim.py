"""Flat AdamW with on-device global-norm clipping, and LR schedules.

The reference runs ``clip_grad_norm_`` then ``torch.optim.AdamW`` over each
role's LoRA parameters (``h3_a100/trainer_loop.py:130-133,203-206``;
``h3_a100/trainer.py:202-218``).  Here each role is one flat buffer, so one
optimizer step is: reduce gradients across ranks, one sum-of-squares pass,
then one fused pass that applies ``min(1, max_norm / (norm + 1e-6))`` and the
decoupled-weight-decay AdamW update to fp32 master weights and writes the
bf16 compute copy.  The clip coefficient stays on the device (no host sync).

With ``shard_states`` the fp32 master/moment buffers hold only this rank's
1/world slice (ZeRO-1): gradients are reduce-scattered, the slice is updated
and the new bf16 parameters are all-gathered.
"""

from __future__ import annotations

import math
from typing import Any

import torch


class LRSchedule:
    """constant | constant_with_warmup | linear | cosine (transformers-style)."""

    def __init__(self, base_lr: float, kind: str = "constant", warmup: int = 0, total: int = 1) -> None:
        self.base_lr, self.kind = float(base_lr), str(kind)
        self.warmup, self.total = int(warmup), max(1, int(total))
        self.last_step = 0
        if self.kind not in {"constant", "constant_with_warmup", "linear", "cosine"}:
            raise ValueError(f"unknown lr_scheduler {kind!r}")

    def _factor(self, step: int) -> float:
        if self.warmup and step < self.warmup:
            return step / max(1, self.warmup)
        if self.kind in {"constant", "constant_with_warmup"}:
            return 1.0
        progress = (step - self.warmup) / max(1, self.total - self.warmup)
        progress = min(max(progress, 0.0), 1.0)
        if self.kind == "linear":
            return 1.0 - progress
        return 0.5 * (1.0 + math.cos(math.pi * progress))

    def get_last_lr(self) -> list[float]:
        return [self.base_lr * self._factor(self.last_step)]

    def step(self) -> None:
        self.last_step += 1

    def state_dict(self) -> dict[str, Any]:
        return {"last_step": self.last_step, "base_lr": self.base_lr, "kind": self.kind,
                "warmup": self.warmup, "total": self.total}

    def load_state_dict(self, state: dict[str, Any]) -> None:
        self.last_step = int(state["last_step"])


class FlatAdamW:
    def __init__(self, store, *, lr: float, betas=(0.9, 0.999), weight_decay: float = 0.01, eps: float = 1e-8,
                 max_grad_norm: float = 1.0, kernels=None, comm=None, shard_states: bool = False) -> None:
        self.store = store
        self.lr, self.betas, self.weight_decay, self.eps = float(lr), tuple(betas), float(weight_decay), float(eps)
        self.max_grad_norm = float(max_grad_norm)
        self.kernels, self.comm = kernels, comm
        world = comm.world_size if comm is not None else 1
        # The peer-memory transport runs the whole step (reduce-scatter, norm,
        # clip, AdamW on the local shard, all-gather of the new parameters) in
        # one kernel, so it always shards the optimizer state.
        self.fused = world > 1 and hasattr(comm, "lora_step")
        self.shard = (bool(shard_states) or self.fused) and world > 1
        param = store.flat
        n = param.numel()
        if self.shard:
            self.chunk = (n + world - 1) // world
            self.padded = self.chunk * world
            lo = comm.rank * self.chunk
            hi = min(n, lo + self.chunk)
            self.lo, self.hi = lo, hi
            master = torch.zeros(self.chunk, dtype=torch.float32, device=param.device)
            master[:max(0, hi - lo)].copy_(param[lo:hi].float())
        else:
            self.chunk, self.padded, self.lo, self.hi = n, n, 0, n
            master = param.detach().float().clone()
        self.master = master
        self.exp_avg = torch.zeros_like(master)
        self.exp_avg_sq = torch.zeros_like(master)
        self.step_count = 0
        self.last_grad_norm: torch.Tensor | None = None

    def zero_grad(self) -> None:
        self.store.zero_grad()

    def state_bytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (self.master, self.exp_avg, self.exp_avg_sq))

    def step(self, lr: float | None = None) -> torch.Tensor:
        """Reduce grads, clip by global norm and update; returns the (device) pre-clip norm."""
        lr = self.lr if lr is None else float(lr)
        grad = self.store.ensure_grad()
        comm = self.comm
        k = self.kernels
        if self.fused:
            self.step_count += 1
            comm.lora_step(self, lr)
            self.last_grad_norm = comm.scratch[15:16]
            return self.last_grad_norm
        if self.shard:
            full = grad if grad.numel() == self.padded else torch.nn.functional.pad(grad, (0, self.padded - grad.numel()))
            local = torch.empty(self.chunk, dtype=torch.float32, device=grad.device)
            comm.reduce_scatter_(local, full, op="avg")
            sq = k.sum_squares(local)
            comm.all_reduce_(sq, op="sum")
        else:
            if comm is not None and comm.world_size > 1:
                comm.all_reduce_(grad, op="avg")
            local = grad
            sq = k.sum_squares(local)
        norm = sq.sqrt()
        self.step_count += 1
        b1, b2 = self.betas
        if self.shard:
            param_local = torch.empty(self.chunk, dtype=self.store.flat.dtype, device=grad.device)
            k.adamw_step(self.master, self.exp_avg, self.exp_avg_sq, local, param_local, norm,
                         lr=lr, beta1=b1, beta2=b2, eps=self.eps, weight_decay=self.weight_decay,
                         step=self.step_count, max_norm=self.max_grad_norm)
            gathered = torch.empty(self.padded, dtype=param_local.dtype, device=grad.device)
            comm.all_gather_into_(gathered, param_local)
            self.store.flat.copy_(gathered[:self.store.flat.numel()])
        else:
            k.adamw_step(self.master, self.exp_avg, self.exp_avg_sq, local, self.store.flat, norm,
                         lr=lr, beta1=b1, beta2=b2, eps=self.eps, weight_decay=self.weight_decay,
                         step=self.step_count, max_norm=self.max_grad_norm)
        self.last_grad_norm = norm
        return norm

    def state_dict(self) -> dict[str, Any]:
        return {"step": self.step_count, "master": self.master.cpu(), "exp_avg": self.exp_avg.cpu(),
                "exp_avg_sq": self.exp_avg_sq.cpu(), "lr": self.lr, "betas": self.betas,
                "weight_decay": self.weight_decay, "eps": self.eps, "shard": self.shard,
                "lo": self.lo, "hi": self.hi}

    def load_state_dict(self, state: dict[str, Any]) -> None:
        if (state["lo"], state["hi"]) != (self.lo, self.hi):
            raise RuntimeError("optimizer shard layout mismatch (world size changed?)")
        self.step_count = int(state["step"])
        self.master.copy_(state["master"])
        self.exp_avg.copy_(state["exp_avg"])
        self.exp_avg_sq.copy_(state["exp_avg_sq"])
