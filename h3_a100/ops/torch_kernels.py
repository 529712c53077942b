"""PyTorch implementation of the kernel set.

Two jobs: it is the fp32 CPU oracle every CUDA kernel is tested against, and,
with ``kernels.backend: torch`` on a GPU, it is the reference-equivalent
library path (cuBLAS GEMMs, SDPA attention) that the hand-written sm_100a
kernels are measured against.  Every function computes in fp32 and returns
the dtype of its main input unless stated otherwise.

Conventions shared with the native kernels (``h3_a100/ops/native.py``):

* hidden states are 2-D ``[T, H]`` (batch 1 per rank, as in the matched
  contract);
* a modulation row is chosen per token: tokens ``< split`` use row 0, the rest
  row 1 (video+text tokens come first, audio tokens last);
* LoRA for a linear with S output sections (the fused QKV has 3) is stored as
  ``A_cat [S*r, in]`` and ``B_cat [out, r]``; section ``s`` of the output uses
  rows ``s*r:(s+1)*r`` of ``A_cat`` and its own rows of ``B_cat``.  The LoRA
  scale ``s = alpha/r`` is applied exactly once, in ``lora_down``
  (``U = s * x A^T``) and in ``lora_dyb`` (``dyb = s * dy B``); every other
  LoRA term uses those scaled tensors;
* RoPE rotates interleaved pairs ``(2i, 2i+1)`` of every head with per-token
  tables ``cos, sin: [T, head_dim/2]`` (fp32).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

GELU_C = math.sqrt(2.0 / math.pi)


@dataclass
class Rope:
    cos: torch.Tensor
    sin: torch.Tensor
    head_dim: int
    section_width: int  # columns per output section (hidden size H)
    sections: tuple[int, ...] = (0, 1)  # output sections rotated (q and k)


@dataclass
class GatedResidual:
    residual: torch.Tensor
    gate: torch.Tensor  # [R, H]
    split: int


def _rows(t: int, split: int, table: torch.Tensor) -> torch.Tensor:
    """Expand a [R, H] table to [T, H] by the split rule (fp32)."""
    table = table.float()
    if table.shape[0] == 1 or split >= t:
        return table[0].expand(t, -1)
    if split <= 0:
        return table[1].expand(t, -1)
    return torch.cat([table[0].expand(split, -1), table[1].expand(t - split, -1)], 0)


def gelu_tanh(x: torch.Tensor) -> torch.Tensor:
    return 0.5 * x * (1.0 + torch.tanh(GELU_C * (x + 0.044715 * x * x * x)))


def gelu_tanh_grad(x: torch.Tensor) -> torch.Tensor:
    inner = GELU_C * (x + 0.044715 * x * x * x)
    th = torch.tanh(inner)
    return 0.5 * (1.0 + th) + 0.5 * x * (1.0 - th * th) * GELU_C * (1.0 + 3 * 0.044715 * x * x)


def rope_apply(y: torch.Tensor, rope: Rope, inverse: bool = False) -> torch.Tensor:
    """Rotate the selected sections of ``y [T, S*H]`` (returns a new fp32 tensor)."""
    t = y.shape[0]
    out = y.float().clone()
    sec_width = rope.section_width
    cos = rope.cos.float()[:, None, :]
    sin = rope.sin.float()[:, None, :]
    if inverse:
        sin = -sin
    for s in rope.sections:
        part = out[:, s * sec_width:(s + 1) * sec_width].view(t, -1, rope.head_dim // 2, 2)
        even, odd = part[..., 0].clone(), part[..., 1].clone()
        part[..., 0] = even * cos - odd * sin
        part[..., 1] = even * sin + odd * cos
    return out


class TorchKernels:
    name = "torch"
    native = False

    # ---------------- norm + AdaLN modulate ----------------
    def norm_modulate(self, x, shift, scale, split, eps=1e-6):
        xf = x.float()
        r = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
        y = xf * r * (1.0 + _rows(x.shape[0], split, scale)) + _rows(x.shape[0], split, shift)
        return y.to(x.dtype)

    def norm_modulate_bwd(self, x, dy, scale, split, eps=1e-6, add=None, gate=None):
        """dx = add + d(norm_modulate)/dx^T dy; with ``gate`` also returns gate[row] * dx."""
        xf, g = x.float(), dy.float() * (1.0 + _rows(x.shape[0], split, scale))
        r = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
        n = xf * r
        dx = r * (g - n * (g * n).mean(-1, keepdim=True))
        if add is not None:
            dx = dx + add.float()
        dx = dx.to(x.dtype)
        if gate is None:
            return dx
        return dx, (dx.float() * _rows(x.shape[0], split, gate)).to(x.dtype)

    # ---------------- linear layers with LoRA ----------------
    def lora_down(self, x, a_cat, scale=1.0):
        return (scale * (x.float() @ a_cat.float().t())).to(x.dtype)

    def _lora_up(self, y, u, b_cat, sections):
        n = y.shape[1]
        r = u.shape[1] // sections
        width = n // sections
        for s in range(sections):
            y[:, s * width:(s + 1) * width] += (
                u[:, s * r:(s + 1) * r].float() @ b_cat[s * width:(s + 1) * width].float().t()
            )
        return y

    def linear(self, x, w, b=None, u=None, b_cat=None, sections=1, epilogue=None):
        """y = x w^T + b (+ U B^T, the LoRA up-projection) then the epilogue.

        epilogue: None | "gelu" (returns (pre, post)) | Rope | GatedResidual.
        """
        if x.dtype == torch.float32:
            y = x @ w.t()
            if b is not None:
                y = y + b
        else:
            y = (torch.addmm(b, x, w.t()) if b is not None else x @ w.t()).float()
        if u is not None:
            y = self._lora_up(y, u, b_cat, sections)
        if epilogue is None:
            return y.to(x.dtype)
        if epilogue == "gelu":
            pre = y.to(x.dtype)
            return pre, gelu_tanh(pre.float()).to(x.dtype)
        if isinstance(epilogue, Rope):
            return rope_apply(y.to(x.dtype), epilogue).to(x.dtype)
        if isinstance(epilogue, GatedResidual):
            gate = _rows(x.shape[0], epilogue.split, epilogue.gate)
            return (epilogue.residual.float() + gate * y.to(x.dtype).float()).to(x.dtype)
        raise ValueError(f"unknown epilogue {epilogue!r}")

    def lora_dyb(self, dy, b_cat, sections, scale=1.0):
        n = dy.shape[1]
        width = n // sections
        parts = [dy[:, s * width:(s + 1) * width].float() @ b_cat[s * width:(s + 1) * width].float()
                 for s in range(sections)]
        return (scale * torch.cat(parts, 1)).to(dy.dtype)

    def linear_dx(self, dy, w, dyb=None, a_cat=None, gelu_pre=None):
        """dx = dy w + dyb A_cat; with ``gelu_pre`` also applies the GELU derivative."""
        if dy.dtype == torch.float32:
            dx = dy @ w
        else:
            dx = (dy @ w).float()
        if dyb is not None:
            dx = dx + dyb.float() @ a_cat.float()
        dx = dx.to(dy.dtype)
        if gelu_pre is not None:
            dx = self.gelu_bwd(dx, gelu_pre)
        return dx

    def lora_wgrad(self, dy, x, u, dyb, sections, grad_a, grad_b):
        """Accumulate dA_cat = dyb^T x and dB_s = dy_s^T U_s into the fp32 sinks."""
        grad_a += dyb.float().t() @ x.float()
        n = dy.shape[1]
        width = n // sections
        r = u.shape[1] // sections
        for s in range(sections):
            grad_b[s * width:(s + 1) * width] += (
                dy[:, s * width:(s + 1) * width].float().t() @ u[:, s * r:(s + 1) * r].float()
            )

    # ---------------- elementwise helpers ----------------
    def gelu_bwd(self, dy, pre):
        return (dy.float() * gelu_tanh_grad(pre.float())).to(dy.dtype)

    def gate_mul(self, dout, gate, split):
        return (dout.float() * _rows(dout.shape[0], split, gate)).to(dout.dtype)

    def rope_bwd(self, dqkv, rope: Rope):
        return rope_apply(dqkv, rope, inverse=True).to(dqkv.dtype)

    # ---------------- attention ----------------
    @staticmethod
    def _split_heads(qkv, heads, head_dim):
        t = qkv.shape[0]
        q, k, v = qkv.view(t, 3, heads, head_dim).permute(1, 2, 0, 3).unbind(0)
        return q, k, v

    def attention_fwd(self, qkv, heads, head_dim):
        q, k, v = self._split_heads(qkv, heads, head_dim)
        if qkv.dtype == torch.float32:
            s = (q @ k.transpose(-1, -2)) / math.sqrt(head_dim)
            lse = torch.logsumexp(s, -1)
            o = torch.softmax(s, -1) @ v
        else:
            o = F.scaled_dot_product_attention(q[None], k[None], v[None])[0]
            lse = None
        return o.transpose(0, 1).reshape(qkv.shape[0], heads * head_dim), lse

    def attention_bwd(self, qkv, o, lse, do, heads, head_dim):
        with torch.enable_grad():
            qkv_ = qkv.detach().requires_grad_(True)
            q, k, v = self._split_heads(qkv_, heads, head_dim)
            if qkv.dtype == torch.float32:
                p = torch.softmax((q @ k.transpose(-1, -2)) / math.sqrt(head_dim), -1)
                out = p @ v
            else:
                out = F.scaled_dot_product_attention(q[None], k[None], v[None])[0]
            out = out.transpose(0, 1).reshape(qkv.shape[0], heads * head_dim)
            (dqkv,) = torch.autograd.grad(out, qkv_, do)
        return dqkv

    # ---------------- small projections ----------------
    def adaln_project(self, temb, w, b):
        """SiLU(temb) @ w^T + b in fp32; temb [R, D_t], w [6H, D_t] -> [R, 6H]."""
        return F.silu(temb.float()) @ w.float().t() + b.float()

    # ---------------- optimizer ----------------
    def sum_squares(self, t):
        return t.float().pow(2).sum().reshape(1)

    def adamw_step(self, master, exp_avg, exp_avg_sq, grad, param_out, norm, *, lr, beta1, beta2, eps,
                   weight_decay, step, max_norm):
        g = grad.float()
        if max_norm and max_norm > 0:
            g = g * torch.clamp(max_norm / (norm.float() + 1e-6), max=1.0)
        master.mul_(1.0 - lr * weight_decay)
        exp_avg.mul_(beta1).add_(g, alpha=1.0 - beta1)
        exp_avg_sq.mul_(beta2).addcmul_(g, g, value=1.0 - beta2)
        bc1, bc2 = 1.0 - beta1 ** step, 1.0 - beta2 ** step
        denom = (exp_avg_sq.sqrt() / math.sqrt(bc2)).add_(eps)
        master.addcdiv_(exp_avg, denom, value=-lr / bc1)
        param_out.copy_(master[:param_out.numel()])

    # ---------------- DMD / flow elementwise ----------------
    def flow_step(self, xt, velocity, sigma, sigma_next, out_dtype):
        """(x0 = xt + sigma*v, xt' = xt + (sigma - sigma')*v) in one pass; x0 in fp32."""
        x0 = xt.float() + sigma * velocity.float()
        nxt = (xt.float() + (sigma - sigma_next) * velocity.float()).to(out_dtype)
        return x0, nxt

    def x0_from_velocity(self, xt, velocity, sigma):
        return xt.float() + sigma * velocity.float()

    def add_noise(self, x0, noise, sigma):
        return ((1.0 - sigma) * x0.float() + sigma * noise.float()).to(x0.dtype)

    def randn(self, shape, dtype, device, generator=None):
        return torch.randn(shape, dtype=dtype, device=device, generator=generator)

    def dmd_loss(self, generated, x0_fake, x0_real):
        from ..trainer.dmd_math import dmd_loss
        return dmd_loss(generated, x0_fake, x0_real)

    def mse_loss(self, pred, target):
        return torch.mean((pred.float() - target.float()) ** 2)
