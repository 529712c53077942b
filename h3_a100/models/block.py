"""The H3-shaped DiT block with a hand-written forward and backward.

One block is: RMSNorm + AdaLN shift/scale -> fused QKV (+LoRA, RoPE in the
epilogue) -> bidirectional attention -> O-proj (+LoRA) with the gated
residual in the epilogue -> RMSNorm + shift/scale -> FF0 (+LoRA) + GELU(tanh)
-> FF2 (+LoRA) with the gated residual.  The reference runs the same structure
through Diffusers + PEFT + FA3 (``h3_a100/model.py:40-75`` shows the
``block(hidden_states, temb, adaln_indices, rotary_emb)`` signature and
``output_train.log:732-750`` the ``ff.net.0.proj`` / GELU / ``ff.net.2`` FFN).

Why an explicit backward: the base is frozen, so the only parameter
gradients are LoRA ones.  The backward writes them straight into the active
role's flat fp32 gradient sink (``LoRAStore.grad``) and returns only the
hidden-state gradient to autograd.  That keeps per-block LoRA gradients final
as soon as the block's backward returns (so they can be reduced per block),
and it lets every step be one kernel of the kernel set ``K`` (hand-written
sm_100a kernels, or the PyTorch oracle).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import nn

from ..ops.torch_kernels import GatedResidual, Rope

# modulation slots inside the [R, 6, H] table
SHIFT_MSA, SCALE_MSA, GATE_MSA, SHIFT_MLP, SCALE_MLP, GATE_MLP = range(6)


@dataclass
class BlockContext:
    """Everything a block call needs besides its input (captured for replay)."""

    kernels: object
    modulation: torch.Tensor          # [R, 6, H] fp32
    split: int
    rope: Rope | None
    heads: int
    head_dim: int
    eps: float
    lora: dict | None                 # linear -> (A_cat, B_cat) of the active role
    lora_scale: float
    grad_sinks: dict | None           # linear -> (dA_cat, dB_cat) fp32 views


def block_forward(ctx: BlockContext, x: torch.Tensor, w: dict[str, torch.Tensor], save: bool):
    K, mod, split, lo, s = ctx.kernels, ctx.modulation, ctx.split, ctx.lora, ctx.lora_scale

    def down(name, inp):
        return K.lora_down(inp, lo[name][0], s) if lo is not None else None

    def up(name):
        return lo[name][1] if lo is not None else None

    h1 = K.norm_modulate(x, mod[:, SHIFT_MSA], mod[:, SCALE_MSA], split, ctx.eps)
    u_qkv = down("qkv", h1)
    qkv = K.linear(h1, w["qkv_weight"], w["qkv_bias"], u_qkv, up("qkv"), 3, epilogue=ctx.rope)
    o, lse = K.attention_fwd(qkv, ctx.heads, ctx.head_dim)
    u_o = down("o", o)
    x1 = K.linear(o, w["out_weight"], w["out_bias"], u_o, up("o"), 1,
                  epilogue=GatedResidual(x, mod[:, GATE_MSA], split))
    h2 = K.norm_modulate(x1, mod[:, SHIFT_MLP], mod[:, SCALE_MLP], split, ctx.eps)
    u_f0 = down("ff0", h2)
    pre, act = K.linear(h2, w["ff0_weight"], w["ff0_bias"], u_f0, up("ff0"), 1, epilogue="gelu")
    u_f2 = down("ff2", act)
    out = K.linear(act, w["ff2_weight"], w["ff2_bias"], u_f2, up("ff2"), 1,
                   epilogue=GatedResidual(x1, mod[:, GATE_MLP], split))
    if not save:
        return out, None
    saved = dict(x=x, h1=h1, u_qkv=u_qkv, qkv=qkv, o=o, lse=lse, u_o=u_o, x1=x1, h2=h2,
                 u_f0=u_f0, pre=pre, act=act, u_f2=u_f2)
    return out, saved


def block_backward(ctx: BlockContext, dout: torch.Tensor, w: dict[str, torch.Tensor], sv: dict):
    K, mod, split, lo, s, sinks = ctx.kernels, ctx.modulation, ctx.split, ctx.lora, ctx.lora_scale, ctx.grad_sinks

    def lora_part(name, dy, inp, u, sections):
        """LoRA gradients of one linear; returns (s*dy*B, A_cat) for the input-gradient GEMM."""
        if lo is None:
            return None, None
        a_cat, b_cat = lo[name]
        dyb = K.lora_dyb(dy, b_cat, sections, s)
        if sinks is not None:
            K.lora_wgrad(dy, inp, u, dyb, sections, sinks[name][0], sinks[name][1])
        return dyb, a_cat

    # FF2 with gated residual: out = x1 + g_mlp * y2;  y2 = GELU(pre) W2^T + ...
    dy2 = K.gate_mul(dout, mod[:, GATE_MLP], split)
    dyb, a_cat = lora_part("ff2", dy2, sv["act"], sv["u_f2"], 1)
    dpre = K.linear_dx(dy2, w["ff2_weight"], dyb, a_cat, gelu_pre=sv["pre"])
    dyb, a_cat = lora_part("ff0", dpre, sv["h2"], sv["u_f0"], 1)
    dh2 = K.linear_dx(dpre, w["ff0_weight"], dyb, a_cat)
    # x1 feeds the MLP norm and the residual; its gradient also gives the O-proj branch (x1 = x + g_msa * y_o).
    dx1, dyo = K.norm_modulate_bwd(sv["x1"], dh2, mod[:, SCALE_MLP], split, ctx.eps, add=dout,
                                   gate=mod[:, GATE_MSA])
    dyb, a_cat = lora_part("o", dyo, sv["o"], sv["u_o"], 1)
    do = K.linear_dx(dyo, w["out_weight"], dyb, a_cat)
    dqkv = K.attention_bwd(sv["qkv"], sv["o"], sv["lse"], do, ctx.heads, ctx.head_dim)
    if ctx.rope is not None:
        dqkv = K.rope_bwd(dqkv, ctx.rope)
    dyb, a_cat = lora_part("qkv", dqkv, sv["h1"], sv["u_qkv"], 3)
    dh1 = K.linear_dx(dqkv, w["qkv_weight"], dyb, a_cat)
    return K.norm_modulate_bwd(sv["x"], dh1, mod[:, SCALE_MSA], split, ctx.eps, add=dx1)


class _BlockFn(torch.autograd.Function):
    """Autograd node of one block: saves activations, runs the explicit backward."""

    @staticmethod
    def forward(fctx, x, block, ctx):
        weights = block.weights()
        out, saved = block_forward(ctx, x, weights, save=True)
        names = [k for k, v in saved.items() if v is not None]
        fctx.names = names
        fctx.block, fctx.ctx = block, ctx
        fctx.save_for_backward(*[saved[k] for k in names])
        block.release_weights()
        return out

    @staticmethod
    def backward(fctx, dout):
        saved = dict(zip(fctx.names, fctx.saved_tensors))
        for key in ("u_qkv", "u_o", "u_f0", "u_f2", "lse"):
            saved.setdefault(key, None)
        weights = fctx.block.weights(backward=True)
        dx = block_backward(fctx.ctx, dout.contiguous(), weights, saved)
        fctx.block.release_weights()
        fctx.block.note_backward_done()
        return dx, None, None


class H3Block(nn.Module):
    """Frozen block weights (possibly sharded); the AdaLN projection lives in the DiT's bank."""

    WEIGHT_NAMES = ("qkv_weight", "qkv_bias", "out_weight", "out_bias",
                    "ff0_weight", "ff0_bias", "ff2_weight", "ff2_bias")

    def __init__(self, hidden: int, ffn: int, prefix: str, *, dtype: torch.dtype, device) -> None:
        super().__init__()
        self.prefix = prefix
        self.hidden, self.ffn = hidden, ffn

        def frozen(*shape):
            return nn.Parameter(torch.empty(*shape, dtype=dtype, device=device), requires_grad=False)

        self.qkv_weight, self.qkv_bias = frozen(3 * hidden, hidden), frozen(3 * hidden)
        self.out_weight, self.out_bias = frozen(hidden, hidden), frozen(hidden)
        self.ff0_weight, self.ff0_bias = frozen(ffn, hidden), frozen(ffn)
        self.ff2_weight, self.ff2_bias = frozen(hidden, ffn), frozen(hidden)
        object.__setattr__(self, "_unit", None)   # sharded-parameter unit, if any
        object.__setattr__(self, "_on_backward_done", None)

    # -- weights (local or gathered through the sharded runtime) -------------
    def attach_unit(self, unit) -> None:
        object.__setattr__(self, "_unit", unit)

    def weights(self, backward: bool = False) -> dict[str, torch.Tensor]:
        if self._unit is not None:
            return self._unit.gather(backward=backward)
        return {name: getattr(self, name) for name in self.WEIGHT_NAMES}

    def release_weights(self) -> None:
        if self._unit is not None:
            self._unit.release()

    def set_backward_hook(self, fn) -> None:
        object.__setattr__(self, "_on_backward_done", fn)

    def note_backward_done(self) -> None:
        if self._on_backward_done is not None:
            self._on_backward_done(self)

    def forward(self, x: torch.Tensor, ctx: BlockContext) -> torch.Tensor:
        if torch.is_grad_enabled() and (x.requires_grad or ctx.lora is not None):
            return _BlockFn.apply(x, self, ctx)
        weights = self.weights()
        out, _ = block_forward(ctx, x, weights, save=False)
        self.release_weights()
        return out
