"""Synthetic MiniMax-H3-shaped text-to-audio+video DiT.

The reference trains Diffusers' ``MiniMaxH3Transformer3DModel`` (external; not
in its tree).  This is our own model with the structure the reference
exposes: a token refiner for the text conditioning
(``h3_a100/model.py:417``), a sinusoidal ``time_proj`` + ``time_embedder`` MLP
(``h3_a100/model.py:360-363``), 50 joint blocks each with its own large AdaLN
projection (``h3_a100/adaln_cache.py:3-11``), ``norm_out`` modulated by the
time embedding and per-modality output projections.

Sequence layout (per sample, batch 1 per rank): ``[video | text | audio]``.
Video latents ``[1, Cv, F, H, W]`` are patchified by ``patch=(1, 2, 2)``; audio
latents ``[1, Ca, L]`` give one token per latent frame.  The time table has two
rows (video sigma, audio sigma): video and text tokens are modulated by row 0,
audio tokens by row 1, which is how the reference's per-row timesteps
(``build_row_timesteps(layout, sigma_video, sigma_audio)``,
``h3_a100/trainer_runtime.py:75-78``) enter the blocks.

Weights are random-init and deterministic in ``synthetic.base_seed`` (same on
every rank); there is no checkpoint to load.
"""

from __future__ import annotations

import contextlib
import math
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F
from torch import nn

from ..memory.checkpoint import BlockCheckpointing
from ..ops.torch_kernels import Rope
from .adaln import AdaLNBank
from .block import BlockContext, H3Block
from .rope import rope_tables


@dataclass
class DiTConfig:
    hidden: int = 256
    heads: int = 4
    head_dim: int = 64
    ffn: int = 1024
    time_embed_dim: int = 384
    num_blocks: int = 4
    num_refiner_blocks: int = 2
    text_dim: int = 256
    video_channels: int = 16
    audio_channels: int = 0
    patch: tuple[int, int, int] = (1, 2, 2)
    freq_dim: int = 256
    rope_base: float = 10000.0
    eps: float = 1e-6
    num_train_timesteps: int = 1000
    extra: dict = field(default_factory=dict)

    def __post_init__(self) -> None:
        if self.heads * self.head_dim != self.hidden:
            raise ValueError(f"heads*head_dim={self.heads * self.head_dim} != hidden={self.hidden}")
        self.patch = tuple(int(p) for p in self.patch)

    @classmethod
    def from_dict(cls, d: dict) -> "DiTConfig":
        known = {f for f in cls.__dataclass_fields__}
        return cls(**{k: v for k, v in d.items() if k in known})

    def param_counts(self) -> dict[str, int]:
        h, f, dt = self.hidden, self.ffn, self.time_embed_dim
        block = 3 * h * h + 3 * h + h * h + h + f * h + f + h * f + h
        adaln = 6 * h * dt + 6 * h
        pc = self.video_channels * self.patch[0] * self.patch[1] * self.patch[2]
        misc = (self.freq_dim * dt + dt + dt * dt + dt          # time embedder
                + self.text_dim * h + h                         # text embed
                + pc * h + h + h * pc + pc                      # video in/out
                + 2 * h * dt + 2 * h)                           # norm_out
        if self.audio_channels:
            misc += 2 * (self.audio_channels * h) + h + self.audio_channels
        return {
            "blocks": self.num_blocks * block,
            "refiner": self.num_refiner_blocks * block,
            "adaln": self.num_blocks * adaln,
            "misc": misc,
            "frozen_total": (self.num_blocks + self.num_refiner_blocks) * block + self.num_blocks * adaln + misc,
        }


def timestep_embedding(t: torch.Tensor, dim: int, max_period: float = 10000.0) -> torch.Tensor:
    """Sinusoidal embedding [len(t), dim], cos half first."""
    half = dim // 2
    freqs = torch.exp(-math.log(max_period) * torch.arange(half, dtype=torch.float32, device=t.device) / half)
    args = t.float()[:, None] * freqs[None]
    return torch.cat([torch.cos(args), torch.sin(args)], -1)


class TimeEmbedder(nn.Module):
    def __init__(self, freq_dim: int, dim: int, dtype, device) -> None:
        super().__init__()
        self.linear_1 = nn.Linear(freq_dim, dim, dtype=dtype, device=device)
        self.linear_2 = nn.Linear(dim, dim, dtype=dtype, device=device)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.linear_2(F.silu(self.linear_1(x)))


class AdaLNProjection(nn.Module):
    """SiLU(temb) -> Linear(D_t, 6H); output [R, 6, H] fp32."""

    def __init__(self, dim_in: int, hidden: int, dtype, device) -> None:
        super().__init__()
        self.hidden = hidden
        self.weight = nn.Parameter(torch.empty(6 * hidden, dim_in, dtype=dtype, device=device), requires_grad=False)
        self.bias = nn.Parameter(torch.empty(6 * hidden, dtype=dtype, device=device), requires_grad=False)
        object.__setattr__(self, "_unit", None)
        object.__setattr__(self, "kernels", None)

    def attach_unit(self, unit) -> None:
        object.__setattr__(self, "_unit", unit)

    def forward(self, temb: torch.Tensor) -> torch.Tensor:
        if self._unit is not None:
            w = self._unit.gather()
            weight, bias = w["weight"], w["bias"]
        else:
            weight, bias = self.weight, self.bias
        kern = self.kernels
        if kern is None:
            out = F.silu(temb.float()) @ weight.float().t() + bias.float()
        else:
            out = kern.adaln_project(temb, weight, bias)
        if self._unit is not None:
            self._unit.release()
        return out.view(temb.shape[0], 6, self.hidden)


class _NormOutFn(torch.autograd.Function):
    @staticmethod
    def forward(fctx, x, shift, scale, split, kernels, eps):
        fctx.save_for_backward(x, scale)
        fctx.split, fctx.kernels, fctx.eps = split, kernels, eps
        return kernels.norm_modulate(x, shift, scale, split, eps)

    @staticmethod
    def backward(fctx, dy):
        x, scale = fctx.saved_tensors
        return fctx.kernels.norm_modulate_bwd(x, dy.contiguous(), scale, fctx.split, fctx.eps), None, None, None, None, None


@dataclass
class TokenLayout:
    grid: tuple[int, int, int]   # latent patch grid (F, H/ph, W/pw)
    n_video: int
    n_text: int
    n_audio: int

    @property
    def total(self) -> int:
        return self.n_video + self.n_text + self.n_audio

    @property
    def split(self) -> int:
        return self.n_video + self.n_text


class H3DiT(nn.Module):
    def __init__(self, cfg: DiTConfig, *, dtype=torch.bfloat16, device="cpu") -> None:
        super().__init__()
        self.cfg = cfg
        h = cfg.hidden
        pc = cfg.video_channels * cfg.patch[0] * cfg.patch[1] * cfg.patch[2]
        self.patch_embed = nn.Linear(pc, h, dtype=dtype, device=device)
        self.text_embed = nn.Linear(cfg.text_dim, h, dtype=dtype, device=device)
        self.audio_embed = nn.Linear(cfg.audio_channels, h, dtype=dtype, device=device) if cfg.audio_channels else None
        self.time_embedder = TimeEmbedder(cfg.freq_dim, cfg.time_embed_dim, dtype, device)
        self.token_refiner = nn.Module()
        self.token_refiner.refiner_blocks = nn.ModuleList(
            [H3Block(h, cfg.ffn, f"token_refiner.refiner_blocks.{i}", dtype=dtype, device=device)
             for i in range(cfg.num_refiner_blocks)]
        )
        self.transformer_blocks = nn.ModuleList(
            [H3Block(h, cfg.ffn, f"transformer_blocks.{i}", dtype=dtype, device=device)
             for i in range(cfg.num_blocks)]
        )
        # One projection per joint block, owned by the bank (each its own sharded unit).
        self.adaln_bank = AdaLNBank([AdaLNProjection(cfg.time_embed_dim, h, dtype, device)
                                     for _ in range(cfg.num_blocks)])
        self.norm_out = nn.Linear(cfg.time_embed_dim, 2 * h, dtype=dtype, device=device)
        self.proj_out = nn.Linear(h, pc, dtype=dtype, device=device)
        self.proj_out_audio = nn.Linear(h, cfg.audio_channels, dtype=dtype, device=device) if cfg.audio_channels else None
        self.requires_grad_(False)
        self.checkpointing: BlockCheckpointing | None = None
        # Optional ``probe(block_index, "before"|"after")`` around every joint
        # block execution (per-block memory attribution); None costs nothing.
        self.block_probe = None
        self._rope_cache: dict = {}
        self.kernels = None

    # ---------------- init ----------------
    @torch.no_grad()
    def init_weights(self, seed: int) -> None:
        """Deterministic N(0, 1/fan_in) weights, zero biases except AdaLN (small)."""
        gen = torch.Generator(device="cpu").manual_seed(int(seed))
        for name, p in self.named_parameters(recurse=True):
            if "lora" in name:
                continue
            sub = torch.Generator(device=p.device if p.device.type == "cuda" else "cpu")
            sub.manual_seed(int(torch.randint(0, 2**62, (1,), generator=gen)))
            if p.dim() >= 2:
                std = 1.0 / math.sqrt(p.shape[-1])
                p.copy_(torch.randn(p.shape, generator=sub, device=sub.device, dtype=torch.float32).mul_(std).to(p.dtype))
            else:
                p.copy_(torch.randn(p.shape, generator=sub, device=sub.device, dtype=torch.float32).mul_(0.02).to(p.dtype))

    def set_kernels(self, kernels) -> None:
        self.kernels = kernels
        for module in self.modules():
            if isinstance(module, AdaLNProjection):
                object.__setattr__(module, "kernels", kernels)

    def enable_gradient_checkpointing(self, segment_size: int = 1) -> BlockCheckpointing:
        """Checkpoint every block (or every ``segment_size`` blocks) in grad forwards."""
        self.checkpointing = BlockCheckpointing(self.cfg.num_blocks, segment_size=segment_size)
        return self.checkpointing

    @property
    def gradient_checkpointing(self) -> bool:
        return self.checkpointing is not None

    # ---------------- layout helpers ----------------
    def token_layout(self, video_shape, audio_shape, text_len: int) -> TokenLayout:
        _, _, f, hh, ww = video_shape
        pf, ph, pw = self.cfg.patch
        grid = (f // pf, hh // ph, ww // pw)
        n_audio = int(audio_shape[-1]) if (audio_shape is not None and self.cfg.audio_channels) else 0
        return TokenLayout(grid, grid[0] * grid[1] * grid[2], int(text_len), n_audio)

    def rope(self, layout: TokenLayout, device) -> Rope:
        key = (layout.grid, layout.n_text, layout.n_audio, str(device))
        if key not in self._rope_cache:
            cos, sin = rope_tables(layout.grid, layout.n_text, layout.n_audio, self.cfg.head_dim,
                                   self.cfg.rope_base, device)
            self._rope_cache[key] = Rope(cos, sin, self.cfg.head_dim, self.cfg.hidden, (0, 1))
        return self._rope_cache[key]

    def patchify(self, video: torch.Tensor) -> torch.Tensor:
        b, c, f, hh, ww = video.shape
        pf, ph, pw = self.cfg.patch
        x = video.reshape(b, c, f // pf, pf, hh // ph, ph, ww // pw, pw)
        x = x.permute(0, 2, 4, 6, 1, 3, 5, 7)
        return x.reshape(b * (f // pf) * (hh // ph) * (ww // pw), c * pf * ph * pw)

    def unpatchify(self, tokens: torch.Tensor, video_shape) -> torch.Tensor:
        b, c, f, hh, ww = video_shape
        pf, ph, pw = self.cfg.patch
        x = tokens.reshape(b, f // pf, hh // ph, ww // pw, c, pf, ph, pw)
        x = x.permute(0, 4, 1, 5, 2, 6, 3, 7)
        return x.reshape(b, c, f, hh, ww)

    # ---------------- time embedding ----------------
    def time_embedding(self, timesteps: torch.Tensor) -> torch.Tensor:
        freq = timestep_embedding(timesteps, self.cfg.freq_dim)
        return self.time_embedder(freq.to(self.time_embedder.linear_1.weight.dtype))

    def adaln_projections(self):
        return list(self.adaln_bank.projections)

    def project_adaln(self, index: int, temb: torch.Tensor) -> torch.Tensor:
        """Block ``index``'s modulation ``[R, 6, H]`` fp32 from the time embedding.

        Uses the row-sharded projection when the bank is sharded across ranks
        (``sharded_projections``), else the bank's own weights.
        """
        sharded = getattr(self, "sharded_projections", None)
        if sharded:
            return sharded[index](temb).view(temb.shape[0], 6, self.cfg.hidden)
        return self.adaln_bank[index](temb)

    # ---------------- forward ----------------
    def forward(self, video: torch.Tensor, audio: torch.Tensor | None, text: torch.Tensor,
                timesteps: torch.Tensor, *, role: str = "student", lora_store=None, adaln_key=None,
                modulations=None):
        """Predict (video velocity, audio velocity).

        ``timesteps``: [2] (video t, audio t) in [0, num_train_timesteps].
        ``role``: the logical role of this forward (counted by the checkpoint plan).
        ``lora_store``: the active role's LoRAStore, or None for the Teacher.
        ``adaln_key`` + ``modulations``: the ``ModulationCache`` key whose table
        was precomputed; without them each block projects ``temb`` itself.
        """
        plan = self.checkpointing
        grad = torch.is_grad_enabled()
        with plan.forward(role, grad) if plan is not None else contextlib.nullcontext():
            return self._forward(video, audio, text, timesteps, lora_store, adaln_key, modulations,
                                 plan if grad else None)

    def _forward(self, video, audio, text, timesteps, lora_store, adaln_key, modulations, plan):
        kern = self.kernels
        dtype = self.patch_embed.weight.dtype
        layout = self.token_layout(video.shape, None if audio is None else audio.shape, text.shape[1])
        rope = self.rope(layout, video.device)
        grad_lora = torch.is_grad_enabled() and lora_store is not None
        scale = lora_store.scale if lora_store is not None else 1.0

        def block_ctx(block, modulation, split, rope_):
            return BlockContext(
                kernels=kern, modulation=modulation, split=split, rope=rope_,
                heads=self.cfg.heads, head_dim=self.cfg.head_dim, eps=self.cfg.eps,
                lora=None if lora_store is None else lora_store.adapters(block.prefix),
                lora_scale=scale,
                grad_sinks=lora_store.grad_sinks(block.prefix) if grad_lora else None,
            )

        # --- text refiner (unmodulated blocks over text tokens only) ---
        txt = F.linear(text[0].to(dtype), self.text_embed.weight, self.text_embed.bias)
        if grad_lora:
            txt = txt.detach().requires_grad_(False)
        ident = torch.zeros(1, 6, self.cfg.hidden, dtype=torch.float32, device=video.device)
        ident[:, 2] = 1.0
        ident[:, 5] = 1.0
        for blk in self.token_refiner.refiner_blocks:
            txt = blk(txt, block_ctx(blk, ident, txt.shape[0], None))

        # --- joint sequence ---
        vid = F.linear(self.patchify(video.to(dtype)), self.patch_embed.weight, self.patch_embed.bias)
        parts = [vid, txt]
        if layout.n_audio:
            aud = F.linear(audio[0].t().to(dtype), self.audio_embed.weight, self.audio_embed.bias)
            parts.append(aud)
        x = torch.cat(parts, 0).contiguous()

        with torch.no_grad():
            temb = self.time_embedding(timesteps)
        calls = [BlockCall(blk, block_ctx(blk, None, layout.split, rope), index, adaln_key, modulations,
                           self.project_adaln, temb, self.block_probe)
                 for index, blk in enumerate(self.transformer_blocks)]
        if plan is not None:
            for unit in plan.segments(calls):
                x = plan.run(unit, x)
        else:
            for call in calls:
                x = call(x)

        # --- output head ---
        with torch.no_grad():
            mod_out = (F.silu(temb.float()) @ self.norm_out.weight.float().t() + self.norm_out.bias.float())
            mod_out = mod_out.view(temb.shape[0], 2, self.cfg.hidden)
        x = _NormOutFn.apply(x, mod_out[:, 0], mod_out[:, 1], layout.split, kern, self.cfg.eps)
        v_tok = F.linear(x[:layout.n_video], self.proj_out.weight, self.proj_out.bias)
        v_video = self.unpatchify(v_tok, video.shape)
        v_audio = None
        if layout.n_audio:
            a_tok = F.linear(x[layout.split:], self.proj_out_audio.weight, self.proj_out_audio.bias)
            v_audio = a_tok.t().unsqueeze(0)
        return v_video, v_audio


class BlockCall:
    """One joint block with everything its execution needs, for the original run and replay.

    The LoRA views, RoPE table and AdaLN key are captured when the forward
    builds the call, so a checkpoint replay recomputes the block on exactly
    the same inputs.  Each execution reads the block's modulation once,
    through ``fetch(key, index)`` when it is given one (the replay audit's
    counting fetch) or the cache's own ``fetch``; with no key it projects
    ``temb`` itself (AdaLN cache disabled).
    """

    __slots__ = ("block", "ctx", "index", "key", "cache", "project", "temb", "probe")
    fetches = 1

    def __init__(self, block, ctx, index, key, cache, project, temb, probe=None):
        self.block, self.ctx, self.index = block, ctx, index
        self.key, self.cache, self.project, self.temb = key, cache, project, temb
        self.probe = probe

    def modulation(self, fetch=None) -> torch.Tensor:
        if self.key is not None and self.cache is not None:
            value = (fetch or self.cache.fetch)(self.key, self.index)
            if value is None:
                raise RuntimeError(f"AdaLN modulation for key {self.key!r} block {self.index} was not precomputed")
            return value
        return self.project(self.index, self.temb)

    def __call__(self, x, fetch=None):
        ctx = BlockContext(**{**self.ctx.__dict__, "modulation": self.modulation(fetch)})
        if self.probe is None:
            return self.block(x, ctx)
        self.probe(self.index, "before")
        out = self.block(x, ctx)
        self.probe(self.index, "after")
        return out
