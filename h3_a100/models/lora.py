"""Native multi-adapter LoRA storage: one flat buffer per role.

The reference adds two named PEFT adapters ("student", "fake") to the frozen
backbone and switches them with ``set_adapter`` / ``disable_adapters``
(``h3_a100/model.py:200-333``).  Here each role owns one contiguous buffer that
holds every LoRA matrix of every block, so that

* the optimizer, the gradient reduce-scatter and the checkpoint writer work on
  one flat tensor per role (no per-parameter launches);
* a block's adapters are views into that buffer, laid out so the fused QKV
  GEMM reads ``A_cat = [A_q; A_k; A_v]`` and ``B_cat = [B_q; B_k; B_v]``
  directly;
* the Teacher role is "no adapter" (the frozen base alone).

Init follows PEFT's "gaussian" mode: ``A ~ N(0, (1/r)^2)``, ``B = 0``, so all
three roles coincide at step 0 (the reference's first-cycle ``dmd=0``).
Checkpoint keys use the Diffusers LoRA naming
(``transformer_blocks.{i}.attn.to_q.lora_A.weight``).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

STUDENT = "student"
FAKE = "fake"
TEACHER = "teacher"
TRAINABLE_ROLES = (STUDENT, FAKE)
DEFAULT_TARGETS = ("to_q", "to_k", "to_v", "to_out.0", "ff.net.0.proj", "ff.net.2")


@dataclass(frozen=True)
class LinearSpec:
    """One LoRA-carrying linear group of a block (QKV is one group of 3 sections)."""

    name: str            # "qkv", "o", "ff0", "ff2"
    in_features: int
    out_features: int    # total over sections
    sections: int
    module_names: tuple[str, ...]  # Diffusers module name per section


def block_linear_specs(hidden: int, ffn: int) -> tuple[LinearSpec, ...]:
    return (
        LinearSpec("qkv", hidden, 3 * hidden, 3, ("attn.to_q", "attn.to_k", "attn.to_v")),
        LinearSpec("o", hidden, hidden, 1, ("attn.to_out.0",)),
        LinearSpec("ff0", hidden, ffn, 1, ("ff.net.0.proj",)),
        LinearSpec("ff2", ffn, hidden, 1, ("ff.net.2",)),
    )


_TARGET_OF_MODULE = {
    "attn.to_q": "to_q",
    "attn.to_k": "to_k",
    "attn.to_v": "to_v",
    "attn.to_out.0": "to_out.0",
    "ff.net.0.proj": "ff.net.0.proj",
    "ff.net.2": "ff.net.2",
}


@dataclass(frozen=True)
class Segment:
    block: str           # module prefix, e.g. "transformer_blocks.7"
    linear: str          # "qkv" | "o" | "ff0" | "ff2"
    kind: str            # "A" or "B"
    offset: int
    rows: int
    cols: int

    @property
    def numel(self) -> int:
        return self.rows * self.cols


class LoRALayout:
    """Offsets of every A_cat / B_cat matrix inside a role's flat buffer."""

    def __init__(self, block_prefixes: list[str], hidden: int, ffn: int, rank: int) -> None:
        self.rank = int(rank)
        self.hidden, self.ffn = int(hidden), int(ffn)
        self.specs = block_linear_specs(hidden, ffn)
        self.segments: dict[tuple[str, str, str], Segment] = {}
        self.block_ranges: dict[str, tuple[int, int]] = {}
        offset = 0
        for prefix in block_prefixes:
            start = offset
            for spec in self.specs:
                a = Segment(prefix, spec.name, "A", offset, spec.sections * rank, spec.in_features)
                offset += a.numel
                b = Segment(prefix, spec.name, "B", offset, spec.out_features, rank)
                offset += b.numel
                self.segments[(prefix, spec.name, "A")] = a
                self.segments[(prefix, spec.name, "B")] = b
            self.block_ranges[prefix] = (start, offset)
        self.numel = offset
        self.block_prefixes = list(block_prefixes)

    def spec(self, linear: str) -> LinearSpec:
        return next(s for s in self.specs if s.name == linear)

    def diffusers_keys(self):
        """Yield (key, block, linear, kind, section) for the Diffusers state dict."""
        for prefix in self.block_prefixes:
            for spec in self.specs:
                for section, module in enumerate(spec.module_names):
                    for kind in ("A", "B"):
                        yield (f"{prefix}.{module}.lora_{kind}.weight", prefix, spec.name, kind, section)


class LoRAStore:
    """Flat bf16/fp32 parameters of one role plus an fp32 gradient sink."""

    def __init__(self, role: str, layout: LoRALayout, *, alpha: float, dtype: torch.dtype,
                 device: torch.device, seed: int, alloc=None, pad_to: int = 1) -> None:
        if role not in TRAINABLE_ROLES:
            raise ValueError(f"role {role!r} has no adapter")
        self.role = role
        self.layout = layout
        self.scale = float(alpha) / float(layout.rank)
        # Flat buffers are padded (zeros) so they split evenly over ranks for the
        # sharded optimizer; `alloc` may place them in peer-mapped memory.
        pad_to = max(1, int(pad_to))
        self.padded_numel = (layout.numel + pad_to - 1) // pad_to * pad_to
        self._alloc = alloc or (lambda n, dt: torch.zeros(n, dtype=dt, device=device))
        self.flat = self._alloc(self.padded_numel, dtype)
        self.grad: torch.Tensor | None = None
        gen = torch.Generator(device=device).manual_seed(int(seed))
        std = 1.0 / layout.rank
        for seg in layout.segments.values():
            if seg.kind == "A":
                view = self.flat[seg.offset:seg.offset + seg.numel]
                view.copy_(torch.randn(seg.numel, generator=gen, device=device, dtype=torch.float32) * std)

    # -- views --------------------------------------------------------------
    def view(self, block: str, linear: str, kind: str, flat: torch.Tensor | None = None) -> torch.Tensor:
        seg = self.layout.segments[(block, linear, kind)]
        src = self.flat if flat is None else flat
        return src[seg.offset:seg.offset + seg.numel].view(seg.rows, seg.cols)

    def adapters(self, block: str) -> dict[str, tuple[torch.Tensor, torch.Tensor]]:
        return {spec.name: (self.view(block, spec.name, "A"), self.view(block, spec.name, "B"))
                for spec in self.layout.specs}

    def ensure_grad(self) -> torch.Tensor:
        if self.grad is None:
            self.grad = self._alloc(self.padded_numel, torch.float32)
        return self.grad

    def grad_sinks(self, block: str) -> dict[str, tuple[torch.Tensor, torch.Tensor]]:
        grad = self.ensure_grad()
        return {spec.name: (self.view(block, spec.name, "A", grad), self.view(block, spec.name, "B", grad))
                for spec in self.layout.specs}

    def zero_grad(self) -> None:
        if self.grad is not None:
            self.grad.zero_()

    def numel(self) -> int:
        """Number of LoRA parameters (without padding)."""
        return self.layout.numel

    # -- Diffusers-format state dict -------------------------------------------
    def _section_view(self, flat: torch.Tensor, block: str, linear: str, kind: str, section: int) -> torch.Tensor:
        spec = self.layout.spec(linear)
        full = self.view(block, linear, kind, flat)
        if spec.sections == 1:
            return full
        rows = full.shape[0] // spec.sections
        return full[section * rows:(section + 1) * rows]

    def state_dict(self, flat: torch.Tensor | None = None) -> dict[str, torch.Tensor]:
        src = self.flat if flat is None else flat
        return {key: self._section_view(src, block, linear, kind, section).detach().cpu().contiguous()
                for key, block, linear, kind, section in self.layout.diffusers_keys()}

    def load_state_dict(self, state: dict[str, torch.Tensor], *, strict: bool = True) -> None:
        seen = set()
        for key, block, linear, kind, section in self.layout.diffusers_keys():
            if key not in state:
                if strict:
                    raise KeyError(f"missing LoRA key {key}")
                continue
            dst = self._section_view(self.flat, block, linear, kind, section)
            if tuple(state[key].shape) != tuple(dst.shape):
                raise ValueError(f"{key}: shape {tuple(state[key].shape)} != {tuple(dst.shape)}")
            dst.copy_(state[key].to(dst.dtype))
            seen.add(key)
        extra = set(state) - seen
        if strict and extra:
            raise KeyError(f"unexpected LoRA keys: {sorted(extra)[:4]}")


def target_modules_supported(targets) -> None:
    if tuple(sorted(targets)) != tuple(sorted(DEFAULT_TARGETS)):
        raise ValueError(
            f"LoRA target_modules must be {list(DEFAULT_TARGETS)} (the fused block layout); got {list(targets)}"
        )
