"""One physical frozen backbone serving three logical roles.

Parity with the reference's ``MiniMaxH3A100Model``
(``h3_a100/model.py:154-453``): Student LoRA, Fake LoRA and Teacher (adapters
off) share one frozen DiT; both adapter sets are trainable and owned by
disjoint optimizers; the AdaLN bank is installed before sharding; modulations
are precomputed per exact timestep key.  Differences by design:

* the role is an explicit argument of every forward (``predict_velocity``);
  ``role_scope`` only sets the default role of calls that name none;
* AdaLN keys are explicit too: ``precompute_adaln`` builds a key's table and
  every forward/backward that reads it names it (``adaln_scope`` holds the
  table resident meanwhile);
* adapters are flat per-role buffers (``LoRAStore``), not PEFT modules;
* sharding is this package's own runtime (``h3_a100.parallel.sharded``), with
  the reference's unit plan: time embedder, each AdaLN projection, each
  refiner/transformer block, root.
"""

from __future__ import annotations

import contextlib
import os
from collections.abc import Iterator
from typing import Any

import torch
from safetensors.torch import load_file, save_file

from ..config import get
from ..parallel.sharded import ShardedProjection, ShardedUnit, link_order
from ..utils.log import logger
from .adaln import ModulationCache
from .block import H3Block
from .dit import DiTConfig, H3DiT
from .lora import FAKE, STUDENT, TEACHER, TRAINABLE_ROLES, LoRALayout, LoRAStore, target_modules_supported

STUDENT_ADAPTER, FAKE_ADAPTER, BASE_ROLE = STUDENT, FAKE, TEACHER
LORA_FILE = "pytorch_lora_weights.safetensors"


def dit_config_from(config: dict[str, Any]) -> DiTConfig:
    model = dict(get(config, "synthetic.model", {}) or {})
    model.setdefault("video_channels", int(get(config, "model.video_latent_channels", 16)))
    if "audio_channels" not in model:
        model["audio_channels"] = int(get(config, "model.audio_latent_channels", 0)) if get(
            config, "synthetic.audio_tokens", 0) else 0
    if "patch" not in model:
        model["patch"] = tuple(get(config, "model.patch_size", (1, 2, 2)))
    return DiTConfig.from_dict(model)


def sequence_tokens(config: dict[str, Any]) -> int:
    """Joint sequence length: patchified video + text + audio tokens."""
    dit = dit_config_from(config)
    v = get(config, "synthetic.video_latent_shape", [0, 0, 0, 0])
    tokens = (v[1] // dit.patch[0]) * (v[2] // dit.patch[1]) * (v[3] // dit.patch[2])
    tokens += int((get(config, "synthetic.text_shape") or [0])[0])
    tokens += int((get(config, "synthetic.audio_latent_shape") or [0, 0])[1])
    return tokens


class H3SharedBackbone:
    def __init__(self, config: dict[str, Any], *, device: torch.device, kernels, comm=None) -> None:
        self.config = config
        self.device = device
        self.kernels = kernels
        self.comm = comm
        self.dit_config = dit_config_from(config)
        dtype_name = str(get(config, "model.transformer_param_dtype", "bf16"))
        self.param_dtype = {"bf16": torch.bfloat16, "fp32": torch.float32, "fp16": torch.float16}[dtype_name]
        self.base_seed = int(get(config, "synthetic.base_seed", 1234))
        self.transformer = H3DiT(self.dit_config, dtype=self.param_dtype, device=device)
        self.transformer.init_weights(self.base_seed)
        self.transformer.set_kernels(kernels)
        self._default_role = STUDENT
        self.modulations: ModulationCache | None = None
        self.lora: dict[str, LoRAStore] = {}
        self.units: list[ShardedUnit] = []
        self.projections: list[ShardedProjection] = []
        self._ready = False

    # ------------------------------------------------------------------ setup
    def denoiser_module(self) -> H3DiT:
        return self.transformer

    def prepare_shared_backbone(self, *, student_lora: dict, fake_lora: dict, cache_enabled: bool = True,
                                max_dynamic_cache_keys: int = 2, alloc=None, pad_to: int = 1) -> None:
        if self._ready:
            return
        dit = self.transformer
        dit.requires_grad_(False)
        self.modulations = ModulationCache.attach(dit.adaln_bank, dit.time_embedder, enabled=cache_enabled,
                                                  max_dynamic_keys=max_dynamic_cache_keys)
        prefixes = [b.prefix for b in dit.token_refiner.refiner_blocks] + [b.prefix for b in dit.transformer_blocks]
        for role, lcfg in ((STUDENT, student_lora), (FAKE, fake_lora)):
            target_modules_supported(lcfg.get("target_modules", ()))
            rank = int(lcfg["rank"])
            layout = LoRALayout(prefixes, self.dit_config.hidden, self.dit_config.ffn, rank)
            seed = self.base_seed * 7919 + (1 if role == STUDENT else 2)
            self.lora[role] = LoRAStore(role, layout, alpha=float(lcfg.get("alpha", rank)),
                                        dtype=self.param_dtype, device=self.device, seed=seed,
                                        alloc=alloc, pad_to=pad_to)
        counts = {role: store.numel() for role, store in self.lora.items()}
        if not all(counts.values()):
            raise RuntimeError(f"failed to build LoRA adapters: {counts}")
        self._ready = True
        logger.info("[h3-a100] shared backbone ready student_lora_params={} fake_lora_params={}",
                    counts[STUDENT], counts[FAKE])

    def apply_sharding(self, comm, *, block_reshard: bool = True, root_reshard: bool = False) -> None:
        """Shard frozen weights with the reference unit plan (time MLP, AdaLN each, blocks, root)."""
        self.comm = comm
        dit = self.transformer
        units = []
        for blk in list(dit.token_refiner.refiner_blocks) + list(dit.transformer_blocks):
            unit = ShardedUnit(blk.prefix, blk, list(H3Block.WEIGHT_NAMES), comm,
                               reshard_after_forward=block_reshard)
            blk.attach_unit(unit)
            units.append(unit)
        link_order(units)
        self.units = units
        if comm.world_size > 1:
            self.projections = [ShardedProjection(p, comm, self.kernels) for p in dit.adaln_bank.projections]
            dit.sharded_projections = self.projections
        # time embedder, embeds and heads are small: kept replicated (root unit, not resharded).
        del root_reshard
        torch.cuda.empty_cache() if torch.cuda.is_available() else None

    def is_sharded(self) -> bool:
        return bool(self.units) and self.units[0].world > 1

    # ------------------------------------------------------------------ roles
    def role_parameters(self, role: str) -> list[torch.Tensor]:
        if role not in TRAINABLE_ROLES:
            raise ValueError(f"role {role!r} has no trainable parameters")
        return [self.lora[role].flat]

    def lora_store(self, role: str) -> LoRAStore | None:
        if role == TEACHER:
            return None
        if role not in self.lora:
            raise ValueError(f"unknown role {role!r}")
        return self.lora[role]

    @contextlib.contextmanager
    def role_scope(self, role: str) -> Iterator[None]:
        """Default role of ``predict_velocity`` calls that name none, for the duration."""
        if role not in (STUDENT, FAKE, TEACHER):
            raise ValueError(f"unknown role {role!r}")
        previous, self._default_role = self._default_role, role
        try:
            yield
        finally:
            self._default_role = previous

    def current_role(self) -> str:
        return self._default_role

    # ------------------------------------------------------------------ AdaLN
    def adaln_cache(self) -> ModulationCache:
        if self.modulations is None:
            raise RuntimeError("the AdaLN modulation cache is set up by prepare_shared_backbone")
        return self.modulations

    @contextlib.contextmanager
    def adaln_scope(self, key: Any) -> Iterator[None]:
        """Keep ``key``'s modulation table resident while a forward or backward reads it."""
        with self.adaln_cache().hold(key):
            yield

    def precompute_adaln(self, key: Any, timesteps: torch.Tensor, *, persistent: bool) -> None:
        """Materialise every block's modulation for one exact timestep table (no-op if present)."""
        dit = self.transformer
        if not self.adaln_cache().enabled:
            return     # cache off: every block projects its own modulation
        self.adaln_cache().build(key, persistent=persistent,
                                 temb=lambda: dit.time_embedding(timesteps.to(self.device)),
                                 project=dit.project_adaln)

    def drop_adaln_key(self, key: Any) -> None:
        self.adaln_cache().release(key)

    def log_adaln_stats(self, prefix: str = "[h3-a100]") -> None:
        s = self.adaln_cache().stats()
        logger.info("{} AdaLN cache hits={} misses={} stores={} evictions={} persistent_keys={} "
                    "dynamic_keys={} memory_mib={:.2f}", prefix, s.hits, s.misses, s.stores, s.evictions,
                    s.persistent_keys, s.dynamic_keys, s.bytes / 1024**2)

    # ------------------------------------------------------------------ forward
    def predict_velocity(self, role: str | None, latents, timesteps: torch.Tensor, condition: dict, *,
                         adaln_key=None):
        role = role or self._default_role
        video, audio = latents
        cache = self.modulations if (self.modulations is not None and self.modulations.enabled) else None
        return self.transformer(video, audio, condition["text"], timesteps, role=role,
                                lora_store=self.lora_store(role), adaln_key=adaln_key if cache else None,
                                modulations=cache)

    # ------------------------------------------------------------------ LoRA IO
    def save_all_role_loras(self, student_dir: str, fake_dir: str, *, main_process: bool = True) -> None:
        """Rank 0 writes both roles in Diffusers key format (adapters are replicated)."""
        if not main_process:
            return
        for role, out in ((STUDENT, student_dir), (FAKE, fake_dir)):
            os.makedirs(out, exist_ok=True)
            save_file(self.lora[role].state_dict(), os.path.join(out, LORA_FILE))

    def load_role_lora(self, load_dir: str, role: str) -> None:
        state = load_file(os.path.join(load_dir, LORA_FILE))
        self.lora[role].load_state_dict(state)

    def memory_report(self) -> dict[str, int]:
        frozen_local = sum(u.local_bytes() for u in self.units) + sum(p.local_bytes() for p in self.projections)
        lora = {role: s.flat.numel() * s.flat.element_size() for role, s in self.lora.items()}
        return {"frozen_local_bytes": int(frozen_local), **{f"lora_{k}_bytes": v for k, v in lora.items()}}
