"""Same-topology checkpoint / resume in the reference layout.

Layout (``h3_a100/checkpointing.py:57-97``; ``docs/DESIGN.md:103-115`` of the
reference)::

    checkpoint-%09d/
      student/pytorch_lora_weights.safetensors   (Diffusers LoRA keys, rank 0)
      fake/pytorch_lora_weights.safetensors
      rank-%04d.pt        optimizers x2, schedulers x2, torch/cuda/python/numpy RNG, world_size
      trainer_state.pt    {iteration, world_size, format: "h3-a100-shared-backbone-v1", base_seed, config_hash}
      _SUCCESS

The frozen base is synthetic, so ``trainer_state.pt`` also records the base
seed and a hash of the model config: resume rebuilds the same base and
refuses a different one.  Only directories with ``_SUCCESS`` are resumable;
``save_total_limit`` prunes the oldest complete checkpoints.
"""

from __future__ import annotations

import hashlib
import json
import os
import random
import re
import shutil

import numpy as np
import torch

from ..models.lora import FAKE, STUDENT
from ..parallel import distributed as pdist
from ..utils.log import logger

FORMAT = "h3-a100-shared-backbone-v1"
_DIR_RE = re.compile(r"^checkpoint-(\d{9})$")


def config_hash(config: dict) -> str:
    model = {k: config.get(k) for k in ("synthetic", "model")}
    blob = json.dumps(model, sort_keys=True, default=str).encode()
    return hashlib.sha256(blob).hexdigest()[:16]


def complete_checkpoints(output_dir: str) -> list[tuple[int, str]]:
    if not os.path.isdir(output_dir):
        return []
    found = []
    for name in os.listdir(output_dir):
        match = _DIR_RE.match(name)
        path = os.path.join(output_dir, name)
        if match and os.path.isfile(os.path.join(path, "_SUCCESS")):
            found.append((int(match.group(1)), path))
    return sorted(found)


def find_latest_checkpoint(output_dir: str) -> tuple[str | None, int]:
    found = complete_checkpoints(output_dir)
    if not found:
        return None, 0
    iteration, path = found[-1]
    return path, iteration


def prune_checkpoints(output_dir: str, keep: int) -> None:
    """Keep at most ``keep - 1`` old complete checkpoints (room for the one being written)."""
    if not keep or keep <= 0:
        return
    found = complete_checkpoints(output_dir)
    for _, path in found[: max(0, len(found) - (keep - 1))]:
        shutil.rmtree(path, ignore_errors=True)


class CheckpointMixin:
    def _resolve_resume_a100(self):
        if not self.auto_resume:
            return None, 0
        return find_latest_checkpoint(self.output_train_dir)

    def _load_role_weights_before_sharding(self, checkpoint_dir: str) -> None:
        state_path = os.path.join(checkpoint_dir, "trainer_state.pt")
        if os.path.isfile(state_path):
            state = torch.load(state_path, map_location="cpu", weights_only=False)
            if state.get("format") != FORMAT:
                raise RuntimeError(f"unknown checkpoint format {state.get('format')!r}")
            if state.get("config_hash") not in (None, config_hash(self.config)):
                raise RuntimeError("checkpoint was written for a different synthetic base model")
        for role in (STUDENT, FAKE):
            role_dir = os.path.join(checkpoint_dir, role)
            if not os.path.isdir(role_dir):
                raise RuntimeError(f"checkpoint is missing {role} LoRA dir: {checkpoint_dir}")
            self.model.load_role_lora(role_dir, role)

    def _rank_state_path(self, checkpoint_dir: str) -> str:
        return os.path.join(checkpoint_dir, f"rank-{pdist.get_rank():04d}.pt")

    def _load_rank_state_after_sharding(self, checkpoint_dir: str) -> None:
        path = self._rank_state_path(checkpoint_dir)
        if not os.path.isfile(path):
            raise RuntimeError(f"rank-local checkpoint state not found: {path}")
        state = torch.load(path, map_location="cpu", weights_only=False)
        if int(state["world_size"]) != pdist.get_world_size():
            raise RuntimeError(f"Checkpoint world_size={state['world_size']} does not match current "
                               f"{pdist.get_world_size()}")
        self.optimizers[STUDENT].load_state_dict(state["student_optimizer"])
        self.optimizers[FAKE].load_state_dict(state["fake_optimizer"])
        self.lr_schedulers[STUDENT].load_state_dict(state["student_scheduler"])
        self.lr_schedulers[FAKE].load_state_dict(state["fake_scheduler"])
        torch.set_rng_state(state["torch_rng"])
        if torch.cuda.is_available() and state.get("cuda_rng") is not None:
            torch.cuda.set_rng_state(state["cuda_rng"])
        random.setstate(state["python_rng"])
        np.random.set_state(state["numpy_rng"])
        if state.get("host_rng") is not None:
            self.host_rng.set_state(state["host_rng"])
        self._score_serial = int(state.get("score_serial", 0))
        logger.info("[h3-a100] resumed rank-local state from {}", path)

    def save_checkpoint_a100(self, iteration: int) -> str:
        main = pdist.is_main_process()
        if main:
            prune_checkpoints(self.output_train_dir, self.save_total_limit)
        ckpt = os.path.join(self.output_train_dir, f"checkpoint-{int(iteration):09d}")
        student_dir, fake_dir = os.path.join(ckpt, STUDENT), os.path.join(ckpt, FAKE)
        if main:
            os.makedirs(student_dir, exist_ok=True)
            os.makedirs(fake_dir, exist_ok=True)
        pdist.barrier()
        self.model.save_all_role_loras(student_dir, fake_dir, main_process=main)
        pdist.barrier()
        torch.save({
            "iteration": int(iteration),
            "world_size": pdist.get_world_size(),
            "student_optimizer": self.optimizers[STUDENT].state_dict(),
            "fake_optimizer": self.optimizers[FAKE].state_dict(),
            "student_scheduler": self.lr_schedulers[STUDENT].state_dict(),
            "fake_scheduler": self.lr_schedulers[FAKE].state_dict(),
            "torch_rng": torch.get_rng_state(),
            "cuda_rng": torch.cuda.get_rng_state() if torch.cuda.is_available() else None,
            "python_rng": random.getstate(),
            "numpy_rng": np.random.get_state(),
            "host_rng": self.host_rng.get_state(),
            "score_serial": self._score_serial,
        }, self._rank_state_path(ckpt))
        pdist.barrier()
        if main:
            torch.save({"iteration": int(iteration), "world_size": pdist.get_world_size(), "format": FORMAT,
                        "base_seed": self.model.base_seed, "config_hash": config_hash(self.config)},
                       os.path.join(ckpt, "trainer_state.pt"))
            with open(os.path.join(ckpt, "_SUCCESS"), "w", encoding="utf-8") as fh:
                fh.write("ok\n")
        pdist.barrier()
        logger.info("[h3-a100] checkpoint saved iteration={} path={}", iteration, ckpt)
        return ckpt
