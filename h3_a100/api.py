"""Programmatic construction of the full training stack from a config dict.

``build_trainer(config)`` is what the CLI and the benchmark call: it brings up
the process group, seeds ``base_seed + global rank`` (python / numpy / torch
/ cuda, as the reference's ``_seed_rank`` at ``h3_a100/entrypoint.py:32-40``),
selects the kernel set, builds the synthetic shared backbone and the data
loader, and returns a trainer that has not been set up yet.
"""

from __future__ import annotations

import random
from typing import Any

import numpy as np
import torch

from .config import get
from .models.shared_backbone import H3SharedBackbone
from .ops import get_kernels
from .parallel import distributed as pdist
from .trainer.data import PinnedLoader, SyntheticLatentDataset
from .trainer.trainer import H3DmdTrainer


def seed_rank(config: dict[str, Any]) -> int:
    seed = int(get(config, "training.seed", 42)) + pdist.get_rank()
    random.seed(seed)
    np.random.seed(seed % (2**32 - 1))
    torch.manual_seed(seed)
    if torch.cuda.is_available():
        torch.cuda.manual_seed_all(seed)
    return seed


def build_trainer(config: dict[str, Any], *, with_data: bool = True) -> H3DmdTrainer:
    pdist.init_distributed_a100(config)
    device = pdist.device()
    seed_rank(config)
    kernels = get_kernels(get(config, "kernels.backend", "native"), device)
    trainer = H3DmdTrainer(config, kernels=kernels, device=device)
    trainer.set_model(H3SharedBackbone(config, device=device, kernels=kernels))
    if with_data:
        dataset = SyntheticLatentDataset(config)
        loader = PinnedLoader(dataset, rank=pdist.get_rank(), world=pdist.get_world_size(),
                              pin_memory=bool(get(config, "data.train.pin_memory", True)),
                              shuffle=bool(get(config, "data.train.shuffle", True)))
        trainer.set_data(loader)
    return trainer
