"""CLI entry point: ``python -m h3_a100.entrypoint --config <yaml>``.

Same flow as the reference (``h3_a100/entrypoint.py:26-71``): parse
``--config``, enable TF32, initialise distributed, seed ``base + rank``, build
data / model / trainer, ``train()``, and always tear the process group down.
"""

from __future__ import annotations

import argparse

import torch

from .api import build_trainer
from .config import load_config
from .parallel import distributed as pdist
from .utils.log import logger, setup_logger


def parse_args(argv=None):
    parser = argparse.ArgumentParser(description="Train the H3-shaped DMD student on B200")
    parser.add_argument("--config", required=True, help="Path to the YAML config")
    return parser.parse_args(argv)


def main(argv=None) -> None:
    args = parse_args(argv)
    config = load_config(args.config)
    torch.backends.cuda.matmul.allow_tf32 = True
    torch.backends.cudnn.allow_tf32 = True
    setup_logger(config)
    try:
        trainer = build_trainer(config)
        logger.info("[h3-a100] deterministic matched seed={} global_rank={}",
                    int(config.get("training", {}).get("seed", 42)) + pdist.get_rank(), pdist.get_rank())
        trainer.train()
    except Exception:
        logger.exception("H3 DMD training failed")
        raise
    finally:
        pdist.cleanup_distributed()


if __name__ == "__main__":
    main()
