"""Logging: loguru with a rank field, as the reference's LightX2V logger does."""

from __future__ import annotations

import os
import sys

from loguru import logger

_CONFIGURED = {"done": False}


def setup_logger(config: dict | None = None, *, rank: int | None = None, log_file: str | None = None) -> None:
    rank = int(os.environ.get("RANK", 0)) if rank is None else rank
    rank_zero_only = bool(((config or {}).get("logging", {}) or {}).get("rank_zero_only", True))
    logger.remove()
    level = os.environ.get("H3_LOG_LEVEL", "INFO")
    if not rank_zero_only or rank == 0:
        logger.add(sys.stderr, level=level,
                   format="{time:YYYY-MM-DD HH:mm:ss.SSS} | {level} | rank=" + str(rank) + " | {message}")
    if log_file:
        logger.add(log_file, level=level)
    _CONFIGURED["done"] = True


__all__ = ["logger", "setup_logger"]
