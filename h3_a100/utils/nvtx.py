"""NVTX ranges with the reference's names (``h3/student_step`` ...); no-ops without CUDA."""

from __future__ import annotations

import contextlib

import torch


@contextlib.contextmanager
def nvtx(name: str):
    if torch.cuda.is_available():
        torch.cuda.nvtx.range_push(name)
        try:
            yield
        finally:
            torch.cuda.nvtx.range_pop()
    else:
        yield
