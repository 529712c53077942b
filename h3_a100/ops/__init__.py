"""Kernel sets: the hand-written sm_100a kernels, or the PyTorch path.

``get_kernels(backend, device)`` is called once when the model is built
(``kernels.backend`` in the config): ``native`` selects ``NativeKernels``
(the compiled extension, required on a GPU; it raises if the extension is
missing rather than falling back), ``torch`` selects ``TorchKernels`` (the
CPU oracle, and on a GPU the cuBLAS/SDPA baseline).  Nothing inside the hot
path re-dispatches per call.
"""

from __future__ import annotations

import torch

from .torch_kernels import GatedResidual, Rope, TorchKernels

__all__ = ["GatedResidual", "Rope", "TorchKernels", "get_kernels"]


def get_kernels(backend: str, device: torch.device):
    backend = str(backend)
    if backend == "torch" or device.type != "cuda":
        return TorchKernels()
    if backend == "native":
        from .native import NativeKernels

        return NativeKernels(device)
    raise ValueError(f"unknown kernels.backend {backend!r} (expected 'native' or 'torch')")
