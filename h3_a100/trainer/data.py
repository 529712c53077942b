"""Synthetic latent dataset and a pinned, prefetching host loader.

The reference reads a LightX2V latent/prompt cache (``latent_dataset``, 96
samples, ``node0_timing.log:7``) with ``pin_memory: true``.  There is no
dataset here, so each sample is generated deterministically from
``(data_seed, global index)``: N(0,1) video and audio latents of the
configured shape and N(0,1) text conditioning embeddings.  Samples carry a
rank-qualified identity in ``meta`` (``row_index``, ``id``, ``lmdb_path``) so
the matched-compute census can prove every rank consumed distinct samples.

Data parallelism: rank ``r`` of ``W`` reads indices ``r, r+W, r+2W, ...`` of an
epoch permutation (seeded, identical on all ranks), so samples never repeat
across ranks within an epoch.  ``PinnedLoader`` builds the next samples on a
host thread into pinned memory; ``to_device`` issues the host->device copies
with ``non_blocking=True`` (the only per-step input traffic).
"""

from __future__ import annotations

import queue
import threading
from typing import Any, Iterator

import torch

from ..config import get


class SyntheticLatentDataset:
    def __init__(self, config: dict[str, Any]) -> None:
        syn = get(config, "synthetic", {}) or {}
        self.size = int(syn.get("num_samples", 96))
        self.seed = int(syn.get("data_seed", 20260817))
        self.video_shape = tuple(int(v) for v in syn["video_latent_shape"])      # [C, F, H, W]
        audio = syn.get("audio_latent_shape")
        self.audio_shape = tuple(int(v) for v in audio) if audio else None      # [C, L]
        self.text_shape = tuple(int(v) for v in syn["text_shape"])               # [L, D]
        self.dtype = {"bf16": torch.bfloat16, "fp32": torch.float32}[str(syn.get("data_dtype", "bf16"))]
        self.path = f"synthetic://h3/{self.seed}"

    def __len__(self) -> int:
        return self.size

    def sample(self, index: int, *, pin: bool = False) -> dict[str, Any]:
        gen = torch.Generator().manual_seed(self.seed * 1_000_003 + int(index))

        def normal(shape):
            t = torch.randn((1,) + tuple(shape), generator=gen, dtype=torch.float32).to(self.dtype)
            return t.pin_memory() if pin else t

        out = {
            "video_latent": normal(self.video_shape),
            "audio_latent": normal(self.audio_shape) if self.audio_shape else None,
            "text": normal(self.text_shape),
            "meta": {"id": f"h3-synthetic-{index:08d}", "row_index": int(index), "lmdb_path": self.path},
        }
        return out


def rank_indices(size: int, rank: int, world: int, seed: int, epoch: int) -> list[int]:
    gen = torch.Generator().manual_seed(int(seed) * 31 + int(epoch))
    perm = torch.randperm(size, generator=gen).tolist()
    usable = size - size % world
    return perm[rank:usable:world]


class PinnedLoader:
    """Infinite per-rank iterator over the dataset with a host prefetch thread."""

    def __init__(self, dataset: SyntheticLatentDataset, *, rank: int, world: int, pin_memory: bool,
                 prefetch: int = 6, shuffle: bool = True) -> None:
        if len(dataset) < world:
            raise ValueError(f"dataset of {len(dataset)} samples cannot feed {world} ranks")
        self.dataset, self.rank, self.world = dataset, rank, world
        self.pin = bool(pin_memory) and torch.cuda.is_available()
        self.shuffle = shuffle
        self._queue: queue.Queue = queue.Queue(maxsize=max(1, prefetch))
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._produce, daemon=True)
        self._thread.start()

    def _indices(self) -> Iterator[int]:
        epoch = 0
        while True:
            if self.shuffle:
                idx = rank_indices(len(self.dataset), self.rank, self.world, self.dataset.seed, epoch)
            else:
                usable = len(self.dataset) - len(self.dataset) % self.world
                idx = list(range(self.rank, usable, self.world))
            yield from idx
            epoch += 1

    def _produce(self) -> None:
        for index in self._indices():
            if self._stop.is_set():
                return
            item = self.dataset.sample(index, pin=self.pin)
            while not self._stop.is_set():
                try:
                    self._queue.put(item, timeout=0.1)
                    break
                except queue.Full:
                    continue

    def __iter__(self):
        return self

    def __next__(self) -> dict[str, Any]:
        return self._queue.get()

    def close(self) -> None:
        """Stop the producer and join it (a daemon thread killed inside a torch
        call at interpreter exit can abort the process)."""
        self._stop.set()
        if self._thread.is_alive() and self._thread is not threading.current_thread():
            self._thread.join(timeout=30)


def to_device(sample: dict[str, Any], device: torch.device) -> dict[str, Any]:
    """Host->device copies of one sample's tensors (non-blocking from pinned memory)."""
    out = {}
    for key, value in sample.items():
        out[key] = value.to(device, non_blocking=True) if torch.is_tensor(value) else value
    return out


def sample_nbytes(sample: dict[str, Any]) -> int:
    return sum(v.numel() * v.element_size() for v in sample.values() if torch.is_tensor(v))
