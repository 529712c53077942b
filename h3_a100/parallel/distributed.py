"""Process-group bring-up and the small collective helpers the trainer uses.

One process per GPU, ``torch.distributed`` for the plumbing: NCCL on CUDA,
gloo on CPU (tests).  Mirrors ``init_distributed_a100`` in the reference
(``h3_a100/distributed.py:63-127``): with ``distributed.hybrid_shard.enabled``
the ranks form a (replicate, shard) placement, but the data-parallel group is
always the whole world so every rank draws its own sample and RNG stream
(``h3_a100/distributed.py:109-115``).
"""

from __future__ import annotations

import os
from datetime import timedelta
from typing import Any

import torch
import torch.distributed as dist

from ..config import get
from .topology import HybridTopology, resolve_hybrid_topology

_STATE: dict[str, Any] = {
    "topology": None,
    "shard_group": None,
    "replicate_group": None,
    "device": torch.device("cpu"),
}


def is_initialized() -> bool:
    return dist.is_available() and dist.is_initialized()


def get_rank() -> int:
    return dist.get_rank() if is_initialized() else int(os.environ.get("RANK", 0))


def get_world_size() -> int:
    return dist.get_world_size() if is_initialized() else int(os.environ.get("WORLD_SIZE", 1))


def get_local_rank() -> int:
    return int(os.environ.get("LOCAL_RANK", 0))


def is_main_process() -> bool:
    return get_rank() == 0


def device() -> torch.device:
    return _STATE["device"]


def topology() -> HybridTopology:
    topo = _STATE["topology"]
    if topo is None:
        topo = resolve_hybrid_topology(get_world_size(), get_rank(), get_world_size())
    return topo


def shard_group():
    """Process group over which frozen parameters are sharded (None = world)."""
    return _STATE["shard_group"]


def shard_group_size() -> int:
    return topology().shard_size


def shard_group_rank() -> int:
    return topology().shard_rank


def init_distributed_a100(config: dict[str, Any] | None = None, *, backend: str | None = None) -> HybridTopology:
    """Initialise the process group (idempotent) and the shard placement.

    Single-process runs without ``RANK`` in the environment stay
    uninitialised; everything downstream treats that as world size 1.
    """
    config = config or {}
    use_cuda = torch.cuda.is_available() and get(config, "kernels.device", "cuda") != "cpu"
    if use_cuda:
        torch.cuda.set_device(get_local_rank())
        _STATE["device"] = torch.device("cuda", get_local_rank())
    else:
        _STATE["device"] = torch.device("cpu")

    if "RANK" in os.environ and "WORLD_SIZE" in os.environ and not is_initialized():
        chosen = backend or get(config, "distributed.backend", "nccl")
        if not use_cuda:
            chosen = "gloo"
        timeout = timedelta(minutes=float(get(config, "distributed.timeout_minutes", 120)))
        kwargs: dict[str, Any] = {"backend": chosen, "timeout": timeout}
        if chosen == "nccl":
            kwargs["device_id"] = _STATE["device"]
        dist.init_process_group(**kwargs)

    world, rank = get_world_size(), get_rank()
    if get(config, "distributed.hybrid_shard.enabled", False):
        shard_size = int(get(config, "distributed.hybrid_shard.shard_size",
                             int(os.environ.get("LOCAL_WORLD_SIZE", world))))
    else:
        shard_size = world
    topo = resolve_hybrid_topology(world, rank, shard_size)
    _STATE["topology"] = topo
    if is_initialized() and topo.replicate_size > 1:
        # new_group must be called by every rank for every group, in order.
        for rep in range(topo.replicate_size):
            ranks = list(range(rep * topo.shard_size, (rep + 1) * topo.shard_size))
            group = dist.new_group(ranks)
            if rep == topo.replicate_rank:
                _STATE["shard_group"] = group
        for shard in range(topo.shard_size):
            ranks = [r * topo.shard_size + shard for r in range(topo.replicate_size)]
            group = dist.new_group(ranks)
            if shard == topo.shard_rank:
                _STATE["replicate_group"] = group
    else:
        _STATE["shard_group"] = None
        _STATE["replicate_group"] = None
    return topo


def replicate_group():
    return _STATE["replicate_group"]


def barrier() -> None:
    if is_initialized():
        if dist.get_backend() == "nccl":
            dist.barrier(device_ids=[torch.cuda.current_device()])
        else:
            dist.barrier()


def reduce_mean(value: float | torch.Tensor) -> float:
    """Mean of a scalar over ranks (logging only; outside any timed region)."""
    if not is_initialized():
        return float(value)
    dev = device() if dist.get_backend() == "nccl" else torch.device("cpu")
    tensor = torch.tensor([float(value)], dtype=torch.float64, device=dev)
    dist.all_reduce(tensor)
    return float(tensor.item()) / get_world_size()


def all_reduce_max(value: float) -> float:
    if not is_initialized():
        return float(value)
    dev = device() if dist.get_backend() == "nccl" else torch.device("cpu")
    tensor = torch.tensor([float(value)], dtype=torch.float64, device=dev)
    dist.all_reduce(tensor, op=dist.ReduceOp.MAX)
    return float(tensor.item())


def all_gather_object(obj: Any) -> list[Any]:
    if not is_initialized():
        return [obj]
    out: list[Any] = [None] * get_world_size()
    dist.all_gather_object(out, obj)
    return out


def cleanup_distributed() -> None:
    if is_initialized():
        dist.destroy_process_group()
    _STATE["topology"] = None
    _STATE["shard_group"] = None
    _STATE["replicate_group"] = None
