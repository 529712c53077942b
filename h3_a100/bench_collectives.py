"""Collective sweep: peer-memory kernels against the NCCL path, with rooflines.

``torchrun --nproc-per-node N -m h3_a100.bench_collectives --config
configs/h3_fused_collective_sweep.yaml`` times, on every rank with CUDA events
(after warm-up; the reported time is the max over ranks):

* ``weight_gather``: one transformer block's frozen-weight unit, all-gathered
  from the per-rank shards (NCCL ``all_gather_into_tensor`` vs the peer-memory
  gather: copy engines by default, ``H3_P2P_GATHER=kernel`` for the pull kernel);
* ``gather_interference`` (p2p): the QKV GEMM timed alone and while a unit
  gather runs beside it on the communication stream, with the pull kernel and
  with the copy engines: what a hidden prefetch costs the compute;
* ``adaln``: the row-sharded AdaLN projection of one block for the two
  timestep rows (GEMV on the local rows + NCCL all-gather of the outputs, vs
  the fused GEMV whose epilogue stores into every rank's output);
* ``lora_step``: one role's optimizer step on the r128 LoRA of the config
  (NCCL reduce-scatter + norm all-reduce + AdamW + all-gather, vs the single
  cooperative peer-memory kernel);
* ``allgather_qkv_gemm``: the fused QKV GEMM on a weight sharded by rows across
  the ranks (NCCL all-gather then the GEMM, vs the GEMM whose gather warps pull
  each N-tile from its owner while earlier tiles are multiplied).

Each line carries the path's roofline: the slower of its HBM bytes at the
measured copy bandwidth and its NVLink bytes per GPU at 770 GB/s per direction
(the measured peer-copy rate on this hardware), and the achieved fraction.
Reference counterparts: FSDP2's per-block all-gather, and
``clip_grad_norm_`` + ``AdamW`` after FSDP2's reduce-scatter
(``h3_a100/model.py:410-438``; ``h3_a100/trainer_loop.py:130-133,203-206``).
"""

from __future__ import annotations

import argparse
import json
import os
from datetime import timedelta

import torch
import torch.distributed as dist

NVLINK_GBS = 770.0


def _peaks() -> dict:
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "MEASURED_PEAKS.json")
    try:
        with open(path) as fh:
            return json.load(fh)
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def _time(fn, iters: int, warmup: int = 3) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(iters):
        fn()
    end.record()
    torch.cuda.synchronize()
    ms = torch.tensor([start.elapsed_time(end) / iters], device="cuda")
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    return float(ms.item())


def _interference(comm, shard, padded, K, cfg, args, lines, world) -> None:
    """How much a prefetched frozen-weight gather slows the compute it hides
    behind: the QKV GEMM of the sweep model timed alone, then while gathers of
    one block's unit run back to back on the communication stream, once with
    the pull kernel (SMs) and once on the copy engines (``gather_engine``)."""
    from .models.shared_backbone import sequence_tokens

    h = cfg.hidden
    m_tok = sequence_tokens(_cfg_of(args))
    x = (torch.randn(m_tok, h, device="cuda") * 0.5).to(torch.bfloat16)
    w = (torch.randn(3 * h, h, device="cuda") * 0.02).to(torch.bfloat16)
    iters = max(10, args.iters)

    def gemm():
        K.linear(x, w)

    base = _time(gemm, iters)
    result = {"op": "gather_interference", "impl": "p2p", "n_gpus": world, "gemm_alone_ms": round(base, 4),
              "unit_bytes": padded * 2}
    saved = comm.gather_engine
    for engine in ("kernel", "copy"):
        comm.gather_engine = engine

        def gemm_under_gather():
            # one gather of the unit per GEMM, issued first on the comm stream
            out = comm.all_gather_async(shard, padded)
            K.linear(x, w)
            comm.recycle(comm.wait(out))

        ms = _time(gemm_under_gather, iters)
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        g0.record(comm._stream)
        for _ in range(5):
            comm.recycle(comm.wait(comm.all_gather_async(shard, padded)))
        g1.record(comm._stream)
        torch.cuda.synchronize()
        gather_alone = g0.elapsed_time(g1) / 5
        result[f"gemm_with_{engine}_gather_ms"] = round(ms, 4)
        result[f"{engine}_gather_alone_ms"] = round(gather_alone, 4)
    comm.gather_engine = saved
    lines.append(result)


def _cfg_of(args):
    from .config import load_config

    return load_config(args.config)


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--config", default=os.path.join("configs", "h3_fused_collective_sweep.yaml"))
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--which", default="nccl,p2p")
    args = p.parse_args(argv)

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(minutes=5), device_id=dev)
    world, rank = dist.get_world_size(), dist.get_rank()

    from .config import load_config
    from .models.shared_backbone import dit_config_from
    from .ops.native import NativeKernels
    from .parallel.comm import TorchComm
    from .parallel.p2p import PeerComm
    from .trainer.optim import FlatAdamW

    cfg = dit_config_from(load_config(args.config))
    peaks = _peaks()
    hbm = float(peaks["hbm_gbs"])
    K = NativeKernels(dev)
    h, f, dt = cfg.hidden, cfg.ffn, cfg.time_embed_dim
    block_params = 3 * h * h + 3 * h + h * h + h + f * h + f + h * f + h
    adaln_rows = 6 * h
    rank_lora = 128
    lora_numel = (cfg.num_blocks + cfg.num_refiner_blocks) * rank_lora * (10 * h + 2 * f)
    comms = {}
    if "nccl" in args.which:
        comms["nccl"] = TorchComm(dist.group.WORLD, dev)
    if "p2p" in args.which and world > 1:
        comms["p2p"] = PeerComm(dist.group.WORLD, dev, kernels=K)
    lines = []

    def emit(op, impl, ms, hbm_bytes, link_bytes, extra=None):
        roof_ms = max(hbm_bytes / (hbm * 1e9), link_bytes / (NVLINK_GBS * 1e9)) * 1e3
        line = {"op": op, "impl": impl, "n_gpus": world, "ms": round(ms, 4),
                "roofline_ms": round(roof_ms, 4), "frac_of_roofline": round(roof_ms / ms, 3) if ms > 0 else None,
                "hbm_bytes": int(hbm_bytes), "nvlink_bytes_per_gpu": int(link_bytes)}
        if extra:
            line.update(extra)
        lines.append(line)

    for impl, comm in comms.items():
        # ---- per-block frozen-weight all-gather (bf16)
        quantum = world * 64
        padded = (block_params + quantum - 1) // quantum * quantum
        shard = comm.alloc_shard(padded // world, torch.bfloat16)
        shard.normal_()

        def gather():
            out = comm.wait(comm.all_gather_async(shard, padded))
            comm.recycle(out)

        ms = _time(gather, args.iters)
        nbytes = padded * 2
        emit("weight_gather", impl, ms, hbm_bytes=nbytes + nbytes / world,
             link_bytes=nbytes * (world - 1) / world, extra={"unit_bytes": nbytes})
        if impl == "p2p":
            _interference(comm, shard, padded, K, cfg, args, lines, world)

        # ---- AdaLN projection (row-sharded) for two timestep rows
        rows = adaln_rows // world
        w_rows = (torch.randn(rows, dt, device=dev) * 0.02).to(torch.bfloat16)
        b_rows = torch.zeros(rows, device=dev, dtype=torch.bfloat16)
        temb = torch.randn(2, dt, device=dev).to(torch.bfloat16)
        if impl == "p2p":
            out = comm.alloc_symmetric(2 * world * rows, torch.float32).view(2, world * rows)

            def adaln():
                comm.adaln_project(temb, w_rows, b_rows, out)
        else:
            def adaln():
                local_rows = K.adaln_project(temb, w_rows, b_rows)
                comm.all_gather_rows(local_rows)

        ms = _time(adaln, args.iters)
        emit("adaln", impl, ms, hbm_bytes=rows * dt * 2, link_bytes=2 * rows * 4 * (world - 1))
        if impl == "p2p":
            comm.check_status()

        # ---- LoRA optimizer step (one role)
        class _Store:
            def __init__(self, flat, grad):
                self.flat, self.grad = flat, grad

            def ensure_grad(self):
                return self.grad

            def zero_grad(self):
                self.grad.zero_()

        n = (lora_numel + 4 * world - 1) // (4 * world) * (4 * world)
        flat = comm.alloc_symmetric(n, torch.bfloat16)
        grad = comm.alloc_symmetric(n, torch.float32)
        flat.normal_()
        grad.normal_()
        opt = FlatAdamW(_Store(flat, grad), lr=1e-4, weight_decay=0.01, max_grad_norm=1.0, kernels=K, comm=comm,
                        shard_states=True)

        ms = _time(lambda: opt.step(1e-4), max(3, args.iters // 4))
        chunk = n // world
        # HBM: read world fp32 grad chunks (local part) + write chunk, master/m/v read+write, bf16 param stores
        hbm_bytes = chunk * 4 * 2 + chunk * 4 * 6 + n * 2
        link = (world - 1) * chunk * 4 + (world - 1) * chunk * 2
        emit("lora_step", impl, ms, hbm_bytes=hbm_bytes, link_bytes=link, extra={"params": n, "fused": opt.fused})
        if impl == "p2p":
            comm.check_status()
        K.check_status()

        # ---- QKV GEMM on a row-sharded weight: all-gather then GEMM (NCCL) vs
        # the GEMM whose gather warps pull each N-tile from its owner (p2p)
        from .models.shared_backbone import sequence_tokens

        m_tok = sequence_tokens(load_config(args.config))
        n_q, k_q = 3 * h, h
        rows_q = n_q // world
        x_q = (torch.randn(m_tok, k_q, device=dev) * 0.5).to(torch.bfloat16)
        w_shard = comm.alloc_shard(rows_q * k_q, torch.bfloat16).view(rows_q, k_q)
        w_shard.normal_(0, 0.02)
        w_full = torch.empty(n_q, k_q, dtype=torch.bfloat16, device=dev)
        torch.cuda.synchronize()
        dist.barrier()
        if impl == "p2p":
            flags = torch.zeros((n_q + 255) // 256, dtype=torch.int32, device=dev)

            def ag_gemm():
                K.linear_allgather(x_q, w_full, comm.gather_spec(w_shard, rows_q, flags))
        else:
            def ag_gemm():
                dist.all_gather_into_tensor(w_full, w_shard)
                K.linear(x_q, w_full)

        ms = _time(ag_gemm, max(5, args.iters // 2))
        flops = 2.0 * m_tok * n_q * k_q
        link = n_q * k_q * 2 * (world - 1) / world
        roof_ms = max(flops / (float(peaks.get("bf16_tflops", 1590.0)) * 1e12), link / (NVLINK_GBS * 1e9)) * 1e3
        lines.append({"op": "allgather_qkv_gemm", "impl": impl, "n_gpus": world, "ms": round(ms, 4),
                      "roofline_ms": round(roof_ms, 4), "frac_of_roofline": round(roof_ms / ms, 3),
                      "tflops": round(flops / ms / 1e9, 1), "m": m_tok, "n": n_q, "k": k_q,
                      "nvlink_bytes_per_gpu": int(link)})
        K.check_status()
        if impl == "p2p":
            comm.check_status()
        del shard, flat, grad, opt, w_shard, w_full, x_q
        torch.cuda.synchronize()
        dist.barrier()

    if rank == 0:
        for line in lines:
            print(json.dumps(line), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
