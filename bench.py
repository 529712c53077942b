"""Headline benchmark: seconds per matched DMD outer cycle, H3-shaped, B1/rank.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl native|torch|reference]

One rank per GPU (``torchrun`` for N > 1).  W untimed warm-up cycles, then
K cycles bracketed by a barrier and ``torch.cuda.synchronize()`` on both
sides, timed with CUDA events on the compute stream; the reported value is
the maximum over ranks.  A cycle takes minutes, so a wall budget
(``--max-seconds``, default 820 s for the whole process) caps the work: at
least three warm-up cycles always run, then as many of the K timed cycles as
fit (at least one); ``steps``/``warmup`` in the JSON line are the counts that
ran, next to the requested ones.  Weights (66 GB) are far larger than L2, so no
flush is needed between cycles.  Every cycle goes through the public API
(``trainer.run_cycle``): each sample's tensors are copied host->device from
pinned memory and the cycle's losses are read back to the host, so the same
K cycles also give the end-to-end number (host wall clock, max over ranks).

``--impl native`` uses the hand-written sm_100a kernels, ``--impl torch`` the
PyTorch/cuBLAS/SDPA path of the same trainer, and ``--impl reference`` tries
the unmodified reference package installed in ``baseline/_ref``.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time

PROCESS_T0 = time.time()
ROOT = os.path.dirname(os.path.abspath(__file__))
MIN_WARMUP = 3                 # warm-up cycles always run (fewer only if --warmup asks for fewer)
CYCLE_SAFETY = 1.04            # margin on the warm-cycle estimate when planning timed cycles
TEARDOWN_RESERVE_S = 25.0      # kept free for the final collectives, the JSON line and teardown
REFERENCE_S_PER_CYCLE = 912.718721   # the reference's published cycle time (16x A100-40GB, world16)
# One cycle takes minutes, so K + W cycles can outlast a caller's time limit;
# the default budget keeps a whole run (setup, 3 warm-up cycles, the timed
# cycles, teardown) under 14 minutes.
DEFAULT_BUDGET_S = 820.0
METRIC = "s per matched DMD cycle @768x1344x124f (max over ranks); peak GiB/rank"


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=1)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="native", choices=["native", "torch", "reference"])
    p.add_argument("--config", default=os.path.join(ROOT, "configs", "h3_dmd_b200_world8.yaml"))
    p.add_argument("--max-seconds", type=float,
                   default=float(os.environ.get("H3_BENCH_BUDGET_S", DEFAULT_BUDGET_S)),
                   help="wall budget of the whole process; warm-up beyond 3 cycles and timed cycles "
                        "beyond what fits are dropped (the JSON line reports the counts actually run)")
    p.add_argument("--num-blocks", type=int, default=None,
                   help="development only: fewer blocks (the result is then not the headline config)")
    return p.parse_args()


def run_reference(args) -> None:
    ref = os.path.join(ROOT, "baseline", "_ref")
    line = {"impl": "reference", "metric": METRIC, "n_gpus": args.gpus}
    if not os.path.isdir(os.path.join(ref, "h3_a100")):
        line["unavailable"] = "reference package not installed in baseline/_ref"
        print(json.dumps(line))
        return
    probe = subprocess.run(
        [sys.executable, "-c", "import sys; sys.path.insert(0, sys.argv[1]); import h3_a100.entrypoint", ref],
        capture_output=True, text=True, timeout=300, cwd="/tmp")
    if probe.returncode != 0:
        err = (probe.stderr.strip().splitlines() or ["unknown import failure"])[-1]
        line["unavailable"] = ("the reference's public API (h3_a100.entrypoint) cannot import offline: it needs "
                               "LightX2V-train, a Diffusers build with MiniMaxH3Transformer3DModel, PEFT and the "
                               f"FA3 hub kernel, none of which exist in this image ({err})")
        print(json.dumps(line))
        return
    line["unavailable"] = "reference imported but needs the MiniMax-H3 checkpoint and prompt cache, which are not available"
    print(json.dumps(line))


def plan_timed_cycles(requested: int, budget_s: float, elapsed_s: float, cycle_s: float,
                      reserve_s: float = TEARDOWN_RESERVE_S) -> int:
    """How many whole timed cycles fit in what is left of the wall budget (at least one)."""
    if requested <= 0:
        return 0
    room = budget_s - elapsed_s - reserve_s
    fits = int(room // max(cycle_s, 1e-6)) if cycle_s > 0 else requested
    return max(1, min(int(requested), fits))


def main() -> None:
    args = parse_args()
    if args.impl == "reference":
        if int(os.environ.get("RANK", "0")) == 0:
            run_reference(args)
        return

    import torch

    sys.path.insert(0, ROOT)
    from h3_a100.api import build_trainer
    from h3_a100.config import load_config
    from h3_a100.parallel import distributed as pdist
    from h3_a100.utils.benchmark import ClockSampler
    from h3_a100.utils.log import setup_logger

    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch N>1 with torchrun")
    overrides = {
        "kernels": {"backend": args.impl},
        "training": {"max_train_iters": args.warmup + args.steps, "save_every_iters": 0,
                     "a100": {"matched_compute": {"expected_world_size": world}}},
        "logging": {"rank_zero_only": True, "train_log_every_iters": 1000000},
    }
    if args.num_blocks:
        overrides["synthetic"] = {"model": {"num_blocks": args.num_blocks}}
    os.environ.setdefault("WORLD_SIZE", str(world))
    config = load_config(args.config, overrides)
    torch.backends.cuda.matmul.allow_tf32 = True
    setup_logger(config)
    trainer = build_trainer(config)
    trainer.setup()
    model_cfg = trainer.model.dit_config
    native = getattr(trainer.kernels, "native", False)
    rank = pdist.get_rank()
    samples = trainer.samples()

    def log(msg: str) -> None:
        if rank == 0:
            print(msg, file=sys.stderr, flush=True)

    # ---- warm-up: at least min(W, 3) cycles; more only if the timed cycles still fit.
    mandatory = min(args.warmup, MIN_WARMUP)
    warm_times: list[float] = []
    warmed = 0
    while warmed < args.warmup:
        if warmed >= mandatory:
            est = pdist.all_reduce_max(max(warm_times[1:] or warm_times))
            need = est * (1 + args.warmup - warmed + args.steps)
            if pdist.all_reduce_max(time.time() - PROCESS_T0) + need + TEARDOWN_RESERVE_S > args.max_seconds:
                break
        t0 = time.perf_counter()
        losses = trainer.run_cycle(samples, warmed)
        torch.cuda.synchronize()
        warm_times.append(time.perf_counter() - t0)
        log(f"warmup cycle {warmed}: {warm_times[-1]:.1f} s losses {losses}")
        warmed += 1

    # ---- plan the timed cycles from the slowest warm cycle (the first one pays one-off costs).
    est_cycle = pdist.all_reduce_max(max(warm_times[1:] or warm_times or [0.0]))
    elapsed = pdist.all_reduce_max(time.time() - PROCESS_T0)
    steps = plan_timed_cycles(args.steps, args.max_seconds, elapsed, est_cycle * CYCLE_SAFETY)
    log(f"budget {args.max_seconds:.0f} s, {elapsed:.0f} s used, cycle ~{est_cycle:.1f} s: "
        f"timing {steps} of {args.steps} requested cycles")

    torch.cuda.synchronize()
    pdist.barrier()
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats()
    launches0 = trainer.kernels.launch_count() if native else 0
    h2d0 = trainer.h2d_bytes
    sampler = ClockSampler([int(os.environ.get("LOCAL_RANK", "0")) + i for i in range(world)]
                           if rank == 0 else None)
    if rank == 0:
        sampler.start()
    marks = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    receipts = []
    wall0 = time.perf_counter()
    marks[0].record()
    last = None
    for k in range(steps):
        last = trainer.run_cycle(samples, warmed + k)
        marks[k + 1].record()
        receipts.append(dict(trainer.last_cycle_receipt))
    torch.cuda.synchronize()
    wall = time.perf_counter() - wall0
    pdist.barrier()
    torch.cuda.synchronize()
    clocks = sampler.stop() if rank == 0 else {}
    cycle_ms = [marks[i].elapsed_time(marks[i + 1]) for i in range(steps)]
    cycle_ms = [pdist.all_reduce_max(v) for v in cycle_ms]
    dev_ms = pdist.all_reduce_max(marks[0].elapsed_time(marks[steps]))
    launches = (trainer.kernels.launch_count() - launches0) if native else 0
    peak_gib = pdist.all_reduce_max(torch.cuda.max_memory_allocated() / 1024**3)
    wall = pdist.all_reduce_max(wall)
    launches = int(pdist.all_reduce_max(launches))
    phases = _mean_over_cycles([r.get("phases_s", {}) for r in receipts], pdist)
    exposed = _mean_over_cycles([r.get("exposed_comm_s", {}) for r in receipts], pdist)
    h2d_per_step = (trainer.h2d_bytes - h2d0) / max(1, steps)
    s_per_cycle = dev_ms / 1000.0 / steps
    from h3_a100.config import get as cfg_get
    from h3_a100.models.shared_backbone import sequence_tokens

    dmd = cfg_get(config, "training.dmd", {}) or {}
    canvas = f"{dmd.get('height', 768)}x{dmd.get('width', 1344)}x{dmd.get('num_frames', 124)}f"
    # only the full 50-block model on the 768x1344x124 canvas is the published metric's config
    headline = args.num_blocks is None and canvas == "768x1344x124f"
    staging = trainer.boundary_staging_report()
    if rank == 0:
        tokens = sequence_tokens(config)
        metric = METRIC if canvas == "768x1344x124f" else METRIC.replace("768x1344x124f", canvas)
        counts = model_cfg.param_counts()
        lora_params = trainer.model.lora["student"].numel()
        line = {
            "metric": metric,
            "value": round(s_per_cycle, 4),
            "unit": "s/cycle",
            "n_gpus": world,
            "steps": steps,
            "warmup": warmed,
            "steps_requested": args.steps,
            "warmup_requested": args.warmup,
            "ms_per_step": round(dev_ms / steps, 2),
            "higher_is_better": False,
            "scaling": "weak",
            "vs_baseline": round(s_per_cycle / REFERENCE_S_PER_CYCLE, 5) if headline else None,
            "dtype": "bf16",
            "data": "synthetic: seeded N(0,1) video/audio latents and text conditioning; random-init weights",
            "impl": args.impl,
            "peak_gib_per_rank": round(peak_gib, 2),
            "cycle_s": [round(v / 1e3, 3) for v in cycle_ms],
            "phases_s": phases,
            "exposed_comm_s": exposed,
            "boundary_staging": staging,
            "budget": {"max_seconds": args.max_seconds, "process_s": round(time.time() - PROCESS_T0, 1),
                       "warm_cycle_s": [round(t, 2) for t in warm_times]},
            "config": {
                "model": (f"H3-shaped DiT {model_cfg.num_blocks} blocks hidden {model_cfg.hidden} "
                          f"ffn {model_cfg.ffn} ({counts['frozen_total'] / 1e9:.1f}B frozen + "
                          f"2x{lora_params / 1e6:.1f}M LoRA r128)"),
                "global_batch": world,
                "seq_len": tokens,
                "parallelism": f"fsdp{world}" if world > 1 else "single",
                "comm": getattr(trainer.comm, "name", "none") if world > 1 else "none",
                "cycle": "Student x1 + Fake x5 (24/6/1 forwards, 1/5 backwards), 300 boundary copies",
                "l2": "no flush: every cycle streams 66 GB of weights, far larger than the 126 MB L2",
                "headline_config": headline,
            },
            "clocks": clocks,
            "e2e": {"value": round(wall / steps, 4), "unit": "s/cycle",
                    "h2d_bytes_per_step": int(h2d_per_step), "d2h_bytes_per_step": 8},
            "gpu_launches": launches,
            "losses": last,
            "receipt": trainer.last_cycle_receipt,
        }
        print(json.dumps(line), flush=True)
    trainer.data.close()
    pdist.cleanup_distributed()


def _mean_over_cycles(items: list[dict], pdist) -> dict:
    """Mean per key over the timed cycles, then max over ranks (same key order on every rank)."""
    keys = sorted({k for d in items for k in d})
    return {k: round(pdist.all_reduce_max(sum(d.get(k, 0.0) for d in items) / max(1, len(items))), 3)
            for k in keys}


if __name__ == "__main__":
    main()
