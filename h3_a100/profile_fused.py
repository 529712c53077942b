"""One-GPU loopback runs of the fused collective kernels, for ncu captures.

    python -m h3_a100.profile_fused --op lora_step [--iters 3]
    ncu --set full --clock-control none -k regex:lora_rs_adamw -c 1 \\
        python -m h3_a100.profile_fused --op lora_step --iters 1

Each op calls one peer-memory kernel of ``csrc/comm/p2p.cu`` (or the GEMM
with gather warps) with a world of one: every "peer" pointer is this GPU's
own buffer, so the kernel runs its whole code path (flag protocol, reduction,
optimizer math, stores to every replica) on local memory.  That isolates the
kernel's compute and HBM behaviour, which is what an ncu capture on one GPU
can show; the NVLink side is measured by ``h3_a100.bench_collectives`` at
2-8 GPUs.  Sizes are small cases (a few hundred MB, all above the 126 MB L2):

* ``weight_gather``   pull all-gather of a 256 MB frozen-weight unit
* ``adaln_gather``    row-sharded AdaLN GEMV (a quarter of one H3 projection,
                      8,064 x 8,064 bf16) with its output stores and flag
* ``lora_step``       reduce-scatter + norm + clip + AdamW + all-gather of a
                      64 M-parameter LoRA (fp32 gradients, master and moments)
* ``allgather_gemm``  the fused-QKV GEMM (8,192 x 16,128 x 5,376) whose gather
                      warps copy each weight N-tile before the TMA loads

Prints one JSON line per op: CUDA-event milliseconds (mean of ``--iters``
after two warm-ups) and the bytes or FLOPs the op must move or do.
"""

from __future__ import annotations

import argparse
import json

import torch

from .parallel.p2p import LORA_SCRATCH_FLOATS

OPS = ("weight_gather", "adaln_gather", "lora_step", "allgather_gemm")


def _time(fn, iters: int) -> float:
    for _ in range(2):
        fn()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(iters):
        fn()
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end) / iters


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--op", default=",".join(OPS), help=f"comma-separated subset of {OPS}")
    p.add_argument("--iters", type=int, default=3)
    args = p.parse_args(argv)
    from . import _C
    from .ops.native import NativeKernels

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    K = NativeKernels(dev)
    status = torch.zeros(4, dtype=torch.int32, device=dev)
    limit = int(10e9)
    flags = torch.zeros(64, dtype=torch.int32, device=dev)
    epoch = [0]

    def next_epoch() -> int:
        epoch[0] += 1
        return epoch[0]

    for op in args.op.split(","):
        if op == "weight_gather":
            shard = torch.randn(128 * 2**20, device=dev).to(torch.bfloat16)        # 256 MB
            out = torch.empty_like(shard)
            nbytes = shard.numel() * 2

            def run():
                _C.p2p_all_gather([shard.data_ptr()], nbytes, out)

            ms = _time(run, args.iters)
            assert torch.equal(out, shard)
            line = {"op": op, "ms": round(ms, 4), "bytes": 2 * nbytes, "gbs": round(2 * nbytes / ms / 1e6, 1)}
        elif op == "adaln_gather":
            rows, dt = 8064, 8064
            w = (torch.randn(rows, dt, device=dev) * 0.02).to(torch.bfloat16)
            b = torch.zeros(rows, device=dev, dtype=torch.bfloat16)
            temb = torch.randn(2, dt, device=dev).to(torch.bfloat16)
            out = torch.zeros(2, rows, device=dev)

            def run():
                _C.adaln_project_gather(temb, w, b, [out.data_ptr()], [flags.data_ptr()], 0, next_epoch(), 3,
                                        status, limit)

            ms = _time(run, args.iters)
            ref = torch.nn.functional.silu(temb.float()) @ w.float().t()
            torch.testing.assert_close(out, ref, rtol=2e-2, atol=2e-2)
            nbytes = w.numel() * 2
            line = {"op": op, "ms": round(ms, 4), "bytes": nbytes, "gbs": round(nbytes / ms / 1e6, 1)}
        elif op == "lora_step":
            n = 64 * 2**20
            grad = torch.randn(n, device=dev)
            param = torch.randn(n, device=dev).to(torch.bfloat16)
            master, m, v = param.float(), torch.zeros(n, device=dev), torch.zeros(n, device=dev)
            scratch = torch.zeros(LORA_SCRATCH_FLOATS, device=dev)
            bar = torch.zeros(2, dtype=torch.int32, device=dev)
            step = [0]

            def run():
                step[0] += 1
                _C.lora_rs_adamw([grad.data_ptr()], [param.data_ptr()], [flags.data_ptr()], 0, next_epoch(),
                                 master, m, v, scratch, bar, 1e-4, 0.9, 0.999, 1e-8, 0.01, step[0], 1.0, status,
                                 limit, 0, 0)

            ms = _time(run, args.iters)
            # grad read, master/m/v read + write, bf16 param store
            nbytes = n * 4 + 3 * 2 * n * 4 + n * 2
            line = {"op": op, "ms": round(ms, 4), "params": n, "bytes": nbytes,
                    "gbs": round(nbytes / ms / 1e6, 1)}
        elif op == "allgather_gemm":
            mt, nq, kq = 8192, 16128, 5376
            x = (torch.randn(mt, kq, device=dev) * 0.5).to(torch.bfloat16)
            w = (torch.randn(nq, kq, device=dev) * 0.02).to(torch.bfloat16)
            w_local = torch.zeros_like(w)
            tile_flags = torch.zeros((nq + 255) // 256, dtype=torch.int32, device=dev)

            def run():
                K.linear_allgather(x, w_local, ([w.data_ptr()], nq, tile_flags))

            ms = _time(run, args.iters)
            assert torch.equal(w_local, w)
            flops = 2.0 * mt * nq * kq
            line = {"op": op, "ms": round(ms, 4), "flops": flops, "tflops": round(flops / ms / 1e9, 1)}
        else:
            raise SystemExit(f"unknown op {op!r}; choose from {OPS}")
        code = int(status[0].item())
        K.check_status()
        if code:
            raise SystemExit(f"{op}: kernel status {code}")
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
