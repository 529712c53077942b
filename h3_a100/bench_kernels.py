"""Per-kernel microbenchmark of one DiT block (native kernels vs the PyTorch path).

    python -m h3_a100.bench_kernels [--tokens 125504] [--hidden 3072] [--heads 24] [--ffn 12288] [--rank 128]

Default shape is the single-B200 block microbench: hidden 3072, 24 heads x
128, FFN 12288, 124,992 video + 512 text tokens, LoRA r128.  Each op is timed
with CUDA events after warm-up (median of ``--iters``), and reported as
achieved TFLOP/s or GB/s and as a fraction of the measured peaks in
``MEASURED_PEAKS.json`` (bf16 GEMM burst, HBM copy).  Operands are larger
than L2 for the GEMMs and the memory-bound ops, so no flush is needed.
"""

from __future__ import annotations

import argparse
import json
import os

import torch

from .ops.torch_kernels import GatedResidual, Rope, TorchKernels

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def peaks() -> dict:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as fh:
            d = json.load(fh)
        return {"tflops": float(d["bf16_tflops"]), "gbs": float(d["hbm_gbs"]), "source": "measured"}
    return {"tflops": 1590.0, "gbs": 6650.0, "source": "fallback"}


def timeit(fn, iters: int) -> float:
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b))
    times.sort()
    return times[len(times) // 2]


def main(argv=None) -> None:
    p = argparse.ArgumentParser()
    p.add_argument("--tokens", type=int, default=124992 + 512)
    p.add_argument("--hidden", type=int, default=3072)
    p.add_argument("--heads", type=int, default=24)
    p.add_argument("--ffn", type=int, default=12288)
    p.add_argument("--rank", type=int, default=128)
    p.add_argument("--iters", type=int, default=5)
    p.add_argument("--which", default="native,torch")
    p.add_argument("--skip-attention", action="store_true")
    p.add_argument("--only", default="", help="comma-separated op labels (prefix match) to run")
    args = p.parse_args(argv)
    from .ops.native import NativeKernels

    dev = torch.device("cuda", 0)
    pk = peaks()
    t, h, f, r, hd = args.tokens, args.hidden, args.ffn, args.rank, args.hidden // args.heads
    g = torch.Generator(device=dev).manual_seed(0)

    def bf(*shape, scale=1.0):
        return (torch.randn(*shape, device=dev, generator=g) * scale).to(torch.bfloat16)

    x = bf(t, h)
    w_qkv, b_qkv = bf(3 * h, h, scale=h ** -0.5), bf(3 * h)
    w_o, b_o = bf(h, h, scale=h ** -0.5), bf(h)
    w0, b0 = bf(f, h, scale=h ** -0.5), bf(f)
    w2, b2 = bf(h, f, scale=f ** -0.5), bf(h)
    a_qkv, bq = bf(3 * r, h, scale=0.01), bf(3 * h, r, scale=0.01)
    a_f, b_f = bf(r, h, scale=0.01), bf(f, r, scale=0.01)
    mod = torch.randn(2, 6, h, device=dev) * 0.1
    ang = torch.rand(t, hd // 2, device=dev)
    rope = Rope(ang.cos(), ang.sin(), hd, h, (0, 1))
    results = []
    for name in args.which.split(","):
        K = NativeKernels(dev) if name == "native" else TorchKernels()
        u_qkv = K.lora_down(x, a_qkv, 1.0)
        u_f = K.lora_down(x, a_f, 1.0)
        qkv = K.linear(x, w_qkv, b_qkv, u_qkv, bq, 3, epilogue=rope)
        pre, act = K.linear(x, w0, b0, u_f, b_f, 1, epilogue="gelu")
        dy = bf(t, h)
        cases = [
            ("qkv_fwd(+lora,+rope)", lambda: K.linear(x, w_qkv, b_qkv, u_qkv, bq, 3, epilogue=rope),
             2.0 * t * h * 3 * h + 2.0 * t * 3 * r * 3 * h / 3, "flop"),
            ("ff0_fwd(+lora,+gelu)", lambda: K.linear(x, w0, b0, u_f, b_f, 1, epilogue="gelu"),
             2.0 * t * h * f + 2.0 * t * r * f, "flop"),
            ("ff2_fwd(+gated_res)", lambda: K.linear(act, w2, b2, None, None, 1,
                                                     epilogue=GatedResidual(x, mod[:, 5], t - 4000)),
             2.0 * t * f * h, "flop"),
            ("o_fwd(+gated_res)", lambda: K.linear(x, w_o, b_o, None, None, 1,
                                                   epilogue=GatedResidual(x, mod[:, 2], t - 4000)),
             2.0 * t * h * h, "flop"),
            ("ff2_dx(+gelu_bwd)", lambda: K.linear_dx(dy, w2, gelu_pre=pre), 2.0 * t * h * f, "flop"),
            ("qkv_dx(+lora)", lambda: K.linear_dx(qkv, w_qkv, K.lora_dyb(qkv, bq, 3, 1.0), a_qkv),
             2.0 * t * 3 * h * h + 2.0 * t * 3 * r * h + 2.0 * t * 3 * h * r, "flop"),
            ("lora_down_qkv", lambda: K.lora_down(x, a_qkv, 1.0), 2.0 * t * h * 3 * r, "flop"),
            ("norm_modulate_fwd", lambda: K.norm_modulate(x, mod[:, 0], mod[:, 1], t - 4000), 2.0 * t * h * 2, "byte"),
            ("norm_modulate_bwd(+add,+gate)", lambda: K.norm_modulate_bwd(x, dy, mod[:, 1], t - 4000, 1e-6, add=dy,
                                                                          gate=mod[:, 2]), 5.0 * t * h * 2, "byte"),
        ]
        if not args.skip_attention:
            heads = args.heads
            cases.append(("attention_fwd", lambda: K.attention_fwd(qkv, heads, hd), 4.0 * t * t * h, "flop"))
            o_att, lse_att = K.attention_fwd(qkv, heads, hd)
            do_att = bf(t, h)
            cases.append(("attention_bwd", lambda: K.attention_bwd(qkv, o_att, lse_att, do_att, heads, hd),
                          10.0 * t * t * h, "flop"))
        only = [o for o in args.only.split(",") if o]
        for label, fn, work, kind in cases:
            if only and not any(label.startswith(o) for o in only):
                continue
            try:
                ms = timeit(fn, args.iters)
            except Exception as exc:  # noqa: BLE001 - report and continue
                results.append({"impl": name, "op": label, "error": str(exc)[:200]})
                continue
            if kind == "flop":
                achieved = work / ms / 1e9
                frac = achieved / pk["tflops"]
                results.append({"impl": name, "op": label, "ms": round(ms, 3), "tflops": round(achieved, 1),
                                f"frac_of_{pk['source']}_bf16": round(frac, 3)})
            else:
                achieved = work / ms / 1e6
                results.append({"impl": name, "op": label, "ms": round(ms, 3), "gbs": round(achieved, 1),
                                f"frac_of_{pk['source']}_hbm": round(achieved / pk["gbs"], 3)})
        if name == "native":
            K.check_status()
        del K
        torch.cuda.empty_cache()
    for row in results:
        print(json.dumps(row))


if __name__ == "__main__":
    main()
