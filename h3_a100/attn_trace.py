"""Phase timing inside the attention-forward kernel (diagnostic).

    python -m h3_a100.attn_trace [--tokens 37730] [--heads 42]

Runs the tcgen05 attention forward once with a trace buffer: CTA (0, 0)
records ``clock64`` at each phase of the first lane band of each query tile's
softmax warpgroup and of the MMA issuer.  Prints the median cycles per KV step
of every phase, which is how the softmax's critical path is split between
waiting for S, reading S from TMEM, the row max, the exponentials and the
hand-off, and how long the MMA issuer waits for P.
"""

from __future__ import annotations

import argparse
import json
import statistics

import torch

PHASES = ["wait_s", "tmem_load", "max", "exp_pack", "rescale_arrive"]


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--tokens", type=int, default=37730)
    p.add_argument("--heads", type=int, default=42)
    args = p.parse_args(argv)
    from . import _C

    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    h = args.heads * 128
    qkv = torch.randn(args.tokens, 3 * h, device=dev).to(torch.bfloat16)
    status = torch.zeros(4, dtype=torch.int32, device=dev)
    n_kv = (args.tokens + 127) // 128
    _C.attention_fwd(qkv, args.heads, 128, status, int(10e9))          # warm-up
    slots = 12
    trace = torch.zeros(2 * n_kv * slots, dtype=torch.int64, device=dev)
    _C.attention_fwd(qkv, args.heads, 128, status, int(10e9), trace)
    torch.cuda.synchronize()
    t = trace.view(2, n_kv, slots).cpu().tolist()
    out = {"n_kv": n_kv}
    skip = min(4, n_kv // 4)          # leave out the pipeline fill
    for tile in range(2):
        rows = t[tile][skip:n_kv - 1]
        per = {name: statistics.median(r[i + 1] - r[i] for r in rows) for i, name in enumerate(PHASES)}
        per["softmax_total"] = statistics.median(r[5] - r[1] for r in rows)
        per["step_period"] = statistics.median(b[1] - a[1] for a, b in zip(rows, rows[1:]))
        # MMA side: from the softmax's arrive to the PV issue, and from PV issue to S(j+1) issue
        per["arrive_to_pv_issue"] = statistics.median(r[6] - r[5] for r in rows)
        per["pv_to_next_s_issue"] = statistics.median(r[7] - r[6] for r in rows)
        # hand-off skew: each lane band's arrive relative to band 0's (slots 5, 8, 9, 10)
        per["band_arrive_after_band0"] = [statistics.median(r[s] - r[5] for r in rows) for s in (8, 9, 10)]
        per["last_band_arrive_to_pv_issue"] = statistics.median(r[6] - max(r[5], r[8], r[9], r[10]) for r in rows)
        out[f"tile{tile}"] = per
    out["tile1_start_after_tile0"] = statistics.median(t[1][j][1] - t[0][j][1] for j in range(skip, n_kv - 1))
    # backward: warpgroup 0's first lane band and the MMA issuer of CTA (0, 0)
    do = torch.randn(args.tokens, h, device=dev).to(torch.bfloat16)
    o, lse = _C.attention_fwd(qkv, args.heads, 128, status, int(10e9))
    _C.attention_bwd(qkv, o, lse, do, args.heads, 128, status, int(10e9))    # warm-up
    n_q = n_kv
    bt = torch.zeros(n_q * 12, dtype=torch.int64, device=dev)
    _C.attention_bwd(qkv, o, lse, do, args.heads, 128, status, int(10e9), bt)
    torch.cuda.synchronize()
    b = bt.view(n_q, 12).cpu().tolist()[skip:n_q - 1]
    med = lambda f: statistics.median(f(r) for r in b)   # noqa: E731
    bwd = {
        "wait_s": med(lambda r: r[1] - r[0]),
        "load_s_dp": med(lambda r: r[2] - r[1]),
        "p_ds_compute_store": med(lambda r: r[4] - r[2]),
        "prev_reduce_wait": med(lambda r: r[5] - r[4]),
        "wait_dq": med(lambda r: r[6] - r[5]),
        "dq_tmem_read_release": med(lambda r: r[9] - r[6]),
        "wait_stage_read": med(lambda r: r[7] - r[9]),
        "dq_stage": med(lambda r: r[8] - r[7]),
        "step_period": statistics.median(y[1] - x[1] for x, y in zip(b, b[1:])),
        "mma_sdp_issue_to_p_full": med(lambda r: r[11] - r[10]),
        "dq_empty_to_next_sdp_issue": statistics.median(y[10] - x[9] for x, y in zip(b, b[1:])),
    }
    out["backward"] = bwd
    print(json.dumps(out, indent=1))


if __name__ == "__main__":
    main()
