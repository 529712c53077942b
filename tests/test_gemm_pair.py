"""2-CTA pair mode of the tcgen05 GEMM against the single-CTA kernel.

In pair mode a cluster of two CTAs computes each 256 x 256 tile with
``tcgen05.mma.cta_group::2``: each CTA stages its own 128 rows of A and its
128-row half of B, and each keeps its 128 x 256 accumulator in its own TMEM.
Every output element still sums the same products in the same K order, so the
pair kernel must reproduce the single-CTA kernel bit for bit.  The single-CTA
results come from a child process started with ``H3_GEMM_PAIR=0`` (the switch
is read once per process).  Shapes are ragged in M and N so the second CTA of
the last pair tile sees rows past M.
"""

from __future__ import annotations

import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def compute_all() -> dict[str, torch.Tensor]:
    """Every pair-eligible GEMM form on seeded inputs (the same in any process)."""
    from h3_a100.ops.native import NativeKernels
    from h3_a100.ops.torch_kernels import GatedResidual, Rope

    dev = torch.device("cuda", 0)
    K = NativeKernels(dev, wait_limit_s=5.0)
    g = torch.Generator(device=dev).manual_seed(31)

    def bf(*shape, scale=1.0):
        return (torch.randn(*shape, device=dev, generator=g) * scale).to(torch.bfloat16)

    t, h, f, r, hd = 700, 512, 1280, 64, 128
    x = bf(t, h)
    out = {}
    w, b = bf(1300, h, scale=0.05), bf(1300)
    out["plain"] = K.linear(x, w, b)
    w0, b0 = bf(f, h, scale=0.05), bf(f)
    out["gelu_pre"], out["gelu_post"] = K.linear(x, w0, b0, epilogue="gelu")
    wq, bq = bf(3 * h, h, scale=0.05), bf(3 * h)
    a_cat, b_cat = bf(3 * r, h, scale=0.05), bf(3 * h, r, scale=0.05)
    ang = torch.rand(t, hd // 2, device=dev, generator=g) * 6.28
    rope = Rope(ang.cos(), ang.sin(), hd, h, (0, 1))
    u = K.lora_down(x, a_cat, 0.5)
    out["qkv_lora_rope"] = K.linear(x, wq, bq, u, b_cat, 3, epilogue=rope)
    w2, b2 = bf(h, f, scale=0.04), bf(h)
    res, gate = bf(t, h), torch.randn(2, h, device=dev, generator=g)
    out["gated_res"] = K.linear(out["gelu_post"], w2, b2, epilogue=GatedResidual(res, gate, 333))
    dy = bf(t, h)
    out["dx_gelu"] = K.linear_dx(dy, w2, gelu_pre=out["gelu_pre"])
    dyb = K.lora_dyb(bf(t, 3 * h), b_cat, 3, 2.0)
    out["dx_lora"] = K.linear_dx(bf(t, 3 * h), wq, dyb, a_cat)
    torch.cuda.synchronize()
    K.check_status()
    return {k: v.cpu() for k, v in out.items()}


def test_pair_mode_matches_single_cta(tmp_path):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    if os.environ.get("H3_GEMM_PAIR", "1") == "0":
        pytest.skip("pair mode switched off in this process")
    got = compute_all()
    ref_file = tmp_path / "single_cta.pt"
    code = ("import sys, torch; sys.path.insert(0, sys.argv[1]); sys.path.insert(0, sys.argv[2]); "
            "import test_gemm_pair as t; torch.save(t.compute_all(), sys.argv[3])")
    env = dict(os.environ, H3_GEMM_PAIR="0")
    proc = subprocess.run([sys.executable, "-c", code, ROOT, os.path.join(ROOT, "tests"), str(ref_file)],
                          env=env, capture_output=True, text=True, timeout=600)
    assert proc.returncode == 0, proc.stderr[-2000:]
    ref = torch.load(ref_file)
    for name, v in ref.items():
        assert torch.isfinite(got[name].float()).all(), name
        assert torch.equal(got[name], v), f"{name}: pair mode differs from the single-CTA kernel"
