"""The bounds-checked build (``h3_a100._C_checked``, built with H3_CHECKED_BUILD=1).

It is the same kernel source compiled with ``-DH3_BOUNDS_CHECK``: every global
store whose index arithmetic is this code's own (the GEMM epilogue's row
stores and fp32 accumulation, the fused gather's copies, the attention
outputs) is checked against the real extent of its allocation, skipped if
outside, and reported as status 7.  These tests run the kernels through it on
ragged shapes and require (a) no report and (b) results equal to the normal
build's bit for bit (within rounding where fp32 atomics add in no fixed
order), and (c) that the checks do fire: with the output
allocation declared one row short (a host-side test hook), the last row must
be reported and left unwritten.
"""

from __future__ import annotations

import os

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def kernels():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    try:
        from h3_a100 import _C_checked
    except ImportError:
        pytest.skip("bounds-checked extension not built (H3_CHECKED_BUILD=1 python setup.py build_ext --inplace)")
    from h3_a100.ops.native import NativeKernels

    dev = torch.device("cuda", 0)
    return NativeKernels(dev, wait_limit_s=5.0), NativeKernels(dev, wait_limit_s=5.0, extension=_C_checked)


def bf(*shape, scale=1.0):
    return (torch.randn(*shape, device="cuda") * scale).to(torch.bfloat16)


def _all_forms(K):
    """GEMM (pair and single-CTA, row-store fallback, MN-major B, fp32 split-K,
    fused gather) and attention forward / backward on ragged shapes."""
    from h3_a100.ops.native import EPI_BF16, EPI_F32_ACC

    g = torch.Generator(device="cuda").manual_seed(50)

    def r(*shape, scale=1.0):
        return (torch.randn(*shape, device="cuda", generator=g) * scale).to(torch.bfloat16)

    out = {}
    m, n, k = 700, 1320, 512
    x, w, b = r(m, k), r(n, k, scale=0.05), r(n)
    out["pair"] = K.linear(x, w, b)
    single = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    K._gemm(x, False, w, False, m, n, k, EPI_BF16, single, bias=b, block_n=128)
    out["single"] = single
    storage = torch.empty(m, n + 1, dtype=torch.bfloat16, device="cuda")
    K._gemm(x, False, w, False, m, n, k, EPI_BF16, storage[:, :n], bias=b, block_n=128)
    out["row_store"] = storage[:, :n].clone()
    pre_post = K.linear(x, w[:1280], b[:1280], epilogue="gelu")
    out["dx_gelu"] = K.linear_dx(r(m, 512), r(512, 512, scale=0.05), gelu_pre=r(m, 512))
    acc = torch.zeros(512, 512, device="cuda")
    K._gemm(r(m, 512), True, pre_post[1][:, :512].contiguous(), True, 512, 512, m, EPI_F32_ACC, acc, splits=3,
            block_n=128)
    out["f32acc"] = acc
    rows = 440
    shards = [w[i * rows:(i + 1) * rows].clone() for i in range(3)]
    flags = torch.zeros((n + 255) // 256, dtype=torch.int32, device="cuda")
    out["gather"] = K.linear_allgather(x, torch.zeros_like(w), ([t.data_ptr() for t in shards], rows, flags), bias=b)
    t, heads, hd = 700, 2, 128
    qkv = r(t, 3 * heads * hd)
    o, lse = K.attention_fwd(qkv, heads, hd)
    out["attn_o"], out["attn_lse"] = o, lse
    out["attn_dqkv"] = K.attention_bwd(qkv, o, lse, r(t, heads * hd), heads, hd)
    torch.cuda.synchronize()
    K.check_status()
    return {key: v.cpu() for key, v in out.items()}


def test_checked_build_matches_normal_build(kernels):
    normal, checked = kernels
    ref = _all_forms(normal)
    got = _all_forms(checked)          # check_status() raises on any out-of-bounds report
    for key, v in ref.items():
        if key == "f32acc":   # split-K fp32 atomics: the summation order differs run to run
            torch.testing.assert_close(got[key], v, rtol=1e-5, atol=1e-4)
        elif key == "attn_dqkv":   # dQ is summed over key tiles by TMA reduce-adds, in no fixed order
            torch.testing.assert_close(got[key].float(), v.float(), rtol=1e-2, atol=1e-3)
        else:
            assert torch.equal(got[key], v), f"{key}: the checked build computes something else"


def test_bounds_check_catches_a_short_allocation(kernels):
    """Host-side fault injection: the output is declared one row short, so the
    checked epilogue must report the last row's stores and skip them."""
    from h3_a100.ops.native import EPI_BF16

    _, checked = kernels
    m, n, k = 300, 264, 256
    x, w = bf(m, k), bf(n, k, scale=0.05)
    storage = torch.full((m, n + 1), float("nan"), dtype=torch.bfloat16, device="cuda")   # row-store path
    os.environ["H3_BOUNDS_SHRINK"] = str(n + 1)
    try:
        checked._gemm(x, False, w, False, m, n, k, EPI_BF16, storage[:, :n], block_n=128)
        torch.cuda.synchronize()
    finally:
        del os.environ["H3_BOUNDS_SHRINK"]
    code = int(checked.status[0])
    checked.status.zero_()
    assert code == 7, f"expected an out-of-bounds report, got status {code}"
    assert bool(torch.isnan(storage[m - 1, :n].float()).all()), "the reported stores were not skipped"
    assert not bool(torch.isnan(storage[: m - 1, :n].float()).any()), "rows inside the allocation were not written"
