"""tcgen05 attention at the production sequence length.

The small-shape tests in test_native_kernels.py cover the tile logic; these
run the H3 joint sequence (37,730 tokens = 295 KV tiles, the last one 98 rows
deep) with all 42 heads, so every CTA of the real grid runs, and compare a few
heads against an fp32 oracle.  The oracle is PyTorch's scaled-dot-product
attention on fp32 inputs (its memory-efficient kernel), because the explicit
T x T score matrix of the plain fp32 formula does not fit at this length.
"""

from __future__ import annotations

import math

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

T, HEADS, HD = 37730, 42, 128
CHECK_HEADS = (0, 41)


@pytest.fixture(scope="module")
def K():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from h3_a100.ops.native import NativeKernels

    k = NativeKernels(torch.device("cuda", 0), wait_limit_s=5.0)
    return k


def _sub_qkv(qkv: torch.Tensor, heads: tuple[int, ...]) -> torch.Tensor:
    v = qkv.view(T, 3, HEADS, HD)[:, :, list(heads)]
    return v.reshape(T, 3 * len(heads) * HD)


def _oracle(qkv_sub: torch.Tensor, n: int, do_sub: torch.Tensor | None = None):
    x = qkv_sub.float().view(T, 3, n, HD).permute(1, 2, 0, 3)      # [3, n, T, hd]
    q, k, v = (t.contiguous().requires_grad_(do_sub is not None) for t in x)
    with torch.enable_grad():
        o = F.scaled_dot_product_attention(q[None], k[None], v[None])[0]   # [n, T, hd]
        grads = None
        if do_sub is not None:
            dov = do_sub.float().view(T, n, HD).permute(1, 0, 2)
            grads = torch.autograd.grad(o, (q, k, v), dov)
    lse = torch.empty(n, T, device=qkv_sub.device)
    for h in range(n):
        for s in range(0, T, 4096):
            lse[h, s:s + 4096] = torch.logsumexp(q[h, s:s + 4096].detach() @ k[h].detach().t() / math.sqrt(HD), -1)
    return o.detach().permute(1, 0, 2).reshape(T, n * HD), lse, grads


def _rel(a: torch.Tensor, b: torch.Tensor) -> float:
    return ((a.float() - b.float()).abs().max() / (b.float().abs().max() + 1e-6)).item()


@pytest.mark.parametrize("scale", [1.0, 3.0])
def test_attention_forward_full_sequence(K, scale):
    torch.manual_seed(21)
    qkv = (torch.randn(T, 3 * HEADS * HD, device="cuda") * scale).to(torch.bfloat16)
    o, lse = K.attention_fwd(qkv, HEADS, HD)
    torch.cuda.synchronize()
    K.check_status()
    assert torch.isfinite(o).all() and torch.isfinite(lse).all()
    o_r, lse_r, _ = _oracle(_sub_qkv(qkv, CHECK_HEADS), len(CHECK_HEADS))
    o_sub = o.view(T, HEADS, HD)[:, list(CHECK_HEADS)].reshape(T, -1)
    assert _rel(o_sub, o_r) < 3e-2
    assert (lse[list(CHECK_HEADS)].float() - lse_r).abs().max().item() < 2e-2 * max(1.0, lse_r.abs().max().item())


def test_attention_backward_full_sequence(K):
    torch.manual_seed(22)
    qkv = (torch.randn(T, 3 * HEADS * HD, device="cuda") * 2.0).to(torch.bfloat16)
    do = torch.randn(T, HEADS * HD, device="cuda").to(torch.bfloat16)
    o, lse = K.attention_fwd(qkv, HEADS, HD)
    dqkv = K.attention_bwd(qkv, o, lse, do, HEADS, HD)
    torch.cuda.synchronize()
    K.check_status()
    assert torch.isfinite(dqkv).all()
    n = len(CHECK_HEADS)
    do_sub = do.view(T, HEADS, HD)[:, list(CHECK_HEADS)].reshape(T, -1)
    _, _, (dq, dk, dv) = _oracle(_sub_qkv(qkv, CHECK_HEADS), n, do_sub)
    got = dqkv.view(T, 3, HEADS, HD)[:, :, list(CHECK_HEADS)]
    for s, ref in enumerate((dq, dk, dv)):
        assert _rel(got[:, s].permute(1, 0, 2), ref) < 5e-2, f"d{'qkv'[s]} mismatch"
