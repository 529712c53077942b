"""Native sm_100a kernels vs the PyTorch fp32 oracle (same bf16 inputs)."""

from __future__ import annotations

import pytest
import torch

from h3_a100.ops.torch_kernels import GatedResidual, Rope, TorchKernels

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def K():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from h3_a100.ops.native import NativeKernels

    return NativeKernels(torch.device("cuda", 0), wait_limit_s=5.0)


R = TorchKernels()


def bf(*shape, scale=1.0):
    return (torch.randn(*shape, device="cuda") * scale).to(torch.bfloat16)


def close(a, b, tol=2e-2):
    a, b = a.float(), b.float()
    err = (a - b).abs().max().item()
    ref = b.abs().max().item() + 1e-6
    assert err <= tol * ref, f"max err {err:.4g} vs ref max {ref:.4g}"


def test_gemm_plain_and_bias(K):
    torch.manual_seed(0)
    x, w, b = bf(300, 384), bf(512, 384, scale=0.05), bf(512)
    close(K.linear(x, w, b), R.linear(x.float(), w.float(), b.float()))
    K.check_status()


def test_gemm_row_store_fallback(K):
    """An output whose row stride is not a multiple of 16 bytes cannot have a
    TMA tensor map: the epilogue falls back to per-row stores."""
    from h3_a100.ops.native import EPI_BF16

    torch.manual_seed(4)
    x, w, b = bf(200, 256), bf(264, 256, scale=0.05), bf(264)
    storage = torch.empty(200, 265, dtype=torch.bfloat16, device="cuda")   # 530-byte rows
    out = storage[:, :264]
    K._gemm(x, False, w, False, 200, 264, 256, EPI_BF16, out, bias=b, block_n=128)
    close(out, R.linear(x.float(), w.float(), b.float()))
    K.check_status()


def test_gemm_fused_gather_local_owners(K):
    """The all-gather fused into the GEMM, on one GPU: the weight's rows are
    split over three 'owner' buffers in local memory (the peer case differs
    only in where those pointers point); the gathered weight and the product
    must equal the plain GEMM on the full weight, on two calls in a row."""
    torch.manual_seed(5)
    n, k, m = 1000, 512, 300
    rows = 334                                      # owners hold 334, 334, 332 rows
    w, b = bf(n, k, scale=0.05), bf(n)
    x = bf(m, k)
    shards = [w[i * rows:(i + 1) * rows].clone() for i in range(3)]
    flags = torch.zeros((n + 255) // 256, dtype=torch.int32, device="cuda")
    ref = K.linear(x, w, b)
    for _ in range(2):
        w_local = torch.zeros_like(w)
        y = K.linear_allgather(x, w_local, ([t.data_ptr() for t in shards], rows, flags), bias=b)
        torch.cuda.synchronize()
        K.check_status()
        assert torch.equal(w_local, w)
        assert torch.equal(y, ref)


def test_gemm_large_tiles(K):
    torch.manual_seed(1)
    x, w = bf(1000, 1024), bf(1536, 1024, scale=0.03)
    close(K.linear(x, w), R.linear(x.float(), w.float()))
    K.check_status()


def test_gemm_lora_sections_rope(K):
    torch.manual_seed(2)
    t, h, hd, r = 333, 256, 128, 64
    x = bf(t, h)
    w, b = bf(3 * h, h, scale=0.05), bf(3 * h)
    a_cat, b_cat = bf(3 * r, h, scale=0.05), bf(3 * h, r, scale=0.05)
    ang = torch.rand(t, hd // 2, device="cuda") * 6.28
    rope = Rope(ang.cos(), ang.sin(), hd, h, (0, 1))
    u = K.lora_down(x, a_cat, 0.5)
    close(u, R.lora_down(x.float(), a_cat.float(), 0.5))
    y = K.linear(x, w, b, u, b_cat, 3, epilogue=rope)
    y_ref = R.linear(x.float(), w.float(), b.float(), u.float(), b_cat.float(), 3, epilogue=rope)
    close(y, y_ref)
    K.check_status()


def test_gemm_gelu_and_gated_residual(K):
    torch.manual_seed(3)
    t, h, f = 257, 256, 512
    x, w0, b0 = bf(t, h), bf(f, h, scale=0.06), bf(f)
    pre, post = K.linear(x, w0, b0, epilogue="gelu")
    pre_r, post_r = R.linear(x.float(), w0.float(), b0.float(), epilogue="gelu")
    close(pre, pre_r)
    close(post, post_r)
    res, gate = bf(t, h), torch.randn(2, h, device="cuda")
    w2, b2 = bf(h, f, scale=0.04), bf(h)
    ep = GatedResidual(res, gate, 100)
    close(K.linear(post, w2, b2, epilogue=ep),
          R.linear(post.float(), w2.float(), b2.float(), epilogue=GatedResidual(res.float(), gate, 100)))
    K.check_status()


def test_backward_gemms(K):
    torch.manual_seed(4)
    t, n, k, r = 515, 384, 256, 64
    dy, w = bf(t, n), bf(n, k, scale=0.05)
    b_cat, a_cat = bf(n, r, scale=0.05), bf(3 * r, k, scale=0.05)
    dyb = K.lora_dyb(dy, bf(n, r, scale=0.05), 1, 1.0)
    dyb3 = K.lora_dyb(dy, b_cat, 3, 2.0)
    b_sec = b_cat
    close(dyb3, R.lora_dyb(dy.float(), b_sec.float(), 3, 2.0))
    dx = K.linear_dx(dy, w, dyb3, a_cat)
    close(dx, R.linear_dx(dy.float(), w.float(), dyb3.float(), a_cat.float()))
    pre = bf(t, k)
    close(K.linear_dx(dy, w, gelu_pre=pre), R.linear_dx(dy.float(), w.float(), gelu_pre=pre.float()), tol=3e-2)
    assert dyb.shape == (t, r)
    K.check_status()


def test_lora_wgrad_split_k(K):
    torch.manual_seed(5)
    t, n, k, r = 4000, 384, 256, 64
    dy, x = bf(t, n, scale=0.1), bf(t, k)
    u, dyb = bf(t, 3 * r), bf(t, 3 * r, scale=0.1)
    ga = torch.ones(3 * r, k, device="cuda")
    gb = torch.ones(n, r, device="cuda")
    ga_r, gb_r = ga.clone(), gb.clone()
    K.lora_wgrad(dy, x, u, dyb, 3, ga, gb)
    R.lora_wgrad(dy.float(), x.float(), u.float(), dyb.float(), 3, ga_r, gb_r)
    close(ga, ga_r, tol=1e-2)
    close(gb, gb_r, tol=1e-2)
    K.check_status()


def test_norm_modulate_and_gate(K):
    torch.manual_seed(6)
    t, h, split = 77, 512, 50
    x, dy, add = bf(t, h), bf(t, h), bf(t, h)
    mod = torch.randn(2, 6, h, device="cuda") * 0.3
    close(K.norm_modulate(x, mod[:, 0], mod[:, 1], split), R.norm_modulate(x.float(), mod[:, 0], mod[:, 1], split))
    dx, g = K.norm_modulate_bwd(x, dy, mod[:, 1], split, add=add, gate=mod[:, 2])
    dx_r, g_r = R.norm_modulate_bwd(x.float(), dy.float(), mod[:, 1], split, add=add.float(), gate=mod[:, 2])
    close(dx, dx_r)
    close(g, g_r)
    close(K.gate_mul(dy, mod[:, 5], split), R.gate_mul(dy.float(), mod[:, 5], split))
    K.check_status()


def test_rope_inverse_roundtrip(K):
    torch.manual_seed(7)
    t, h, hd = 90, 256, 128
    y = bf(t, 3 * h)
    ang = torch.rand(t, hd // 2, device="cuda") * 6.28
    rope = Rope(ang.cos(), ang.sin(), hd, h, (0, 1))
    close(K.rope_bwd(y.clone(), rope), R.rope_bwd(y.float(), rope))


def test_adaln_project(K):
    torch.manual_seed(8)
    temb, w, b = bf(2, 1024), bf(6 * 256, 1024, scale=0.03), bf(6 * 256)
    close(K.adaln_project(temb, w, b), R.adaln_project(temb.float(), w.float(), b.float()), tol=1e-2)


def test_flow_dmd_mse_ops(K):
    torch.manual_seed(9)
    xt, v = torch.randn(1, 24, 3, 8, 8, device="cuda"), torch.randn(1, 24, 3, 8, 8, device="cuda")
    x0, nxt = K.flow_step(xt, v, 0.7, 0.4, torch.float32)
    x0_r, nxt_r = R.flow_step(xt, v, 0.7, 0.4, torch.float32)
    close(x0, x0_r, 1e-5)
    close(nxt, nxt_r, 1e-5)
    noise = torch.randn_like(xt)
    close(K.add_noise(xt, noise, 0.3), R.add_noise(xt, noise, 0.3), 1e-5)
    gen = torch.randn_like(xt, requires_grad=True)
    fake, real = torch.randn_like(xt), torch.randn_like(xt)
    l = K.dmd_loss(gen, fake, real)
    l.backward()
    g_native = gen.grad.clone()
    gen.grad = None
    l_r = R.dmd_loss(gen, fake, real)
    l_r.backward()
    close(l, l_r, 1e-4)
    close(g_native, gen.grad, 1e-4)
    p = torch.randn_like(xt, requires_grad=True)
    m = K.mse_loss(p, real)
    m.backward()
    gp = p.grad.clone()
    p.grad = None
    R.mse_loss(p, real).backward()
    close(m, R.mse_loss(p, real), 1e-4)
    close(gp, p.grad, 1e-4)


def test_x0_autograd(K):
    xt = torch.randn(1, 4, 2, 4, 4, device="cuda")
    v = torch.randn_like(xt, requires_grad=True)
    x0 = K.x0_from_velocity(xt, v, 0.6)
    x0.sum().backward()
    close(x0, xt + 0.6 * v.detach(), 1e-6)
    close(v.grad, torch.full_like(v, 0.6), 1e-6)


def test_adamw_matches_reference(K):
    torch.manual_seed(10)
    n = 10_001
    master = torch.randn(n, device="cuda")
    grad = torch.randn(n, device="cuda")
    states = [(master.clone(), torch.zeros(n, device="cuda"), torch.zeros(n, device="cuda")) for _ in range(2)]
    params = [torch.empty(n, dtype=torch.bfloat16, device="cuda") for _ in range(2)]
    norm_n = K.sum_squares(grad).sqrt()
    norm_r = R.sum_squares(grad).sqrt()
    close(norm_n, norm_r, 1e-5)
    for step in (1, 2):
        K.adamw_step(*states[0], grad, params[0], norm_n, lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8,
                     weight_decay=0.01, step=step, max_norm=1.0)
        R.adamw_step(*states[1], grad, params[1], norm_r, lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8,
                     weight_decay=0.01, step=step, max_norm=1.0)
    close(states[0][0], states[1][0], 1e-5)
    close(params[0], params[1], 1e-2)


def test_block_forward_backward_matches_oracle(K):
    """Whole DiT block with LoRA: native forward/backward vs the fp32 oracle on the same weights."""
    from h3_a100.models.block import BlockContext, block_backward, block_forward

    torch.manual_seed(11)
    t, h, f, heads, hd, r = 200, 256, 512, 2, 128, 64
    w = {"qkv_weight": bf(3 * h, h, scale=0.06), "qkv_bias": bf(3 * h, scale=0.1),
         "out_weight": bf(h, h, scale=0.06), "out_bias": bf(h, scale=0.1),
         "ff0_weight": bf(f, h, scale=0.06), "ff0_bias": bf(f, scale=0.1),
         "ff2_weight": bf(h, f, scale=0.04), "ff2_bias": bf(h, scale=0.1)}
    lora = {"qkv": (bf(3 * r, h, scale=0.05), bf(3 * h, r, scale=0.05)), "o": (bf(r, h, scale=0.05), bf(h, r, scale=0.05)),
            "ff0": (bf(r, h, scale=0.05), bf(f, r, scale=0.05)), "ff2": (bf(r, f, scale=0.05), bf(h, r, scale=0.05))}
    mod = torch.randn(2, 6, h, device="cuda") * 0.2
    ang = torch.rand(t, hd // 2, device="cuda") * 6.28
    rope = Rope(ang.cos(), ang.sin(), hd, h, (0, 1))
    x, dout = bf(t, h), bf(t, h)

    def run(kern, cast):
        sinks = {k: (torch.zeros(a.shape, device="cuda"), torch.zeros(b.shape, device="cuda")) for k, (a, b) in lora.items()}
        ctx = BlockContext(kern, mod, 150, rope, heads, hd, 1e-6,
                           {k: (cast(a), cast(b)) for k, (a, b) in lora.items()}, 1.0, sinks)
        ww = {k: cast(v) for k, v in w.items()}
        out, saved = block_forward(ctx, cast(x), ww, save=True)
        dx = block_backward(ctx, cast(dout), ww, saved)
        return out, dx, sinks

    out_n, dx_n, sink_n = run(K, lambda v: v)
    out_r, dx_r, sink_r = run(R, lambda v: v.float())
    close(out_n, out_r, 3e-2)
    close(dx_n, dx_r, 5e-2)
    for name in lora:
        close(sink_n[name][0], sink_r[name][0], 5e-2)
        close(sink_n[name][1], sink_r[name][1], 5e-2)
    K.check_status()


@pytest.mark.parametrize("t,heads", [(300, 2), (1000, 3), (128, 1)])
def test_attention_forward_matches_oracle(K, t, heads):
    torch.manual_seed(12)
    hd = 128
    qkv = bf(t, 3 * heads * hd)
    o, lse = K.attention_fwd(qkv, heads, hd)
    o_r, lse_r = R.attention_fwd(qkv.float(), heads, hd)
    close(o, o_r, 3e-2)
    close(lse, lse_r, 1e-3)
    K.check_status()


def test_attention_forward_large_logits(K):
    """Rows whose max grows across KV tiles exercise the lazy O rescaling."""
    torch.manual_seed(13)
    t, heads, hd = 700, 2, 128
    qkv = bf(t, 3 * heads * hd, scale=4.0)
    o, lse = K.attention_fwd(qkv, heads, hd)
    o_r, lse_r = R.attention_fwd(qkv.float(), heads, hd)
    close(o, o_r, 3e-2)
    close(lse, lse_r, 2e-3)
    K.check_status()


def test_attention_forward_max_jumps_late(K):
    """A key tile far past the first one (and the masked last tile) raises
    some rows' max by much more than the lazy-rescale threshold, so O and the
    row sum must be rescaled mid-sequence."""
    torch.manual_seed(15)
    t, heads, hd = 640, 2, 128
    qkv = bf(t, 3 * heads * hd, scale=2.0).float()
    h = heads * hd
    qkv[384:512, h:2 * h] *= 4.0          # keys of KV tile 3
    qkv[600:, h:2 * h] *= 6.0             # and of the masked last tile
    qkv = qkv.to(torch.bfloat16)
    o, lse = K.attention_fwd(qkv, heads, hd)
    o_r, lse_r = R.attention_fwd(qkv.float(), heads, hd)
    close(o, o_r, 3e-2)
    close(lse, lse_r, 2e-3)
    K.check_status()


@pytest.mark.parametrize("t,heads", [(300, 2), (640, 1), (1000, 3)])
def test_attention_backward_matches_oracle(K, t, heads):
    if not hasattr(K.C, "attention_bwd"):
        pytest.skip("extension built without the tcgen05 attention backward")
    torch.manual_seed(14)
    hd = 128
    qkv = bf(t, 3 * heads * hd)
    o, lse = K.attention_fwd(qkv, heads, hd)
    do = bf(t, heads * hd)
    dqkv = K.attention_bwd(qkv, o, lse, do, heads, hd)
    dqkv_r = R.attention_bwd(qkv.float(), o.float(), None, do.float(), heads, hd)
    h = heads * hd
    for s in range(3):
        close(dqkv[:, s * h:(s + 1) * h], dqkv_r[:, s * h:(s + 1) * h], 4e-2)
    K.check_status()
