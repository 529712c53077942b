"""The hand-written block backward vs autograd of a plain fp32 PyTorch block."""

import math

import torch

from h3_a100.models.block import BlockContext, block_backward, block_forward
from h3_a100.ops.torch_kernels import Rope, TorchKernels, gelu_tanh


def _rows(t, split, table):
    return torch.cat([table[0].expand(split, -1), table[1].expand(t - split, -1)], 0)


def _rope(y, cos, sin, hd, width):
    out = y.clone()
    for s in (0, 1):
        part = y[:, s * width:(s + 1) * width].reshape(y.shape[0], -1, hd // 2, 2)
        e, o = part[..., 0], part[..., 1]
        c, sn = cos[:, None, :], sin[:, None, :]
        rot = torch.stack([e * c - o * sn, e * sn + o * c], -1).reshape(y.shape[0], width)
        out = torch.cat([out[:, :s * width], rot, out[:, (s + 1) * width:]], 1)
    return out


def naive_block(x, w, lora, mod, cos, sin, split, heads, hd, scale, eps=1e-6):
    t, h = x.shape

    def norm(v, sh, sc):
        n = v * torch.rsqrt(v.pow(2).mean(-1, keepdim=True) + eps)
        return n * (1 + _rows(t, split, sc)) + _rows(t, split, sh)

    def lin(v, name, wk, bk, sections=1):
        a, b = lora[name]
        y = v @ w[wk].t() + w[bk]
        r = a.shape[0] // sections
        width = y.shape[1] // sections
        ups = [scale * (v @ a[s * r:(s + 1) * r].t()) @ b[s * width:(s + 1) * width].t() for s in range(sections)]
        return y + torch.cat(ups, 1)

    h1 = norm(x, mod[:, 0], mod[:, 1])
    qkv = _rope(lin(h1, "qkv", "qkv_weight", "qkv_bias", 3), cos, sin, hd, h)
    q, k, v = qkv.view(t, 3, heads, hd).permute(1, 2, 0, 3).unbind(0)
    o = (torch.softmax(q @ k.transpose(-1, -2) / math.sqrt(hd), -1) @ v).transpose(0, 1).reshape(t, h)
    x1 = x + _rows(t, split, mod[:, 2]) * lin(o, "o", "out_weight", "out_bias")
    h2 = norm(x1, mod[:, 3], mod[:, 4])
    act = gelu_tanh(lin(h2, "ff0", "ff0_weight", "ff0_bias"))
    return x1 + _rows(t, split, mod[:, 5]) * lin(act, "ff2", "ff2_weight", "ff2_bias")


def test_explicit_backward_matches_autograd():
    torch.manual_seed(0)
    t, h, f, heads, hd, r, split, scale = 23, 32, 48, 2, 16, 4, 15, 0.5
    g = lambda *s, k=0.2: (torch.randn(*s) * k).double()  # noqa: E731
    w = {"qkv_weight": g(3 * h, h), "qkv_bias": g(3 * h), "out_weight": g(h, h), "out_bias": g(h),
         "ff0_weight": g(f, h), "ff0_bias": g(f), "ff2_weight": g(h, f), "ff2_bias": g(h)}
    lora = {"qkv": (g(3 * r, h), g(3 * h, r)), "o": (g(r, h), g(h, r)), "ff0": (g(r, h), g(f, r)),
            "ff2": (g(r, f), g(h, r))}
    mod = g(2, 6, h)
    ang = torch.rand(t, hd // 2).double() * 6
    cos, sin = ang.cos(), ang.sin()
    x, dout = g(t, h, k=1.0), g(t, h, k=1.0)

    x_ag = x.clone().requires_grad_(True)
    lora_ag = {k: (a.clone().requires_grad_(True), b.clone().requires_grad_(True)) for k, (a, b) in lora.items()}
    out_ag = naive_block(x_ag, w, lora_ag, mod, cos, sin, split, heads, hd, scale)
    out_ag.backward(dout)

    sinks = {k: (torch.zeros_like(a), torch.zeros_like(b)) for k, (a, b) in lora.items()}
    ctx = BlockContext(TorchKernels(), mod, split, Rope(cos, sin, hd, h, (0, 1)), heads, hd, 1e-6, lora, scale, sinks)
    out, saved = block_forward(ctx, x, w, save=True)
    dx = block_backward(ctx, dout, w, saved)
    torch.testing.assert_close(out, out_ag.detach(), rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(dx, x_ag.grad, rtol=1e-4, atol=1e-5)
    for name, (a, b) in lora_ag.items():
        torch.testing.assert_close(sinks[name][0], a.grad, rtol=1e-4, atol=1e-5)
        torch.testing.assert_close(sinks[name][1], b.grad, rtol=1e-4, atol=1e-5)
