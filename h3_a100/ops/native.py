"""Kernel set backed by the hand-written sm_100a extension ``h3_a100._C``.

Same interface as ``TorchKernels``.  Every GEMM-shaped op runs on the
tcgen05 GEMM (``csrc/gemm/gemm_tcgen05.cu``) with its epilogue fused:

* ``linear``      y = x W^T + U_s B^T in ONE accumulation (second K-phase),
                  then bias + RoPE / GELU / gated residual in the epilogue;
* ``linear_dx``   dx = dy W + dyb A_cat in one accumulation, GELU' fused for FF2;
* ``lora_down``   U_s = s * x A_cat^T (alpha = s folded into the epilogue);
* ``lora_dyb``    dyb = s * dy_sec B_sec per section;
* ``lora_wgrad``  dA_cat += dyb^T x and dB_sec += dy_sec^T U_sec, fp32
                  accumulate epilogue, split over K with atomics.

Norm/modulate, gate, RoPE-inverse, AdaLN projection, flow/DMD elementwise
passes, sum-of-squares and AdamW are the kernels of
``csrc/elementwise/elementwise.cu``; attention is ``csrc/attn``.

Importing this module without the compiled extension raises: on a GPU the
native path never falls back silently.
"""

from __future__ import annotations

import torch

try:
    from .. import _C
except ImportError as exc:  # pragma: no cover - exercised only on broken installs
    raise ImportError(
        "h3_a100._C (the sm_100a extension) is not built; run `python setup.py build_ext --inplace`"
    ) from exc

from .torch_kernels import GatedResidual, Rope

EPI_BF16, EPI_GELU, EPI_ROPE = _C.EPI_BF16, _C.EPI_GELU, _C.EPI_ROPE
EPI_GATED_RES, EPI_GELU_BWD, EPI_F32_ACC = _C.EPI_GATED_RES, _C.EPI_GELU_BWD, _C.EPI_F32_ACC
STATUS_NAMES = {1: "timeout waiting for a TMA stage", 2: "timeout waiting for a free stage",
                3: "timeout waiting for an accumulator", 4: "timeout waiting for the epilogue",
                5: "timeout waiting for a peer GPU", 6: "bad argument",
                7: "out-of-bounds access caught by the bounds-checked build"}


def _num_sms(device: torch.device) -> int:
    return torch.cuda.get_device_properties(device).multi_processor_count


class NativeKernels:
    name = "native"
    native = True

    def __init__(self, device: torch.device, *, wait_limit_s: float = 10.0, extension=None) -> None:
        """``extension``: the compiled module to run (default ``h3_a100._C``;
        tests pass ``h3_a100._C_checked``, the bounds-checked build)."""
        if device.type != "cuda":
            raise ValueError("NativeKernels needs a CUDA device")
        self.device = device
        self.C = extension if extension is not None else _C
        self.status = torch.zeros(4, dtype=torch.int32, device=device)
        self.limit_ns = int(wait_limit_s * 1e9)
        self.sms = _num_sms(device)
        self._ones = torch.ones(1, dtype=torch.float32, device=device)
        missing = [name for name in ("gemm", "attention_fwd", "attention_bwd") if not hasattr(_C, name)]
        if missing:
            raise RuntimeError(f"the sm_100a extension lacks {missing}; rebuild it (python setup.py build_ext --inplace)")

    # ------------------------------------------------------------ bookkeeping
    def launch_count(self) -> int:
        return int(self.C.launch_count())

    def check_status(self) -> None:
        """Raise if any kernel recorded a bounded-wait timeout (synchronizes)."""
        code, block, detail, count = (int(v) for v in self.status.tolist())
        if code != 0:
            self.status.zero_()
            raise RuntimeError(f"native kernel error: {STATUS_NAMES.get(code, code)} "
                               f"(block {block}, detail {detail}, {count} reports)")

    def _gemm(self, A, a_mn, B, b_mn, M, N, K, epi, out, *, A2=(), B2=None, K2=0, section_n=0, out2=None,
              bias=None, res=None, gate=None, split_row=0, cos=None, sin=None, rope_cols=0, head_dim=0,
              pre=None, alpha=1.0, splits=1, block_n=256, gather=None):
        """``gather`` = (owner shard pointers, rows per owner, int32 per-N-tile counters) fuses
        the all-gather of a row-sharded K-major B into the GEMM (B is then the local destination)."""
        g_src, g_rows, g_flags = gather if gather is not None else ([], 0, None)
        self.C.gemm(A, a_mn, B, b_mn, int(M), int(N), int(K), list(A2), B2, int(K2), int(section_n), int(epi),
                    out, out2, bias, res, gate, int(split_row), cos, sin, int(rope_cols), int(head_dim), pre,
                    float(alpha), int(splits), int(block_n), self.status, self.limit_ns, list(g_src), int(g_rows),
                    g_flags)

    def _splits(self, tiles: int, k: int) -> int:
        kb = (k + 63) // 64
        want = max(1, (2 * self.sms + tiles - 1) // tiles)
        return int(max(1, min(want, kb // 8 if kb >= 8 else 1)))

    # ------------------------------------------------------------ norms
    def norm_modulate(self, x, shift, scale, split, eps=1e-6):
        return self.C.norm_modulate_fwd(x, shift, scale, int(split), float(eps))

    def norm_modulate_bwd(self, x, dy, scale, split, eps=1e-6, add=None, gate=None):
        out = self.C.norm_modulate_bwd(x, dy, scale, int(split), float(eps), add, gate)
        return out[0] if gate is None else (out[0], out[1])

    def gate_mul(self, dout, gate, split):
        return self.C.gate_mul(dout, gate, int(split))

    # ------------------------------------------------------------ linears
    def lora_down(self, x, a_cat, scale=1.0):
        m, k = x.shape
        n = a_cat.shape[0]
        out = torch.empty(m, n, dtype=x.dtype, device=x.device)
        self._gemm(x, False, a_cat, False, m, n, k, EPI_BF16, out, alpha=scale, block_n=128)
        return out

    def linear(self, x, w, b=None, u=None, b_cat=None, sections=1, epilogue=None):
        m, k = x.shape
        n = w.shape[0]
        out = torch.empty(m, n, dtype=x.dtype, device=x.device)
        kw = {}
        if u is not None:
            r = u.shape[1] // sections
            section_n = n // sections if sections > 1 else 0
            kw = dict(A2=[u[:, s * r:(s + 1) * r] for s in range(sections)], B2=b_cat, K2=r, section_n=section_n,
                      block_n=256 if section_n % 256 == 0 else 128)
        if epilogue is None:
            self._gemm(x, False, w, False, m, n, k, EPI_BF16, out, bias=b, **kw)
            return out
        if epilogue == "gelu":
            post = torch.empty_like(out)
            self._gemm(x, False, w, False, m, n, k, EPI_GELU, out, out2=post, bias=b, **kw)
            return out, post
        if isinstance(epilogue, Rope):
            rope_cols = epilogue.section_width * len(epilogue.sections)
            self._gemm(x, False, w, False, m, n, k, EPI_ROPE, out, bias=b, cos=epilogue.cos, sin=epilogue.sin,
                       rope_cols=rope_cols, head_dim=epilogue.head_dim, **kw)
            return out
        if isinstance(epilogue, GatedResidual):
            self._gemm(x, False, w, False, m, n, k, EPI_GATED_RES, out, bias=b, res=epilogue.residual,
                       gate=epilogue.gate, split_row=epilogue.split, **kw)
            return out
        raise ValueError(f"unknown epilogue {epilogue!r}")

    def lora_dyb(self, dy, b_cat, sections, scale=1.0):
        m, n = dy.shape
        r = b_cat.shape[1]
        width = n // sections
        out = torch.empty(m, sections * r, dtype=dy.dtype, device=dy.device)
        for s in range(sections):
            self._gemm(dy[:, s * width:(s + 1) * width], False, b_cat[s * width:(s + 1) * width], True,
                       m, r, width, EPI_BF16, out[:, s * r:(s + 1) * r], alpha=scale, block_n=128)
        return out

    def linear_dx(self, dy, w, dyb=None, a_cat=None, gelu_pre=None):
        m, n_out = dy.shape
        k_in = w.shape[1]
        out = torch.empty(m, k_in, dtype=dy.dtype, device=dy.device)
        kw = {}
        if dyb is not None:
            kw = dict(A2=[dyb], B2=a_cat, K2=dyb.shape[1])
        if gelu_pre is not None:
            self._gemm(dy, False, w, True, m, k_in, n_out, EPI_GELU_BWD, out, pre=gelu_pre, **kw)
        else:
            self._gemm(dy, False, w, True, m, k_in, n_out, EPI_BF16, out, **kw)
        return out

    def lora_wgrad(self, dy, x, u, dyb, sections, grad_a, grad_b):
        t, n = dy.shape
        k_in = x.shape[1]
        rs = dyb.shape[1]
        tiles = ((rs + 127) // 128) * ((k_in + 255) // 256)
        self._gemm(dyb, True, x, True, rs, k_in, t, EPI_F32_ACC, grad_a, splits=self._splits(tiles, t))
        r = u.shape[1] // sections
        width = n // sections
        for s in range(sections):
            tiles = ((width + 127) // 128) * ((r + 127) // 128)
            self._gemm(dy[:, s * width:(s + 1) * width], True, u[:, s * r:(s + 1) * r], True, width, r, t,
                       EPI_F32_ACC, grad_b[s * width:(s + 1) * width], splits=self._splits(tiles, t), block_n=128)

    def gelu_bwd(self, dy, pre):
        raise NotImplementedError("the native kernel set fuses the GELU backward into the FF2 input-gradient "
                                  "GEMM: call linear_dx(..., gelu_pre=pre)")

    def rope_bwd(self, dqkv, rope: Rope):
        self.C.rope_inverse_(dqkv, rope.cos, rope.sin, rope.section_width * len(rope.sections), rope.head_dim)
        return dqkv

    # ------------------------------------------------------------ attention
    def attention_fwd(self, qkv, heads, head_dim):
        o, lse = self.C.attention_fwd(qkv, int(heads), int(head_dim), self.status, self.limit_ns)
        return o, lse

    def attention_bwd(self, qkv, o, lse, do, heads, head_dim):
        if lse is None:
            raise ValueError("the tcgen05 attention backward needs the forward's log-sum-exp rows")
        return self.C.attention_bwd(qkv, o, lse, do, int(heads), int(head_dim), self.status, self.limit_ns)

    # ------------------------------------------------------------ small projections
    def adaln_project(self, temb, w, b):
        return self.C.adaln_project(temb.to(torch.bfloat16).contiguous(), w, b)

    # ------------------------------------------------------------ optimizer
    def sum_squares(self, t):
        return self.C.sum_squares(t)

    def adamw_step(self, master, exp_avg, exp_avg_sq, grad, param_out, norm, *, lr, beta1, beta2, eps,
                   weight_decay, step, max_norm):
        self.C.adamw_step(master, exp_avg, exp_avg_sq, grad, param_out, norm, lr, beta1, beta2, eps,
                          weight_decay, int(step), max_norm)

    def linear_allgather(self, x, w_local, gather, bias=None, block_n=256):
        """y = x W^T + b where W's rows live sharded on the peers: the GEMM's
        gather warps pull each N-tile's rows into ``w_local`` (this rank's
        full-size buffer) while the tensor core works on the tiles already
        there.  ``gather`` comes from ``PeerComm.gather_spec``."""
        m, k = x.shape
        n = w_local.shape[0]
        out = torch.empty(m, n, dtype=torch.bfloat16, device=x.device)
        self._gemm(x.contiguous(), False, w_local, False, m, n, k, EPI_BF16, out, bias=bias, block_n=block_n,
                   gather=gather)
        return out

    # ------------------------------------------------------------ flow / DMD
    def flow_step(self, xt, velocity, sigma, sigma_next, out_dtype):
        x0, nxt = self.C.flow_step(xt.contiguous(), velocity.contiguous(), float(sigma), float(sigma_next),
                                   True, True, out_dtype)
        return x0, nxt

    def x0_from_velocity(self, xt, velocity, sigma):
        return _X0.apply(xt, velocity, float(sigma), self)

    def add_noise(self, x0, noise, sigma):
        return self.C.add_noise(x0.contiguous(), noise.contiguous(), float(sigma))

    def randn(self, shape, dtype, device, generator=None):
        return torch.randn(shape, dtype=dtype, device=device, generator=generator)

    def dmd_loss(self, generated, x0_fake, x0_real):
        return _DMDLoss.apply(generated, x0_fake.contiguous(), x0_real.contiguous(), self)

    def mse_loss(self, pred, target):
        return _MSELoss.apply(pred, target.contiguous(), self)


class _X0(torch.autograd.Function):
    """x0 = xt + sigma * v (fp32); gradient sigma * dx0 flows to v only."""

    @staticmethod
    def forward(ctx, xt, v, sigma, k):
        ctx.sigma, ctx.k, ctx.v_dtype = sigma, k, v.dtype
        x0, _ = k.C.flow_step(xt.contiguous(), v.contiguous(), sigma, sigma, True, False, torch.float32)
        return x0

    @staticmethod
    def backward(ctx, g):
        dv = ctx.k.C.scale_copy(g.contiguous().float(), ctx.sigma, ctx.k._ones, ctx.v_dtype)
        return None, dv, None, None


class _DMDLoss(torch.autograd.Function):
    @staticmethod
    def forward(ctx, generated, x0_fake, x0_real, k):
        loss, grad = k.C.dmd_forward(generated.contiguous(), x0_fake, x0_real)
        ctx.save_for_backward(grad)
        ctx.k, ctx.dtype, ctx.n = k, generated.dtype, generated.numel()
        return loss.reshape(())

    @staticmethod
    def backward(ctx, g):
        (grad,) = ctx.saved_tensors
        dgen = ctx.k.C.scale_copy(grad, 1.0 / ctx.n, g.reshape(1).float().contiguous(), ctx.dtype)
        return dgen, None, None, None


class _MSELoss(torch.autograd.Function):
    @staticmethod
    def forward(ctx, pred, target, k):
        ctx.save_for_backward(pred, target)
        ctx.k = k
        return k.C.mse_forward(pred.contiguous(), target).reshape(())

    @staticmethod
    def backward(ctx, g):
        pred, target = ctx.saved_tensors
        return ctx.k.C.mse_backward(pred.contiguous(), target, g.reshape(1).float().contiguous()), None, None
