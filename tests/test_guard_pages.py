"""Guard pages and canaries around the memory the kernels write.

compute-sanitizer is not available on the GPU pool, so out-of-bounds writes
and unwritten elements are caught structurally:

* every caller-provided output is a view into a larger buffer whose 4 KB
  before and after the view, and the gap columns of a row stride wider than
  the row, hold a sentinel byte pattern; after the kernel every sentinel byte
  must be intact;
* the output's own elements start as NaN and must all be overwritten;
* inputs sit in guarded buffers too and must come back bit for bit unchanged.

Shapes are ragged (M and N not multiples of the tiles) so the edge tiles of
the GEMM (single-CTA and 2-CTA pair mode), the attention tiles past T and
the elementwise tails all run.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

GUARD_BYTES = 4096
SENTINEL = 0xA5


class Guarded:
    """A [rows, cols] view with row stride ``ld`` inside a sentinel-filled buffer."""

    def __init__(self, rows, cols, dtype, ld=None, fill=float("nan")):
        self.rows, self.cols, self.ld = rows, cols, ld or cols
        self.itemsize = torch.empty(0, dtype=dtype).element_size()
        self.pad = GUARD_BYTES // self.itemsize
        self.buf = torch.empty(2 * self.pad + rows * self.ld, dtype=dtype, device="cuda")
        self.buf.view(torch.uint8).fill_(SENTINEL)
        self.body = self.buf[self.pad:self.pad + rows * self.ld].view(rows, self.ld)
        self.view = self.body[:, :cols]
        if fill is not None:
            self.view.copy_(fill if isinstance(fill, torch.Tensor) else torch.full_like(self.view, fill))

    def check(self, name, written=True):
        raw = self.buf.view(torch.uint8)
        head = raw[:self.pad * self.itemsize]
        tail = raw[(self.pad + self.rows * self.ld) * self.itemsize:]
        assert bool((head == SENTINEL).all()), f"{name}: write before the output"
        assert bool((tail == SENTINEL).all()), f"{name}: write after the output"
        if self.ld > self.cols:
            gap = self.body[:, self.cols:].contiguous().view(torch.uint8)
            assert bool((gap == SENTINEL).all()), f"{name}: write past the end of a row"
        if written:
            assert not bool(torch.isnan(self.view.float()).any()), f"{name}: output elements left unwritten"


def guarded_input(t: torch.Tensor) -> tuple[Guarded, torch.Tensor]:
    g = Guarded(t.shape[0], t.shape[1], t.dtype, fill=t)
    return g, t.clone()


def check_input(g: Guarded, copy: torch.Tensor, name: str) -> None:
    g.check(name, written=False)
    assert torch.equal(g.view, copy), f"{name}: an input was modified"


@pytest.fixture(scope="module")
def K():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from h3_a100.ops.native import NativeKernels

    return NativeKernels(torch.device("cuda", 0), wait_limit_s=5.0)


def bf(*shape, scale=1.0):
    return (torch.randn(*shape, device="cuda") * scale).to(torch.bfloat16)


def test_gemm_epilogues_stay_inside_their_outputs(K):
    """Every bf16 epilogue on ragged M/N (256-column tiles, 2-CTA pair mode),
    and the plain bf16 epilogue of the single-CTA 128-column kernel."""
    from h3_a100.ops.native import EPI_BF16, EPI_GATED_RES, EPI_GELU, EPI_ROPE

    torch.manual_seed(40)
    m, n, k, hd = 700, 1280 + 40, 512, 128
    xg, xc = guarded_input(bf(m, k))
    wg, wc = guarded_input(bf(n, k, scale=0.05))
    b = bf(n)
    ld = n + 72                                   # 2,784-byte rows: TMA-storable, with an 72-column gap
    out = Guarded(m, n, torch.bfloat16, ld=ld)
    K._gemm(xg.view, False, wg.view, False, m, n, k, EPI_BF16, out.view, bias=b)
    out128 = Guarded(m, n, torch.bfloat16, ld=ld)
    K._gemm(xg.view, False, wg.view, False, m, n, k, EPI_BF16, out128.view, bias=b, block_n=128)
    out2a, out2b = Guarded(m, n, torch.bfloat16, ld=ld), Guarded(m, n, torch.bfloat16, ld=ld)
    K._gemm(xg.view, False, wg.view, False, m, n, k, EPI_GELU, out2a.view, out2=out2b.view, bias=b)
    ang = torch.rand(m, hd // 2, device="cuda") * 6.28
    rope = Guarded(m, n, torch.bfloat16, ld=ld)
    K._gemm(xg.view, False, wg.view, False, m, n, k, EPI_ROPE, rope.view, bias=b, cos=ang.cos().contiguous(),
            sin=ang.sin().contiguous(), rope_cols=1024, head_dim=hd)
    resg, resc = guarded_input(bf(m, n))
    gate = torch.randn(2, n, device="cuda")
    gres = Guarded(m, n, torch.bfloat16, ld=ld)
    K._gemm(xg.view, False, wg.view, False, m, n, k, EPI_GATED_RES, gres.view, bias=b, res=resg.view, gate=gate,
            split_row=300)
    torch.cuda.synchronize()
    K.check_status()
    for name, g in (("bf16", out), ("bf16 128", out128), ("gelu pre", out2a), ("gelu post", out2b),
                    ("rope", rope), ("gated", gres)):
        g.check(name)
    torch.testing.assert_close(out.view.float(), (xc.float() @ wc.float().t() + b.float()), rtol=2e-2, atol=2e-2)
    check_input(xg, xc, "x")
    check_input(wg, wc, "w")
    check_input(resg, resc, "residual")


def test_gemm_row_store_and_input_gradient_forms(K):
    """The per-row store fallback (row stride not a multiple of 16 bytes), the
    MN-major B forms of the input gradient, and the fp32 split-K accumulate."""
    from h3_a100.ops.native import EPI_BF16, EPI_F32_ACC, EPI_GELU_BWD

    torch.manual_seed(41)
    m, n, k = 333, 264, 256
    x, w, b = bf(m, k), bf(n, k, scale=0.05), bf(n)
    odd = Guarded(m, n, torch.bfloat16, ld=n + 1)            # 530-byte rows: no tensor map
    K._gemm(x, False, w, False, m, n, k, EPI_BF16, odd.view, bias=b, block_n=128)
    t, n_out, k_in = 515, 768, 512
    dyg, dyc = guarded_input(bf(t, n_out))
    w2 = bf(n_out, k_in, scale=0.05)
    preg, prec = guarded_input(bf(t, k_in))
    dx = Guarded(t, k_in, torch.bfloat16, ld=k_in + 64)
    K._gemm(dyg.view, False, w2, True, t, k_in, n_out, EPI_GELU_BWD, dx.view, pre=preg.view)
    dx_plain = Guarded(t, k_in, torch.bfloat16, ld=k_in + 64)
    K._gemm(dyg.view, False, w2, True, t, k_in, n_out, EPI_BF16, dx_plain.view)
    # fp32 accumulate over a split K (atomic adds): the body starts at zero
    acc = Guarded(n_out, k_in, torch.float32, ld=k_in + 32, fill=0.0)
    K._gemm(dyg.view, True, preg.view, True, n_out, k_in, t, EPI_F32_ACC, acc.view, splits=3, block_n=128)
    torch.cuda.synchronize()
    K.check_status()
    odd.check("row-store fallback")
    dx.check("dx + gelu backward")
    dx_plain.check("dx")
    acc.check("fp32 split-K accumulate")
    torch.testing.assert_close(acc.view, dyc.float().t() @ prec.float(), rtol=2e-2, atol=2e-1)
    check_input(dyg, dyc, "dy")
    check_input(preg, prec, "gelu input")


def test_attention_and_norm_leave_inputs_untouched(K):
    """Kernels that allocate their outputs: the inputs (and their guards) are read only."""
    torch.manual_seed(42)
    t, heads, hd = 700, 2, 128
    qkvg, qkvc = guarded_input(bf(t, 3 * heads * hd))
    o, lse = K.attention_fwd(qkvg.view, heads, hd)
    dog, doc = guarded_input(bf(t, heads * hd))
    dqkv = K.attention_bwd(qkvg.view, o, lse, dog.view, heads, hd)
    xg, xc = guarded_input(bf(t, 512))
    mod = torch.randn(2, 6, 512, device="cuda") * 0.1
    y = K.norm_modulate(xg.view, mod[:, 0], mod[:, 1], 300)
    dyg, dyc = guarded_input(bf(t, 512))
    dx = K.norm_modulate_bwd(xg.view, dyg.view, mod[:, 1], 300, add=dyg.view, gate=mod[:, 2])
    torch.cuda.synchronize()
    K.check_status()
    outs = [("o", o), ("lse", lse), ("dqkv", dqkv), ("norm", y)]
    outs += [(f"norm bwd {i}", v) for i, v in enumerate(dx if isinstance(dx, (tuple, list)) else (dx,))
             if v is not None]
    for name, v in outs:
        assert bool(torch.isfinite(v.float()).all()), name
    check_input(qkvg, qkvc, "qkv")
    check_input(dog, doc, "do")
    check_input(xg, xc, "x")
    check_input(dyg, dyc, "dy")


def test_in_place_kernels_stay_inside_their_buffers(K):
    """RoPE inverse (in place on a strided view) and the fused AdamW step."""
    from h3_a100.ops.torch_kernels import Rope

    torch.manual_seed(43)
    t, h, hd = 301, 256, 128
    src = bf(t, 3 * h)
    g = Guarded(t, 3 * h, torch.bfloat16, ld=3 * h + 64, fill=src)
    ang = torch.rand(t, hd // 2, device="cuda")
    K.rope_bwd(g.view, Rope(ang.cos().contiguous(), ang.sin().contiguous(), hd, h, (0, 1)))
    n = 3 * 2**16 + 12
    master = Guarded(1, n, torch.float32, fill=torch.randn(1, n, device="cuda"))
    m1 = Guarded(1, n, torch.float32, fill=0.0)
    v1 = Guarded(1, n, torch.float32, fill=0.0)
    grad_g, grad_c = guarded_input(torch.randn(1, n, device="cuda"))
    param = Guarded(1, n, torch.bfloat16)
    norm = torch.ones(1, device="cuda")
    K.adamw_step(master.view[0], m1.view[0], v1.view[0], grad_g.view[0], param.view[0], norm, lr=1e-3, beta1=0.9,
                 beta2=0.999, eps=1e-8, weight_decay=0.01, step=1, max_norm=1.0)
    torch.cuda.synchronize()
    K.check_status()
    g.check("rope inverse")
    for name, b in (("master", master), ("exp_avg", m1), ("exp_avg_sq", v1), ("param", param)):
        b.check(name)
    check_input(grad_g, grad_c, "grad")


def test_peer_kernels_stay_inside_their_buffers():
    """The peer-memory kernels on one GPU (every peer pointer is this GPU's
    own buffer): pull all-gather, fused AdaLN GEMV + gather, fused LoRA step."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from h3_a100 import _C
    from h3_a100.parallel.p2p import LORA_SCRATCH_FLOATS

    torch.manual_seed(44)
    status = torch.zeros(4, dtype=torch.int32, device="cuda")
    units = 2**20 + 8
    shard_g, shard_c = guarded_input(torch.randn(1, units, device="cuda").to(torch.bfloat16))
    out = Guarded(1, units, torch.bfloat16)
    _C.p2p_all_gather([shard_g.view.data_ptr()], units * 2, out.view[0])
    rows, kk = 1030, 1024
    w = (torch.randn(rows, kk, device="cuda") * 0.05).to(torch.bfloat16)
    b = torch.randn(rows, device="cuda").to(torch.bfloat16)
    temb = torch.randn(2, kk, device="cuda").to(torch.bfloat16)
    flags = torch.zeros(64, dtype=torch.int32, device="cuda")
    ada = Guarded(2, rows, torch.float32)
    _C.adaln_project_gather(temb, w, b, [ada.view.data_ptr()], [flags.data_ptr()], 0, 1, 3, status, int(5e9))
    n = 2**18 + 64
    grad_g, grad_c = guarded_input(torch.randn(1, n, device="cuda"))
    param = Guarded(1, n, torch.bfloat16)
    master = Guarded(1, n, torch.float32, fill=torch.randn(1, n, device="cuda"))
    m1, v1 = Guarded(1, n, torch.float32, fill=0.0), Guarded(1, n, torch.float32, fill=0.0)
    lflags = torch.zeros(64, dtype=torch.int32, device="cuda")
    scratch = torch.zeros(LORA_SCRATCH_FLOATS, device="cuda")
    bar = torch.zeros(2, dtype=torch.int32, device="cuda")
    _C.lora_rs_adamw([grad_g.view.data_ptr()], [param.view.data_ptr()], [lflags.data_ptr()], 0, 1, master.view[0],
                     m1.view[0], v1.view[0], scratch, bar, 1e-2, 0.9, 0.999, 1e-8, 0.01, 1, 1.0, status, int(5e9),
                     0, 0)
    torch.cuda.synchronize()
    assert int(status[0]) == 0
    out.check("all-gather")
    assert torch.equal(out.view, shard_c)
    check_input(shard_g, shard_c, "shard")
    ada.check("adaln gather")
    for name, g in (("param", param), ("master", master), ("exp_avg", m1), ("exp_avg_sq", v1)):
        g.check(name)
    # the fused step reduces the (single-rank) gradient in place, averaged over the world of one
    torch.testing.assert_close(grad_g.view, grad_c)
    grad_g.check("grad", written=False)
