"""Race detection for the peer-memory kernels without a sanitizer: each fused
kernel runs twice from the same inputs (one GPU, every peer pointer this
GPU's own buffer) and the outputs must agree bit for bit, and with the
PyTorch fp32 statement of the op within tolerance."""

import pytest
import torch

from h3_a100.parallel.p2p import LORA_SCRATCH_FLOATS

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def C():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from h3_a100 import _C

    return _C


def _status():
    return torch.zeros(4, dtype=torch.int32, device="cuda")


def test_lora_step_is_bitwise_deterministic_and_matches_adamw(C):
    torch.manual_seed(0)
    n = 3 * 2**20 + 64
    grad = torch.randn(n, device="cuda")
    param0 = torch.randn(n, device="cuda").to(torch.bfloat16)
    outs = []
    for _ in range(2):
        param = param0.clone()
        master, m, v = param0.float(), torch.zeros(n, device="cuda"), torch.zeros(n, device="cuda")
        flags = torch.zeros(64, dtype=torch.int32, device="cuda")
        scratch = torch.zeros(LORA_SCRATCH_FLOATS, device="cuda")
        bar = torch.zeros(2, dtype=torch.int32, device="cuda")
        st = _status()
        C.lora_rs_adamw([grad.data_ptr()], [param.data_ptr()], [flags.data_ptr()], 0, 1, master, m, v, scratch, bar,
                        1e-2, 0.9, 0.999, 1e-8, 0.01, 1, 1.0, st, int(5e9), 0, 0)
        torch.cuda.synchronize()
        assert int(st[0]) == 0
        outs.append((param, master, m, v, scratch[15].clone()))
    for a, b in zip(outs[0], outs[1]):
        assert torch.equal(a, b)
    # fp32 oracle: clip by the global norm, then AdamW step 1
    norm = grad.norm()
    g = grad * min(1.0, 1.0 / (float(norm) + 1e-6))
    m_ref = 0.1 * g
    v_ref = 0.001 * g * g
    upd = (m_ref / 0.1) / ((v_ref / 0.001).sqrt() + 1e-8)
    master_ref = param0.float() * (1 - 1e-2 * 0.01) - 1e-2 * upd
    torch.testing.assert_close(outs[0][1], master_ref, rtol=1e-4, atol=1e-5)
    assert torch.equal(outs[0][0], outs[0][1].to(torch.bfloat16))   # the bf16 replica is the rounded master


def test_pull_all_gather_and_adaln_gather_are_bitwise_deterministic(C):
    torch.manual_seed(1)
    shard = torch.randn(4 * 2**20, device="cuda").to(torch.bfloat16)
    outs = []
    for _ in range(2):
        out = torch.empty_like(shard)
        C.p2p_all_gather([shard.data_ptr()], shard.numel() * 2, out)
        outs.append(out)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], shard) and torch.equal(outs[1], shard)
    rows, k = 1030, 1024
    w = (torch.randn(rows, k, device="cuda") * 0.05).to(torch.bfloat16)
    b = torch.randn(rows, device="cuda").to(torch.bfloat16)
    temb = torch.randn(2, k, device="cuda").to(torch.bfloat16)
    flags = torch.zeros(64, dtype=torch.int32, device="cuda")
    res = []
    for epoch in (1, 2):
        out = torch.full((2, rows), float("nan"), device="cuda")
        st = _status()
        C.adaln_project_gather(temb, w, b, [out.data_ptr()], [flags.data_ptr()], 0, epoch, 3, st, int(5e9))
        torch.cuda.synchronize()
        assert int(st[0]) == 0
        res.append(out)
    assert torch.equal(res[0], res[1])
    ref = torch.nn.functional.silu(temb.float()) @ w.float().t() + b.float()
    torch.testing.assert_close(res[0], ref, rtol=1e-3, atol=1e-3)
