"""Failure detection on the GPU without a GPU fault.

Every device-side spin-wait in the peer-memory kernels is bounded: when the
flag it waits for never arrives, the kernel records kStatusTimeoutPeer (5) in
a status word and returns, so the context stays usable and the host raises.
These tests make a wait run out on purpose -- a flag that nothing sets, with a
limit of a fraction of a second -- and check the status.  Nothing traps,
faults or spins unbounded.  The two-GPU case waits on 1 GPU for a flag in the
other GPU's memory (plain peer loads, no multicast) that the other side never
posts.
"""

from __future__ import annotations

import time

import pytest
import torch

pytestmark = pytest.mark.gpu

TIMEOUT_PEER = 5
LIMIT_NS = 200_000_000          # 0.2 s


@pytest.fixture(scope="module")
def C():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from h3_a100 import _C

    return _C


def _status(dev):
    return torch.zeros(4, dtype=torch.int32, device=dev)


def test_withheld_flag_times_out_and_context_survives(C):
    dev = torch.device("cuda", 0)
    flag, status = torch.zeros(1, dtype=torch.int32, device=dev), _status(dev)
    t0 = time.monotonic()
    C.wait_flag_test(flag, 1, status, LIMIT_NS)
    torch.cuda.synchronize()
    assert time.monotonic() - t0 < 10.0
    code, _, detail, count = status.tolist()
    assert (code, detail, count) == (TIMEOUT_PEER, 99, 1)
    # the context is still usable
    x = torch.arange(1024, device=dev, dtype=torch.float32)
    assert float(x.sum()) == 1023 * 1024 / 2


def test_posted_flag_passes(C):
    dev = torch.device("cuda", 0)
    flag, status = torch.ones(1, dtype=torch.int32, device=dev), _status(dev)
    C.wait_flag_test(flag, 1, status, LIMIT_NS)
    torch.cuda.synchronize()
    assert status.tolist() == [0, 0, 0, 0]


def test_native_kernels_raise_on_timeout_status(C):
    from h3_a100.ops.native import NativeKernels

    K = NativeKernels(torch.device("cuda", 0), wait_limit_s=0.2)
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    C.wait_flag_test(flag, 3, K.status, LIMIT_NS)
    with pytest.raises(RuntimeError, match="native kernel error"):
        K.check_status()
    K.check_status()        # the status word was cleared: the next step runs


def test_peer_flag_withheld_by_other_gpu(C):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    C.enable_peer_access(0, 1)
    flag = torch.zeros(1, dtype=torch.int32, device="cuda:1")     # lives on GPU 1, never posted
    status = _status("cuda:0")                                    # the wait runs on GPU 0
    C.wait_flag_test(flag, 1, status, LIMIT_NS)
    torch.cuda.synchronize(0)
    assert status[0].item() == TIMEOUT_PEER
    flag.fill_(1)                                                 # GPU 1 posts; the next wait passes
    torch.cuda.synchronize(1)
    status.zero_()
    C.wait_flag_test(flag, 1, status, LIMIT_NS)
    torch.cuda.synchronize(0)
    assert status[0].item() == 0
