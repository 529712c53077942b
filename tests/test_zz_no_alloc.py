"""The allocation-free DMD loss entry point, called through its exported C symbol.

It is for callers that may not allocate device memory (their host
application owns the whole device-memory budget), so the test hands it
caller-owned buffers only and compares it with the regular entry point
(``h3_a100._C.dmd_forward``) on two calls in a row.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

MAX_SAMPLES = 1024


@pytest.fixture(scope="module")
def entry():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import h3_a100._C as C

    lib = ctypes.CDLL(C.__file__)
    fn = lib.h3_dmd_loss_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_longlong, ctypes.c_longlong,
                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    return C, fn


def _call(fn, gen, fake, real, loss, grad, samples):
    stream = torch.cuda.current_stream().cuda_stream
    return fn(gen.data_ptr(), fake.data_ptr(), real.data_ptr(), samples, gen.numel() // samples,
              loss.data_ptr(), grad.data_ptr(), stream)


@pytest.mark.parametrize("shape_a,shape_b", [((1, 24, 3, 8, 8), (1, 32, 50)), ((1, 4, 1000), (1, 4, 1000))])
def test_noalloc_matches_regular_entry_point_twice(entry, shape_a, shape_b):
    C, fn = entry
    torch.manual_seed(0)
    for shape in (shape_a, shape_b):
        gen = torch.randn(shape, device="cuda")
        real = torch.randn(shape, device="cuda")
        fake = real + 0.1 * torch.randn(shape, device="cuda")
        loss = torch.full((1,), -1.0, device="cuda")
        grad = torch.full_like(gen, float("nan"))
        assert _call(fn, gen, fake, real, loss, grad, 1) == 0
        ref_loss, ref_grad = C.dmd_forward(gen, fake, real)
        torch.cuda.synchronize()
        torch.testing.assert_close(loss, ref_loss, rtol=1e-4, atol=1e-6)
        torch.testing.assert_close(grad, ref_grad, rtol=1e-4, atol=1e-6)


@pytest.mark.parametrize("samples,per_sample", [(3, 5000), (MAX_SAMPLES, 300)])
def test_noalloc_multi_sample_matches_fp32_formula(entry, samples, per_sample):
    """Several samples per call: per-sample normalisers (one grid row each), the
    second accumulator half and the final sum over samples, against the fp32
    PyTorch statement of the DMD loss, on two calls in a row (the second call
    finds the first call's sums in the shared scratch and must clear them)."""
    from h3_a100.trainer.dmd_math import dmd_direction, dmd_loss

    _, fn = entry
    torch.manual_seed(1)
    for call in range(2):
        gen = torch.randn(samples, per_sample, device="cuda") * (1.0 + call)
        real = torch.randn(samples, per_sample, device="cuda")
        # per-sample scale so every sample has its own normaliser
        real = real * torch.linspace(0.5, 2.0, samples, device="cuda")[:, None]
        fake = real + 0.1 * torch.randn(samples, per_sample, device="cuda")
        loss = torch.full((1,), -1.0, device="cuda")
        grad = torch.full_like(gen, float("nan"))
        assert _call(fn, gen, fake, real, loss, grad, samples) == 0
        torch.cuda.synchronize()
        ref_grad = dmd_direction(gen, fake, real)
        ref_loss = dmd_loss(gen, fake, real)
        torch.testing.assert_close(grad, ref_grad, rtol=1e-4, atol=1e-5)
        torch.testing.assert_close(loss[0], ref_loss, rtol=1e-4, atol=1e-6)


def test_noalloc_rejects_too_many_samples(entry):
    _, fn = entry
    gen = torch.zeros(MAX_SAMPLES + 1, 8, device="cuda")
    loss = torch.full((1,), 7.0, device="cuda")
    grad = torch.full_like(gen, 3.0)
    assert _call(fn, gen, gen, gen, loss, grad, MAX_SAMPLES + 1) == -2
    torch.cuda.synchronize()
    assert float(loss) == 7.0 and bool((grad == 3.0).all())
