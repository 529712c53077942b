"""Flow-matching / DMD identities the runtime relies on."""

import torch

from h3_a100.ops.torch_kernels import TorchKernels
from h3_a100.trainer.dmd_math import (
    add_noise, dmd_direction, dmd_loss, dmd_loss_pair, euler_step, shift_sigma, shifted_sigmas, weighted_mse_pair,
    x0_from_velocity)


def test_velocity_parametrisation_round_trip():
    torch.manual_seed(0)
    x0, eps = torch.randn(2, 5), torch.randn(2, 5)
    sigma, nxt = 0.7, 0.3
    xt = add_noise(x0, eps, sigma)
    v = x0 - eps
    torch.testing.assert_close(x0_from_velocity(xt, v, sigma), x0)
    torch.testing.assert_close(euler_step(xt, v, sigma, nxt, torch.float32), add_noise(x0, eps, nxt))


def test_schedule_is_shifted_and_ends_at_zero():
    s = shifted_sigmas(4, 6.0)
    assert s.shape == (5,) and s[0] == 1.0 and s[-1] == 0.0
    assert torch.all(s[:-1] > s[1:])
    assert abs(float(shift_sigma(torch.tensor(0.5), 3.0)) - 0.75) < 1e-6


def test_dmd_loss_zero_when_fake_equals_teacher_and_gradient():
    torch.manual_seed(1)
    gen = torch.randn(1, 3, 4, requires_grad=True)
    real = torch.randn(1, 3, 4)
    assert float(dmd_loss(gen, real, real)) == 0.0
    fake = real + 0.1 * torch.randn(1, 3, 4)
    loss = dmd_loss(gen, fake, real)
    loss.backward()
    direction = dmd_direction(gen.detach(), fake, real)
    torch.testing.assert_close(gen.grad, direction / gen.numel())
    torch.testing.assert_close(loss, 0.5 * direction.pow(2).mean())


def test_pair_losses_and_kernel_set_agree():
    torch.manual_seed(2)
    K = TorchKernels()
    gen = (torch.randn(1, 2, 3), torch.randn(1, 4, 5))
    fake = (torch.randn(1, 2, 3), torch.randn(1, 4, 5))
    real = (torch.randn(1, 2, 3), torch.randn(1, 4, 5))
    ref = dmd_loss_pair(gen, fake, real, 1.0, 0.5)
    mine = K.dmd_loss(gen[0], fake[0], real[0]) + 0.5 * K.dmd_loss(gen[1], fake[1], real[1])
    torch.testing.assert_close(ref, mine)
    mse = weighted_mse_pair(gen, real, 1.0, 2.0)
    torch.testing.assert_close(mse, K.mse_loss(gen[0], real[0]) + 2.0 * K.mse_loss(gen[1], real[1]))
    x0, nxt = K.flow_step(gen[0], fake[0], 0.6, 0.2, torch.float32)
    torch.testing.assert_close(x0, gen[0] + 0.6 * fake[0])
    torch.testing.assert_close(nxt, gen[0] + 0.4 * fake[0])
