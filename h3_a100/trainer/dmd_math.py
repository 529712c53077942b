"""Flow-matching and DMD math (re-derived; LightX2V's versions are external).

What the reference shows (``h3_a100/trainer_runtime.py:80-212``) fixes the
parametrisation, and everything here is consistent with it:

* noising ``x_sigma = (1 - sigma) * x0 + sigma * eps`` (rectified flow);
* the model predicts ``v = x0 - eps``, so ``x0 = x_sigma + sigma * v`` and the
  Euler step from ``sigma`` to ``sigma'`` is ``x + (sigma - sigma') * v``;
* the Fake (critic) regresses ``v`` onto ``x0 - eps``;
* the rollout schedule is ``linspace(1, 0, steps + 1)`` warped by the usual
  flow shift ``s*t / (1 + (s - 1)*t)`` (video 6.0, audio 3.0);
* the renoise level is continuous, ``u ~ U(sigma_min, sigma_max)``, warped by
  the same per-modality shift.

The DMD generator loss is DMD2's (Yin et al., 2024): with
``g = (x0_fake - x0_real) / mean|x - x0_real|`` (per sample, no grad), the
loss is ``0.5 * mean((x - stop_grad(x - g))^2)`` whose gradient w.r.t. ``x``
is ``g / numel``.  When Fake == Teacher (cycle 1: LoRA B starts at zero) the
loss is exactly 0, as in the reference log (``dmd=0.000000``).

The elementwise passes run through the kernel set (native sm_100a kernels on
GPU); these functions define the math and are the CPU oracle.
"""

from __future__ import annotations

import torch


def shifted_sigmas(num_steps: int, shift: float) -> torch.Tensor:
    base = torch.linspace(1.0, 0.0, int(num_steps) + 1, dtype=torch.float64)
    return (shift * base / (1.0 + (shift - 1.0) * base)).float()


def shift_sigma(u: torch.Tensor, shift: float) -> torch.Tensor:
    return shift * u / (1.0 + (shift - 1.0) * u)


def add_noise(x0: torch.Tensor, noise: torch.Tensor, sigma) -> torch.Tensor:
    return ((1.0 - sigma) * x0.float() + sigma * noise.float()).to(x0.dtype)


def x0_from_velocity(xt: torch.Tensor, velocity: torch.Tensor, sigma) -> torch.Tensor:
    return xt.float() + sigma * velocity.float()


def euler_step(xt: torch.Tensor, velocity: torch.Tensor, sigma, sigma_next, out_dtype) -> torch.Tensor:
    return (xt.float() + (sigma - sigma_next) * velocity.float()).to(out_dtype)


def dmd_direction(generated: torch.Tensor, x0_fake: torch.Tensor, x0_real: torch.Tensor) -> torch.Tensor:
    g = generated.float()
    real = x0_real.float()
    dims = tuple(range(1, g.dim()))
    normalizer = (g - real).abs().mean(dim=dims, keepdim=True).clamp_min(1e-12)
    return torch.nan_to_num((x0_fake.float() - real) / normalizer)


def dmd_loss(generated: torch.Tensor, x0_fake: torch.Tensor, x0_real: torch.Tensor) -> torch.Tensor:
    with torch.no_grad():
        grad = dmd_direction(generated, x0_fake, x0_real)
        target = generated.float() - grad
    return 0.5 * torch.mean((generated.float() - target) ** 2)


def dmd_loss_pair(generated, x0_fake, x0_teacher, w_video: float, w_audio: float) -> torch.Tensor:
    loss = w_video * dmd_loss(generated[0], x0_fake[0], x0_teacher[0])
    if generated[1] is not None and w_audio:
        loss = loss + w_audio * dmd_loss(generated[1], x0_fake[1], x0_teacher[1])
    return loss


def weighted_mse_pair(pred, target, w_video: float, w_audio: float) -> torch.Tensor:
    loss = w_video * torch.mean((pred[0].float() - target[0].float()) ** 2)
    if pred[1] is not None and w_audio:
        loss = loss + w_audio * torch.mean((pred[1].float() - target[1].float()) ** 2)
    return loss
