"""DMD runtime: rollouts, the Student DMD loss and the Fake (critic) loss.

Same algorithm and call counts as the reference's ``H3A100RuntimeMixin``
(``h3_a100/trainer_runtime.py:17-216``):

* ``run_back_simulation``: 4 Student evaluations at the rollout sigmas, grad
  only at the fixed end step 3; per step ``x0 = xt + sigma*v`` and the Euler
  step in fp32 cast to the latent dtype; each step's AdaLN modulations are a
  persistent key ``("rollout", i)``.
* ``forward_student_loss``: grad rollout -> continuous renoise sigma -> fp32
  noise -> Fake and Teacher no-grad predictions under one dynamic key
  ``("score", n)`` -> DMD loss.
* ``prepare_fake_update``: a no-grad rollout + renoise (the critic's input).
* ``fake_loss``: grad Fake prediction regressed onto ``x0 - eps``.

Every DiT call names its role explicitly and is counted by the census.
"""

from __future__ import annotations

import dataclasses
from typing import Any

import torch

from ..models.lora import FAKE, STUDENT, TEACHER
from .dmd_math import shift_sigma, shifted_sigmas
from .matched_contract import FAKE_ROLE, STUDENT_ROLE, TEACHER_ROLE

_LOGICAL = {STUDENT: STUDENT_ROLE, FAKE: FAKE_ROLE, TEACHER: TEACHER_ROLE}


@dataclasses.dataclass
class PreparedFakeUpdate:
    latent_shape: dict[str, Any]
    condition: dict[str, torch.Tensor]
    generated: tuple[torch.Tensor, torch.Tensor | None]
    noises: tuple[torch.Tensor, torch.Tensor | None]
    renoised: tuple[torch.Tensor, torch.Tensor | None]
    sigmas: tuple[float, float]
    cache_key: tuple[str, int]


class DMDRuntimeMixin:
    # ---------------------------------------------------------------- schedule
    def _init_schedule(self) -> None:
        self.video_sigmas_cpu = shifted_sigmas(self.num_inference_steps, self.video_flow_shift)
        self.audio_sigmas_cpu = shifted_sigmas(self.num_inference_steps, self.audio_flow_shift)
        self._score_serial = 0

    def _sample_synced_int(self, low: int, high: int) -> int:
        if self.matched_compute_enabled and int(low) == 0 and int(high) == int(self.num_inference_steps):
            return int(self.matched_fixed_end_step_idx)
        return int(torch.randint(int(low), int(high), (1,), generator=self.host_rng).item())

    def _sample_renoise_sigmas(self) -> tuple[float, float]:
        u = torch.empty(1).uniform_(self.renoise_sigma_min, self.renoise_sigma_max, generator=self.host_rng)
        return float(shift_sigma(u, self.video_flow_shift)), float(shift_sigma(u, self.audio_flow_shift))

    def _timesteps(self, sigmas) -> torch.Tensor:
        t = torch.tensor([float(sigmas[0]), float(sigmas[1])], dtype=torch.float32) * self.num_train_timesteps
        return t.to(self.device, non_blocking=True)

    def sample_initial_latents(self, latent_shape) -> tuple[torch.Tensor, torch.Tensor | None]:
        video = torch.randn(latent_shape["video"], device=self.device, dtype=torch.float32).to(self.latent_dtype)
        audio = None
        if latent_shape.get("audio") is not None:
            audio = torch.randn(latent_shape["audio"], device=self.device, dtype=torch.float32).to(self.latent_dtype)
        return video, audio

    @staticmethod
    def _randn_like_exact(t: torch.Tensor | None) -> torch.Tensor | None:
        return None if t is None else torch.randn_like(t, dtype=torch.float32)

    def _next_score_key(self) -> tuple[str, int]:
        self._score_serial += 1
        return ("score", self._score_serial)

    # ---------------------------------------------------------------- forwards
    def _predict(self, role: str, latents, sigmas, condition, key):
        grad = bool(torch.is_grad_enabled())
        self.matched_cycle_census.note_forward(_LOGICAL[role], grad_enabled=grad)
        timesteps = self._timesteps(sigmas)
        with self.timeline.span("compute", f"{role}_forward{'_grad' if grad else ''}"):
            return self.model.predict_velocity(role, latents, timesteps, condition, adaln_key=key)

    def _pair(self, fn, a, b):
        return fn(a[0], b[0], 0), (None if a[1] is None else fn(a[1], b[1], 1))

    def run_back_simulation(self, condition, latent_shape, end_step_idx: int, grad_enabled: bool, xt=None):
        K = self.kernels
        if xt is None:
            xt = self.sample_initial_latents(latent_shape)
        x0, backward_key = None, None
        for step in range(end_step_idx + 1):
            sig = (float(self.video_sigmas_cpu[step]), float(self.audio_sigmas_cpu[step]))
            nxt = (float(self.video_sigmas_cpu[step + 1]), float(self.audio_sigmas_cpu[step + 1]))
            key = ("rollout", int(step))
            self.model.precompute_adaln(key, self._timesteps(sig), persistent=True)
            with_grad = grad_enabled and step == end_step_idx
            with torch.set_grad_enabled(with_grad), self.model.adaln_scope(key):
                velocity = self._predict(STUDENT, xt, sig, condition, key)
            if with_grad:
                backward_key = key
                # The grad step is the last: only x0 carries the graph.
                x0 = tuple(None if v is None else K.x0_from_velocity(x, v, s)
                           for x, v, s in zip(xt, velocity, sig))
            else:
                outs = [None if v is None else K.flow_step(x, v, s, n, self.latent_dtype)
                        for x, v, s, n in zip(xt, velocity, sig, nxt)]
                x0 = tuple(None if o is None else o[0] for o in outs)
                xt = tuple(None if o is None else o[1] for o in outs)
        if x0 is None:
            raise RuntimeError("rollout produced no x0 prediction")
        gen = tuple(None if t is None else t.to(self.latent_dtype) for t in x0)
        return gen, backward_key

    def forward_student_loss(self, latent_shape, condition) -> dict[str, Any]:
        K = self.kernels
        end = self._sample_synced_int(0, self.num_inference_steps)
        generated, backward_key = self.run_back_simulation(condition, latent_shape, end, grad_enabled=True)
        sigmas = self._sample_renoise_sigmas()
        noises = (self._randn_like_exact(generated[0]), self._randn_like_exact(generated[1]))
        renoised = tuple(None if g is None else K.add_noise(g.detach(), n, s)
                         for g, n, s in zip(generated, noises, sigmas))
        score_key = self._next_score_key()
        self.model.precompute_adaln(score_key, self._timesteps(sigmas), persistent=False)
        with torch.no_grad(), self.model.adaln_scope(score_key):
            v_fake = self._predict(FAKE, renoised, sigmas, condition, score_key)
            v_teacher = self._predict(TEACHER, renoised, sigmas, condition, score_key)
            x0_fake = tuple(None if v is None else K.x0_from_velocity(r, v, s)
                            for r, v, s in zip(renoised, v_fake, sigmas))
            x0_teacher = tuple(None if v is None else K.x0_from_velocity(r, v, s)
                               for r, v, s in zip(renoised, v_teacher, sigmas))
        self.model.drop_adaln_key(score_key)
        loss = self.video_loss_weight * K.dmd_loss(generated[0], x0_fake[0], x0_teacher[0])
        if generated[1] is not None and self.audio_loss_weight:
            loss = loss + self.audio_loss_weight * K.dmd_loss(generated[1], x0_fake[1], x0_teacher[1])
        if backward_key is None:
            raise RuntimeError("Student DMD loss has no rollout backward cache key")
        return {"loss": loss, "dmd": loss.detach(), "backward_key": backward_key}

    @torch.no_grad()
    def prepare_fake_update(self, latent_shape, condition) -> PreparedFakeUpdate:
        K = self.kernels
        end = self._sample_synced_int(0, self.num_inference_steps)
        generated, _ = self.run_back_simulation(condition, latent_shape, end, grad_enabled=False)
        sigmas = self._sample_renoise_sigmas()
        noises = (self._randn_like_exact(generated[0]), self._randn_like_exact(generated[1]))
        renoised = tuple(None if g is None else K.add_noise(g, n, s) for g, n, s in zip(generated, noises, sigmas))
        return PreparedFakeUpdate(latent_shape, condition, generated, noises, renoised, sigmas, self._next_score_key())

    def fake_loss(self, item: PreparedFakeUpdate) -> torch.Tensor:
        K = self.kernels
        self.model.precompute_adaln(item.cache_key, self._timesteps(item.sigmas), persistent=False)
        with self.model.adaln_scope(item.cache_key):
            v_fake = self._predict(FAKE, item.renoised, item.sigmas, item.condition, item.cache_key)
            loss = self.video_loss_weight * K.mse_loss(v_fake[0], item.generated[0].float() - item.noises[0])
            if v_fake[1] is not None and self.audio_loss_weight:
                loss = loss + self.audio_loss_weight * K.mse_loss(
                    v_fake[1], item.generated[1].float() - item.noises[1])
        return loss
