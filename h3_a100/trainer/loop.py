"""Outer DMD cycle: Student step, reordered critic phase, fail-closed validation.

Same schedule as the reference's ``H3A100LoopMixin``
(``h3_a100/trainer_loop.py:33-293``): one Student update, then the critic
phase with rollout reordering (all 5 no-grad Student rollouts first, then the
5 ordered Fake updates).  After every cycle the census (local + gathered
global), the boundary-staging deltas (6/1/5/0/300/300) and the exact-replay
deltas (300/600/600/0) are checked and a violation raises.

``run_cycle`` is the public one-cycle entry point (used by ``train`` and by the
benchmark); it returns the cycle's losses as host floats, which is the one
device->host read per cycle.
"""

from __future__ import annotations

from typing import Any, Iterator

import torch

from ..memory.exact_replay import cycle_delta, expected_cycle_counts
from ..models.lora import FAKE, STUDENT
from ..parallel import distributed as pdist
from ..utils.log import logger
from ..utils.memory import log_cuda_memory
from ..utils.nvtx import nvtx
from .data import to_device
from .matched_contract import FAKE_ROLE, STUDENT_ROLE, validate_global_snapshots
from .runtime import PreparedFakeUpdate


class LoopMixin:
    # ---------------------------------------------------------------- public
    def train(self) -> None:
        resume_path, current = self._resolve_resume_a100()
        self.setup(resume_ckpt_path=resume_path)
        pdist.barrier()
        samples = self.samples()
        logger.info("[h3-a100] train start iter={}/{} world={} grad_accum={} fake_ratio={} reorder={}",
                    current, self.max_train_iters, pdist.get_world_size(), self.gradient_accumulation_iters,
                    self.fake_update_ratio, self.reorder_critic_rollouts)
        if torch.cuda.is_available():
            torch.cuda.reset_peak_memory_stats()
        while current < self.max_train_iters:
            losses = self.run_cycle(samples, current)
            current += 1
            if current == 1 or current % self.train_log_every_iters == 0:
                dmd, fake = pdist.reduce_mean(losses["dmd"]), pdist.reduce_mean(losses["fake"])
                lr = self.lr_schedulers[STUDENT].get_last_lr()[0]
                logger.info("[h3-a100] iter={}/{} dmd={:.6f} fake={:.6f} lr={:.8f}", current,
                            self.max_train_iters, dmd, fake, lr)
                self.metrics.append({"iter": current, "train/dmd": dmd, "train/fake": fake, "train/lr": lr})
                self.model.log_adaln_stats()
                log_cuda_memory(f"iter_{current}")
            if self.save_every_iters and current % self.save_every_iters == 0:
                self.save_checkpoint_a100(current)
        logger.info("[h3-a100] train finished iter={}/{}", current, self.max_train_iters)

    def samples(self) -> Iterator[dict[str, Any]]:
        if self.data is None:
            raise RuntimeError("trainer has no data; call set_data()")
        return iter(self.data)

    def run_cycle(self, samples: Iterator[dict[str, Any]], current_iter: int = 0, *,
                  validate: bool = True) -> dict[str, float]:
        """One matched cycle: Student x1, Fake x5 (reordered), then the contract checks."""
        self.matched_cycle_census.reset()
        self._begin_cycle_counters()
        self.timeline.start_cycle()
        self.timer.start("student_step")
        with nvtx("h3/student_step"):
            dmd = self._student_step(samples)
        self.timer.stop("student_step")
        self.timer.start("critic_phase")
        with nvtx("h3/critic_phase"):
            fake = self._fake_steps(samples)
        self.timer.stop("critic_phase")
        values = torch.stack([dmd.reshape(()).float(), fake.reshape(()).float()]).cpu()
        self._record_cycle_times()
        self._record_timeline(current_iter)
        if validate:
            self._validate_cycle(current_iter)
        return {"dmd": float(values[0]), "fake": float(values[1])}

    def _record_timeline(self, current_iter: int) -> None:
        """Lane unions of this cycle (and a Chrome trace) when ``H3_TIMELINE`` is set."""
        if not self.timeline.enabled:
            return
        import os

        rows = self.timeline.collect()
        self.last_cycle_receipt["timeline"] = self.timeline.unions(rows)
        path = os.path.join(self.timeline.out_dir, f"timeline_rank{pdist.get_rank():02d}_iter{current_iter:04d}.json")
        self.timeline.write_chrome_trace(rows, path, pid=pdist.get_rank())
        logger.info("[h3-a100][timeline] iter={} rank={} {}", current_iter, pdist.get_rank(),
                    self.last_cycle_receipt["timeline"])

    def _record_cycle_times(self) -> None:
        """Per-phase device seconds and exposed (non-overlapped) collective time of this cycle.

        Phases come from CUDA events on the compute stream; ``optimizer_step``
        is the device time of the six optimizer steps, which contain the LoRA
        gradient reduce-scatter (fused with clip + AdamW on the peer-memory
        transport); ``all_gather`` is the time the compute stream stalled on
        the prefetched frozen-weight gathers.
        """
        phases = self.timer.take()
        stalls = self.stall_ledger.collect()
        self.last_cycle_receipt["phases_s"] = {k: round(v / 1e3, 4) for k, v in sorted(phases.items())}
        self.last_cycle_receipt["exposed_comm_s"] = {
            "all_gather": round(stalls.get("all_gather", 0.0) / 1e3, 4),
            "optimizer_step_incl_reduce_scatter": round(phases.get("optimizer_step", 0.0) / 1e3, 4),
        }

    # ---------------------------------------------------------------- steps
    def _next_sample(self, samples, stage: str):
        sample = next(samples)
        self.matched_cycle_census.note_sample(stage, sample)
        self.h2d_bytes += sum(v.numel() * v.element_size() for v in sample.values() if torch.is_tensor(v))
        return to_device(sample, self.device)

    def _student_step(self, samples) -> torch.Tensor:
        opt = self.optimizers[STUDENT]
        opt.zero_grad()
        running = torch.zeros((), device=self.device)
        for _ in range(self.gradient_accumulation_iters):
            sample = self._next_sample(samples, "student")
            condition, latent_shape = self._encode_conditions(sample), self._latent_shape(sample)
            self.residency("before_student_grad_forward")
            with self._activation_offload_scope("student") as offload:
                result = self.forward_student_loss(latent_shape, condition)
                self.residency("after_student_grad_forward")
                if offload is not None:
                    offload.begin_backward()
                with self.model.adaln_scope(result["backward_key"]):
                    self.matched_cycle_census.note_backward(STUDENT_ROLE)
                    with self.timeline.span("compute", "student_backward"):
                        (result["loss"] / self.gradient_accumulation_iters).backward()
                self.residency("after_student_backward")
            running = running + result["dmd"] / self.gradient_accumulation_iters
        self.timer.start("optimizer_step")
        with self.timeline.span("compute", "student_optimizer_step"):
            opt.step(self.lr_schedulers[STUDENT].get_last_lr()[0])
        self.timer.stop("optimizer_step")
        self.lr_schedulers[STUDENT].step()
        opt.zero_grad()
        return running

    def _fake_steps(self, samples) -> torch.Tensor:
        running = torch.zeros((), device=self.device)
        if self.reorder_critic_rollouts:
            self.timer.start("critic_prepare")
            with nvtx("h3/critic_prepare_5xG"):
                groups = [self._prepare_one_fake_group(samples, i) for i in range(self.fake_update_ratio)]
            self.timer.stop("critic_prepare")
            self.timer.start("critic_updates")
            for group in groups:
                with nvtx("h3/critic_update_F"):
                    running = running + self._apply_one_fake_group(group) / self.fake_update_ratio
            self.timer.stop("critic_updates")
            return running
        for i in range(self.fake_update_ratio):
            group = self._prepare_one_fake_group(samples, i)
            running = running + self._apply_one_fake_group(group) / self.fake_update_ratio
        return running

    def _prepare_one_fake_group(self, samples, fake_index: int) -> list[PreparedFakeUpdate]:
        group = []
        for _ in range(self.gradient_accumulation_iters):
            sample = self._next_sample(samples, f"fake_{fake_index}")
            group.append(self.prepare_fake_update(self._latent_shape(sample), self._encode_conditions(sample)))
            self.residency(f"after_fake_{fake_index}_rollout_prepare")
        return group

    def _apply_one_fake_group(self, group: list[PreparedFakeUpdate]) -> torch.Tensor:
        opt = self.optimizers[FAKE]
        opt.zero_grad()
        total = torch.zeros((), device=self.device)
        for micro, item in enumerate(group):
            with self._activation_offload_scope(f"fake_{micro}") as offload:
                loss = self.fake_loss(item)
                if offload is not None:
                    offload.begin_backward()
                with self.model.adaln_scope(item.cache_key):
                    self.matched_cycle_census.note_backward(FAKE_ROLE)
                    with self.timeline.span("compute", "fake_backward"):
                        (loss / len(group)).backward()
            self.model.drop_adaln_key(item.cache_key)
            total = total + loss.detach() / len(group)
        self.timer.start("optimizer_step")
        with self.timeline.span("compute", "fake_optimizer_step"):
            opt.step(self.lr_schedulers[FAKE].get_last_lr()[0])
        self.timer.stop("optimizer_step")
        self.lr_schedulers[FAKE].step()
        opt.zero_grad()
        return total

    # ---------------------------------------------------------------- checks
    def _begin_cycle_counters(self) -> None:
        staging = self.boundary_staging
        self._boundary_start = None if staging is None else dict(staging.stats)
        audit = self.replay_audit
        self._replay_start = None if audit is None else dict(audit.stats)

    def _validate_cycle(self, current_iter: int) -> None:
        if self.matched_compute_enabled:
            self._validate_matched_cycle(current_iter)
        self._validate_boundary_offload_cycle(current_iter)
        self._validate_exact_replay_cycle(current_iter)

    def _validate_boundary_offload_cycle(self, current_iter: int) -> None:
        reg = self.boundary_staging
        if reg is None:
            return
        if self._boundary_start is None:
            raise RuntimeError("checkpoint-boundary staging cycle baseline is missing")
        blocks = reg.expected_block_count
        expected = {
            "grad_transformer_forward_count": 6,
            "student_grad_forward_count": 1,
            "fake_grad_forward_count": 5,
            "other_grad_forward_count": 0,
            "grad_checkpoint_call_count": 6 * blocks,
            "cpu_copy_count": 6 * blocks,
        }
        observed = {k: int(reg.stats[k]) - int(self._boundary_start.get(k, 0)) for k in expected}
        errors = [f"{k}={observed[k]} expected={v}" for k, v in expected.items() if observed[k] != v]
        if errors:
            raise RuntimeError(f"checkpoint-boundary CPU staging contract failed at outer iteration "
                               f"{current_iter}: {'; '.join(errors)}")
        offloaded = int(reg.stats["offloaded_storage_bytes"]) - int(self._boundary_start.get("offloaded_storage_bytes", 0))
        self.last_cycle_receipt["boundary"] = {**observed, "offloaded_gib": offloaded / 1024**3,
                                               "staging": self.boundary_staging_report()}
        logger.info("[h3-a100][boundary-offload] iter={} rank={} policy={} observed={} offloaded_gib={:.2f}",
                    current_iter, pdist.get_rank(), reg.receipt()["policy"], observed, offloaded / 1024**3)

    def _validate_exact_replay_cycle(self, current_iter: int) -> None:
        rep = self.replay_audit
        if rep is None:
            return
        if self._replay_start is None:
            raise RuntimeError("exact AdaLN replay cycle baseline is missing")
        expected = expected_cycle_counts(self.model.dit_config.num_blocks,
                                         segment_size=self.activation_checkpoint_segment_size)
        observed = cycle_delta(rep.stats, self._replay_start)
        errors = [f"{k}={observed[k]} expected={v}" for k, v in expected.items() if observed[k] != v]
        if errors:
            raise RuntimeError(f"exact AdaLN checkpoint-replay contract failed at outer iteration "
                               f"{current_iter}: {'; '.join(errors)}")
        self.last_cycle_receipt["exact_replay"] = observed
        logger.info("[h3-a100][exact-adaln-replay] iter={} observed={}", current_iter, observed)

    def _validate_matched_cycle(self, current_iter: int) -> None:
        census = self.matched_cycle_census
        local = census.validate_local()
        snapshot = census.snapshot()
        snapshots = pdist.all_gather_object(snapshot)
        errors = local + validate_global_snapshots(
            snapshots, expected_world_size=self.matched_expected_world_size,
            require_unique_samples=self.matched_require_unique_samples)
        if errors:
            raise RuntimeError(f"Matched compute contract failed at outer iteration {current_iter}: "
                               f"{'; '.join(errors[:12])}")
        self.last_cycle_receipt["census"] = {
            "forwards": snapshot["forward_counts"], "grad_forwards": snapshot["grad_forward_counts"],
            "backwards": snapshot["backward_counts"], "samples": len(snapshot["samples"]),
            "world": pdist.get_world_size()}
        logger.info("[h3-a100][matched] iter={} rank={} forwards={} grad_forwards={} backwards={} samples={} world={}",
                    current_iter, pdist.get_rank(), snapshot["forward_counts"], snapshot["grad_forward_counts"],
                    snapshot["backward_counts"], len(snapshot["samples"]), pdist.get_world_size())
