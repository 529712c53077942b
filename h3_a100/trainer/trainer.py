"""The shared-backbone DMD trainer: configuration, contracts and setup.

Parity with ``MiniMaxH3A100DmdTrainer`` (``h3_a100/trainer.py:28-316``):
reads ``training.a100.*`` (alias ``training.b200``) plus the same environment
overrides, validates the static matched contract (fixed end step 3, 4
inference steps, fake ratio 5, no gradient accumulation, no in-run
inference) and the policy combinations, and sets up in the same order:
shared backbone -> segments -> reorder contract -> [resume LoRA] -> sharding ->
checkpointing -> boundary staging -> role parameters -> disjointness
contract -> two AdamW + two schedulers (Fake: ``max_iters * 5`` steps, no
warmup) -> [resume rank state] -> exact AdaLN replay (outermost wrapper).
"""

from __future__ import annotations

import os
from pathlib import Path
from typing import Any

import torch

from ..config import env_flag, get, training_system_section
from ..memory.boundary import POLICY_NAME as CHECKPOINT_BOUNDARY_CPU
from ..memory.boundary import BoundaryStaging, PinnedSlabPool, choose_staging_target
from ..memory.exact_replay import ReplayAudit
from ..memory.saved_tensor_offload import offload_scope
from ..models.lora import FAKE, STUDENT
from ..parallel import distributed as pdist
from ..utils.log import logger
from ..utils.memory import BlockResidencyProbe, ResidencyLogger, log_cuda_memory
from ..utils.timeline import StreamTimeline
from ..utils.timing import PhaseTimer, StallLedger
from .checkpointing import CheckpointMixin
from .loop import LoopMixin
from .matched_contract import FIXED_END_STEP_IDX, MatchedCycleCensus
from .optim import FlatAdamW, LRSchedule
from .runtime import DMDRuntimeMixin

_DTYPES = {"bf16": torch.bfloat16, "fp32": torch.float32, "fp16": torch.float16}


class H3DmdTrainer(CheckpointMixin, LoopMixin, DMDRuntimeMixin):
    trainer_name = "minimax_h3_t2av_dmd_a100"

    def __init__(self, config: dict[str, Any], *, kernels, device: torch.device) -> None:
        self.config = config
        self.kernels = kernels
        self.device = device
        tr = get(config, "training", {}) or {}
        dmd = tr.get("dmd", {}) or {}
        h3 = tr.get("minimax_h3", {}) or {}
        sysc = training_system_section(config)

        self.student_train_type = get(tr, "student.train_type", "lora")
        self.fake_train_type = get(tr, "fake.train_type", "lora")
        if self.student_train_type != "lora" or self.fake_train_type != "lora":
            raise ValueError("shared-backbone training requires student/fake train_type=lora")
        self.student_lora_config = dict(get(tr, "student.lora", {}) or {})
        self.fake_lora_config = dict(get(tr, "fake.lora", {}) or {})
        self.student_optimizer_config = dict(get(tr, "student.optimizer", {}) or {})
        self.fake_optimizer_config = dict(get(tr, "fake.optimizer", {}) or {})

        self.seed = int(tr.get("seed", 42))
        self.max_train_iters = int(tr.get("max_train_iters", 1))
        self.gradient_accumulation_iters = max(1, int(tr.get("gradient_accumulation_iters", 1)))
        self.gradient_checkpointing = bool(tr.get("gradient_checkpointing", True))
        self.max_grad_norm = float(tr.get("max_grad_norm", 1.0))
        self.lr_scheduler_kind = str(tr.get("lr_scheduler", "constant"))
        self.lr_warmup_iters = int(tr.get("lr_warmup_iters", 0))
        self.save_every_iters = int(tr.get("save_every_iters", 0) or 0)
        self.save_total_limit = int(tr.get("save_total_limit", 3) or 0)
        self.output_train_dir = str(tr.get("output_dir", "./output_train"))
        self.train_log_every_iters = max(1, int(get(config, "logging.train_log_every_iters", 1)))
        self.auto_resume = bool(get(config, "resume.auto_resume", False))
        self.infer_every_iters = get(config, "inference.infer_every_iters", None)

        self.num_inference_steps = int(dmd.get("num_inference_steps", 4))
        self.fake_update_ratio = int(dmd.get("fake_update_ratio", 5))
        self.renoise_sigma_min = float(dmd.get("renoise_sigma_min", 0.02))
        self.renoise_sigma_max = float(dmd.get("renoise_sigma_max", 0.98))
        self.video_flow_shift = float(h3.get("video_flow_shift", 6.0))
        self.audio_flow_shift = float(h3.get("audio_flow_shift", 3.0))
        self.video_loss_weight = float(h3.get("video_loss_weight", 1.0))
        self.audio_loss_weight = float(h3.get("audio_loss_weight", 1.0))
        self.latent_dtype = _DTYPES[str(h3.get("latent_dtype", "fp32"))]
        self.num_train_timesteps = int(get(config, "scheduler.num_train_timesteps", 1000))

        cache = sysc.get("adaln_cache", {}) or {}
        reorder = sysc.get("critic_rollout_reorder", {}) or {}
        matched = sysc.get("matched_compute", {}) or {}
        ckpt = sysc.get("activation_checkpointing", {}) or {}
        policy = sysc.get("activation_policy", {}) or {}
        self.adaln_cache_enabled = bool(cache.get("enabled", True))
        self.adaln_dynamic_keys = int(cache.get("max_dynamic_keys", 2))
        self.reorder_critic_rollouts = bool(reorder.get("enabled", True))
        self.critic_rollout_group_size = int(reorder.get("group_size", self.fake_update_ratio))
        if self.critic_rollout_group_size != self.fake_update_ratio:
            raise ValueError("critic_rollout_reorder.group_size must equal "
                             f"fake_update_ratio={self.fake_update_ratio} to preserve optimizer-step semantics")
        self.matched_compute_enabled = bool(matched.get("enabled", True))
        self.matched_fixed_end_step_idx = int(matched.get("fixed_end_step_idx", FIXED_END_STEP_IDX))
        self.matched_expected_world_size = int(matched.get("expected_world_size", pdist.get_world_size()))
        self.matched_require_unique_samples = bool(matched.get("require_unique_samples", True))
        self.matched_cycle_census = MatchedCycleCensus(
            enabled=self.matched_compute_enabled, fixed_end_step_idx=self.matched_fixed_end_step_idx,
            expected_world_size=self.matched_expected_world_size,
            require_unique_samples=self.matched_require_unique_samples)

        self.activation_checkpoint_segment_size = int(os.environ.get(
            "H3_ACTIVATION_CHECKPOINT_SEGMENT", ckpt.get("segment_size", 1)))
        if self.activation_checkpoint_segment_size < 1:
            raise ValueError("H3_ACTIVATION_CHECKPOINT_SEGMENT must be >= 1, got "
                             f"{self.activation_checkpoint_segment_size}")
        self.activation_policy = str(os.environ.get("H3_ACTIVATION_POLICY", policy.get("name", "none")))
        if self.activation_policy not in {"none", CHECKPOINT_BOUNDARY_CPU}:
            raise ValueError(f"H3_ACTIVATION_POLICY must be 'none' or '{CHECKPOINT_BOUNDARY_CPU}', "
                             f"got {self.activation_policy!r}")
        self.boundary_offload_pin_memory = env_flag("H3_BOUNDARY_OFFLOAD_PIN_MEMORY", policy.get("pin_memory", True))
        self.boundary_offload_events = env_flag("H3_BOUNDARY_OFFLOAD_EVENTS", policy.get("detailed_events", False))
        self.boundary_staging_target = str(os.environ.get("H3_BOUNDARY_STAGING_TARGET",
                                                          policy.get("staging_target", "host")))
        self.activation_offload_enabled = env_flag("H3_ACTIVATION_OFFLOAD", False)
        self.activation_offload_min_bytes = int(os.environ.get("H3_ACTIVATION_OFFLOAD_MIN_BYTES", 128 * 1024 * 1024))
        self.activation_offload_pin_memory = env_flag("H3_ACTIVATION_OFFLOAD_PIN_MEMORY", True)
        if self.activation_offload_min_bytes < 0:
            raise ValueError("H3_ACTIVATION_OFFLOAD_MIN_BYTES must be >= 0")
        if self.activation_policy == CHECKPOINT_BOUNDARY_CPU:
            if self.activation_checkpoint_segment_size != 1:
                raise ValueError("checkpoint_boundary_cpu requires native per-block checkpointing: "
                                 "H3_ACTIVATION_CHECKPOINT_SEGMENT must be 1")
            if self.activation_offload_enabled:
                raise ValueError("checkpoint_boundary_cpu is mutually exclusive with the legacy "
                                 "H3_ACTIVATION_OFFLOAD threshold policy")
            if not self.gradient_checkpointing:
                raise ValueError("checkpoint_boundary_cpu requires gradient_checkpointing=true")
        self.require_exact_replay = bool(sysc.get("exact_adaln_replay", self.activation_policy == CHECKPOINT_BOUNDARY_CPU))
        self.shard_optimizer_states = bool(get(config, "distributed.shard_optimizer_states", False))
        self._validate_matched_static_contract()

        self.model = None
        self.data = None
        self.optimizers: dict[str, FlatAdamW] = {}
        self.lr_schedulers: dict[str, LRSchedule] = {}
        self.boundary_staging: BoundaryStaging | None = None
        self.replay_audit: ReplayAudit | None = None
        self.boundary_pool: PinnedSlabPool | None = None
        self.host_rng = torch.Generator().manual_seed(self.seed + pdist.get_rank())
        self.timer = PhaseTimer(enabled=True)
        self.stall_ledger = StallLedger()
        self.timeline = StreamTimeline()
        self.residency = ResidencyLogger(self)
        self.metrics: list[dict] = []
        self.last_cycle_receipt: dict[str, Any] = {}
        self.h2d_bytes = 0
        self._init_schedule()

    # ---------------------------------------------------------------- wiring
    def set_model(self, model) -> None:
        self.model = model

    def set_data(self, train_loader, eval_loader=None) -> None:
        self.data = train_loader
        self.eval_data = eval_loader

    @property
    def shared_model(self):
        return self.model

    def _validate_matched_static_contract(self) -> None:
        if not self.matched_compute_enabled:
            return
        if self.matched_fixed_end_step_idx != FIXED_END_STEP_IDX:
            raise ValueError(f"matched_compute.fixed_end_step_idx must be {FIXED_END_STEP_IDX}, "
                             f"got {self.matched_fixed_end_step_idx}")
        if self.num_inference_steps != 4:
            raise ValueError("matched benchmark requires num_inference_steps=4")
        if self.fake_update_ratio != 5:
            raise ValueError("matched benchmark requires fake_update_ratio=5")
        if self.gradient_accumulation_iters != 1:
            raise ValueError("matched benchmark requires gradient_accumulation_iters=1")
        if self.infer_every_iters:
            raise ValueError("matched benchmark forbids in-run inference")

    def _encode_conditions(self, sample: dict[str, Any]) -> dict[str, torch.Tensor]:
        return {"text": sample["text"]}

    def _latent_shape(self, sample: dict[str, Any]) -> dict[str, Any]:
        audio = sample.get("audio_latent")
        return {"video": tuple(sample["video_latent"].shape), "audio": None if audio is None else tuple(audio.shape)}

    def _activation_offload_scope(self, component: str):
        return offload_scope(
            self.model.denoiser_module(), enabled=self.activation_offload_enabled, label=component,
            min_bytes=self.activation_offload_min_bytes, pin_memory=self.activation_offload_pin_memory,
            include_cpu=self.device.type == "cpu")

    # ---------------------------------------------------------------- setup
    def _build_comm(self):
        """NCCL baseline or the peer-memory kernels (``distributed.comm``), chosen once."""
        from ..parallel.comm import TorchComm

        kind = str(get(self.config, "distributed.comm", "nccl"))
        world = pdist.get_world_size()
        if kind == "p2p" and world > 1 and self.device.type == "cuda" and getattr(self.kernels, "native", False):
            from ..parallel.p2p import PeerComm

            if pdist.topology().replicate_size != 1:
                raise ValueError("distributed.comm=p2p needs a single shard group (one NVLink domain)")
            return PeerComm(pdist.shard_group(), self.device, kernels=self.kernels)
        if kind not in {"nccl", "p2p"}:
            raise ValueError(f"distributed.comm must be 'nccl' or 'p2p', got {kind!r}")
        return TorchComm(pdist.shard_group(), self.device)

    def setup(self, resume_ckpt_path: str | None = None, *, comm=None) -> None:
        model = self.model
        self.comm = comm or self._build_comm()
        self.comm.ledger = self.stall_ledger
        if self.timeline.enabled:
            self.comm.timeline = self.timeline
        pad = 4 * max(1, self.comm.world_size)
        model.prepare_shared_backbone(student_lora=self.student_lora_config, fake_lora=self.fake_lora_config,
                                      cache_enabled=self.adaln_cache_enabled,
                                      max_dynamic_cache_keys=self.adaln_dynamic_keys,
                                      alloc=self.comm.alloc_symmetric if self.comm.world_size > 1 else None,
                                      pad_to=pad)
        dit = model.denoiser_module()
        self._validate_reorder_contract()
        if resume_ckpt_path is not None:
            self._load_role_weights_before_sharding(resume_ckpt_path)
        reshard = get(self.config, "distributed.fsdp2.reshard_after_forward", {}) or {}
        fsdp_enabled = bool(get(self.config, "distributed.fsdp2.enabled", True))
        shard_comm = self.comm if fsdp_enabled else _LocalComm(self.device)
        model.apply_sharding(shard_comm, block_reshard=bool(reshard.get("block_reshard", True)),
                             root_reshard=bool(reshard.get("root_reshard", False)))
        plan = None
        if self.gradient_checkpointing:
            plan = dit.enable_gradient_checkpointing(self.activation_checkpoint_segment_size)
            if self.activation_checkpoint_segment_size > 1:
                logger.info("[h3-a100] SAC activation checkpoint segments enabled segment_size={} blocks={} "
                            "segments={} (diagnostic)", self.activation_checkpoint_segment_size,
                            model.dit_config.num_blocks, plan.calls_per_grad_forward)
        if self.activation_policy == CHECKPOINT_BOUNDARY_CPU:
            event_path = None
            if self.boundary_offload_events:
                event_path = Path(self.output_train_dir) / "checkpoint_boundary_offload" / f"rank_{pdist.get_rank():03d}.jsonl"
            per_rank = self._boundary_bytes_per_rank(model)
            local_ranks = int(os.environ.get("LOCAL_WORLD_SIZE", "1"))
            self.boundary_staging_target = choose_staging_target(
                self.boundary_staging_target, per_rank, local_ranks, self.device)
            self.boundary_pool = PinnedSlabPool(self.boundary_offload_pin_memory, self.boundary_staging_target,
                                                self.device)
            self.boundary_staging = BoundaryStaging(
                expected_block_count=model.dit_config.num_blocks, pool=self.boundary_pool,
                pin_memory=self.boundary_offload_pin_memory, require_cuda=self.device.type == "cuda",
                event_path=event_path)
            plan.attach_staging(self.boundary_staging)
            if self.timeline.enabled:
                self.boundary_staging.stager.timeline = self.timeline
        self.trainable_params = model.role_parameters(STUDENT)
        self.fake_trainable_params = model.role_parameters(FAKE)
        self._validate_shared_parameter_contract()
        world_comm = self.comm
        if pdist.topology().replicate_size > 1:
            # The adapters are replicated on every rank and every rank draws its
            # own sample, so LoRA gradients average over the whole world (the
            # shard group only spans one replica).
            from ..parallel.comm import TorchComm

            world_comm = TorchComm(None, self.device)
        for role, ocfg, total in ((STUDENT, self.student_optimizer_config, self.max_train_iters),
                                  (FAKE, self.fake_optimizer_config, self.max_train_iters * self.fake_update_ratio)):
            self.optimizers[role] = FlatAdamW(
                model.lora[role], lr=float(ocfg.get("learning_rate", 1e-4)),
                betas=(float(ocfg.get("adam_beta1", 0.9)), float(ocfg.get("adam_beta2", 0.999))),
                weight_decay=float(ocfg.get("weight_decay", 0.01)), eps=float(ocfg.get("adam_epsilon", 1e-8)),
                max_grad_norm=self.max_grad_norm, kernels=self.kernels, comm=world_comm,
                shard_states=self.shard_optimizer_states)
            self.lr_schedulers[role] = LRSchedule(
                float(ocfg.get("learning_rate", 1e-4)), self.lr_scheduler_kind,
                warmup=self.lr_warmup_iters if role == STUDENT else 0, total=max(1, total))
        if resume_ckpt_path is not None:
            self._load_rank_state_after_sharding(resume_ckpt_path)
        if self.require_exact_replay and self.gradient_checkpointing:
            if not self.adaln_cache_enabled:
                raise RuntimeError("exact replay requires exact AdaLN caching enabled")
            self.replay_audit = ReplayAudit(model.adaln_cache())
            plan.attach_replay(self.replay_audit)
        probe = BlockResidencyProbe()
        if probe.enabled:
            dit.block_probe = probe
            self.block_residency = probe
        log_cuda_memory("after_setup")
        logger.info("[h3-a100] setup physical_backbones=1 logical_roles=3 student_params={} fake_params={} "
                    "sharded={} critic_reorder={} matched_compute={} kernels={}",
                    model.lora[STUDENT].numel(), model.lora[FAKE].numel(), model.is_sharded(),
                    self.reorder_critic_rollouts, self.matched_compute_enabled, self.kernels.name)
        logger.info("[h3-a100] activation policy={} checkpoint_segment={} boundary_pin={} boundary_target={} "
                    "boundary_events={} legacy_threshold_offload={}", self.activation_policy,
                    self.activation_checkpoint_segment_size, self.boundary_offload_pin_memory,
                    self.boundary_staging_target, self.boundary_offload_events, self.activation_offload_enabled)

    def boundary_staging_report(self) -> dict[str, Any]:
        """Where the checkpoint boundaries went: the reference pins them in host memory.

        ``device`` keeps the same copies and counters in HBM slabs; it is not
        like-for-like with the reference's host staging (no PCIe traffic).
        """
        pool = self.boundary_pool
        if pool is None:
            return {"policy": self.activation_policy, "target": None, "pinned": False,
                    "like_for_like_with_reference": False}
        return {"policy": self.activation_policy, "target": pool.target, "pinned": bool(pool.pin_memory),
                "slab_gib": round(pool.allocated_bytes / 1024**3, 2),
                "like_for_like_with_reference": pool.target == "host" and bool(pool.pin_memory)}

    def _boundary_bytes_per_rank(self, model) -> int:
        """Bytes of one grad forward's boundaries (one bf16 hidden state per block)."""
        from ..models.shared_backbone import sequence_tokens

        cfg = model.dit_config
        return sequence_tokens(self.config) * cfg.hidden * 2 * cfg.num_blocks

    def reserve_boundary_slabs(self, per_forward: int, numel: int, dtype: torch.dtype) -> None:
        """Allocate the pinned boundary pool up front (one grad forward's worth)."""
        if self.boundary_pool is not None:
            self.boundary_pool.reserve(per_forward, numel, dtype)

    def _validate_reorder_contract(self) -> None:
        if not self.reorder_critic_rollouts:
            return
        bad = [(n, m.p) for n, m in self.model.denoiser_module().named_modules()
               if isinstance(m, torch.nn.Dropout) and float(m.p) != 0.0]
        if bad:
            raise RuntimeError("Critic rollout reordering requires deterministic forwards; found nonzero dropout "
                               f"modules: {', '.join(f'{n}:p={p}' for n, p in bad[:6])}")

    def _validate_shared_parameter_contract(self) -> None:
        student = {id(p) for p in self.trainable_params}
        fake = {id(p) for p in self.fake_trainable_params}
        if student & fake:
            raise RuntimeError(f"Student/Fake optimizers share {len(student & fake)} parameter objects")
        s_ptr = {p.untyped_storage().data_ptr() for p in self.trainable_params}
        f_ptr = {p.untyped_storage().data_ptr() for p in self.fake_trainable_params}
        if s_ptr & f_ptr:
            raise RuntimeError("Student/Fake adapters share storage")
        trainable_base = [n for n, p in self.model.denoiser_module().named_parameters() if p.requires_grad]
        if trainable_base:
            raise RuntimeError(f"shared base has trainable parameters: {', '.join(trainable_base[:6])}")


class _LocalComm:
    """No-op communicator: replicated frozen weights (fsdp2.enabled: false)."""

    world_size, rank, name = 1, 0, "local"

    def __init__(self, device) -> None:
        self.device = device

    def recycle(self, buf) -> None:
        pass
