"""Fail-closed matched-compute census for one DMD outer cycle.

Same constants and API as the reference (``h3_a100/matched_contract.py:16-160``):
per rank and cycle the application issues 24/6/1 Student/Fake/Teacher DiT
forwards (1/5/0 of them with grad), 1/5 backward graphs, and consumes six
samples in the stage order ``student, fake_0..fake_4`` with no reuse, locally
or across the world.  Checkpoint recomputation is not an application forward.
"""

from __future__ import annotations

import json
from dataclasses import dataclass, field
from typing import Any

STUDENT_ROLE = "student"
FAKE_ROLE = "fake"
TEACHER_ROLE = "teacher"

FIXED_END_STEP_IDX = 3
EXPECTED_FORWARD_COUNTS = {STUDENT_ROLE: 24, FAKE_ROLE: 6, TEACHER_ROLE: 1}
EXPECTED_GRAD_FORWARD_COUNTS = {STUDENT_ROLE: 1, FAKE_ROLE: 5, TEACHER_ROLE: 0}
EXPECTED_BACKWARD_COUNTS = {STUDENT_ROLE: 1, FAKE_ROLE: 5}
EXPECTED_SAMPLE_STAGES = ["student"] + [f"fake_{i}" for i in range(5)]

_IDENTITY_KEYS = (
    "id",
    "row_index",
    "condition_path",
    "prompt_path",
    "lmdb_path",
    "video_latent_path",
    "audio_latent_path",
)


def sample_identity(sample: Any) -> str:
    """Stable identity of a sample, comparable across ranks (JSON of its meta keys)."""
    meta = sample.get("meta", {}) if isinstance(sample, dict) else {}
    if not isinstance(meta, dict):
        raise RuntimeError(f"sample meta must be a dict, got {type(meta)!r}")
    identity = {k: str(meta[k]) for k in _IDENTITY_KEYS if meta.get(k) is not None}
    if not identity:
        raise RuntimeError(
            "matched timing needs a rank-qualified sample identity in meta "
            "(id/row_index/condition_path/lmdb_path/...)"
        )
    return json.dumps(identity, sort_keys=True, separators=(",", ":"))


@dataclass
class MatchedCycleCensus:
    enabled: bool = True
    fixed_end_step_idx: int = FIXED_END_STEP_IDX
    expected_world_size: int = 8
    require_unique_samples: bool = True
    forward_counts: dict[str, int] = field(default_factory=dict)
    grad_forward_counts: dict[str, int] = field(default_factory=dict)
    backward_counts: dict[str, int] = field(default_factory=dict)
    samples: list[dict[str, str]] = field(default_factory=list)

    def __post_init__(self) -> None:
        self.reset()

    def reset(self) -> None:
        self.forward_counts = dict.fromkeys(EXPECTED_FORWARD_COUNTS, 0)
        self.grad_forward_counts = dict.fromkeys(EXPECTED_GRAD_FORWARD_COUNTS, 0)
        self.backward_counts = dict.fromkeys(EXPECTED_BACKWARD_COUNTS, 0)
        self.samples = []

    def note_forward(self, role: str, *, grad_enabled: bool) -> None:
        if not self.enabled:
            return
        if role not in self.forward_counts:
            raise RuntimeError(f"unknown DiT role {role!r}")
        self.forward_counts[role] += 1
        if grad_enabled:
            self.grad_forward_counts[role] += 1

    def note_backward(self, role: str) -> None:
        if not self.enabled:
            return
        if role not in self.backward_counts:
            raise RuntimeError(f"unknown backward role {role!r}")
        self.backward_counts[role] += 1

    def note_sample(self, stage: str, sample: Any) -> None:
        if self.enabled:
            self.samples.append({"stage": str(stage), "identity": sample_identity(sample)})

    def snapshot(self) -> dict[str, Any]:
        return {
            "fixed_end_step_idx": int(self.fixed_end_step_idx),
            "forward_counts": dict(self.forward_counts),
            "grad_forward_counts": dict(self.grad_forward_counts),
            "backward_counts": dict(self.backward_counts),
            "samples": [dict(s) for s in self.samples],
        }

    def validate_local(self) -> list[str]:
        if not self.enabled:
            return []
        errors: list[str] = []
        if self.fixed_end_step_idx != FIXED_END_STEP_IDX:
            errors.append(f"fixed_end_step_idx={self.fixed_end_step_idx} != matched baseline {FIXED_END_STEP_IDX}")
        if self.forward_counts != EXPECTED_FORWARD_COUNTS:
            errors.append(f"forward_counts={self.forward_counts} != {EXPECTED_FORWARD_COUNTS}")
        if self.grad_forward_counts != EXPECTED_GRAD_FORWARD_COUNTS:
            errors.append(f"grad_forward_counts={self.grad_forward_counts} != {EXPECTED_GRAD_FORWARD_COUNTS}")
        if self.backward_counts != EXPECTED_BACKWARD_COUNTS:
            errors.append(f"backward_counts={self.backward_counts} != {EXPECTED_BACKWARD_COUNTS}")
        stages = [s["stage"] for s in self.samples]
        if stages != EXPECTED_SAMPLE_STAGES:
            errors.append(f"sample_stages={stages} != {EXPECTED_SAMPLE_STAGES}")
        ids = [s["identity"] for s in self.samples]
        if self.require_unique_samples and len(set(ids)) != len(ids):
            errors.append("same rank reused a sample inside one Student1/Fake5 cycle")
        return errors


def validate_global_snapshots(
    snapshots: list[dict[str, Any]],
    *,
    expected_world_size: int,
    require_unique_samples: bool,
) -> list[str]:
    """World-wide check of per-rank snapshots (counts, stage order, uniqueness)."""
    if len(snapshots) != expected_world_size:
        return [f"world snapshots={len(snapshots)} != expected {expected_world_size}"]
    errors: list[str] = []
    identities: list[str] = []
    for rank, snap in enumerate(snapshots):
        if snap.get("forward_counts") != EXPECTED_FORWARD_COUNTS:
            errors.append(f"rank {rank} forward census mismatch")
        if snap.get("grad_forward_counts") != EXPECTED_GRAD_FORWARD_COUNTS:
            errors.append(f"rank {rank} grad-forward census mismatch")
        if snap.get("backward_counts") != EXPECTED_BACKWARD_COUNTS:
            errors.append(f"rank {rank} backward census mismatch")
        samples = snap.get("samples", [])
        stages = [s.get("stage") for s in samples]
        if stages != EXPECTED_SAMPLE_STAGES:
            errors.append(f"rank {rank} sample stage sequence mismatch: {stages}")
        identities.extend(str(s.get("identity")) for s in samples)
    expected = expected_world_size * len(EXPECTED_SAMPLE_STAGES)
    if len(identities) != expected:
        errors.append(f"sample identities={len(identities)} != expected {expected}")
    if require_unique_samples and len(set(identities)) != len(identities):
        errors.append(f"global sample reuse detected: unique={len(set(identities))} total={len(identities)}")
    return errors
