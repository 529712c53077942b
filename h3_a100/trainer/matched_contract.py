"""Fail-closed matched-compute census of one DMD outer cycle.

The contract is the reference's (``h3_a100/matched_contract.py:16-160``), and
its constants are kept verbatim because they define the benchmark's cycle:
per rank, 24/6/1 Student/Fake/Teacher DiT application forwards (1/5/0 with
grad), 1/5 backward graphs, and six samples consumed in the stage order
``student, fake_0..fake_4`` with no reuse, on the rank or across the world.
Checkpoint recomputation is not an application forward.

Design here: the census keeps ``Counter`` tallies and a sample list; a
snapshot is a plain dict (it crosses ranks through ``all_gather_object``).
Local and global validation share one snapshot check (``snapshot_errors``);
the global pass adds the world size and the world-wide uniqueness of the
``world x 6`` sample identities.
"""

from __future__ import annotations

from collections import Counter
from collections.abc import Iterator
from typing import Any

STUDENT_ROLE = "student"
FAKE_ROLE = "fake"
TEACHER_ROLE = "teacher"
ROLES = (STUDENT_ROLE, FAKE_ROLE, TEACHER_ROLE)

FIXED_END_STEP_IDX = 3
EXPECTED_FORWARD_COUNTS = {STUDENT_ROLE: 24, FAKE_ROLE: 6, TEACHER_ROLE: 1}
EXPECTED_GRAD_FORWARD_COUNTS = {STUDENT_ROLE: 1, FAKE_ROLE: 5, TEACHER_ROLE: 0}
EXPECTED_BACKWARD_COUNTS = {STUDENT_ROLE: 1, FAKE_ROLE: 5}
EXPECTED_SAMPLE_STAGES = ["student"] + [f"fake_{i}" for i in range(5)]

# sample ``meta`` fields that name a sample (any subset may be present)
IDENTITY_FIELDS = ("id", "row_index", "condition_path", "prompt_path", "lmdb_path", "video_latent_path",
                   "audio_latent_path")

_COUNT_FIELDS = (("forward_counts", EXPECTED_FORWARD_COUNTS),
                 ("grad_forward_counts", EXPECTED_GRAD_FORWARD_COUNTS),
                 ("backward_counts", EXPECTED_BACKWARD_COUNTS))


def sample_identity(sample: Any) -> str:
    """``field=value`` pairs of the sample's identifying meta fields, sorted and joined by ``|``."""
    meta = sample.get("meta") if isinstance(sample, dict) else None
    if not isinstance(meta, dict):
        raise RuntimeError(f"a sample needs a dict 'meta' to be identified, got {type(meta).__name__}")
    parts = sorted(f"{name}={meta[name]}" for name in IDENTITY_FIELDS if meta.get(name) is not None)
    if not parts:
        raise RuntimeError("matched timing needs a rank-qualified sample identity in meta "
                           f"(one of {', '.join(IDENTITY_FIELDS)})")
    return "|".join(parts)


def snapshot_errors(snapshot: dict[str, Any], who: str = "local") -> Iterator[str]:
    """Every way one rank's snapshot departs from the contract."""
    for name, expected in _COUNT_FIELDS:
        got = snapshot.get(name)
        if got != expected:
            yield f"{who}: {name}={got} != {expected}"
    stages = [s.get("stage") for s in snapshot.get("samples", [])]
    if stages != EXPECTED_SAMPLE_STAGES:
        yield f"{who}: sample stages {stages} != {EXPECTED_SAMPLE_STAGES}"


def _duplicates(identities: list[str]) -> list[str]:
    return sorted(i for i, n in Counter(identities).items() if n > 1)


class MatchedCycleCensus:
    """Per-rank tallies of one cycle's forwards, backwards and samples."""

    def __init__(self, *, enabled: bool = True, fixed_end_step_idx: int = FIXED_END_STEP_IDX,
                 expected_world_size: int = 8, require_unique_samples: bool = True) -> None:
        self.enabled = bool(enabled)
        self.fixed_end_step_idx = int(fixed_end_step_idx)
        self.expected_world_size = int(expected_world_size)
        self.require_unique_samples = bool(require_unique_samples)
        self.reset()

    def reset(self) -> None:
        self._forwards: Counter[str] = Counter()
        self._grad_forwards: Counter[str] = Counter()
        self._backwards: Counter[str] = Counter()
        self._samples: list[dict[str, str]] = []

    # ------------------------------------------------------------ notes
    def note_forward(self, role: str, *, grad_enabled: bool) -> None:
        if not self.enabled:
            return
        if role not in ROLES:
            raise RuntimeError(f"unknown DiT role {role!r} (expected one of {ROLES})")
        self._forwards[role] += 1
        self._grad_forwards[role] += bool(grad_enabled)

    def note_backward(self, role: str) -> None:
        if not self.enabled:
            return
        if role not in EXPECTED_BACKWARD_COUNTS:
            raise RuntimeError(f"role {role!r} has no backward graph in the matched cycle")
        self._backwards[role] += 1

    def note_sample(self, stage: str, sample: Any) -> None:
        if self.enabled:
            self._samples.append({"stage": str(stage), "identity": sample_identity(sample)})

    # ------------------------------------------------------------ views
    @property
    def forward_counts(self) -> dict[str, int]:
        return {role: self._forwards[role] for role in EXPECTED_FORWARD_COUNTS}

    @property
    def grad_forward_counts(self) -> dict[str, int]:
        return {role: self._grad_forwards[role] for role in EXPECTED_GRAD_FORWARD_COUNTS}

    @property
    def backward_counts(self) -> dict[str, int]:
        return {role: self._backwards[role] for role in EXPECTED_BACKWARD_COUNTS}

    @property
    def samples(self) -> list[dict[str, str]]:
        return [dict(s) for s in self._samples]

    def snapshot(self) -> dict[str, Any]:
        return {"fixed_end_step_idx": self.fixed_end_step_idx, "forward_counts": self.forward_counts,
                "grad_forward_counts": self.grad_forward_counts, "backward_counts": self.backward_counts,
                "samples": self.samples}

    # ------------------------------------------------------------ checks
    def validate_local(self) -> list[str]:
        if not self.enabled:
            return []
        errors = []
        if self.fixed_end_step_idx != FIXED_END_STEP_IDX:
            errors.append(f"local: fixed_end_step_idx={self.fixed_end_step_idx} != {FIXED_END_STEP_IDX}")
        errors.extend(snapshot_errors(self.snapshot()))
        if self.require_unique_samples:
            dup = _duplicates([s["identity"] for s in self._samples])
            if dup:
                errors.append(f"local: a sample was reused inside one Student1/Fake5 cycle: {dup[:3]}")
        return errors


def validate_global_snapshots(snapshots: list[dict[str, Any]], *, expected_world_size: int,
                              require_unique_samples: bool) -> list[str]:
    """World-wide check of every rank's snapshot (counts, stage order, world x 6 unique samples)."""
    if len(snapshots) != int(expected_world_size):
        return [f"global: {len(snapshots)} rank snapshots, expected world size {expected_world_size}"]
    errors = [e for rank, snap in enumerate(snapshots) for e in snapshot_errors(snap, f"rank {rank}")]
    identities = [str(s.get("identity")) for snap in snapshots for s in snap.get("samples", [])]
    expected = int(expected_world_size) * len(EXPECTED_SAMPLE_STAGES)
    if len(identities) != expected:
        errors.append(f"global: {len(identities)} sample identities, expected {expected}")
    if require_unique_samples:
        dup = _duplicates(identities)
        if dup:
            errors.append(f"global sample reuse: {len(dup)} identities seen more than once, e.g. {dup[:3]}")
    return errors
