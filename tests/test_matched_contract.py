"""Matched-compute census (reference behaviour: tests/test_matched_contract.py)."""

import pytest

from h3_a100.trainer.matched_contract import (
    EXPECTED_BACKWARD_COUNTS,
    EXPECTED_FORWARD_COUNTS,
    EXPECTED_GRAD_FORWARD_COUNTS,
    EXPECTED_SAMPLE_STAGES,
    MatchedCycleCensus,
    sample_identity,
    validate_global_snapshots,
)


def _sample(i):
    return {"meta": {"lmdb_path": "synthetic://h3", "row_index": i}}


def _complete(rank=0, world=8):
    c = MatchedCycleCensus(expected_world_size=world)
    for i in range(24):
        c.note_forward("student", grad_enabled=i == 23)
    for i in range(6):
        c.note_forward("fake", grad_enabled=i != 0)
    c.note_forward("teacher", grad_enabled=False)
    c.note_backward("student")
    for _ in range(5):
        c.note_backward("fake")
    for i, stage in enumerate(EXPECTED_SAMPLE_STAGES):
        c.note_sample(stage, _sample(rank * 100 + i))
    return c


def test_exact_inventory_passes():
    c = _complete()
    assert c.forward_counts == EXPECTED_FORWARD_COUNTS
    assert c.grad_forward_counts == EXPECTED_GRAD_FORWARD_COUNTS
    assert c.backward_counts == EXPECTED_BACKWARD_COUNTS
    assert c.validate_local() == []


def test_missing_forward_fails():
    c = MatchedCycleCensus()
    for _ in range(23):
        c.note_forward("student", grad_enabled=False)
    assert any("forward_counts" in e for e in c.validate_local())


def test_extra_backward_fails():
    c = _complete()
    c.note_backward("fake")
    assert any("backward_counts" in e for e in c.validate_local())


def test_reused_sample_fails_locally():
    c = MatchedCycleCensus()
    for stage in EXPECTED_SAMPLE_STAGES:
        c.note_sample(stage, _sample(7))
    assert any("reused" in e for e in c.validate_local())


def test_stage_order_is_checked():
    c = _complete()
    snap = c.snapshot()
    snap["samples"][0], snap["samples"][1] = snap["samples"][1], snap["samples"][0]
    errors = validate_global_snapshots([snap], expected_world_size=1, require_unique_samples=True)
    assert any("sample stages" in e for e in errors)


@pytest.mark.parametrize("world", [8, 16])
def test_global_contract_requires_unique_samples(world):
    snaps = [_complete(r, world).snapshot() for r in range(world)]
    assert validate_global_snapshots(snaps, expected_world_size=world, require_unique_samples=True) == []
    snaps[-1]["samples"][5]["identity"] = snaps[0]["samples"][0]["identity"]
    errors = validate_global_snapshots(snaps, expected_world_size=world, require_unique_samples=True)
    assert any("global sample reuse" in e for e in errors)


def test_wrong_world_size_fails():
    snaps = [_complete(r).snapshot() for r in range(4)]
    assert validate_global_snapshots(snaps, expected_world_size=8, require_unique_samples=True)


def test_identity_requires_meta():
    with pytest.raises(RuntimeError):
        sample_identity({"meta": {}})
    assert sample_identity({"meta": {"row_index": 3, "id": "a"}}) == "id=a|row_index=3"
    assert sample_identity({"meta": {"row_index": 3, "id": "a"}}) != sample_identity({"meta": {"row_index": 4, "id": "a"}})


def test_unknown_role_rejected():
    with pytest.raises(RuntimeError):
        MatchedCycleCensus().note_forward("critic", grad_enabled=False)
