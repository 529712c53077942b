"""Per-block checkpointing with boundary staging, the exact-replay audit, SAC
segments and the saved-tensor offload diagnostic (the reference's
tests/test_checkpoint_boundary_offload.py, tests/test_exact_adaln_replay.py and
tests/test_activation_offload.py, in behaviour), on a toy block stack driven
by this package's own checkpoint plan."""

import json

import pytest
import torch
from torch.utils.checkpoint import checkpoint

from h3_a100.memory.boundary import BoundaryStaging, PinnedSlabPool
from h3_a100.memory.checkpoint import BlockCheckpointing, native_checkpoint
from h3_a100.memory.exact_replay import ReplayAudit, expected_cycle_counts
from h3_a100.memory.saved_tensor_offload import ThresholdOffload, offload_scope
from h3_a100.models.adaln import ModulationCache

WIDTH = 8


class _Block(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.proj = torch.nn.Linear(WIDTH, WIDTH, bias=False)

    def forward(self, h, shift):
        return torch.tanh(self.proj(h) + shift) + h


class _Call:
    """A block call in the DiT's protocol: key, fetch count, ``call(x, fetch)``."""

    fetches = 1

    def __init__(self, block, index, key, cache):
        self.block, self.index, self.key, self.cache = block, index, key, cache

    def __call__(self, x, fetch=None):
        shift = (fetch or self.cache.fetch)(self.key, self.index)
        if shift is None:
            raise RuntimeError("modulation missing")
        return self.block(x, shift)


class _Stack(torch.nn.Module):
    def __init__(self, blocks=3):
        super().__init__()
        self.blocks = torch.nn.ModuleList([_Block() for _ in range(blocks)])
        self.cache = ModulationCache(blocks, max_dynamic_keys=4)
        self.cache.insert("k", torch.linspace(-0.5, 0.5, blocks * WIDTH).view(blocks, WIDTH), persistent=True)
        self.plan = None

    def forward(self, h, role="student", key="k"):
        calls = [_Call(b, i, key, self.cache) for i, b in enumerate(self.blocks)]
        grad = torch.is_grad_enabled()
        if self.plan is None:
            for c in calls:
                h = c(h)
            return h
        with self.plan.forward(role, grad):
            for unit in self.plan.segments(calls):
                h = self.plan.run(unit, h) if grad else self.plan.execute(unit, h)
        return h


def _twins(blocks=3, **plan_kw):
    torch.manual_seed(7)
    ref, cand = _Stack(blocks), _Stack(blocks)
    cand.load_state_dict(ref.state_dict())
    cand.plan = BlockCheckpointing(blocks, **plan_kw)
    return ref, cand


def _staging(blocks, tmp_path=None):
    return BoundaryStaging(expected_block_count=blocks, pool=PinnedSlabPool(False), pin_memory=False,
                           require_cuda=False, event_path=None if tmp_path is None else tmp_path / "events.jsonl")


def _grads_match(ref, cand, x_ref, x):
    torch.testing.assert_close(x.grad, x_ref.grad)
    for a, b in zip(ref.parameters(), cand.parameters()):
        torch.testing.assert_close(b.grad, a.grad)


def test_boundary_staging_preserves_output_and_grads(tmp_path):
    ref, cand = _twins()
    staging = _staging(3, tmp_path)
    cand.plan.attach_staging(staging)
    x_ref = torch.randn(2, 5, WIDTH, requires_grad=True)
    x = x_ref.detach().clone().requires_grad_(True)
    y_ref = ref(x_ref)
    y_ref.square().mean().backward()
    y = cand(x)
    y.square().mean().backward()
    torch.testing.assert_close(y, y_ref)
    _grads_match(ref, cand, x_ref, x)
    s = staging.stats
    assert s["grad_transformer_forward_count"] == 1 and s["student_grad_forward_count"] == 1
    assert s["grad_checkpoint_call_count"] == 3 and s["cpu_copy_count"] == 3 and s["restore_count"] == 3
    assert s["offloaded_logical_bytes"] == 3 * 2 * 5 * WIDTH * 4
    events = [json.loads(line) for line in (tmp_path / "events.jsonl").read_text().splitlines()]
    assert [e["event"] for e in events] == ["boundary_saved"] * 3 + ["grad_forward_complete"]
    assert staging.stager.live() == 0


def test_boundary_staging_tracks_roles_and_prefetches_in_reverse():
    _, model = _twins(blocks=4)
    staging = _staging(4)
    model.plan.attach_staging(staging)
    model(torch.randn(1, 3, WIDTH, requires_grad=True), role="student").sum().backward()
    model(torch.randn(1, 3, WIDTH, requires_grad=True), role="fake").sum().backward()
    s = staging.stats
    assert (s["student_grad_forward_count"], s["fake_grad_forward_count"], s["other_grad_forward_count"]) == (1, 1, 0)
    assert s["grad_checkpoint_call_count"] == 8 and s["cpu_copy_count"] == 8
    assert s["restore_count"] == 8 and s["prefetch_count"] == 8


def test_boundary_staging_skips_no_grad_forward_and_frees_abandoned_slabs():
    _, model = _twins(blocks=2)
    staging = _staging(2)
    model.plan.attach_staging(staging)
    with torch.no_grad():
        assert torch.isfinite(model(torch.randn(1, 3, WIDTH))).all()
    assert staging.stats["grad_transformer_forward_count"] == 0 and staging.stats["cpu_copy_count"] == 0
    assert staging.stats["transformer_forward_count"] == 1
    model(torch.randn(1, 3, WIDTH, requires_grad=True))          # backward never runs
    model(torch.randn(1, 3, WIDTH, requires_grad=True)).sum().backward()
    assert staging.stats["abandoned_count"] == 2 and staging.stager.live() == 0


def test_grad_forward_must_checkpoint_every_block():
    plan = BlockCheckpointing(3)
    plan.attach_staging(_staging(3))
    with pytest.raises(RuntimeError, match="2 checkpoint calls, expected 3"):
        with plan.forward("student", True):
            h = torch.randn(2, WIDTH, requires_grad=True)
            for _ in range(2):
                h = plan.run(lambda x, fetch=None: x * 2, h)


def test_boundary_staging_refuses_to_overwrite_events(tmp_path):
    path = tmp_path / "e.jsonl"
    path.write_text("x")
    with pytest.raises(FileExistsError):
        BoundaryStaging(expected_block_count=3, pin_memory=False, require_cuda=False, event_path=path)


def test_boundary_staging_requires_per_block_checkpoints():
    with pytest.raises(ValueError, match="segment_size 1"):
        BlockCheckpointing(4, segment_size=2).attach_staging(_staging(4))


def test_exact_replay_counts_with_staging_and_never_projects():
    ref, cand = _twins()
    audit = ReplayAudit(cand.cache)
    cand.plan.attach_staging(_staging(3))
    cand.plan.attach_replay(audit)
    x_ref = torch.randn(2, WIDTH, requires_grad=True)
    x = x_ref.detach().clone().requires_grad_(True)
    ref(x_ref).sum().backward()
    cand(x).sum().backward()
    _grads_match(ref, cand, x_ref, x)
    assert audit.stats == expected_cycle_counts(3, grad_forwards=1)
    assert audit.stats == {"checkpoint_wrap_count": 3, "scoped_execution_count": 6, "cache_hit_count": 6,
                           "cache_miss_count": 0, "captured_key_missing_count": 0,
                           "captured_key_incomplete_count": 0, "unexpected_hit_delta_count": 0}


def test_exact_replay_fails_closed_without_key_or_on_incomplete_key():
    _, model = _twins()
    audit = ReplayAudit(model.cache)
    model.plan.attach_replay(audit)
    with pytest.raises(RuntimeError, match="without an AdaLN key"):
        model(torch.randn(2, WIDTH, requires_grad=True), key=None)
    with pytest.raises(RuntimeError, match="no complete modulation table"):
        model(torch.randn(2, WIDTH, requires_grad=True), key="never-built")
    assert audit.stats["captured_key_missing_count"] == 1 and audit.stats["captured_key_incomplete_count"] == 1


def test_exact_replay_fails_closed_when_the_key_vanishes_before_replay():
    _, model = _twins()
    model.cache.insert("s", torch.zeros(3, WIDTH), persistent=False)
    audit = ReplayAudit(model.cache)
    model.plan.attach_replay(audit)
    y = model(torch.randn(2, WIDTH, requires_grad=True), key="s")
    model.cache.release("s")
    with pytest.raises(RuntimeError, match="modulation missing"):
        y.sum().backward()
    assert audit.stats["cache_miss_count"] == 1


def test_exact_replay_rejects_wrong_number_of_reads():
    cache = ModulationCache(1)
    cache.insert("k", torch.ones(1, 2), persistent=True)
    audit = ReplayAudit(cache)

    class Twice:
        key, fetches = "k", 1

        def __call__(self, x, fetch=None):
            return x + fetch("k", 0) + fetch("k", 0)

    with pytest.raises(RuntimeError, match="expected 1 modulation read"):
        audit.execute(Twice(), torch.zeros(2))
    assert audit.stats["unexpected_hit_delta_count"] == 1


@pytest.mark.parametrize("segment", [2, 3])
def test_sac_segments_match_per_block_gradients(segment):
    """segment_size > 1 (diagnostic SAC): one saved boundary per segment, same gradients."""
    ref, cand = _twins(blocks=5, segment_size=segment)
    audit = ReplayAudit(cand.cache)
    cand.plan.attach_replay(audit)
    x_ref = torch.randn(2, WIDTH, requires_grad=True)
    x = x_ref.detach().clone().requires_grad_(True)
    ref(x_ref).sum().backward()
    cand(x).sum().backward()
    _grads_match(ref, cand, x_ref, x)
    assert audit.stats == expected_cycle_counts(5, grad_forwards=1, segment_size=segment)


def test_native_checkpoint_matches_torch_checkpoint():
    torch.manual_seed(3)
    w = torch.randn(WIDTH, WIDTH, requires_grad=True)

    def f(x):
        return torch.tanh(x @ w).sin()

    a = torch.randn(3, WIDTH, requires_grad=True)
    b = a.detach().clone().requires_grad_(True)
    native_checkpoint(f, a).sum().backward()
    ga = w.grad.clone()
    w.grad = None
    checkpoint(f, b, use_reentrant=False).sum().backward()
    torch.testing.assert_close(a.grad, b.grad)
    torch.testing.assert_close(ga, w.grad)


class _Ckpt(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.weight = torch.nn.Parameter(torch.randn(8, 8))

    def forward(self, v):
        return checkpoint(lambda x: torch.tanh(x @ self.weight.t()), v, use_reentrant=False)


def test_saved_tensor_offload_disabled_is_noop():
    m = _Ckpt()
    with offload_scope(m, enabled=False, label="t", min_bytes=128) as scope:
        assert scope is None
        m(torch.randn(2, 8, requires_grad=True)).sum().backward()


def test_saved_tensor_offload_preserves_gradients_and_keeps_replay_on_device():
    torch.manual_seed(7)
    ref, cand = _Ckpt(), _Ckpt()
    cand.load_state_dict(ref.state_dict())
    v_ref = torch.randn(2, 8, requires_grad=True)
    v = v_ref.detach().clone().requires_grad_(True)
    out_ref = ref(v_ref)
    out_ref.sum().backward()
    policy = ThresholdOffload(cand, min_bytes=0, pin_memory=False, include_cpu=True)
    with policy.active():
        out = cand(v)
        policy.begin_backward()
        out.sum().backward()
    torch.testing.assert_close(out, out_ref)
    torch.testing.assert_close(v.grad, v_ref.grad)
    torch.testing.assert_close(cand.weight.grad, ref.weight.grad)
    c = policy.counts
    assert c["saved"] > 0 and c["offloaded"] > 0
    offloaded = c["offloaded"]
    with policy.active():                  # after begin_backward nothing more leaves the device
        cand(v.detach().requires_grad_(True)).sum().backward()
    assert c["offloaded"] == offloaded and c["kept_replay"] > 0
    with pytest.raises(RuntimeError):
        policy.begin_backward()


def test_saved_tensor_offload_keeps_small_tensors_and_parameters():
    m = torch.nn.Linear(8, 8)
    policy = ThresholdOffload(m, min_bytes=1 << 20, pin_memory=False, include_cpu=True)
    with policy.active():
        m(torch.randn(2, 8, requires_grad=True)).sum().backward()
    assert policy.counts["offloaded"] == 0
    assert policy.counts["kept_below_threshold"] + policy.counts["kept_parameter_or_buffer"] == policy.counts["saved"]


def test_staging_target_choice(monkeypatch):
    """`auto` keeps boundary slabs on the host while every local rank's slabs
    fit in half the node's available RAM, else in HBM; explicit targets win;
    CPU devices always stage on the host."""
    from h3_a100.memory import boundary

    gib = 1024**3
    monkeypatch.setattr(boundary, "host_available_bytes", lambda: 200 * gib)
    cuda = torch.device("cuda", 0)
    assert boundary.choose_staging_target("auto", 20 * gib, 4, cuda) == "host"      # 80 <= 100
    assert boundary.choose_staging_target("auto", 20 * gib, 8, cuda) == "device"    # 160 > 100
    assert boundary.choose_staging_target("host", 20 * gib, 8, cuda) == "host"
    assert boundary.choose_staging_target("device", 1, 1, cuda) == "device"
    assert boundary.choose_staging_target("auto", 20 * gib, 8, torch.device("cpu")) == "host"
    monkeypatch.setattr(boundary, "host_available_bytes", lambda: 0)                # unreadable meminfo
    assert boundary.choose_staging_target("auto", 1, 1, cuda) == "device"
    with pytest.raises(ValueError):
        boundary.choose_staging_target("disk", 1, 1, cuda)
