"""Boundary staging, exact replay, saved-tensor offload (reference behaviour:
tests/test_checkpoint_boundary_offload.py, tests/test_exact_adaln_replay.py,
tests/test_activation_offload.py), on toy transformers and on our native checkpoint."""

from functools import partial

import pytest
import torch
from torch.utils.checkpoint import checkpoint

from h3_a100.memory.boundary import install_checkpoint_boundary_cpu_offload
from h3_a100.memory.checkpoint import native_checkpoint
from h3_a100.memory.exact_replay import install_exact_adaln_checkpoint_replay_scope
from h3_a100.memory.saved_tensor_offload import SelectiveSavedTensorOffload, maybe_saved_tensor_offload
from h3_a100.models.adaln import AdaLNCacheController


class _Block(torch.nn.Module):
    def __init__(self, width):
        super().__init__()
        self.proj = torch.nn.Linear(width, width, bias=False)

    def forward(self, h):
        return torch.tanh(self.proj(h)) + h


class _Toy(torch.nn.Module):
    def __init__(self, blocks=3, width=8, native=False):
        super().__init__()
        self.transformer_blocks = torch.nn.ModuleList([_Block(width) for _ in range(blocks)])
        self.gradient_checkpointing = True
        self._gradient_checkpointing_func = (
            native_checkpoint if native else (lambda fn, *a, **k: checkpoint(fn, *a, use_reentrant=False, **k)))

    def forward(self, h):
        for b in self.transformer_blocks:
            h = self._gradient_checkpointing_func(b, h)
        return h


@pytest.mark.parametrize("native", [False, True])
def test_boundary_staging_preserves_output_and_grads(tmp_path, native):
    torch.manual_seed(7)
    ref, cand = _Toy(native=native), _Toy(native=native)
    cand.load_state_dict(ref.state_dict())
    x_ref = torch.randn(2, 5, 8, requires_grad=True)
    x = x_ref.detach().clone().requires_grad_(True)
    y_ref = ref(x_ref)
    y_ref.square().mean().backward()
    reg = install_checkpoint_boundary_cpu_offload(cand, role_getter=lambda: "student",
                                                  event_path=tmp_path / "events.jsonl", pin_memory=False,
                                                  expected_block_count=3, require_cuda=False)
    y = cand(x)
    y.square().mean().backward()
    torch.testing.assert_close(y, y_ref)
    torch.testing.assert_close(x.grad, x_ref.grad)
    for a, b in zip(ref.parameters(), cand.parameters()):
        torch.testing.assert_close(b.grad, a.grad)
    s = reg.stats
    assert s["grad_transformer_forward_count"] == 1 and s["student_grad_forward_count"] == 1
    assert s["grad_checkpoint_call_count"] == 3 and s["cpu_copy_count"] == 3
    assert s["offloaded_logical_bytes"] == 3 * 2 * 5 * 8 * 4
    assert (tmp_path / "events.jsonl").is_file()
    assert reg.stager.live() == 0


def test_boundary_staging_tracks_roles_and_prefetches_in_reverse():
    torch.manual_seed(11)
    model = _Toy(blocks=4, native=True)
    role = {"v": "student"}
    reg = install_checkpoint_boundary_cpu_offload(model, role_getter=lambda: role["v"], pin_memory=False,
                                                  expected_block_count=4, require_cuda=False)
    model(torch.randn(1, 3, 8, requires_grad=True)).sum().backward()
    role["v"] = "fake"
    model(torch.randn(1, 3, 8, requires_grad=True)).sum().backward()
    s = reg.stats
    assert (s["student_grad_forward_count"], s["fake_grad_forward_count"], s["other_grad_forward_count"]) == (1, 1, 0)
    assert s["grad_checkpoint_call_count"] == 8 and s["cpu_copy_count"] == 8
    assert s["unpack_count"] == 8 and s["prefetch_count"] == 8


def test_boundary_staging_skips_no_grad_forward():
    model = _Toy(blocks=2)
    reg = install_checkpoint_boundary_cpu_offload(model, role_getter=lambda: "teacher", pin_memory=False,
                                                  expected_block_count=2, require_cuda=False)
    with torch.no_grad():
        assert torch.isfinite(model(torch.randn(1, 3, 8))).all()
    assert reg.stats["grad_transformer_forward_count"] == 0 and reg.stats["cpu_copy_count"] == 0


def test_boundary_staging_fails_closed_on_layout_mismatch():
    with pytest.raises(RuntimeError, match="native per-block layout"):
        install_checkpoint_boundary_cpu_offload(_Toy(blocks=2), role_getter=lambda: "student", pin_memory=False,
                                                expected_block_count=3, require_cuda=False)


def test_boundary_staging_refuses_to_overwrite_events(tmp_path):
    path = tmp_path / "e.jsonl"
    path.write_text("x")
    with pytest.raises(FileExistsError):
        install_checkpoint_boundary_cpu_offload(_Toy(), role_getter=lambda: "student", event_path=path,
                                                pin_memory=False, expected_block_count=3, require_cuda=False)


class _ReplayToy:
    def __init__(self):
        self.gradient_checkpointing = True
        # run twice: original execution + replay
        self._gradient_checkpointing_func = lambda fn, *a, **k: (fn(*a, **k), fn(*a, **k))[0]


def _controller():
    ctl = AdaLNCacheController(enabled=True, max_dynamic_keys=0)
    key = ("rollout", 3)
    ctl.store(key, 0, (torch.tensor([1.0]),), persistent=True)
    ctl.store(key, 1, (torch.tensor([2.0]),), persistent=True)
    return ctl, key


def test_exact_replay_restores_key_and_never_computes():
    tr = _ReplayToy()
    ctl, key = _controller()
    reg = install_exact_adaln_checkpoint_replay_scope(tr, ctl, expected_block_count=2)

    def must_not_run(_):
        raise AssertionError("projection fallback executed")

    for index in (0, 1):
        def block(x, i=index):
            return x + ctl.get_or_compute(i, x, must_not_run)[0]

        with ctl.scope(key, persistent=True):
            tr._gradient_checkpointing_func(block, torch.tensor([3.0]))
    assert reg.stats == {"checkpoint_wrap_count": 2, "scoped_execution_count": 4, "cache_hit_count": 4,
                         "cache_miss_count": 0, "captured_key_missing_count": 0,
                         "captured_key_incomplete_count": 0, "unexpected_hit_delta_count": 0}


@pytest.mark.parametrize("fn", [partial(checkpoint, use_reentrant=False), native_checkpoint])
def test_exact_replay_with_real_checkpoint(fn):
    class Tr:
        gradient_checkpointing = True

    tr = Tr()
    tr._gradient_checkpointing_func = fn
    ctl = AdaLNCacheController(enabled=True, max_dynamic_keys=0)
    key = ("rollout", 3)
    ctl.store(key, 0, (torch.tensor([0.25]),), persistent=True)
    reg = install_exact_adaln_checkpoint_replay_scope(tr, ctl, expected_block_count=1)

    def block(x):
        m = ctl.get_or_compute(0, x, lambda _: (_ for _ in ()).throw(AssertionError("fallback")))[0]
        y = (x + m).sin()
        return y * y

    x = torch.tensor([0.7], requires_grad=True)
    with ctl.scope(key, persistent=True):
        y = tr._gradient_checkpointing_func(block, x)
    y.sum().backward()
    assert x.grad is not None
    assert reg.stats["checkpoint_wrap_count"] == 1
    assert reg.stats["scoped_execution_count"] == 2 and reg.stats["cache_hit_count"] == 2
    assert reg.stats["cache_miss_count"] == 0


def test_exact_replay_fails_closed_without_key():
    tr = _ReplayToy()
    ctl, _ = _controller()
    install_exact_adaln_checkpoint_replay_scope(tr, ctl, expected_block_count=2)
    with pytest.raises(RuntimeError, match="no active cache key"):
        tr._gradient_checkpointing_func(lambda x: x, torch.tensor([1.0]))


def test_exact_replay_fails_closed_on_incomplete_key():
    tr = _ReplayToy()
    ctl, key = _controller()
    install_exact_adaln_checkpoint_replay_scope(tr, ctl, expected_block_count=3)
    with ctl.scope(key, persistent=True), pytest.raises(RuntimeError, match="incomplete"):
        tr._gradient_checkpointing_func(lambda x: x, torch.tensor([1.0]))


class _Ckpt(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.weight = torch.nn.Parameter(torch.randn(8, 8))

    def forward(self, v):
        return checkpoint(lambda x: torch.tanh(x @ self.weight.t()), v, use_reentrant=False)


def test_saved_tensor_offload_disabled_is_noop():
    m = _Ckpt()
    with maybe_saved_tensor_offload(m, enabled=False, logical_component="t", min_offload_bytes=128) as scope:
        assert scope is None
        m(torch.randn(2, 8, requires_grad=True)).sum().backward()


def test_saved_tensor_offload_preserves_gradients():
    torch.manual_seed(7)
    ref, cand = _Ckpt(), _Ckpt()
    cand.load_state_dict(ref.state_dict())
    v_ref = torch.randn(2, 8, requires_grad=True)
    v = v_ref.detach().clone().requires_grad_(True)
    out_ref = ref(v_ref)
    out_ref.sum().backward()
    scope = SelectiveSavedTensorOffload(cand, logical_component="t", min_offload_bytes=0, pin_memory=False,
                                        offload_cpu_tensors=True)
    with scope.context():
        out = cand(v)
        scope.begin_backward()
        out.sum().backward()
    torch.testing.assert_close(out, out_ref)
    torch.testing.assert_close(v.grad, v_ref.grad)
    torch.testing.assert_close(cand.weight.grad, ref.weight.grad)
    assert scope.stats["pack_count"] > 0 and scope.stats["offload_count"] > 0


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
