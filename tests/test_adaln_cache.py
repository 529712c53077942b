"""AdaLN modulation cache (the reference's tests/test_adaln_cache.py, in behaviour):
one exact table per key, computed once; dynamic keys bounded and droppable;
persistent keys never evicted; frozen bank and time MLP required."""

import pytest
import torch
from torch import nn

from h3_a100.models.adaln import AdaLNBank, ModulationCache


class CountingProjection(nn.Module):
    def __init__(self, offset):
        super().__init__()
        self.weight = nn.Parameter(torch.tensor(offset), requires_grad=False)
        self.calls = 0

    def forward(self, temb):
        self.calls += 1
        return (temb[:, :1] + self.weight + torch.arange(6.0)).view(1, 6, 1).expand(1, 6, 3).clone()


def _bank():
    return AdaLNBank([CountingProjection(1.0), CountingProjection(2.0)])


def _build(cache, bank, key, persistent, temb):
    calls = {"temb": 0}

    def make_temb():
        calls["temb"] += 1
        return temb

    cache.build(key, persistent=persistent, temb=make_temb, project=lambda i, t: bank[i](t))
    return calls["temb"]


def test_persistent_key_computes_once_and_is_exact():
    bank = _bank()
    cache = ModulationCache.attach(bank, None, max_dynamic_keys=1)
    temb = torch.tensor([[1.0, 2.0]])
    assert _build(cache, bank, ("rollout", 0), True, temb) == 1
    assert _build(cache, bank, ("rollout", 0), True, temb) == 0          # complete: nothing recomputed
    assert [p.calls for p in bank.projections] == [1, 1]
    first = [cache.fetch(("rollout", 0), i).clone() for i in range(2)]
    second = [cache.fetch(("rollout", 0), i) for i in range(2)]
    for a, b in zip(first, second):
        torch.testing.assert_close(a, b, rtol=0, atol=0)
    torch.testing.assert_close(first[1], bank[1](temb).float(), rtol=0, atol=0)
    s = cache.stats()
    assert (s.misses, s.stores, s.hits, s.persistent_keys) == (2, 2, 4, 1) and s.bytes == 2 * 6 * 3 * 4


def test_dynamic_key_reuse_then_recompute_after_release():
    bank = _bank()
    cache = ModulationCache.attach(bank, None, max_dynamic_keys=1)
    temb = torch.tensor([[3.0, 4.0]])
    _build(cache, bank, ("score", 1), False, temb)
    _build(cache, bank, ("score", 1), False, temb)
    assert bank[0].calls == 1
    cache.release(("score", 1))
    assert not cache.complete(("score", 1))
    _build(cache, bank, ("score", 1), False, temb)
    assert bank[0].calls == 2


def test_eviction_never_drops_persistent_or_held_tables():
    bank = _bank()
    cache = ModulationCache.attach(bank, None, max_dynamic_keys=1)
    temb = torch.ones(1, 2)
    _build(cache, bank, "persistent", True, temb)
    cache.release("persistent")                         # persistent tables survive release
    _build(cache, bank, "dynamic-1", False, temb)
    with cache.hold("dynamic-1"):
        _build(cache, bank, "dynamic-2", False, temb)   # over the bound, but dynamic-1 is held
        assert cache.complete("dynamic-1") and cache.complete("dynamic-2")
    _build(cache, bank, "dynamic-3", False, temb)       # now the oldest unheld ones go
    s = cache.stats()
    assert (s.persistent_keys, s.dynamic_keys, s.evictions) == (1, 1, 2)
    assert cache.complete("persistent") and cache.complete("dynamic-3")


def test_rejects_trainable_projection_or_time_mlp():
    bank = _bank()
    bank[0].weight.requires_grad_(True)
    with pytest.raises(RuntimeError, match="must be frozen"):
        ModulationCache.attach(bank, None)
    with pytest.raises(RuntimeError, match="timestep embedder"):
        ModulationCache.attach(_bank(), nn.Linear(2, 2))


def test_counted_fetch_reports_miss_without_computing():
    bank = _bank()
    cache = ModulationCache.attach(bank, None)
    assert cache.fetch(("rollout", 9), 0) is None
    assert cache.stats().misses == 1 and bank[0].calls == 0


def test_dit_blocks_read_the_precomputed_table():
    """The DiT owns the bank; a forward under a key reads one table row per block."""
    from h3_a100.models.dit import DiTConfig, H3DiT
    from h3_a100.ops.torch_kernels import TorchKernels

    cfg = DiTConfig(hidden=32, heads=2, head_dim=16, ffn=64, time_embed_dim=48, num_blocks=3,
                    num_refiner_blocks=1, text_dim=16, video_channels=4)
    dit = H3DiT(cfg, dtype=torch.float32)
    dit.init_weights(3)
    dit.set_kernels(TorchKernels())
    cache = ModulationCache.attach(dit.adaln_bank, dit.time_embedder)
    t = torch.tensor([500.0, 500.0])
    cache.build(("rollout", 0), persistent=True, temb=lambda: dit.time_embedding(t), project=dit.project_adaln)
    video, text = torch.randn(1, 4, 1, 4, 4), torch.randn(1, 5, 16)
    with torch.no_grad():
        cached, _ = dit(video, None, text, t, adaln_key=("rollout", 0), modulations=cache)
        direct, _ = dit(video, None, text, t)
    torch.testing.assert_close(cached, direct)
    assert cache.stats().hits == cfg.num_blocks
