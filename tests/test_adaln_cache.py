"""AdaLN bank + exact cache (reference behaviour: tests/test_adaln_cache.py)."""

import torch
from torch import nn

from h3_a100.models.adaln import AdaLNProjectionBank, adaln_bank, install_adaln_cache


class CountingProjection(nn.Module):
    def __init__(self, offset):
        super().__init__()
        self.weight = nn.Parameter(torch.tensor(offset))
        self.calls = 0

    def forward(self, temb):
        self.calls += 1
        return tuple(temb + self.weight + i for i in range(6))


class Block(nn.Module):
    def __init__(self, offset):
        super().__init__()
        self.adaln_proj = CountingProjection(offset)


class Transformer(nn.Module):
    def __init__(self):
        super().__init__()
        self.transformer_blocks = nn.ModuleList([Block(1.0), Block(2.0)])
        self.time_embedder = nn.Linear(2, 2, bias=False)


def _installed():
    tr = Transformer()
    tr.requires_grad_(False)
    ctl = install_adaln_cache(tr, max_dynamic_keys=1)
    bank = adaln_bank(tr)
    assert isinstance(bank, AdaLNProjectionBank)
    return tr, bank, ctl


def test_persistent_key_computes_once_and_is_exact():
    tr, bank, ctl = _installed()
    temb = torch.tensor([[1.0, 2.0]])
    with ctl.scope(("rollout", 0), persistent=True):
        first = [b.adaln_proj(temb) for b in tr.transformer_blocks]
    with ctl.scope(("rollout", 0), persistent=True):
        second = [b.adaln_proj(temb) for b in tr.transformer_blocks]
    assert [p.calls for p in bank.projections] == [1, 1]
    for a, b in zip(first, second):
        for x, y in zip(a, b):
            torch.testing.assert_close(x, y, rtol=0, atol=0)
    s = ctl.stats()
    assert (s.misses, s.hits, s.persistent_keys) == (2, 2, 1) and s.bytes > 0


def test_dynamic_key_reuse_then_recompute_after_drop():
    tr, bank, ctl = _installed()
    temb = torch.tensor([[3.0, 4.0]])
    with ctl.scope(("score", 1)):
        tr.transformer_blocks[0].adaln_proj(temb)
        tr.transformer_blocks[0].adaln_proj(temb)
    assert bank.projections[0].calls == 1
    ctl.drop(("score", 1))
    with ctl.scope(("score", 1)):
        tr.transformer_blocks[0].adaln_proj(temb)
    assert bank.projections[0].calls == 2


def test_lru_never_evicts_persistent():
    tr, _, ctl = _installed()
    temb = torch.ones(1, 2)
    with ctl.scope("persistent", persistent=True):
        tr.transformer_blocks[0].adaln_proj(temb)
    for key in ("dynamic-1", "dynamic-2"):
        with ctl.scope(key):
            tr.transformer_blocks[0].adaln_proj(temb)
    s = ctl.stats()
    assert (s.persistent_keys, s.dynamic_keys, s.evictions) == (1, 1, 1)
    assert ctl.has_complete_key("persistent", 1)


def test_rejects_trainable_projection():
    tr = Transformer()
    try:
        install_adaln_cache(tr)
    except RuntimeError as err:
        assert "must be frozen" in str(err)
    else:
        raise AssertionError("trainable AdaLN projections must not be cached")


def test_install_is_idempotent():
    tr, _, first = _installed()
    assert install_adaln_cache(tr) is first


def test_counted_lookup_reports_miss_without_computing():
    _, _, ctl = _installed()
    assert ctl.lookup(("rollout", 9), 0) is None
    assert ctl.stats().misses == 1
