"""Placement arithmetic (reference behaviour: tests/test_topology.py)."""

import pytest

from h3_a100.parallel.topology import resolve_hybrid_topology


def test_two_by_eight_mapping():
    r0, r7, r8, r15 = (resolve_hybrid_topology(16, r, 8) for r in (0, 7, 8, 15))
    assert (r0.replicate_rank, r0.shard_rank) == (0, 0)
    assert (r7.replicate_rank, r7.shard_rank) == (0, 7)
    assert (r8.replicate_rank, r8.shard_rank) == (1, 0)
    assert (r15.replicate_rank, r15.shard_rank) == (1, 7)
    assert r15.replicate_size == 2
    assert r8.shard_group_ranks == list(range(8, 16))
    assert r8.replicate_group_ranks == [0, 8]


def test_one_node_is_one_replica():
    topo = resolve_hybrid_topology(8, 5, 8)
    assert (topo.replicate_size, topo.replicate_rank, topo.shard_rank) == (1, 0, 5)


@pytest.mark.parametrize("world,rank,shard", [(16, 0, 6), (0, 0, 1), (8, 8, 8), (8, -1, 8)])
def test_invalid_topologies(world, rank, shard):
    with pytest.raises(ValueError):
        resolve_hybrid_topology(world, rank, shard)
