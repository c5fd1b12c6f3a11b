"""Structure sharding (independent structures over ranks): partition, sub-batch selection and
result reassembly, single-process and as two gloo ranks on CPU."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from rune_b200.sharding import ShardedEvaluator, partition, select, structure_costs


def _batch(seed=3, count=11):
    rng = np.random.default_rng(seed)
    sizes = rng.integers(1, 9, size=count)
    n = int(sizes.sum())
    positions = rng.normal(size=(n, 3))
    types = rng.integers(0, 4, size=n)
    cells = np.stack([np.eye(3) * rng.uniform(4, 9) for _ in range(count)])
    pbc = np.ones((count, 3), bool)
    return positions, cells, pbc, types, sizes


def _fake_evaluate(positions, cells, pbc, types, sizes):
    """CPU stand-in with structure-local outputs that identify every atom and structure."""
    positions = np.asarray(positions, np.float64)
    types = np.asarray(types)
    energies = positions.sum(axis=1) + types
    ptr = np.concatenate([[0], np.cumsum(sizes)])
    energy = np.array([energies[ptr[s]:ptr[s + 1]].sum() for s in range(len(sizes))])
    forces = positions * (types[:, None] + 1.0)
    virial = np.asarray(cells, np.float64).reshape(-1, 9) * np.asarray(sizes)[:, None]
    return {"energies": energies, "energy": energy, "forces": forces, "virial": virial}


def test_partition_covers_and_balances():
    costs = np.array([5.0, 1.0, 3.0, 3.0, 8.0, 2.0, 2.0, 7.0])
    for world in (1, 2, 3, 4, 8, 11):
        parts = partition(costs, world)
        assert len(parts) == world
        flat = sorted(s for p in parts for s in p)
        assert flat == list(range(len(costs)))
        assert all(p == sorted(p) for p in parts)
        loads = [costs[p].sum() for p in parts]
        assert max(loads) - min(loads) <= costs.max() + 1e-12
        assert parts == partition(costs, world)  # deterministic
    with pytest.raises(ValueError):
        partition(costs, 0)


def test_costs_follow_edge_density():
    sizes = [8, 64, 64]
    cells = np.stack([np.eye(3) * 5.0, np.eye(3) * 10.0, np.eye(3) * 5.0])
    c = structure_costs(sizes, cells)
    assert c[2] > c[1] > c[0]  # same atoms in a smaller cell: more edges


def test_select_and_single_rank_roundtrip():
    positions, cells, pbc, types, sizes = _batch()
    atom_idx, sub = select(sizes, [1, 4, 7])
    ptr = np.concatenate([[0], np.cumsum(sizes)])
    expect = np.concatenate([np.arange(ptr[s], ptr[s + 1]) for s in (1, 4, 7)])
    np.testing.assert_array_equal(atom_idx, expect)
    np.testing.assert_array_equal(sub, sizes[[1, 4, 7]])
    full = _fake_evaluate(positions, cells, pbc, types, sizes)
    got = ShardedEvaluator(_fake_evaluate)(positions, cells, pbc, types, sizes)
    for key in full:
        np.testing.assert_array_equal(got[key], full[key])


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, shard_only):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        positions, cells, pbc, types, sizes = _batch()
        seen = []

        def evaluate(p, c, pb, t, s):
            seen.append(int(np.asarray(s).sum()))
            return _fake_evaluate(p, c, pb, t, s)

        ev = ShardedEvaluator(evaluate)
        got = ev(torch.as_tensor(positions), cells, pbc, torch.as_tensor(types), sizes)
        full = _fake_evaluate(positions, cells, pbc, types, sizes)
        for key in full:
            np.testing.assert_allclose(got[key], full[key], rtol=0, atol=1e-12)
        # this rank evaluated exactly its own shard
        parts = partition(structure_costs(sizes, cells), world)
        assert seen == ([int(sizes[parts[rank]].sum())] if parts[rank] else [])
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(120)
def test_two_gloo_ranks_match_single_process():
    mp.start_processes(_rank_main, args=(2, _free_port(), False), nprocs=2, join=True,
                       start_method="spawn")
