"""Structure sharding for batches of independent structures, one rank per GPU.

Independent periodic structures need no exchange between GPUs: every rank evaluates a subset
of the batch with its own engine and only the per-structure results are gathered. The
reference evaluates a batch on one device (``BatchBuilder`` + ``Mobius.forward``,
rune/mobius/interface/batch.py:124-166, rune/mobius/model.py:307-393); ``ShardedEvaluator``
returns the same outputs, in the same order, from any number of ranks.

Assignment is greedy longest-processing-time on a per-structure cost proportional to the
structure's edge count (atoms x atom density: N^2 / V), plus its atom count.
"""

from __future__ import annotations

from typing import Callable, Sequence

import numpy as np


def structure_costs(sizes: Sequence[int], cells: np.ndarray) -> np.ndarray:
    """Relative evaluation cost per structure: edges (N^2 / V) plus atoms. Structures without
    a volume (no cell) count N^2 / (N * 20 A^3)."""
    sizes = np.asarray(sizes, np.float64)
    cells = np.asarray(cells, np.float64).reshape(-1, 3, 3)
    vol = np.abs(np.linalg.det(cells))
    vol = np.where(vol > 1e-6, vol, np.maximum(sizes, 1.0) * 20.0)
    return sizes * sizes / vol * 60.0 + sizes


def partition(costs: Sequence[float], world: int) -> list[list[int]]:
    """Greedy LPT assignment of structures to `world` ranks.

    Structures are taken by decreasing cost (ties: lower index first) and each goes to the
    rank with the smallest load so far (ties: lower rank). Every rank's list is returned in
    ascending structure order, so the assignment is deterministic and reproducible on every
    rank without communication."""
    if world < 1:
        raise ValueError("world size must be positive")
    costs = np.asarray(costs, np.float64)
    order = sorted(range(len(costs)), key=lambda s: (-costs[s], s))
    load = [0.0] * world
    parts: list[list[int]] = [[] for _ in range(world)]
    for s in order:
        r = min(range(world), key=lambda k: (load[k], k))
        parts[r].append(s)
        load[r] += float(costs[s])
    return [sorted(p) for p in parts]


def select(sizes: Sequence[int], structures: Sequence[int]):
    """Atom index array and sizes of the sub-batch made of `structures` (ascending)."""
    sizes = np.asarray(sizes, np.int64)
    ptr = np.concatenate([[0], np.cumsum(sizes)])
    atoms = [np.arange(ptr[s], ptr[s + 1]) for s in structures]
    atom_idx = np.concatenate(atoms) if atoms else np.zeros(0, np.int64)
    return atom_idx, sizes[list(structures)] if len(structures) else np.zeros(0, np.int64)


class ShardedEvaluator:
    """Evaluate a batch of independent structures across the ranks of a process group.

    ``evaluate_fn(positions, cells, pbc, types, sizes)`` evaluates one sub-batch on this rank
    (for example ``model.evaluate`` of the engine model) and returns a dict with ``energies``
    [n], ``energy`` [b], ``forces`` [n, 3] and ``virial`` [b, 9] (tensors or arrays). The call
    returns the whole batch's outputs on every rank as float64 numpy arrays in the input order.
    With ``group`` None (or one rank) it evaluates everything locally.
    """

    def __init__(self, evaluate_fn: Callable, group=None):
        self.evaluate_fn = evaluate_fn
        self.group = group

    def _world(self):
        import torch.distributed as dist

        if self.group is None and not (dist.is_available() and dist.is_initialized()):
            return 1, 0
        return dist.get_world_size(self.group), dist.get_rank(self.group)

    def shard(self, sizes, cells, world):
        return partition(structure_costs(sizes, cells), world)

    def __call__(self, positions, cells, pbc, types, sizes):
        sizes = np.asarray(sizes, np.int64)
        cells = np.asarray(cells, np.float64).reshape(-1, 9)
        pbc = np.asarray(pbc, bool).reshape(-1, 3)
        world, rank = self._world()
        parts = self.shard(sizes, cells, world)
        mine = parts[rank]
        atom_idx, sub_sizes = select(sizes, mine)
        local = {}
        if len(mine):
            out = self.evaluate_fn(_take(positions, atom_idx), cells[mine], pbc[mine],
                                   _take(types, atom_idx), sub_sizes)
            local = {k: _numpy(v) for k, v in out.items() if v is not None}
        if world == 1:
            gathered = [local]
        else:
            import torch.distributed as dist

            gathered = [None] * world
            dist.all_gather_object(gathered, local, group=self.group)
        return _assemble(gathered, parts, sizes)


def _take(x, idx):
    try:
        import torch

        if isinstance(x, torch.Tensor):
            return x[torch.as_tensor(idx, device=x.device, dtype=torch.long)]
    except ImportError:  # pragma: no cover - torch is a dependency
        pass
    return np.asarray(x)[idx]


def _numpy(v):
    if hasattr(v, "detach"):
        v = v.detach().cpu().numpy()
    return np.asarray(v, np.float64)


def _assemble(gathered, parts, sizes):
    """Per-rank results back into batch order."""
    n = int(sizes.sum())
    b = len(sizes)
    ptr = np.concatenate([[0], np.cumsum(sizes)])
    out = {}
    for res, structures in zip(gathered, parts):
        if not structures:
            continue
        off = 0
        for k, s in enumerate(structures):
            na = int(sizes[s])
            for key, val in res.items():
                if key in ("energy", "virial"):
                    shape = (b,) + val.shape[1:]
                    dst = out.setdefault(key, np.zeros(shape))
                    dst[s] = val[k]
                else:
                    shape = (n,) + val.shape[1:]
                    dst = out.setdefault(key, np.zeros(shape))
                    dst[ptr[s]:ptr[s] + na] = val[off:off + na]
            off += na
    return out
