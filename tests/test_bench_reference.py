"""The reference arm of bench.py splits the oracle over worker processes: each worker evaluates
the subsystem of its centre atoms and their neighbours, renumbered. The centres' energies must
equal those of the whole-structure oracle (a NEP energy depends only on its centre's edges)."""

from __future__ import annotations

import numpy as np

import bench
from oracle import models as om
from oracle.neighbors import neighbor_pairs
from rune_b200.nep.plugin import build_model

from .helpers import GOLDEN, load_params, load_state


def test_worker_subsystem_energies_match_whole_structure():
    g = np.load(GOLDEN / "nep_fcc108.npz")
    params = load_params(g)
    state = {k: np.asarray(v, np.float64) for k, v in load_state(g).items()}
    build_model(params)  # the parameters resolve as the bench's model does
    rng = np.random.default_rng(11)
    a, cells = 3.6, 3
    basis = np.array([[0, 0, 0], [0, .5, .5], [.5, 0, .5], [.5, .5, 0]])
    grid = np.stack(np.meshgrid(*(np.arange(cells),) * 3, indexing="ij"), -1).reshape(-1, 3)
    pos = ((grid[:, None] + basis[None]).reshape(-1, 3)) * a + rng.normal(0, 0.1, (108, 3))
    cell = np.eye(3) * a * cells
    types = rng.integers(0, len(params["elements"]), size=len(pos))
    z = np.arange(1.0, len(params["elements"]) + 1.0)
    rc = (params["rcut_radial"], params["rcut_angular"])
    radial, angular = neighbor_pairs(pos, cell, [True] * 3, rc)
    full = om.nep_forward(params, state, types, om.edges_from_pairs(pos, cell, radial),
                          om.edges_from_pairs(pos, cell, angular), [len(pos)], z)
    payload = (params, state, pos, cell, types, z)
    total = 0.0
    for lo, hi in ((0, 40), (40, 41), (41, 108)):
        r = radial[(radial[:, 0] >= lo) & (radial[:, 0] < hi)]
        q = angular[(angular[:, 0] >= lo) & (angular[:, 0] < hi)]
        energy, _, _ = bench._oracle_shard((lo, hi, payload, r, q))
        np.testing.assert_allclose(energy, full["energies"][lo:hi].sum(), rtol=0, atol=1e-10)
        total += energy
    np.testing.assert_allclose(total, full["energies"].sum(), rtol=0, atol=1e-9)
