"""bench.py's CPU legs. The oracle port (cpu_baseline, and the reference arm's fallback) splits
the oracle over worker processes: each worker evaluates the subsystem of its centre atoms and
their neighbours, renumbered, and the centres' energies must equal those of the whole-structure
oracle. The reference arm feeds the reference's own models batches built here: they must give
the reference's golden outputs."""

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


def _reference_import():
    """The reference package as installed for bench.py's reference arm (skip when absent)."""
    import sys

    import pytest

    if not (bench.REFERENCE_INSTALL / "rune").exists():
        pytest.skip("reference not installed under baseline/_ref")
    for p in (str(bench.ASE_SHIM), str(bench.REFERENCE_INSTALL)):
        if p not in sys.path:
            sys.path.insert(0, p)


def test_reference_arm_batch_reproduces_reference_golden():
    """The padded batch the reference arm builds, fed to the reference's own NEP in float64,
    gives the golden outputs that the reference produced from its own neighbour builder."""
    _reference_import()
    import torch
    from rune.nep.model import NEP

    g = np.load(GOLDEN / "nep_fcc108.npz")
    params = load_params(g)
    model = NEP(params).double()
    model.load_state_dict({k: torch.as_tensor(v) for k, v in load_state(g).items()})
    pos, cell, types = g["positions"], g["cell"], g["types"]
    radial, angular = neighbor_pairs(pos, cell, [True] * 3,
                                     (params["rcut_radial"], params["rcut_angular"]))
    batch = bench.reference_padded_batch(pos, cell, types, radial, angular)
    batch = {k: (v.double() if v.is_floating_point() else v) for k, v in batch.items()}
    batch["positions"] = torch.as_tensor(pos)
    for name in ("radial", "angular"):
        p = radial if name == "radial" else angular
        off = np.zeros(batch[f"{name}_offsets"].shape)
        counts = np.bincount(p[:, 0], minlength=len(pos))
        slot = np.arange(len(p)) - np.repeat(np.cumsum(counts) - counts, counts)
        off[p[:, 0], slot] = p[:, 2:5] @ cell
        batch[f"{name}_offsets"] = torch.as_tensor(off)
    out = model({**batch, "compute_forces": True, "compute_virial": True})
    np.testing.assert_allclose(out["energy"].detach().numpy(), g["energy_f64"], rtol=0,
                               atol=1e-9)
    np.testing.assert_allclose(out["forces"].detach().numpy(), g["forces_f64"], rtol=0,
                               atol=1e-9)


def test_reference_arm_batch_of_cells_matches_single_cells():
    """Independent cells stacked into one reference batch give each cell's own energy."""
    _reference_import()
    import torch
    from rune.nep.model import NEP

    g = np.load(GOLDEN / "nep_fcc108.npz")
    params = load_params(g)
    torch.manual_seed(3)
    model = NEP(params).double()
    pos, cells, types, sizes = bench.random_cells(3, len(params["elements"]), seed=9, n_min=8,
                                                 n_max=12)
    rc = (params["rcut_radial"], params["rcut_angular"])
    batch = bench.reference_batch_of_cells(pos, cells, sizes, types, rc)
    batch = {k: (v.double() if v.is_floating_point() else v) for k, v in batch.items()}
    out = model({**batch, "compute_forces": False, "compute_virial": False})
    start = 0
    for k, n in enumerate(sizes):
        cell = cells[k].reshape(3, 3)
        p = pos[start:start + n]
        radial, angular = neighbor_pairs(p, cell, [True] * 3, rc)
        one = bench.reference_padded_batch(p, cell, types[start:start + n], radial, angular)
        one = {kk: (v.double() if v.is_floating_point() else v) for kk, v in one.items()}
        e = model({**one, "compute_forces": False, "compute_virial": False})["energy"]
        np.testing.assert_allclose(out["energy"][k].item(), e.item(), rtol=0, atol=1e-5)
        start += n
