"""Velocity-Verlet NVE on the device with a Verlet-skin neighbour cache (``rune_md_nve``).

The engine integrates one periodic structure entirely on the GPU: positions and velocities stay
in device memory (float64), forces come from the model's engine each step, and the neighbour
candidates (pairs within max(rc) + skin) are rebuilt when an atom has moved more than skin / 2
since the last build — the cache rule of the reference's native evaluator
(rune/mobius/src/mobius.cu:334-402). Units: A, fs, amu, eV.
"""

from __future__ import annotations

import numpy as np
import torch

from .elements import atomic_masses, atomic_numbers

# 1 amu A^2 / fs^2 in eV, and k_B in eV / K
AMU_A2_FS2_EV = 103.642697
KB_EV = 8.617333262e-5


def maxwell_boltzmann(masses, temperature, seed=0):
    """Velocities (A/fs) drawn at `temperature` (K) from a seeded generator, zero net momentum."""
    masses = np.asarray(masses, np.float64)
    rng = np.random.default_rng(seed)
    sigma = np.sqrt(KB_EV * temperature / (masses * AMU_A2_FS2_EV))
    v = rng.normal(size=(len(masses), 3)) * sigma[:, None]
    v -= (masses[:, None] * v).sum(axis=0) / masses.sum()
    return v


class NVE:
    """Velocity-Verlet NVE of one structure with `model` (an engine model: ``model.engine()``).

    positions [N, 3] (A), cell [3, 3], pbc [3], types [N] (model type indices), masses [N] amu
    (default: standard weights of the model's elements), velocities [N, 3] A/fs (default zero).
    """

    def __init__(self, model, positions, cell, pbc, types, masses=None, velocities=None,
                 dt=1.0, skin=1.0, device=None):
        engine = model.engine()
        self.engine = engine
        self.device = torch.device(device) if device is not None else engine._dev()
        self.types = torch.as_tensor(np.asarray(types), dtype=torch.int32, device=self.device)
        n = int(self.types.shape[0])
        self.positions = torch.as_tensor(np.asarray(positions, np.float64).reshape(n, 3),
                                         device=self.device).clone()
        if masses is None:
            elements = list(getattr(model, "elements", None) or model.params["elements"])
            table = np.array([atomic_masses[atomic_numbers[e]] for e in elements])
            masses = table[np.asarray(types)]
        self.masses = torch.as_tensor(np.asarray(masses, np.float64), device=self.device)
        if velocities is None:
            velocities = np.zeros((n, 3))
        self.velocities = torch.as_tensor(np.asarray(velocities, np.float64).reshape(n, 3),
                                          device=self.device).clone()
        self.cell = np.asarray(cell, np.float64).reshape(9)
        self.pbc = np.asarray(pbc, bool).reshape(3)
        self.dt = float(dt)
        self.skin = float(skin)
        self.forces = torch.zeros((n, 3), dtype=torch.float32, device=self.device)

    def run(self, n_steps, stream=None):
        """Advance n_steps steps. Returns potential, kinetic and total energies (eV) of the
        initial and every following state, and the number of candidate-list builds."""
        energies, rebuilds = self.engine.md_nve(
            self.types, self.positions, self.velocities, self.masses, self.cell, self.pbc,
            self.dt, n_steps, self.skin, forces=self.forces, stream=stream)
        return {"potential": energies[:, 0], "kinetic": energies[:, 1],
                "total": energies.sum(axis=1), "rebuilds": rebuilds}
