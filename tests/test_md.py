"""Velocity-Verlet NVE driver (rune_md_nve): initial velocities on the CPU; on the GPU, the
trajectory against a host loop over the engine's single-point evaluation, the Verlet-skin
cache (rebuilds, final forces), and energy conservation."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from rune_b200.md import AMU_A2_FS2_EV, KB_EV, maxwell_boltzmann

from .helpers import GOLDEN, load_params, load_state

DEV = "cuda"


def test_maxwell_boltzmann_temperature_and_momentum():
    masses = np.full(20000, 63.546)
    v = maxwell_boltzmann(masses, 600.0, seed=4)
    np.testing.assert_allclose((masses[:, None] * v).sum(axis=0), 0.0, atol=1e-9)
    ke = 0.5 * (masses[:, None] * v * v).sum() * AMU_A2_FS2_EV
    temperature = 2.0 * ke / (3.0 * len(masses) * KB_EV)
    assert abs(temperature - 600.0) < 15.0
    np.testing.assert_array_equal(v, maxwell_boltzmann(masses, 600.0, seed=4))


def _nep_fcc(cells=4, seed=7):
    from rune_b200.nep.plugin import build_model

    g = np.load(GOLDEN / "nep_fcc108.npz")
    params = dict(load_params(g))
    model = build_model(params)
    model.load_state_dict({k: torch.as_tensor(v, dtype=torch.float32)
                           for k, v in load_state(g).items()}, strict=True)
    model = model.to(DEV).eval()
    a = 3.6
    basis = np.array([[0, 0, 0], [0, .5, .5], [.5, 0, .5], [.5, .5, 0]])
    grid = np.stack(np.meshgrid(*(np.arange(cells),) * 3, indexing="ij"), -1).reshape(-1, 3)
    pos = ((grid[:, None, :] + basis[None]).reshape(-1, 3)) * a
    rng = np.random.default_rng(seed)
    pos = pos + rng.normal(0.0, 0.05, size=pos.shape)
    cell = np.eye(3) * a * cells
    types = rng.integers(0, len(params["elements"]), size=len(pos))
    from rune_b200.elements import atomic_masses, atomic_numbers

    masses = np.array([atomic_masses[atomic_numbers[e]] for e in params["elements"]])[types]
    return model, pos, cell, types, masses


def _host_verlet(model, pos, cell, types, masses, vel, dt, steps):
    """x, v after `steps` velocity-Verlet steps with forces from the single-point entry."""
    from rune_b200.md import AMU_A2_FS2_EV

    acc = 1.0 / AMU_A2_FS2_EV
    x = torch.as_tensor(pos, dtype=torch.float64, device=DEV).clone()
    v = torch.as_tensor(vel, dtype=torch.float64, device=DEV).clone()
    m = torch.as_tensor(masses, dtype=torch.float64, device=DEV)[:, None]
    t = torch.as_tensor(types, dtype=torch.int32, device=DEV)

    def force(xx):
        out = model.evaluate(xx, cell.reshape(1, 9), np.ones((1, 3), bool), t)
        return out["forces"].double(), float(out["energy"][0])

    f, _ = force(x)
    for _ in range(steps):
        v = v + 0.5 * dt * f / m * acc
        x = x + dt * v
        f, e = force(x)
        v = v + 0.5 * dt * f / m * acc
    return x, v, f


@pytest.mark.gpu
def test_nve_trajectory_matches_host_loop():
    from rune_b200.md import NVE

    model, pos, cell, types, masses = _nep_fcc()
    vel = maxwell_boltzmann(masses, 800.0, seed=1)
    md = NVE(model, pos, cell, [True] * 3, types, masses=masses, velocities=vel, dt=1.0,
             skin=0.3)
    out = md.run(20)
    x_ref, v_ref, f_ref = _host_verlet(model, pos, cell, types, masses, vel, 1.0, 20)
    assert np.max(np.abs((md.positions - x_ref).cpu().numpy())) < 1e-7
    assert np.max(np.abs((md.velocities - v_ref).cpu().numpy())) < 1e-8
    assert np.max(np.abs((md.forces.double() - f_ref).cpu().numpy())) < 1e-4
    assert out["rebuilds"] >= 2  # 800 K over 20 fs moves atoms beyond skin / 2 = 0.15 A


@pytest.mark.gpu
def test_nve_conserves_energy_and_reuses_candidates():
    """Velocity Verlet with consistent forces: the total-energy fluctuation shrinks as dt^2
    (same simulated time at dt and dt / 2) and shows no secular drift; the candidate cache is
    reused between rebuilds; the final forces are the single-point forces. The window is
    150 fs: this random-weight model brings two atoms close near 188 fs, where dt = 1 fs
    leaves the asymptotic dt^2 regime (the error there shrinks faster than dt^2 with dt)."""
    from rune_b200.md import NVE

    model, pos, cell, types, masses = _nep_fcc(cells=5)
    vel = maxwell_boltzmann(masses, 300.0, seed=2)
    n = len(types)
    runs = {}
    for dt, steps in ((1.0, 150), (0.5, 300)):
        md = NVE(model, pos, cell, [True] * 3, types, masses=masses, velocities=vel, dt=dt,
                 skin=1.0)
        out = md.run(steps)
        runs[dt] = (md, out)
    f1 = np.max(np.abs(runs[1.0][1]["total"] - runs[1.0][1]["total"][0])) / n
    f2 = np.max(np.abs(runs[0.5][1]["total"] - runs[0.5][1]["total"][0])) / n
    assert 3.0 < f1 / f2 < 5.5, (f1, f2)
    tot = runs[0.5][1]["total"] / n
    slope = np.polyfit(np.arange(len(tot)) * 0.5e-3, tot, 1)[0]  # eV / atom / ps
    assert abs(slope) < f2 / 0.15, slope  # no drift beyond the fluctuation scale
    md, out = runs[1.0]
    assert out["kinetic"][0] > 0.0
    assert 1 <= out["rebuilds"] < 150  # the cache is reused between rebuilds
    ref = model.evaluate(md.positions, cell.reshape(1, 9), np.ones((1, 3), bool),
                         torch.as_tensor(types, dtype=torch.int32, device=DEV))
    # two float32 evaluations whose rows list the same edges in different orders (candidate
    # rows vs a fresh build): summation-order differences on forces of up to ~8 eV/A
    assert torch.max(torch.abs(ref["forces"] - md.forces)).item() < 5e-5
    assert abs(float(ref["energy"][0]) - out["potential"][-1]) < 1e-6 * n
