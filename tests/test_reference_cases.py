"""The reference's native-evaluator edge cases, rerun against this engine on the GPU with the
float64 oracle (pinned to the reference's own outputs by tests/test_oracle_golden.py) as the
expected values, on the small Fe/C Möbius models of the reference's GPUMD tests (the tiny
golden fixtures, one per message mode):

* the 21-frame neighbour sequence of tests/mobius_neighbor_check.py:24-83 (pairs entering and
  leaving the cutoffs, type changes, box, pbc and triclinic changes, translations by whole
  periods, a cell smaller than the cutoff, a fully non-periodic box), evaluated one after
  another by one engine, with the radial / angular edge counts of the first frames;
* a pair entering the cutoff within the Verlet skin during MD (tests/test_mobius_gpumd.py:255-270):
  the candidate list is built once and reused, and the final forces are the single-point ones;
* workspace reuse with 0 -> 2 -> 4 -> 2 -> 0 directed edges (tests/test_mobius_gpumd.py:272-294);
* rotation and parity symmetry of energy, forces and virial, and finite-difference forces and
  strain virial of the engine's own energy (tests/test_mobius_equivariant.py:152-211)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from tests.helpers import GOLDEN, load_params, load_state, z_of_type

pytestmark = pytest.mark.gpu
DEV = "cuda"
MODES = ["local", "scalar", "equivariant"]


def _tiny(mode):
    from rune_b200.mobius.plugin import build_model

    g = np.load(GOLDEN / f"tiny_{mode}.npz")
    params, state = load_params(g), load_state(g)
    model = build_model(params)
    model.load_state_dict({k: torch.as_tensor(v, dtype=torch.float32) for k, v in state.items()},
                          strict=True)
    # the oracle sees the float32 weights the engine holds
    state32 = {k: np.asarray(v, np.float32).astype(np.float64) for k, v in state.items()}
    return model.to(DEV).eval(), params, state32


def _oracle(params, state, pos, cell, pbc, types):
    from oracle import models as om
    from oracle.neighbors import neighbor_pairs

    radial, angular = neighbor_pairs(pos, cell, pbc, (params["rcut_radial"],
                                                      params["rcut_angular"]))
    out = om.mobius_forward(params, state, np.asarray(types), om.edges_from_pairs(pos, cell, radial),
                            om.edges_from_pairs(pos, cell, angular), [len(pos)],
                            z_of_type(params))
    return out, len(radial), len(angular)


def _engine(model, pos, cell, pbc, types, forces=True, virial=True):
    out = model.evaluate(torch.as_tensor(np.asarray(pos, np.float64), device=DEV),
                         np.asarray(cell, np.float64).reshape(1, 9), np.array([pbc]),
                         torch.as_tensor(np.asarray(types), dtype=torch.int32, device=DEV),
                         compute_forces=forces, compute_virial=virial)
    torch.cuda.synchronize()
    return {k: v.double().cpu().numpy() for k, v in out.items()}


def _close(out, ref, n, label, f_tol=1e-5):
    de = abs(float(out["energy"][0]) - float(ref["energy"][0])) / max(n, 1)
    df = float(np.max(np.abs(out["forces"] - ref["forces"]))) if n else 0.0
    dw = float(np.max(np.abs(out["virial"].reshape(-1) - np.asarray(ref["virial"]).reshape(-1))))
    assert de <= 1e-6 and df <= f_tol and dw <= 1e-5 * max(n, 1), (label, de, df, dw)


def neighbour_frames():
    """(label, positions, cell, pbc, types) of the reference's 21-frame sequence (Fe = 0,
    C = 1), built step by step the way the reference script mutates one structure."""
    frames = []
    pos = np.array([[5., 5., 5.], [8.9, 5., 5.], [17., 17., 17.], [22., 17., 17.]])
    cell = np.eye(3) * 30.0
    pbc = [True, True, True]
    types = np.array([0, 1, 0, 1])

    def add(label):
        frames.append((label, pos.copy(), cell.copy(), list(pbc), types.copy()))

    def wrap():
        nonlocal pos
        frac = pos @ np.linalg.inv(cell)
        frac = np.where(pbc, frac - np.floor(frac), frac)
        pos = frac @ cell

    add("initial_empty_with_cutoff_and_skin_candidates")
    pos[1, 0] = 8.7
    add("enter_radial_cutoff")
    pos[1, 0] = 8.45
    add("enter_angular_cutoff")
    pos[1, 0] = 8.95
    add("leave_both_cutoffs")
    pos[3, 0] = 20.7
    add("new_pair_enters_from_outside_skin")
    types = np.array([1, 0, 1, 0])
    add("types_change_without_geometry_change")
    frac = pos @ np.linalg.inv(cell)
    cell = np.eye(3) * 31.0
    pos = frac @ cell
    add("box_change")
    pbc = [True, False, True]
    add("pbc_change")
    pos[0, 0] += 3 * 31.
    pos[1, 0] -= 2 * 31.
    pos[2, 2] += 4 * 31.
    pos[3, 2] -= 3 * 31.
    add("independent_multiple_box_translations")
    wrap()
    pos[0, 0] = 30.9
    pos[1, 0] = 3.2
    add("boundary_crossing_setup")
    pos[0, 0] = 31.1
    add("cross_periodic_boundary")
    wrap()
    add("explicit_coordinate_rewrap")
    frac = pos @ np.linalg.inv(cell)
    cell = np.array([[31., .3, .5], [.1, 30., .2], [.4, .2, 32.]])
    pos = frac @ cell
    pbc = [True, True, True]
    add("triclinic_box_change")
    pos = pos + np.array([.05, .03, .02])
    add("triclinic_small_displacement")
    frac = pos @ np.linalg.inv(cell)
    cell = np.eye(3) * 30.0
    pos = np.array([[3., 3., 3.], [12., 3., 3.], [3., 12., 3.], [3., 3., 12.]])
    add("return_to_empty_edges")
    pos = pos + .05
    add("reuse_empty_candidate_list")
    cell = np.array([[4.1, .1, .2], [0., 4.3, .1], [.1, 0., 4.5]])
    pos = np.array([[.10, .13, .22], [.82, .21, .37], [.30, .75, .19], [.68, .63, .81]]) @ cell
    add("small_box_multiple_periodic_images")
    pos[1] += [.02, -.01, .01]
    add("small_box_repeated_call")
    cell = np.eye(3) * 30.0
    pbc = [False, False, False]
    pos = np.array([[3., 3., 3.], [12., 3., 3.], [3., 12., 3.], [3., 3., 12.]])
    add("fully_nonperiodic_empty_edges")
    pbc = [True, True, True]
    add("return_to_large_box_after_small_path")
    add("reuse_after_small_path_rebuild")
    return frames


@pytest.mark.parametrize("mode", MODES)
def test_neighbour_frame_sequence(mode):
    """mobius_neighbor_check.py:24-83: every frame through one engine against the oracle, and
    the edge counts of the first five frames (radial 0, 2, 2, 0, 2; angular 0, 0, 2, 0, 0)."""
    model, params, state = _tiny(mode)
    engine = model.engine()
    counts = []
    frames = neighbour_frames()
    assert len(frames) == 21
    for label, pos, cell, pbc, types in frames:
        out = _engine(model, pos, cell, pbc, types)
        ref, nr, na = _oracle(params, state, pos, cell, pbc, types)
        got_r = len(engine.neighbor_pairs("radial"))
        got_a = len(engine.neighbor_pairs("angular"))
        assert (got_r, got_a) == (nr, na), (label, got_r, got_a, nr, na)
        counts.append((nr, na))
        _close(out, ref, len(pos), f"{mode} {label}")
    assert [c[0] for c in counts[:5]] == [0, 2, 2, 0, 2]
    assert [c[1] for c in counts[:5]] == [0, 0, 2, 0, 0]


@pytest.mark.parametrize("mode", MODES)
def test_pair_enters_cutoff_within_skin(mode):
    """Two atoms 4.2 A apart (cutoff 3.8 A) approach by 0.6 A in 60 MD steps: each moves 0.3 A,
    less than skin / 2, so the candidate list of the first build is reused while the radial
    pair appears; the MD forces at the end equal the single-point (and oracle) forces."""
    from rune_b200.md import NVE

    model, params, state = _tiny(mode)
    pos = np.array([[15., 15., 15.], [19.2, 15., 15.]])
    cell = np.eye(3) * 40.0
    types = np.array([0, 1])
    vel = np.array([[.5, 0., 0.], [-.5, 0., 0.]])
    md = NVE(model, pos, cell, [True] * 3, types, masses=np.array([55.845, 12.011]),
             velocities=vel, dt=0.01, skin=1.0)
    out = md.run(60)
    assert out["rebuilds"] == 1
    final = md.positions.cpu().numpy()
    assert np.linalg.norm(final[1] - final[0]) < params["rcut_radial"]
    ref, nr, _ = _oracle(params, state, final, cell, [True] * 3, types)
    assert nr == 2
    np.testing.assert_allclose(md.forces.double().cpu().numpy(), ref["forces"], atol=1e-5)
    assert abs(out["potential"][-1] - float(ref["energy"][0])) < 1e-5


@pytest.mark.parametrize("mode", MODES)
def test_workspace_reuse_with_changing_and_empty_edges(mode):
    """A fast atom passes two separated atoms and leaves both cutoffs: one engine evaluates
    every frame (0 -> 2 -> 4 -> 2 -> 0 directed edges) against the oracle."""
    model, params, state = _tiny(mode)
    cell = np.eye(3) * 40.0
    types = np.array([0, 1, 0])
    counts = []
    for k in range(49):
        pos = np.array([[15., 15., 15.], [20., 15., 15.], [25. - 0.3 * k, 16.3, 15.]])
        out = _engine(model, pos, cell, [True] * 3, types)
        ref, nr, na = _oracle(params, state, pos, cell, [True] * 3, types)
        counts.append(nr)
        _close(out, ref, 3, f"{mode} frame {k}")
    assert counts[0] == 0 and max(counts) >= 4 and len(set(counts)) >= 3
    assert counts[-3:] == [0, 0, 0] or counts[-1] == 0


def _rotation(parity):
    axis = np.array([1.0, -2.0, 3.0])
    axis /= np.linalg.norm(axis)
    k = np.array([[0, -axis[2], axis[1]], [axis[2], 0, -axis[0]], [-axis[1], axis[0], 0]])
    angle = 0.713
    return (np.eye(3) + np.sin(angle) * k + (1 - np.cos(angle)) * (k @ k)) * parity


def _tri():
    cell = np.array([[3.9, 0.1, 0.2], [0.0, 4.1, 0.1], [0.1, 0.0, 4.3]])
    frac = np.array([[.10, .13, .22], [.82, .21, .37], [.30, .75, .19], [.68, .63, .81]])
    return frac @ cell, cell, np.array([0, 1, 0, 1])


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("parity", [1.0, -1.0])
def test_rotation_and_parity_symmetry(mode, parity):
    model, _, _ = _tiny(mode)
    pos, cell, types = _tri()
    rot = _rotation(parity)
    a = _engine(model, pos, cell, [True] * 3, types)
    b = _engine(model, pos @ rot.T, cell @ rot.T, [True] * 3, types)
    scale = max(1.0, float(np.max(np.abs(a["forces"]))))
    assert abs(a["energy"][0] - b["energy"][0]) <= 1e-5 * max(1.0, abs(a["energy"][0]))
    np.testing.assert_allclose(b["forces"], a["forces"] @ rot.T, atol=2e-5 * scale)
    w = a["virial"].reshape(3, 3)
    np.testing.assert_allclose(b["virial"].reshape(3, 3), rot @ w @ rot.T,
                               atol=2e-5 * max(1.0, float(np.max(np.abs(w)))))
    np.testing.assert_allclose(a["forces"].sum(axis=0), 0.0, atol=1e-5 * scale)


@pytest.mark.parametrize("mode", MODES)
def test_finite_difference_forces_and_strain_virial(mode):
    """Central differences (h = 1e-3 A, strain 1e-3) of the engine's own energy; the engine
    evaluates per-atom energies in float32, so the difference quotients carry ~1e-4 eV/A of
    rounding noise."""
    model, _, _ = _tiny(mode)
    pos, cell, types = _tri()
    res = _engine(model, pos, cell, [True] * 3, types)

    def energy(p, c):
        return float(_engine(model, p, c, [True] * 3, types, forces=False,
                             virial=False)["energy"][0])

    h = 1e-3
    f_fd = np.zeros_like(pos)
    for i in range(len(pos)):
        for c in range(3):
            d = np.zeros_like(pos)
            d[i, c] = h
            f_fd[i, c] = -(energy(pos + d, cell) - energy(pos - d, cell)) / (2 * h)
    w_fd = np.zeros((3, 3))
    for r in range(3):
        for c in range(3):
            eps = np.zeros((3, 3))
            eps[r, c] = h
            plus, minus = np.eye(3) + eps, np.eye(3) - eps
            w_fd[r, c] = -(energy(pos @ plus.T, cell @ plus.T) -
                           energy(pos @ minus.T, cell @ minus.T)) / (2 * h)
    print(mode, "max |F - F_fd|", np.max(np.abs(res["forces"] - f_fd)),
          "max |W - W_fd|", np.max(np.abs(res["virial"].reshape(3, 3) - w_fd)))
    np.testing.assert_allclose(res["forces"], f_fd, atol=2e-3, rtol=1e-3)
    np.testing.assert_allclose(res["virial"].reshape(3, 3), w_fd, atol=5e-3, rtol=1e-3)
