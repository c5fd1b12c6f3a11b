"""GPU parity of the Möbius EQ edge products on the tcgen05 tensor cores (kind::i8, exact
integer digit products accumulated in TMEM), selected with RUNE_EQ_TENSOR_CORES=1 when the
engine is created. The same goldens and tolerances as the SIMT path: energy 1e-6 eV/atom,
forces 1e-5 eV/A, virial 1e-5 eV per atom, against the reference's float64 outputs."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from tests.helpers import GOLDEN, WEIGHTS, assert_within, errors, load_params, load_state

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(autouse=True)
def _tensor_cores(monkeypatch):
    monkeypatch.setenv("RUNE_EQ_TENSOR_CORES", "1")


def _evaluate(model, pos, cell, types):
    pos = torch.as_tensor(pos, dtype=torch.float64, device=DEV)
    types = torch.as_tensor(types, dtype=torch.int32, device=DEV)
    res = model.evaluate(pos, np.asarray(cell).reshape(1, 9), np.ones((1, 3), bool), types)
    torch.cuda.synchronize()
    assert model.engine().stats()["tensor_core_layers"] == model.message_layers > 0
    return {k: v.double().cpu().numpy() for k, v in res.items()}


def _ref(g, prefix):
    return (g[f"{prefix}energies_f64"], g[f"{prefix}energy_f64"], g[f"{prefix}forces_f64"],
            g[f"{prefix}virial_f64"])


@pytest.mark.parametrize("name", ["equivariant", "equivariant_tail", "equivariant_zbl_ra",
                                  "equivariant_flexzbl", "equivariant_order1", "equivariant_order2",
                                  "equivariant_order6", "equivariant_order8"])
def test_tiny_eq_tensor_cores(name):
    from rune_b200.mobius.plugin import build_model

    g = np.load(GOLDEN / f"tiny_{name}.npz")
    model = build_model(load_params(g))
    model.load_state_dict({k: torch.as_tensor(v, dtype=torch.float32)
                           for k, v in load_state(g).items()}, strict=True)
    model = model.to(DEV).eval()
    for system in ("tri", "large"):
        prefix = f"{system}:"
        if prefix + "positions" not in g:
            continue
        out = _evaluate(model, g[prefix + "positions"], g[prefix + "cell"], g[prefix + "types"])
        err = errors(out, *_ref(g, prefix))
        print(name, system, err)
        assert_within(err, label=f"{name} {system} tcgen05")


@pytest.mark.parametrize("system", ["mgo64", "si64"])
def test_oam_eq_tensor_cores(system):
    from rune_b200.mobius.plugin import load_model

    path = WEIGHTS / "mobius-oam-eq.pt"
    if not path.exists():
        pytest.skip("repository weights not present")
    g = np.load(GOLDEN / "oam_eq.npz")
    model = load_model(path, device=DEV).eval()
    prefix = f"{system}:"
    out = _evaluate(model, g[prefix + "positions"], g[prefix + "cell"], g[prefix + "types"])
    err = errors(out, *_ref(g, prefix))
    print("eq tcgen05", system, err)
    assert_within(err, label=f"{system} tcgen05")


def test_config4_mgo1728_tensor_cores():
    """OAM-EQ on rocksalt MgO 6x6x6 (1,728 atoms), the config-4 golden, with the tensor-core
    edge products; the result also agrees with the SIMT engine to float32 accumulation-order
    differences."""
    from rune_b200.mobius.plugin import load_model

    path = WEIGHTS / "mobius-oam-eq.pt"
    if not path.exists():
        pytest.skip("repository weights not present")
    g = np.load(GOLDEN / "config4_eq_mgo1728.npz")
    n = len(g["types"])
    model = load_model(path, device=DEV).eval()
    out = _evaluate(model, g["positions"], g["cell"], g["types"])
    de = abs(float(out["energy"].sum()) - float(np.sum(g["energy_f64"]))) / n
    df = float(np.max(np.abs(out["forces"] - g["forces_f64"])))
    dw = float(np.max(np.abs(out["virial"].reshape(-1) - np.asarray(g["virial_f64"]).reshape(-1))))
    print("config4 tcgen05", dict(energy_per_atom=de, forces=df, virial_per_atom=dw / n))
    assert de <= 1e-6 and df <= 1e-5 and dw / n <= 1e-5
