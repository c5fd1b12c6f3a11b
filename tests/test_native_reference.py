"""Same-box comparison with the reference's native FP64 evaluator (``Mobius::compute`` of
rune/mobius/src, the GPUMD adapter), compiled from the reference's own sources against
stand-ins for the GPUMD types it uses (oracle/native). The native build is first pinned to the
float64 golden outputs that the reference's PyTorch models produced for the same inputs (its
own parity with the PyTorch path is ~1e-10, docs/paper.pdf p.7); the engine is then compared
with it at the north-star tolerances.

Cases: OAM-EQ on MgO 6x6x6 (1,728 atoms: the native large-box path with its Verlet-skin
candidate list), OAM-Local on Si-216 and OAM-MP on Si-64 (the native small-box path, every
periodic image enumerated)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import native_ref
from tests.helpers import GOLDEN, WEIGHTS

pytestmark = pytest.mark.gpu

CASES = [("eq", "config4_eq_mgo1728.npz", ""), ("loc", "oam_loc.npz", "si216:"),
         ("mp", "oam_mp.npz", "si64:")]


def _setup(variant, fixture, prefix, tmp_path):
    if not native_ref.available():
        pytest.skip("native reference not built (oracle/native/build.sh)")
    from rune_b200.mobius.plugin import export_model, load_model

    path = WEIGHTS / f"mobius-oam-{variant}.pt"
    if not path.exists():
        pytest.skip(f"{path.name} not present")
    model = load_model(path, device="cuda").eval()
    g = np.load(GOLDEN / fixture)
    pos, cell, types = g[prefix + "positions"], g[prefix + "cell"], g[prefix + "types"]
    model_file = export_model(model, tmp_path / f"oam-{variant}.txt")
    native = native_ref.NativeMobius(model_file, len(pos))
    return model, g, pos, cell, types, native


@pytest.mark.parametrize("variant,fixture,prefix", CASES)
def test_native_build_matches_reference_float64(variant, fixture, prefix, tmp_path):
    _, g, pos, cell, types, native = _setup(variant, fixture, prefix, tmp_path)
    ref = native.compute(types, pos, cell)
    native.close()
    n = len(pos)
    de = abs(ref["energy"] - float(np.sum(g[prefix + "energy_f64"]))) / n
    df = float(np.max(np.abs(ref["forces"] - g[prefix + "forces_f64"])))
    dw = float(np.max(np.abs(ref["virial"].reshape(-1) - g[prefix + "virial_f64"].reshape(-1))))
    print(variant, n, "native vs reference float64:", de, df, dw)
    assert de < 1e-9 and df < 1e-8 and dw < 1e-7, (de, df, dw)


@pytest.mark.parametrize("variant,fixture,prefix", CASES)
def test_engine_matches_native_reference(variant, fixture, prefix, tmp_path):
    model, g, pos, cell, types, native = _setup(variant, fixture, prefix, tmp_path)
    ref = native.compute(types, pos, cell)
    native.close()
    n = len(pos)
    out = model.evaluate(torch.as_tensor(pos, device="cuda"), np.asarray(cell).reshape(1, 9),
                         np.ones((1, 3), bool), torch.as_tensor(types, device="cuda"))
    de = abs(float(out["energy"][0]) - ref["energy"]) / n
    dei = float(np.max(np.abs(out["energies"].double().cpu().numpy() - ref["energies"])))
    df = float(np.max(np.abs(out["forces"].double().cpu().numpy() - ref["forces"])))
    dw = float(np.max(np.abs(out["virial"][0].double().cpu().numpy() -
                             ref["virial"].reshape(-1))))
    print(variant, n, "engine vs native:", dict(energy_per_atom=de, atom_energy=dei, forces=df,
                                               virial=dw, virial_per_atom=dw / n))
    assert de < 1e-6 and df < 1e-5 and dw / n < 1e-5, (de, df, dw)
