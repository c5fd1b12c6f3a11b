"""Golden fixtures for the on-disk model formats, made by running the RUNE reference itself.

Run in a container that holds the reference checkout (read-only is fine)::

    python tests/golden/make_formats.py --reference /path/to/Rune

* ``nep_txt.npz``: GPUMD ``nep.txt`` texts written here from seeded NEP4 models (plain,
  universal ZBL, flexible ZBL, a per-type cutoff line and a short l_max line), each parsed by
  the reference's ``NEP.from_nep_txt`` (rune/nep/model.py:284-489); the fixture keeps the text,
  the parameters and tensors the reference reader produced, and the text the reference's
  ``export_model`` (rune/nep/plugin.py:84-91, ``save_nep_txt`` rune/nep/model.py:491-579)
  writes for that model.
* ``mobius1.npz``: ``mobius1`` texts exported by the reference's ``export_model``
  (rune/mobius/export.py:120-146) from small Möbius models (Local, MP, EQ with flexible ZBL),
  with the exported models' parameters and tensors.
"""

from __future__ import annotations

import argparse
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SEED = 20261201


def _setup(reference: Path):
    sys.path.insert(0, str(HERE / "_ase_shim"))
    sys.path.insert(0, str(reference))
    sys.path.insert(0, str(HERE))


def _state(model):
    return {f"param:{k}": v.detach().cpu().double().numpy() for k, v in
            model.state_dict().items()}


# --------------------------------------------------------------------------- nep.txt
def write_nep_txt(model, zbl_line=None, per_type_cutoff=False, lmax_values=None):
    """A nep.txt text holding `model` (the layout the reference reader parses)."""
    p = model.params
    elements = list(p["elements"])
    t = len(elements)
    lines = [f"nep4{'_zbl' if zbl_line else ''} {t} {' '.join(elements)}"]
    if zbl_line:
        lines.append(zbl_line)
    if per_type_cutoff:
        cut = " ".join(f"{p['rcut_radial']} {p['rcut_angular']}" for _ in range(t))
        lines.append(f"cutoff {cut} {p['max_neighbors_radial']} {p['max_neighbors_angular']}")
    else:
        lines.append(f"cutoff {p['rcut_radial']} {p['rcut_angular']} "
                     f"{p['max_neighbors_radial']} {p['max_neighbors_angular']}")
    lines.append(f"n_max {p['n_desc_radial'] - 1} {p['n_desc_angular'] - 1}")
    lines.append(f"basis_size {p['k_max_radial'] - 1} {p['k_max_angular'] - 1}")
    if lmax_values is None:
        lmax_values = [p["l_max"], 2 if p["has_q_222"] else 0, 1 if p["has_q_1111"] else 0,
                       p["has_q_112"], p["has_q_123"], p["has_q_233"], p["has_q_134"]]
    lines.append("l_max " + " ".join(str(v) for v in lmax_values))
    neurons = p["hidden_dims"][0]
    lines.append(f"ANN {neurons} 0")
    values = []
    for e in elements:
        mlp = model.element_mlps[e]
        values += mlp[0].weight.detach().reshape(-1).tolist()
        values += (-mlp[0].bias.detach()).reshape(-1).tolist()
        values += mlp[-1].weight.detach().reshape(-1).tolist()
    values.append(float(model.shared_bias.detach().reshape(-1)[0]))
    for table in (model.descriptor.radial.c_table, model.descriptor.angular.c_table):
        values += table.detach().permute(2, 3, 0, 1).reshape(-1).tolist()
    values += model.q_scaler.detach().reshape(-1).tolist()
    if zbl_line and zbl_line.split()[1:3] == ["0", "0"]:
        values += [0.5, 2.8, .18175, 3.1998, .50986, .94229, .28022, .4029, .02817, .20162] * (
            t * (t + 1) // 2)
    lines += [" ".join(f"{v:.9g}" for v in values[k:k + 10]) for k in range(0, len(values), 10)]
    return "\n".join(lines) + "\n"


NEP_CASES = {
    "plain": dict(),
    "zbl": dict(zbl_line="zbl 1.0 2.0"),
    "flexzbl": dict(zbl_line="zbl 0 0"),
    "pertype": dict(per_type_cutoff=True),
    "short_lmax": dict(lmax_values=[4, 2]),
}


def make_nep_txt():
    import torch
    from rune.nep.model import NEP
    from rune.nep.plugin import export_model as export_nep
    from rune.nep.plugin import resolve_params

    params = resolve_params(dict(
        elements=["Cu", "Ag", "Au"], rcut_radial=5.0, rcut_angular=4.0, n_max_radial=3,
        n_max_angular=2, basis_size_radial=5, basis_size_angular=4, l_max=4, l_max_4body=2,
        l_max_5body=1, hidden_dims=[7], max_neighbors_radial=90, max_neighbors_angular=40))
    arrays = {}
    for name, case in NEP_CASES.items():
        torch.manual_seed(SEED)
        model = NEP(params)
        with torch.no_grad():
            gen = torch.Generator().manual_seed(SEED + 1)
            model.q_scaler.copy_(torch.rand(model.q_scaler.shape, generator=gen) + 0.5)
            model.shared_bias.add_(0.3)
        text = write_nep_txt(model, **case)
        with tempfile.TemporaryDirectory() as tmp:
            path = Path(tmp) / "nep.txt"
            path.write_text(text)
            ref = NEP.from_nep_txt(path)
            # the reference exporter's output for the model its reader produced
            out = export_nep(ref, Path(tmp) / "model")
            arrays[f"{name}:export"] = np.array(out.read_text())
            arrays[f"{name}:export_name"] = np.array(out.name)
        arrays[f"{name}:text"] = np.array(text)
        arrays[f"{name}:params"] = np.array(repr(ref.params))
        arrays.update({f"{name}:{k}": v for k, v in _state(ref).items()})
    np.savez_compressed(HERE / "nep_txt.npz", **arrays)


# --------------------------------------------------------------------------- mobius1
MOBIUS_CASES = {
    "local": ("local", {}),
    "scalar": ("scalar", {}),
    "equivariant_flexzbl": ("equivariant", dict(zbl=dict(
        rc_inner=0.0, rc_outer=0.0, flexible=True,
        parameters=[[.5, 2.8, .18175, 3.1998, .50986, .94229, .28022, .4029, .02817, .20162]]
        * 3))),
    "scalar_zbl": ("scalar", dict(zbl=[0.8, 2.8])),
}


def make_mobius1():
    import torch
    from make_golden import tiny_params
    from rune.mobius.export import export_model
    from rune.mobius.model import Mobius

    arrays = {}
    for name, (mode, changes) in MOBIUS_CASES.items():
        params = tiny_params(mode, **changes)
        torch.manual_seed(20261021)
        model = Mobius(params)
        with torch.no_grad():
            gen = torch.Generator().manual_seed(SEED)
            for key, value in model.named_parameters():
                if key.endswith("norm.weight") or key.endswith(".bias"):
                    value.add_(0.1 * torch.randn(value.shape, generator=gen, dtype=value.dtype))
        with tempfile.TemporaryDirectory() as tmp:
            path = export_model(model, Path(tmp) / "mobius.txt")
            text = path.read_text()
        arrays[f"{name}:text"] = np.array(text)
        arrays[f"{name}:params"] = np.array(repr(model.params))
        arrays.update({f"{name}:{k}": v for k, v in _state(model).items()})
    np.savez_compressed(HERE / "mobius1.npz", **arrays)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, required=True)
    args = ap.parse_args()
    _setup(args.reference)
    make_nep_txt()
    make_mobius1()


if __name__ == "__main__":
    main()
