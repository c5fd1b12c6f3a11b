"""Golden fixtures at BASELINE configuration sizes, made by running the RUNE reference itself.

Run in a container that holds the reference checkout (read-only is fine)::

    python tests/golden/make_configs.py --reference /path/to/Rune [--only nep mp eq]

Inputs are the benchmark's own seeded workloads (``bench.py``: ``fcc_alloy``, ``random_cells``,
``rocksalt_mgo``); the reference's PyTorch models (``rune.nep.model.NEP``,
``rune.mobius.plugin.load_model`` on the repository checkpoints), cast to float64 and fed exact
float64 offsets ``S @ cell``, give the expected outputs. The reference's training neighbour
builder (``rune/datasets/neighbor.py``) is O(N^2) in memory, so at these sizes the pair lists
come from ``oracle/neighbors.py``, the O(N) cell list whose pair sets the neighbour fixtures
pin bit for bit to that builder.

* ``config2_nep_fcc32k.npz``: BASELINE config 2 in full, NEP4 (seeded initialisation), FCC
  ternary 20x20x20 (32,000 atoms); float64 and float32 reference outputs.
* ``config3_mp_slice256.npz``: the first 256 structures of the config-3 batch (OAM-MP weights);
  float64 and float32 reference outputs.
* ``config4_eq_mgo1728.npz``: OAM-EQ on rocksalt MgO 6x6x6 (1,728 atoms) of the config-4
  lattice and jitter; float64 and float32 reference outputs.
"""

from __future__ import annotations

import argparse
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]


def _setup(reference: Path):
    sys.path.insert(0, str(HERE / "_ase_shim"))
    sys.path.insert(0, str(reference))
    sys.path.insert(0, str(HERE))
    sys.path.insert(0, str(ROOT))
    import torch

    torch.set_num_threads(8)


def _pairs(pos, cell, rc_r, rc_a):
    from oracle.neighbors import neighbor_pairs

    radial, angular = neighbor_pairs(pos, cell, [True] * 3, (rc_r, rc_a))
    return {"radial": radial, "angular": angular}


def _run(model, pos, cell, types, pairs, dtype):
    from make_golden import padded_batch, run_model

    return run_model(model.to(dtype).eval(), padded_batch(pos, cell, types, pairs, dtype))


def make_nep():
    import torch
    from bench import NEP_CONFIG, SEED, fcc_alloy
    from rune.nep.model import NEP
    from rune.nep.plugin import resolve_params

    params = resolve_params(dict(NEP_CONFIG))
    pos, cell, types = fcc_alloy()
    pairs = _pairs(pos, cell, params["rcut_radial"], params["rcut_angular"])
    arrays = dict(positions=pos, cell=cell, types=types, seed=np.array(SEED),
                  params=np.array(repr(params)),
                  n_radial_pairs=np.array(len(pairs["radial"])),
                  n_angular_pairs=np.array(len(pairs["angular"])))
    for tag, dtype in (("f64", torch.float64), ("f32", torch.float32)):
        torch.manual_seed(SEED)
        model = NEP(params)
        out = _run(model, pos, cell, types, pairs, dtype)
        arrays.update({f"{k}_{tag}": v for k, v in out.items()})
    np.savez_compressed(HERE / "config2_nep_fcc32k.npz", **arrays)


def make_mp(reference: Path):
    import torch
    from bench import random_cells
    from make_golden import concat_batches, padded_batch, run_model
    from rune.mobius.plugin import load_model

    count = 256
    pos, cells, types, sizes = random_cells(4096, 89)
    n = int(sum(sizes[:count]))
    arrays = dict(positions=pos[:n], cells=cells[:count], types=types[:n],
                  sizes=np.array(sizes[:count]))
    for tag, dtype in (("f64", torch.float64), ("f32", torch.float32)):
        model = load_model(reference / "models" / "mobius-oam-mp" / "model.pt").to(dtype).eval()
        batches = []
        start = 0
        for s in range(count):
            p, c = pos[start:start + sizes[s]], cells[s].reshape(3, 3)
            t = types[start:start + sizes[s]]
            pairs = _pairs(p, c, 6.0, 5.0)
            batches.append(padded_batch(p, c, t, pairs, dtype))
            start += sizes[s]
        out = run_model(model, concat_batches(batches))
        arrays.update({f"{k}_{tag}": v for k, v in out.items()})
    np.savez_compressed(HERE / "config3_mp_slice256.npz", **arrays)


def make_eq(reference: Path):
    import torch
    from bench import rocksalt_mgo
    from rune.mobius.plugin import load_model

    pos, cell = rocksalt_mgo(6)
    model = load_model(reference / "models" / "mobius-oam-eq" / "model.pt")
    elements = model.elements
    types = np.array([elements.index(s) for s in (["Mg"] * 4 + ["O"] * 4) * (len(pos) // 8)])
    pairs = _pairs(pos, cell, 6.0, 5.0)
    arrays = dict(positions=pos, cell=cell, types=types)
    for tag, dtype in (("f64", torch.float64), ("f32", torch.float32)):
        path = reference / "models" / "mobius-oam-eq" / "model.pt"
        out = _run(load_model(path), pos, cell, types, pairs, dtype)
        arrays.update({f"{k}_{tag}": v for k, v in out.items()})
    np.savez_compressed(HERE / "config4_eq_mgo1728.npz", **arrays)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, required=True)
    ap.add_argument("--only", nargs="*", default=None)
    args = ap.parse_args()
    _setup(args.reference)
    jobs = {"nep": make_nep, "mp": lambda: make_mp(args.reference),
            "eq": lambda: make_eq(args.reference)}
    for name, job in jobs.items():
        if args.only and name not in args.only:
            continue
        t0 = time.time()
        print("generating", name, flush=True)
        job()
        print(f"  {name}: {time.time() - t0:.1f} s", flush=True)


if __name__ == "__main__":
    main()
