"""Generate the golden fixtures in this directory by running the RUNE reference itself.

Run in a container that holds the reference checkout (read-only is fine)::

    python tests/golden/make_golden.py --reference /path/to/Rune

The reference imports ``ase.data`` (and ``ase.geometry`` for its training neighbour builder); the
tiny stand-in under ``_ase_shim/`` supplies both, so the reference PyTorch models import and run
on CPU. Every fixture stores its inputs, the model parameters it used (random-init models) or the
checkpoint name (repository weights), and the reference outputs:

* ``*_f64``: the reference model cast to float64, fed float64 positions and exact float64
  periodic offsets ``S @ cell``. This is the ground truth the fp32 engine is measured against.
* ``*_f32``: the reference model in float32, fed float32 positions and offsets exactly as the
  reference ``BatchBuilder`` does (``interface/batch.py``). This is the fp32 reference result.

Neighbour pair sets come from the reference's own builder ``rune/datasets/neighbor.py`` and are
stored as integer (i, j, S) triples so the engine's neighbour kernel can be checked bit-exactly.
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SEED = 20261201


def _setup(reference: Path):
    sys.path.insert(0, str(HERE / "_ase_shim"))
    sys.path.insert(0, str(reference))
    import torch  # noqa: F401

    torch.set_num_threads(8)


# --------------------------------------------------------------------------- structures
def diamond_si(n, a=5.43, jitter=0.05, seed=SEED):
    basis = np.array(
        [[0, 0, 0], [0, .5, .5], [.5, 0, .5], [.5, .5, 0],
         [.25, .25, .25], [.25, .75, .75], [.75, .25, .75], [.75, .75, .25]]
    )
    return _lattice(basis, ["Si"] * 8, n, a, jitter, seed)


def rocksalt_mgo(n, a=4.21, jitter=0.08, seed=SEED):
    basis = np.array(
        [[0, 0, 0], [0, .5, .5], [.5, 0, .5], [.5, .5, 0],
         [.5, 0, 0], [0, .5, 0], [0, 0, .5], [.5, .5, .5]]
    )
    return _lattice(basis, ["Mg"] * 4 + ["O"] * 4, n, a, jitter, seed)


def fcc_alloy(n, a=3.6, jitter=0.1, n_species=3, seed=SEED):
    basis = np.array([[0, 0, 0], [0, .5, .5], [.5, 0, .5], [.5, .5, 0]])
    pos, cell, _ = _lattice(basis, ["X"] * 4, n, a, jitter, seed)
    rng = np.random.default_rng(seed + 1)
    types = rng.integers(0, n_species, size=len(pos))
    return pos, cell, types


def _lattice(basis, symbols, n, a, jitter, seed):
    rng = np.random.default_rng(seed)
    grid = np.stack(np.meshgrid(*(np.arange(n),) * 3, indexing="ij"), -1).reshape(-1, 3)
    frac = (grid[:, None, :] + basis[None]).reshape(-1, 3) / n
    cell = np.eye(3) * a * n
    pos = frac @ cell + rng.normal(0.0, jitter, size=(len(frac), 3))
    sym = [symbols[k % len(symbols)] for k in range(len(frac))]
    return pos, cell, sym


def random_cells(count, elements, seed=SEED, n_min=8, n_max=64, v_min=12.0, v_max=20.0,
                 d_min=1.7):
    """Independent periodic cubic structures (BASELINE config 3 recipe)."""
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(count):
        n = int(rng.integers(n_min, n_max + 1))
        length = (n * rng.uniform(v_min, v_max)) ** (1.0 / 3.0)
        cell = np.eye(3) * length
        pos = []
        while len(pos) < n:
            p = rng.uniform(0, length, size=3)
            ok = True
            for q in pos:
                d = p - q
                d -= length * np.round(d / length)
                if d @ d < d_min * d_min:
                    ok = False
                    break
            if ok:
                pos.append(p)
        types = rng.integers(0, len(elements), size=n)
        out.append((np.array(pos), cell, types))
    return out


# --------------------------------------------------------------------------- batches
def reference_pairs(pos, cell, pbc, rc_r, rc_a):
    """(i, j, S) triples for the radial and angular lists from ``datasets/neighbor.py``."""
    from rune.datasets.neighbor import build_neighbor_list

    rn, ro, an, ao = build_neighbor_list(pos, cell, pbc, rc_r, rc_a, 4096, 4096)
    inv = np.linalg.inv(cell)
    out = {}
    for name, nb, off in (("radial", rn, ro), ("angular", an, ao)):
        i, slot = np.nonzero(nb >= 0)
        j = nb[i, slot]
        s = np.rint(off[i, slot].astype(np.float64) @ inv).astype(np.int64)
        key = np.lexsort((s[:, 2], s[:, 1], s[:, 0], j, i))
        out[name] = np.concatenate([i[key, None], j[key, None], s[key]], axis=1)
    return out


def padded_batch(pos, cell, types, pairs, dtype):
    """Padded reference batch from (i, j, S) triples, offsets = S @ cell."""
    import torch

    n = len(pos)
    batch = {
        "types": torch.as_tensor(np.asarray(types), dtype=torch.long),
        "positions": torch.as_tensor(np.asarray(pos, np.float64), dtype=dtype),
        "n_atoms_per_structure": torch.tensor([n]),
    }
    for name in ("radial", "angular"):
        p = pairs[name]
        counts = np.bincount(p[:, 0], minlength=n)
        width = max(1, int(counts.max()) if len(p) else 1)
        nb = np.full((n, width), -1, np.int64)
        off = np.zeros((n, width, 3), np.float64)
        starts = np.cumsum(counts) - counts
        slot = np.arange(len(p)) - np.repeat(starts, counts)
        nb[p[:, 0], slot] = p[:, 1]
        off[p[:, 0], slot] = p[:, 2:5].astype(np.float64) @ cell
        batch[f"{name}_neighbors"] = torch.as_tensor(nb)
        batch[f"{name}_offsets"] = torch.as_tensor(off, dtype=dtype)
    return batch


def concat_batches(batches):
    import torch

    out = {}
    offset = 0
    parts = {k: [] for k in batches[0]}
    for b in batches:
        for k, v in b.items():
            if k.endswith("_neighbors"):
                v = v.clone()
                v[v >= 0] += offset
            parts[k].append(v)
        offset += len(b["types"])
    for k, v in parts.items():
        if k.endswith("_neighbors") or k.endswith("_offsets"):
            width = max(x.shape[1] for x in v)
            padded = []
            for x in v:
                pad = width - x.shape[1]
                if pad:
                    fill = -1 if k.endswith("_neighbors") else 0
                    shape = (x.shape[0], pad) + tuple(x.shape[2:])
                    x = torch.cat([x, torch.full(shape, fill, dtype=x.dtype)], 1)
                padded.append(x)
            v = padded
        out[k] = torch.cat(v, 0)
    return out


def run_model(model, batch):
    out = model({**batch, "compute_forces": True, "compute_virial": True})
    return {k: out[k].detach().cpu().numpy().astype(np.float64)
            for k in ("energies", "energy", "forces", "virial")}


def both_precisions(model_f64_factory, pos, cell, types, pairs):
    import torch

    out = {}
    m64 = model_f64_factory(torch.float64).eval()
    for k, v in run_model(m64, padded_batch(pos, cell, types, pairs, torch.float64)).items():
        out[f"{k}_f64"] = v
    m32 = model_f64_factory(torch.float32).eval()
    for k, v in run_model(m32, padded_batch(pos, cell, types, pairs, torch.float32)).items():
        out[f"{k}_f32"] = v
    return out


def state_arrays(model):
    return {f"param:{k}": v.detach().cpu().numpy() for k, v in model.state_dict().items()}


# --------------------------------------------------------------------------- fixtures
def make_basis(reference: Path):
    import torch
    from rune.mobius.descriptor import AngularDescriptor
    from rune.mobius.force import _angular_basis_derivative, _angular_weight

    rng = np.random.default_rng(SEED)
    u = rng.normal(size=(64, 3))
    u /= np.linalg.norm(u, axis=1, keepdims=True)
    desc = AngularDescriptor(2, 3, 4, 5.0, 8, 1, 1, 1, 1, 1, 1).double()
    ut = torch.tensor(u)
    basis = desc._compute_basis(ut, None).numpy()
    grad = _angular_basis_derivative(ut[:, 0], ut[:, 1], ut[:, 2],
                                     desc.basis_derivative_exponents,
                                     desc.basis_derivative_coefficients.double()).numpy()
    # invariants and their moment gradient with every higher-order term enabled, l_max=4
    desc4 = AngularDescriptor(2, 3, 4, 5.0, 4, 1, 1, 1, 1, 1, 1).double()
    moments = torch.tensor(rng.normal(size=(6, 3, 24)))
    q = desc4._compute_q(moments).numpy()

    class _D:
        pass

    d = _D()
    d.angular = desc4
    d.radial = _D()
    d.radial.n_desc = 2
    dq = torch.tensor(rng.normal(size=(6, 2 + 3 * desc4.num_L)))
    weight = _angular_weight(d, dq, moments).numpy()
    np.savez_compressed(HERE / "angular_basis.npz", unit=u, basis=basis, basis_grad=grad,
                        moments=moments.numpy(), q=q, dq=dq.numpy(), weight=weight)


def nep_params():
    from rune.nep.plugin import resolve_params

    return resolve_params(dict(
        elements=["Cu", "Ag", "Au"], rcut_radial=6.0, rcut_angular=4.0,
        n_max_radial=4, n_max_angular=4, basis_size_radial=8, basis_size_angular=8,
        l_max=4, l_max_4body=2, l_max_5body=1, hidden_dims=[30],
        max_neighbors_radial=200, max_neighbors_angular=100))


def make_nep():
    import torch
    from rune.nep.model import NEP

    params = nep_params()
    torch.manual_seed(SEED)
    model = NEP(params)
    state = state_arrays(model)
    pos, cell, types = fcc_alloy(3)
    pairs = reference_pairs(pos, cell, [True] * 3, params["rcut_radial"], params["rcut_angular"])

    def factory(dtype):
        m = NEP(params).to(dtype)
        m.load_state_dict(model.state_dict())
        return m

    out = both_precisions(factory, pos, cell, types, pairs)
    np.savez_compressed(
        HERE / "nep_fcc108.npz", positions=pos, cell=cell, pbc=np.ones(3, bool), types=types,
        radial_pairs=pairs["radial"], angular_pairs=pairs["angular"],
        params=np.array(repr(params)), **state, **out)


def tiny_params(mode, **changes):
    """The reference GPUMD-test model recipe (tests/test_mobius_gpumd.py:model_for)."""
    from rune.mobius.plugin import resolve_params

    config = dict(elements=["Fe", "C"], hidden_dim=8, ffn_dim=12, blocks=1,
                  message_layers=0 if mode == "local" else 2, message_dim=8,
                  message_groups=2, pair_dim=3, vector_channels=2,
                  message_basis_size=3, rcut_radial=3.8, rcut_angular=3.5,
                  n_max_radial=1, n_max_angular=1, basis_size_radial=2, basis_size_angular=2,
                  l_max=4, l_max_4body=2, l_max_5body=1,
                  has_q_112=1, has_q_123=1, has_q_233=1, has_q_134=1,
                  max_neighbors_radial=128, max_neighbors_angular=128)
    if mode == "equivariant":
        config.update(message_mode="equivariant", equivariant_channels=3, equivariant_l_max=4)
    config.update(changes)
    return resolve_params(config)


TINY_CASES = {
    "local": ("local", {}),
    "scalar": ("scalar", {}),
    "equivariant": ("equivariant", {}),
    "local_gelu": ("local", dict(activation="gelu")),
    "local_tanh_wide": ("local", dict(hidden_dim=36, ffn_dim=53, blocks=2, activation="tanh")),
    "scalar_v0": ("scalar", dict(vector_channels=0)),
    "scalar_tail": ("scalar", dict(hidden_dim=36, ffn_dim=53, message_dim=15,
                                   message_groups=3, blocks=2)),
    "equivariant_tail": ("equivariant", dict(hidden_dim=36, ffn_dim=53, message_dim=15,
                                             message_groups=3, blocks=2)),
    "equivariant_zbl_ra": ("equivariant", dict(rcut_radial=3.0, rcut_angular=4.2,
                                               zbl=[0.8, 2.8], equivariant_l_max=2)),
    "equivariant_flexzbl": ("equivariant", dict(zbl=dict(
        rc_inner=0.0, rc_outer=0.0, flexible=True,
        parameters=[[.5, 2.8, .18175, 3.1998, .50986, .94229, .28022, .4029, .02817, .20162]]
        * 3))),
    "local_order1": ("local", dict(l_max=1, l_max_4body=0, has_q_112=0, has_q_123=0,
                                   has_q_233=0, has_q_134=0)),
    "local_order8": ("local", dict(l_max=8)),
    "local_channels5": ("local", dict(n_max_radial=4, n_max_angular=4, basis_size_radial=20,
                                      basis_size_angular=18)),
    # radial channels and basis group boundaries (tests/test_mobius_gpumd.py:245-253)
    **{f"local_channels{c}": ("local", dict(n_max_radial=c - 1, n_max_angular=c - 1,
                                            basis_size_radial=20, basis_size_angular=18))
       for c in (2, 3, 17, 33)},
    # descriptor derivatives across angular orders (tests/test_mobius_gpumd.py:234-243)
    **{f"equivariant_order{o}": ("equivariant", dict(
        l_max=o, equivariant_l_max=min(o, 3), l_max_4body=2 if o >= 2 else 0,
        has_q_112=int(o >= 2), has_q_123=int(o >= 3), has_q_233=int(o >= 3),
        has_q_134=int(o >= 4))) for o in (1, 2, 6, 8)},
}


def small_triclinic():
    """The reference tests' 4-atom triclinic Fe/C cell (tests/test_mobius_gpumd.py)."""
    cell = np.array([[4.1, .1, .2], [.0, 4.3, .1], [.1, .0, 4.5]])
    frac = np.array([[.10, .13, .22], [.82, .21, .37], [.30, .75, .19], [.68, .63, .81]])
    return frac @ cell, cell, np.array([0, 1, 0, 1])


def large_cell():
    pos = np.array([[.2, .3, .4], [19.2, .6, .4], [2., 1., .7], [8., 7., 9.], [9.8, 7.2, 8.1],
                    [14., 14., 14.]])
    cell = np.array([[20., .2, .4], [0., 20.5, .3], [.2, 0., 21.]])
    return pos, cell, np.array([0, 1, 0, 1, 0, 1])


def make_tiny(names=None):
    import torch
    from rune.mobius.model import Mobius

    systems = {"tri": small_triclinic(), "large": large_cell()}
    for name, (mode, changes) in TINY_CASES.items():
        if names and name not in names:
            continue
        params = tiny_params(mode, **changes)
        torch.manual_seed(20261021)
        model = Mobius(params).double()
        model.set_descriptor_scaler(
            torch.linspace(.7, 1.2, model.input_dim, dtype=torch.float64))
        # perturb RMSNorm weights and biases away from their init so they are exercised
        with torch.no_grad():
            gen = torch.Generator().manual_seed(SEED)
            for key, value in model.named_parameters():
                if key.endswith("norm.weight") or key.endswith(".bias"):
                    value.add_(0.1 * torch.randn(value.shape, generator=gen,
                                                 dtype=value.dtype))
        state = state_arrays(model)
        arrays = {}
        for sname, (pos, cell, types) in systems.items():
            if name not in ("local", "scalar", "equivariant") and sname != "tri":
                continue
            pairs = reference_pairs(pos, cell, [True] * 3, params["rcut_radial"],
                                    params["rcut_angular"])

            def factory(dtype):
                m = Mobius(params).to(dtype)
                m.load_state_dict(model.state_dict())
                return m

            res = both_precisions(factory, pos, cell, types, pairs)
            arrays.update({f"{sname}:{k}": v for k, v in res.items()})
            arrays[f"{sname}:positions"] = pos
            arrays[f"{sname}:cell"] = cell
            arrays[f"{sname}:types"] = types
            arrays[f"{sname}:radial_pairs"] = pairs["radial"]
            arrays[f"{sname}:angular_pairs"] = pairs["angular"]
        np.savez_compressed(HERE / f"tiny_{name}.npz", params=np.array(repr(params)),
                            **state, **arrays)


def load_reference_model(reference: Path, variant: str):
    from rune.mobius.plugin import load_model

    return load_model(reference / "models" / f"mobius-oam-{variant}" / "model.pt")


def make_oam(reference: Path):
    from rune.mobius.plugin import load_model  # noqa: F401

    elements = None
    cases = {
        "loc": [("si216", diamond_si(3))],
        "mp": [("si64", diamond_si(2))],
        "eq": [("mgo64", rocksalt_mgo(2)), ("si64", diamond_si(2))],
    }
    for variant, systems in cases.items():
        base = load_reference_model(reference, variant)
        elements = base.elements
        arrays = {}
        for sname, (pos, cell, sym) in systems:
            types = np.array([elements.index(s) for s in sym])
            pairs = reference_pairs(pos, cell, [True] * 3, 6.0, 5.0)
            res = both_precisions(lambda dt: load_reference_model(reference, variant).to(dt),
                                  pos, cell, types, pairs)
            arrays.update({f"{sname}:{k}": v for k, v in res.items()})
            arrays[f"{sname}:positions"] = pos
            arrays[f"{sname}:cell"] = cell
            arrays[f"{sname}:types"] = types
            arrays[f"{sname}:radial_pairs"] = pairs["radial"]
            arrays[f"{sname}:angular_pairs"] = pairs["angular"]
        if variant == "mp":
            # a batch of independent random structures (config 3 recipe, 3 structures)
            structures = random_cells(3, elements, seed=SEED, n_max=24)
            import torch

            b64, b32 = [], []
            for k, (pos, cell, types) in enumerate(structures):
                pairs = reference_pairs(pos, cell, [True] * 3, 6.0, 5.0)
                b64.append(padded_batch(pos, cell, types, pairs, torch.float64))
                b32.append(padded_batch(pos, cell, types, pairs, torch.float32))
                arrays[f"batch{k}:positions"] = pos
                arrays[f"batch{k}:cell"] = cell
                arrays[f"batch{k}:types"] = types
                arrays[f"batch{k}:radial_pairs"] = pairs["radial"]
                arrays[f"batch{k}:angular_pairs"] = pairs["angular"]
            for tag, batches, cast in (("f64", b64, "double"), ("f32", b32, "float")):
                model = getattr(load_reference_model(reference, variant), cast)().eval()
                res = run_model(model, concat_batches(batches))
                arrays.update({f"batch:{k}_{tag}": v for k, v in res.items()})
        np.savez_compressed(HERE / f"oam_{variant}.npz", **arrays)


def make_neighbors():
    """Pair sets from the reference training builder for awkward cells."""
    arrays = {}
    cases = {
        "tri_small": small_triclinic()[:2] + ([True, True, True], 3.8, 3.5),
        "tri_mixed": small_triclinic()[:2] + ([True, False, True], 3.8, 3.5),
        "large": large_cell()[:2] + ([True, True, True], 3.8, 3.5),
        "unwrapped": (np.array([[1., 1., 1.], [64.7, 1., 1.], [8., 8., 8.], [-55.8, 8., 8.]]),
                      np.eye(3) * 20.9, [True, True, True], 6.0, 5.0),
        "si64": diamond_si(2)[:2] + ([True, True, True], 6.0, 5.0),
        "tiny_cell": (np.array([[0.1, 0.2, 0.3], [1.4, 1.1, 0.9]]),
                      np.array([[2.6, 0.0, 0.0], [0.3, 2.5, 0.0], [0.2, 0.4, 2.7]]),
                      [True, True, True], 6.0, 5.0),
    }
    for name, (pos, cell, pbc, rc_r, rc_a) in cases.items():
        pairs = reference_pairs(pos, cell, pbc, rc_r, rc_a)
        arrays[f"{name}:positions"] = pos
        arrays[f"{name}:cell"] = cell
        arrays[f"{name}:pbc"] = np.array(pbc)
        arrays[f"{name}:cutoffs"] = np.array([rc_r, rc_a])
        arrays[f"{name}:radial_pairs"] = pairs["radial"]
        arrays[f"{name}:angular_pairs"] = pairs["angular"]
    np.savez_compressed(HERE / "neighbors.npz", **arrays)


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", type=Path, required=True)
    parser.add_argument("--only", nargs="*", default=None)
    parser.add_argument("--tiny", nargs="*", default=None, help="tiny cases to (re)generate")
    args = parser.parse_args()
    _setup(args.reference)
    jobs = {
        "basis": lambda: make_basis(args.reference),
        "neighbors": make_neighbors,
        "nep": make_nep,
        "tiny": lambda: make_tiny(args.tiny),
        "oam": lambda: make_oam(args.reference),
    }
    for name, job in jobs.items():
        if args.only and name not in args.only:
            continue
        print("generating", name, flush=True)
        job()


if __name__ == "__main__":
    main()
