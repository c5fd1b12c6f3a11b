"""Benchmark: atoms/s for energy + forces + virial on B200, one JSON line on rank 0.

Default workload (``--config eq-halo``): BASELINE config 4's lattice and model, strong-scaled:
OAM-EQ (repository weights) on a periodic rocksalt MgO 36x36x36 supercell (373,248 atoms,
a = 4.21 A, positions jittered by N(0, 0.08 A)), the largest box of that lattice whose EQ
evaluation fits one GPU undivided. On N GPUs (torchrun) every rank owns one spatial domain and
the engine exchanges the ghost rows of each layer's node and direction states with NCCL
all-to-all (``rune_b200.domain.HaloEvaluator``); one GPU evaluates the whole box as one domain.
The total work is fixed ("scaling": "strong"); value = atoms / the slowest rank's time. The
1M-atom config-4 box itself is ``--eq-halo-cells 50`` (four GPUs or more).

``--config nep``: BASELINE config 2 — NEP4, random-init from a seed (the reference's own
initialisation for ``torch.manual_seed(20261201)``), 3 species, rc 6/4 A, n_max 4/4, basis
8/8, l_max 4/2/1, 30 hidden neurons; periodic FCC ternary alloy 20x20x20 cells (32,000 atoms,
a = 3.6 A), species uniform at random, positions jittered by N(0, 0.1 A). A step is one full
evaluation on the device: neighbour list + descriptor + network + analytic forces and virial.
Inputs are resident in HBM; L2 is flushed (a 256 MiB write) between timed steps, outside the
timed events. ``--config local|mp|eq|eq-domains|md``: configs 1, 3, 4 (one domain, or fixed
domains with redundant ghost shells) and 5.

Multi-GPU for the other configs (torchrun): a single structure (configs 1, 2, 4 lattice) runs
as independent replicas ("replicas only", weak scaling); a batch of independent structures
(``--config mp``) is split across the ranks by ``rune_b200.sharding`` (greedy by edge count, no
exchange in the step, strong scaling).

``--impl reference`` times the reference's own CPU implementation of the path (its PyTorch
``NEP.forward`` / ``Mobius.forward``, float32, installed under baseline/_ref) on all host cores;
without that install it falls back to the float64 numpy oracle. ``cpu_baseline`` of the engine
line times the oracle port in one process. ``--impl native`` times the reference's FP64 GPU
evaluator (Möbius configs).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import tempfile
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
SEED = 20261201
NEP_CONFIG = dict(elements=["Cu", "Ag", "Au"], rcut_radial=6.0, rcut_angular=4.0,
                  n_max_radial=4, n_max_angular=4, basis_size_radial=8, basis_size_angular=8,
                  l_max=4, l_max_4body=2, l_max_5body=1, hidden_dims=[30],
                  max_neighbors_radial=200, max_neighbors_angular=100)
METRIC = "atoms/s energy+force+virial"
MD_METRIC = "atom-steps/s (NVE, energy+force each step)"


# --------------------------------------------------------------------------- workload
def fcc_alloy(n_cells=20, a=3.6, jitter=0.1, n_species=3, seed=SEED):
    basis = np.array([[0, 0, 0], [0, .5, .5], [.5, 0, .5], [.5, .5, 0]])
    rng = np.random.default_rng(seed)
    grid = np.stack(np.meshgrid(*(np.arange(n_cells),) * 3, indexing="ij"), -1).reshape(-1, 3)
    frac = (grid[:, None, :] + basis[None]).reshape(-1, 3) / n_cells
    cell = np.eye(3) * a * n_cells
    pos = frac @ cell + rng.normal(0.0, jitter, size=(len(frac), 3))
    types = np.random.default_rng(seed + 1).integers(0, n_species, size=len(pos))
    return pos, cell, types


def diamond_si(n, a=5.43, jitter=0.05, seed=SEED):
    basis = np.array([[0, 0, 0], [0, .5, .5], [.5, 0, .5], [.5, .5, 0],
                      [.25, .25, .25], [.25, .75, .75], [.75, .25, .75], [.75, .75, .25]])
    return _lattice(basis, n, a, jitter, seed)


def rocksalt_mgo(n, a=4.21, jitter=0.08, seed=SEED):
    basis = np.array([[0, 0, 0], [0, .5, .5], [.5, 0, .5], [.5, .5, 0],
                      [.5, 0, 0], [0, .5, 0], [0, 0, .5], [.5, .5, .5]])
    return _lattice(basis, n, a, jitter, seed)


def _lattice(basis, n, a, jitter, seed):
    rng = np.random.default_rng(seed)
    grid = np.stack(np.meshgrid(*(np.arange(n),) * 3, indexing="ij"), -1).reshape(-1, 3)
    frac = (grid[:, None, :] + basis[None]).reshape(-1, 3) / n
    cell = np.eye(3) * a * n
    pos = frac @ cell + rng.normal(0.0, jitter, size=(len(frac), 3))
    return pos, cell


def random_cells(count, n_types, seed=SEED, n_min=8, n_max=64, v_min=12.0, v_max=20.0,
                 d_min=1.7):
    """independent cubic cells, 8-64 atoms, 12-20 A^3/atom, species uniform,
    positions uniform with rejection below d_min."""
    rng = np.random.default_rng(seed)
    pos_all, cells, types, sizes = [], [], [], []
    for _ in range(count):
        n = int(rng.integers(n_min, n_max + 1))
        length = (n * rng.uniform(v_min, v_max)) ** (1.0 / 3.0)
        acc = np.zeros((0, 3))
        while len(acc) < n:
            p = rng.uniform(0, length, size=(32, 3))
            for q in p:
                if len(acc) >= n:
                    break
                d = acc - q
                d -= length * np.round(d / length)
                if len(acc) == 0 or np.min(np.einsum("ij,ij->i", d, d)) >= d_min * d_min:
                    acc = np.vstack([acc, q])
        pos_all.append(acc)
        cells.append(np.eye(3).reshape(9) * length)
        types.append(rng.integers(0, n_types, size=n))
        sizes.append(n)
    return np.concatenate(pos_all), np.stack(cells), np.concatenate(types), sizes


def workload(name, args=None):
    """Positions, cells, pbc, types and structure sizes of a BASELINE configuration."""
    if name == "nep":
        pos, cell, types = fcc_alloy()
        return dict(name="nep-fcc-ternary-20x20x20", family="nep", positions=pos,
                    cells=cell.reshape(1, 9), pbc=np.ones((1, 3), bool), types=types,
                    sizes=[len(pos)])
    if name == "local":  # config 1: Si diamond 3x3x3, OAM Local weights
        pos, cell = diamond_si(3)
        return dict(name="mobius-local-si-diamond-3x3x3", family="mobius", weights="loc",
                    positions=pos, cells=cell.reshape(1, 9), pbc=np.ones((1, 3), bool),
                    symbols=["Si"] * len(pos), sizes=[len(pos)])
    if name == "mp":  # config 3: 4,096 independent random cells, OAM MP weights
        count = args.structures if args is not None else 4096
        pos, cells, types, sizes = random_cells(count, 89)
        return dict(name=f"mobius-mp-random-cells-x{count}", family="mobius", weights="mp",
                    positions=pos, cells=cells, pbc=np.ones((len(sizes), 3), bool), types=types,
                    sizes=sizes)
    if name == "eq":  # config 4 lattice: rocksalt MgO n x n x n, OAM EQ weights
        n = args.eq_cells if args is not None else 20
        pos, cell = rocksalt_mgo(n)
        symbols = (["Mg"] * 4 + ["O"] * 4) * (len(pos) // 8)
        return dict(name=f"mobius-eq-mgo-rocksalt-{n}x{n}x{n}", family="mobius", weights="eq",
                    positions=pos, cells=cell.reshape(1, 9), pbc=np.ones((1, 3), bool),
                    symbols=symbols, sizes=[len(pos)])
    if name == "eq-domains":  # config 4: rocksalt MgO 50 x 50 x 50 (1M atoms), OAM EQ weights
        n = args.eq_domain_cells if args is not None else 50
        pos, cell = rocksalt_mgo(n)
        symbols = (["Mg"] * 4 + ["O"] * 4) * (len(pos) // 8)
        return dict(name=f"mobius-eq-mgo-rocksalt-{n}x{n}x{n}", family="mobius", weights="eq",
                    positions=pos, cells=cell.reshape(1, 9), pbc=np.ones((1, 3), bool),
                    symbols=symbols, sizes=[len(pos)])
    if name == "eq-halo":  # config 4 lattice, one domain per rank with halo exchange
        n = args.eq_halo_cells if args is not None else 36
        pos, cell = rocksalt_mgo(n)
        symbols = (["Mg"] * 4 + ["O"] * 4) * (len(pos) // 8)
        return dict(name=f"mobius-eq-mgo-rocksalt-{n}x{n}x{n}", family="mobius", weights="eq",
                    positions=pos, cells=cell.reshape(1, 9), pbc=np.ones((1, 3), bool),
                    symbols=symbols, sizes=[len(pos)])
    if name == "md":  # config 5: EQ NVE, diamond Si n x n x n, Maxwell-Boltzmann 1000 K
        n = args.md_cells if args is not None else 30
        pos, cell = diamond_si(n)
        return dict(name=f"mobius-eq-nve-si-diamond-{n}x{n}x{n}", family="mobius", weights="eq",
                    positions=pos, cells=cell.reshape(1, 9), pbc=np.ones((1, 3), bool),
                    symbols=["Si"] * len(pos), sizes=[len(pos)])
    raise SystemExit(f"unknown config {name}")


def workload_name(args):
    """Name of the workload ``workload(args.config, args)`` builds, without building it."""
    c = args.config
    if c == "nep":
        return "nep-fcc-ternary-20x20x20"
    if c == "local":
        return "mobius-local-si-diamond-3x3x3"
    if c == "mp":
        return f"mobius-mp-random-cells-x{args.structures}"
    if c in ("eq", "eq-domains", "eq-halo"):
        n = {"eq": args.eq_cells, "eq-domains": args.eq_domain_cells,
             "eq-halo": args.eq_halo_cells}[c]
        return f"mobius-eq-mgo-rocksalt-{n}x{n}x{n}"
    if c == "md":
        return f"mobius-eq-nve-si-diamond-{args.md_cells}x{args.md_cells}x{args.md_cells}"
    raise SystemExit(f"unknown config {c}")


def build_engine_model(wl, dev):
    import torch

    sys.path.insert(0, str(ROOT))
    if wl["family"] == "nep":
        from rune_b200.nep.plugin import build_model

        torch.manual_seed(SEED)
        return build_model(nep_params()).to(dev).eval(), nep_params()
    from rune_b200.mobius.plugin import load_model

    path = ROOT / "weights" / f"mobius-oam-{wl['weights']}.pt"
    if not path.exists():
        raise SystemExit(f"{path} missing: run __graft_entry__.build() where the reference "
                         "checkout is available")
    model = load_model(path, device=dev).eval()
    if "symbols" in wl:
        elements = model.params["elements"]
        wl["types"] = np.array([elements.index(x) for x in wl["symbols"]])
    return model, model.params


def nep_params():
    sys.path.insert(0, str(ROOT))
    from rune_b200.nep.plugin import resolve_params

    return resolve_params(dict(NEP_CONFIG))


# --------------------------------------------------------------------------- distributed
def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def init_dist(world, local):
    import torch
    import torch.distributed as dist

    if world > 1:
        from datetime import timedelta

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return dist


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples (every 20 ms, host timestamps) kept for the timed window."""
    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.path = Path(tempfile.gettempdir()) / f"rune_b200_clocks_{os.getpid()}_{gpu_index}.csv"

    def start(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "20"],
                stdout=self.fh, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self, t0, t1):
        """Summary of the samples taken between host times t0 and t1 (time.time()); when the
        window is shorter than the sampling period, the samples nearest to it."""
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.fh.close()
        text = self.path.read_text()
        self.path.unlink(missing_ok=True)
        from datetime import datetime
        rows = []
        for line in text.splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 10:
                continue
            try:
                ts = datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                rows.append((ts, float(parts[2]), float(parts[3]), parts[6:10]))
            except ValueError:
                continue
        if not rows:
            return None
        inside = [r for r in rows if t0 <= r[0] <= t1]
        window = "timed steps"
        if not inside:
            rows.sort(key=lambda r: min(abs(r[0] - t0), abs(r[0] - t1)))
            inside = rows[:2]
            window = "nearest samples to the timed steps (window shorter than 20 ms)"
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[k] for *_, flags in inside for k, f in enumerate(flags)
                          if f.lower().startswith("active")})
        return {"sm_mhz": statistics.median(r[1] for r in inside),
                "sm_max_mhz": max(r[2] for r in inside), "reasons": reasons,
                "samples": len(inside), "window": window}


# --------------------------------------------------------------------------- roofline
def algorithmic_bytes(kernel, n_atoms, e_radial, e_angular, p):
    """Compulsory HBM bytes of one launch: every array read or written once; an edge record is
    16 B (float32 vector + int32 neighbour), a neighbour-type gather 4 B."""
    na, nr = p["n_desc_angular"], p["n_desc_radial"]
    C = p["l_max"] * (p["l_max"] + 2)
    T = len(p["elements"])
    edge = 16
    if kernel == "k_desc_forward":  # edges (angular = suffix of the radial rows), types
        return ((edge + 4) * e_radial + 4 * n_atoms  # -> q_r, moments s
                + 4 * n_atoms * (nr + na * C))
    if kernel == "k_forces":  # edges, types, contracted radial adjoint, angular gradients + rev
        kp = (p["k_max_radial"] + 3) // 4 * 4
        return ((edge + 4) * e_radial + 4 * n_atoms + 4 * n_atoms * T * kp
                + (16 + 4) * e_angular + n_atoms * (12 + 8 + 72))  # -> F, e_zbl, W_atom
    if kernel == "k_desc_backward":  # s, angular edges -> angular gradients (dq not counted)
        return n_atoms * 4 * na * C + (edge + 16) * e_angular
    if kernel == "k_nbr_build":  # binned positions -> edge records + shifts + row metadata
        return n_atoms * (24 + 32 + 4 + 16) + (16 + 4) * max(e_radial, e_angular)
    return None


def measured_peak(key="hbm_gbs"):
    """Roofline denominator: the pool's measured figure, else the earlier fallback."""
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        if key in data:
            return float(data[key]), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0,
            "bf16_tflops_sustained": 1400.0}[key], "fallback"


# Whole-model FLOPs per atom (forward + dX-only backward, the reference's mathematical form;
# 2 per multiply-add) by workload, used to express a step's arithmetic rate against the FP32
# pipes: NEP ~35 k, Local on Si ~1.2 M, MP on the config-3 cells ~3.9 M, EQ on MgO ~134 M,
# EQ on Si ~70 M.
FLOP_PER_ATOM = {"nep": 35e3, "local": 1.2e6, "mp": 3.9e6, "eq": 134e6, "eq-domains": 134e6,
                 "md": 70e6}


def fp32_peak_tflops(dev):
    """FP32 SIMT throughput measured here: cuBLAS SGEMM 8192^3 with TF32 disabled, best of 5
    (CUDA events). The pool's measured-peaks file has no FP32 entry; this is the denominator
    of the FP32 fraction."""
    import torch

    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        n = 8192
        a = torch.randn(n, n, device=dev)
        b = torch.randn(n, n, device=dev)
        c = a @ b
        best = float("inf")
        for _ in range(5):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            torch.matmul(a, b, out=c)
            e.record()
            e.synchronize()
            best = min(best, s.elapsed_time(e))
        del a, b, c
        return 2.0 * n ** 3 / (best / 1e3) / 1e12
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def fp32_fraction(config, atoms_per_s, peak):
    f = FLOP_PER_ATOM.get(config)
    if not f or not peak:
        return None
    achieved = f * atoms_per_s / 1e12
    return {"flop_per_atom": f, "achieved_tflops": achieved, "peak_tflops": peak,
            "peak_kind": "measured here (cuBLAS SGEMM, TF32 off)", "frac": achieved / peak}


def ncu_traffic():
    path = ROOT / "profiles" / "ncu_traffic.json"
    if path.exists():
        return json.loads(path.read_text())
    return {}


# --------------------------------------------------------------------------- CPU oracle
def _oracle_shard(args):
    """One worker's share: E/F/W of centres [lo, hi) from their own pairs, evaluated on the
    subsystem of those centres and their neighbours (renumbered), so the work is proportional
    to the share."""
    lo, hi, payload, radial, angular = args
    sys.path.insert(0, str(ROOT))
    from oracle import models as om

    params, state, pos, cell, types, z = payload
    atoms = np.unique(np.concatenate([np.arange(lo, hi), radial[:, 1], angular[:, 1]]))

    def local(pairs):
        out = pairs.copy()
        out[:, 0] = np.searchsorted(atoms, pairs[:, 0])
        out[:, 1] = np.searchsorted(atoms, pairs[:, 1])
        return out

    sub = pos[atoms]
    er = om.edges_from_pairs(sub, cell, local(radial))
    ea = om.edges_from_pairs(sub, cell, local(angular))
    out = om.nep_forward(params, state, types[atoms], er, ea, [len(atoms)], z)
    centres = np.searchsorted(atoms, np.arange(lo, hi))
    return out["energies"][centres].sum(), out["forces"], out["virial"]


def _oracle_warm(_):
    sys.path.insert(0, str(ROOT))
    from oracle import models  # noqa: F401  (imports outside the timed region)
    return 0


def oracle_mobius_sample(config, n_cells):
    """cpu_baseline of the Möbius configs: the float64 numpy oracle (one process) on a small
    structure of the config's lattice (MgO rocksalt for config 4, diamond Si for config 5),
    all its atoms; (atoms/s, description)."""
    sys.path.insert(0, str(ROOT))
    import torch

    from oracle import models as om
    from oracle.neighbors import neighbor_pairs

    if config == "md":
        pos, cell = diamond_si(n_cells)
        symbols = ["Si"] * len(pos)
        name = f"Si diamond {n_cells}x{n_cells}x{n_cells}"
    else:
        pos, cell = rocksalt_mgo(n_cells)
        symbols = (["Mg"] * 4 + ["O"] * 4) * (len(pos) // 8)
        name = f"MgO rocksalt {n_cells}x{n_cells}x{n_cells}"
    ckpt = torch.load(ROOT / "weights" / "mobius-oam-eq.pt", map_location="cpu",
                      weights_only=False)
    params = ckpt["model_params"]
    state = {k: v.detach().double().numpy() for k, v in ckpt["model_state_dict"].items()}
    types = np.array([params["elements"].index(x) for x in symbols])
    t0 = time.perf_counter()
    radial, angular = neighbor_pairs(pos, cell, [True] * 3,
                                     (params["rcut_radial"], params["rcut_angular"]))
    from rune_b200.elements import atomic_numbers

    z = np.array([float(atomic_numbers[e]) for e in params["elements"]])
    om.mobius_forward(params, state, types, om.edges_from_pairs(pos, cell, radial),
                      om.edges_from_pairs(pos, cell, angular), [len(pos)], z)
    dt = time.perf_counter() - t0
    return len(pos) / dt, (f"float64 numpy oracle (CPU restatement of rune/mobius, OAM-EQ), "
                           f"{name} ({len(pos)} atoms, neighbour list included), one process")


def oracle_sample(wl, n_centers, processes):
    """E/F/W of ``n_centers`` atoms (all their edges) with the float64 oracle; seconds. The
    pairs are split by centre in the parent, so each worker receives only its own rows."""
    sys.path.insert(0, str(ROOT))
    import torch

    from oracle.neighbors import neighbor_pairs
    from rune_b200.nep.plugin import build_model

    params = nep_params()
    torch.manual_seed(SEED)
    model = build_model(params)
    state = {k: v.detach().double().numpy() for k, v in model.state_dict().items()}
    z = np.array([29.0, 47.0, 79.0])
    cell = wl["cells"][0].reshape(3, 3)
    radial, angular = neighbor_pairs(wl["positions"], cell, wl["pbc"][0], (6.0, 4.0))
    payload = (params, state, wl["positions"], cell, wl["types"], z)
    bounds = np.linspace(0, n_centers, processes + 1).astype(int)
    tasks = []
    for k in range(processes):
        lo, hi = int(bounds[k]), int(bounds[k + 1])
        r = radial[(radial[:, 0] >= lo) & (radial[:, 0] < hi)]
        a = angular[(angular[:, 0] >= lo) & (angular[:, 0] < hi)]
        tasks.append((lo, hi, payload, r, a))
    if processes == 1:
        t0 = time.perf_counter()
        results = [_oracle_shard(tasks[0])]
    else:
        import multiprocessing as mp

        # one BLAS / OpenMP thread per worker process (inherited by the spawned workers)
        for var in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
            os.environ[var] = "1"
        with mp.get_context("spawn").Pool(processes) as pool:
            pool.map(_oracle_warm, range(processes))
            t0 = time.perf_counter()
            results = pool.map(_oracle_shard, tasks, chunksize=1)
    dt = time.perf_counter() - t0
    return dt, results


REFERENCE_INSTALL = ROOT / "baseline" / "_ref"
ASE_SHIM = ROOT / "tests" / "golden" / "_ase_shim"


def reference_padded_batch(pos, cell, types, radial, angular):
    """The reference model's batch dict (``rune/mobius/interface/batch.py`` layout: padded
    ``[N, M]`` neighbour rows with -1, offsets = S @ cell) from (i, j, S) pair triples, in
    float32."""
    import torch

    n = len(pos)
    batch = {"types": torch.as_tensor(np.asarray(types), dtype=torch.long),
             "positions": torch.as_tensor(np.asarray(pos, np.float64), dtype=torch.float32),
             "n_atoms_per_structure": torch.tensor([n])}
    for name, p in (("radial", radial), ("angular", angular)):
        counts = np.bincount(p[:, 0], minlength=n)
        width = max(1, int(counts.max()) if len(p) else 1)
        nb = np.full((n, width), -1, np.int64)
        off = np.zeros((n, width, 3), np.float64)
        slot = np.arange(len(p)) - np.repeat(np.cumsum(counts) - counts, counts)
        nb[p[:, 0], slot] = p[:, 1]
        off[p[:, 0], slot] = p[:, 2:5].astype(np.float64) @ cell
        batch[f"{name}_neighbors"] = torch.as_tensor(nb)
        batch[f"{name}_offsets"] = torch.as_tensor(off, dtype=torch.float32)
    return batch


def reference_batch_of_cells(pos, cells, sizes, types, rc):
    """One reference batch of independent periodic structures (``collate_fn`` form: rows of
    all structures stacked, neighbour indices global, ``n_atoms_per_structure`` = sizes)."""
    import torch

    from oracle.neighbors import neighbor_pairs

    parts, start = [], 0
    for k, n in enumerate(sizes):
        p, cell = pos[start:start + n], cells[k].reshape(3, 3)
        radial, angular = neighbor_pairs(p, cell, [True] * 3, rc)
        parts.append(reference_padded_batch(p, cell, types[start:start + n], radial, angular))
        start += n
    out, offset = {}, 0
    for b in parts:
        for name in ("radial", "angular"):
            b[f"{name}_neighbors"] = torch.where(b[f"{name}_neighbors"] >= 0,
                                                 b[f"{name}_neighbors"] + offset,
                                                 b[f"{name}_neighbors"])
        offset += len(b["types"])
    for key in parts[0]:
        vals = [b[key] for b in parts]
        if key.endswith("_neighbors") or key.endswith("_offsets"):
            width = max(v.shape[1] for v in vals)
            fill = -1 if key.endswith("_neighbors") else 0
            vals = [torch.cat([v, torch.full((v.shape[0], width - v.shape[1], *v.shape[2:]),
                                             fill, dtype=v.dtype)], 1) for v in vals]
        out[key] = torch.cat(vals, 0)
    out["n_atoms_per_structure"] = torch.tensor([int(s) for s in sizes])
    return out


def reference_sample(config):
    """Structure the reference arm evaluates per step: the config's own structure where the
    reference's CPU path handles it in seconds, else the same lattice / distribution at a
    stated smaller size (atoms/s of the reference path is size-independent at these sizes)."""
    if config == "nep":
        pos, cell, types = fcc_alloy()
        return "nep", pos, cell, types, None, "FCC ternary 20x20x20 (the whole config-2 structure)"
    if config == "local":
        pos, cell = diamond_si(3)
        return "loc", pos, cell, None, ["Si"] * len(pos), "Si diamond 3x3x3 (config 1 itself)"
    if config == "mp":
        pos, cells, types, sizes = random_cells(64, 89)
        return ("mp", pos, (cells, sizes), types, None,
                "64 structures from the config-3 batch generator (same seed and distributions)")
    if config in ("eq", "eq-domains", "eq-halo"):
        pos, cell = rocksalt_mgo(3)
        return ("eq", pos, cell, None, (["Mg"] * 4 + ["O"] * 4) * (len(pos) // 8),
                "MgO rocksalt 3x3x3 (216 atoms, config-4 lattice and jitter)")
    pos, cell = diamond_si(3)
    return ("eq", pos, cell, None, ["Si"] * len(pos),
            "Si diamond 3x3x3 (216 atoms, config-5 lattice; one force evaluation per step)")


def run_reference(args):
    """The reference's own CPU implementation of the path: ``NEP.forward`` / ``Mobius.forward``
    (PyTorch, float32, autograd forces) from the pip install under baseline/_ref, on all host
    cores. Neighbour rows come from the oracle's cell list (the reference's ``BatchBuilder``
    needs ASE, which is not installed) and are built outside the timed region."""
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    if not (REFERENCE_INSTALL / "rune").exists():
        return run_reference_port(args)
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ASE_SHIM))
    sys.path.insert(0, str(REFERENCE_INSTALL))
    import torch

    from oracle.neighbors import neighbor_pairs

    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    torch.set_num_threads(cores)
    kind, pos, cell, types, symbols, sample = reference_sample(args.config)
    if kind == "nep":
        from rune.nep.plugin import build_model, resolve_params

        params = resolve_params(dict(NEP_CONFIG))
        torch.manual_seed(SEED)
        model = build_model(params).eval()
        rc = (params["rcut_radial"], params["rcut_angular"])
    else:
        from rune.mobius.plugin import load_model

        model = load_model(str(ROOT / "weights" / f"mobius-oam-{kind}.pt"), device="cpu").eval()
        params = model.params
        rc = (params["rcut_radial"], params["rcut_angular"])
        if symbols is not None:
            types = np.array([params["elements"].index(x) for x in symbols])
    if isinstance(cell, tuple):  # independent cells: one batch over all of them
        batch = reference_batch_of_cells(pos, cell[0], cell[1], types, rc)
    else:
        radial, angular = neighbor_pairs(pos, cell, [True] * 3, rc)
        batch = reference_padded_batch(pos, cell, types, radial, angular)
    batch.update(compute_forces=True, compute_virial=True)
    n = len(pos)
    if args.steps is None:
        args.steps = 5
    times = []
    for step in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        out = model(batch)
        float(out["energy"].sum())
        dt = time.perf_counter() - t0
        if step >= args.warmup:
            times.append(dt)
    total = sum(times)
    value = n * len(times) / total
    desc = (f"reference PyTorch {type(model).__name__}.forward (baseline/_ref, float32, "
            f"autograd forces and virial), {sample}, {n} atoms per step, "
            f"torch threads = {cores}")
    metric, unit = ((MD_METRIC, "atom-steps/s") if args.config == "md" else (METRIC, "atoms/s"))
    print(json.dumps({
        "impl": "reference", "metric": metric, "value": value, "unit": unit,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * total / len(times), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": workload_name(args), "n_atoms": n,
                   "parallelism": f"cpu, {cores} torch threads"},
        "cpu_baseline": {"value": value, "unit": unit, "cores": cores,
                         "kind": "reference", "sample": desc},
        "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)
    return 0


def run_native(args):
    """The reference's native FP64 GPU evaluator (``Mobius::compute``, rune/mobius/src, built
    from the reference's own sources by oracle/native/build.sh) on the config's structure, one
    GPU: the prior-art GPU path the reference ships for GPUMD. Inputs resident on the device;
    one untimed call, then ``steps`` calls timed with CUDA events."""
    world, rank, local = dist_env()
    if rank != 0:
        return 0
    sys.path.insert(0, str(ROOT))
    from oracle import native_ref

    if not native_ref.available():
        print(json.dumps({"impl": "reference-native",
                          "unavailable": "oracle/_ref/libmobius_native_ref.so not built"}))
        return 0
    import torch

    torch.cuda.set_device(local)
    wl = workload(args.config, args)
    if wl["family"] != "mobius" or len(wl["sizes"]) != 1:
        raise SystemExit("--impl native: single-structure Möbius configs (local, eq, md)")
    from rune_b200.mobius.plugin import export_model, load_model

    model = load_model(ROOT / "weights" / f"mobius-oam-{wl['weights']}.pt", device="cpu")
    types = np.array([model.params["elements"].index(x) for x in wl["symbols"]])
    with tempfile.TemporaryDirectory() as tmp:
        path = export_model(model, Path(tmp) / "model.txt")
        native = native_ref.NativeMobius(path, len(types))
    steps = args.steps if args.steps is not None else 5
    for _ in range(max(0, args.warmup - 1)):
        native.compute(types, wl["positions"], wl["cells"][0], reps=0)
    res = native.compute(types, wl["positions"], wl["cells"][0], reps=steps)
    n = len(types)
    value = n / (res["ms"] / 1e3)
    print(json.dumps({
        "impl": "reference-native", "metric": METRIC, "value": value, "unit": "atoms/s",
        "n_gpus": 1, "steps": steps, "warmup": args.warmup, "ms_per_step": res["ms"],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
        "data": "synthetic",
        "config": {"workload": wl["name"], "n_atoms": n,
                   "parallelism": "one GPU, default stream (reference design)"},
        "energy_per_atom": float(res["energy"]) / n}), flush=True)
    return 0


def run_reference_port(args):
    """Fallback reference arm when the reference install is absent: the float64 numpy oracle
    (CPU restatement of rune/nep) on the host cores, on a bounded sample of config 2."""
    world, rank, _ = dist_env()
    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    if args.config != "nep":  # Möbius configs: the float64 Möbius oracle on a small sample
        if args.steps is None:
            args.steps = 3
        vals = []
        for step in range(args.warmup + args.steps):
            v, sample = oracle_mobius_sample("md" if args.config == "md" else "eq", 2)
            if step >= args.warmup:
                vals.append(v)
        value = len(vals) / sum(1.0 / v for v in vals)
        print(json.dumps({
            "impl": "reference", "metric": METRIC, "value": value, "unit": "atoms/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": None, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "config": {"workload": workload_name(args), "parallelism": "cpu, one process"},
            "cpu_baseline": {"value": value, "unit": "atoms/s", "cores": 1, "kind": "port",
                             "sample": sample},
            "e2e": {"value": value, "unit": "atoms/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}), flush=True)
        return 0
    wl = workload("nep")
    n_centers = min(args.reference_atoms, len(wl["types"]))
    if args.steps is None:
        args.steps = 3  # each step is a multi-second CPU sample
    times = []
    for step in range(args.warmup + args.steps):
        dt, _ = oracle_sample(wl, n_centers, cores)
        if step >= args.warmup:
            times.append(dt)
    total = sum(times)
    value = n_centers * len(times) / total
    sample = (f"float64 numpy oracle (CPU restatement of rune/nep), {n_centers} centre atoms "
              f"of the {len(wl['types'])}-atom structure per step, {cores} processes")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "atoms/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * total / len(times), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": {"workload": wl["name"], "n_atoms": int(len(wl["types"])),
                   "parallelism": "cpu processes"},
        "cpu_baseline": {"value": value, "unit": "atoms/s", "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "atoms/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)
    return 0


# --------------------------------------------------------------------------- GPU arm
def run_engine(args):
    import torch

    world, rank, local = dist_env()
    dist = init_dist(world, local)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    sys.path.insert(0, str(ROOT))
    wl = workload(args.config, args)
    model, params = build_engine_model(wl, dev)
    engine = model.engine()
    n_batch = len(wl["types"])
    sharded = world > 1 and len(wl["sizes"]) > 1
    if sharded:
        # independent structures: this rank evaluates its share, no exchange in the step
        from rune_b200.sharding import partition, select, structure_costs

        parts = partition(structure_costs(wl["sizes"], wl["cells"]), world)
        atom_idx, sub_sizes = select(wl["sizes"], parts[rank])
        wl = dict(wl, positions=wl["positions"][atom_idx], types=np.asarray(wl["types"])[atom_idx],
                  cells=wl["cells"][parts[rank]], pbc=wl["pbc"][parts[rank]],
                  sizes=[int(x) for x in sub_sizes])
    n = len(wl["types"])
    types = torch.as_tensor(wl["types"], dtype=torch.int32, device=dev)
    pos = torch.as_tensor(wl["positions"], dtype=torch.float64, device=dev)
    cells = wl["cells"]
    pbc = wl["pbc"]
    atom_ptr = np.concatenate([[0], np.cumsum(wl["sizes"])]).astype(np.int32)
    n_struct = len(wl["sizes"])
    out = engine.allocate(n, n_struct)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        engine.compute(types, pos, cells, pbc, atom_ptr, out=out)

    fp32_peak = fp32_peak_tflops(dev) if rank == 0 else None
    for _ in range(args.warmup):
        flush.fill_(1.0)
        step()
    torch.cuda.synchronize()
    stats0 = engine.stats()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)  # let the sampler start before the timed steps
    if args.steps is None:  # default: enough steps for about a second of timed work
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        step()
        e.record(stream)
        e.synchronize()
        args.steps = int(min(5000, max(20, 1000.0 / max(s.elapsed_time(e), 1e-3))))
    if world > 1:
        # every rank times the same number of steps
        k = torch.tensor([args.steps], device=dev)
        dist.all_reduce(k, op=dist.ReduceOp.MIN)
        args.steps = int(k.item())
        dist.barrier()
    torch.cuda.synchronize()
    t_begin = time.time()
    total_ms = 0.0
    for _ in range(args.steps):
        flush.fill_(float(_))
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        step()
        e.record(stream)
        e.synchronize()
        total_ms += s.elapsed_time(e)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t_end = time.time()
    clock_info = clocks.stop(t_begin, t_end)
    stats1 = engine.stats()
    launches = stats1["kernel_launches"] - stats0["kernel_launches"]

    # ---------------- per-kernel device times: a separate pass with CUDA events around every
    # launch (the events cost host time, so the timed steps above run without them)
    engine.reset_kernel_stats()
    engine.set_profiling(True)
    for _ in range(args.steps):
        flush.fill_(3.0)
        step()
    torch.cuda.synchronize()
    engine.set_profiling(False)
    kstats = engine.kernel_stats()

    # ---------------- e2e through the public API with host buffers
    pin_pos = torch.as_tensor(wl["positions"], dtype=torch.float64).pin_memory()
    pin_types = torch.as_tensor(wl["types"], dtype=torch.int32).pin_memory()
    host = {"energies": torch.empty(n, dtype=torch.float32).pin_memory(),
            "energy": torch.empty(n_struct, dtype=torch.float64).pin_memory(),
            "forces": torch.empty((n, 3), dtype=torch.float32).pin_memory(),
            "virial": torch.empty((n_struct, 9), dtype=torch.float64).pin_memory()}

    def e2e_step():
        p = pin_pos.to(dev, non_blocking=True)
        t = pin_types.to(dev, non_blocking=True)
        res = model.evaluate(p, cells, pbc, t, wl["sizes"])
        for k in host:
            host[k].copy_(res[k], non_blocking=True)

    for _ in range(max(1, args.warmup)):
        e2e_step()
    torch.cuda.synchronize()
    e2e_ms = 0.0
    for _ in range(args.steps):
        flush.fill_(2.0)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        e2e_step()
        e.record(stream)
        e.synchronize()
        e2e_ms += s.elapsed_time(e)
    h2d = n * 3 * 8 + n * 4
    d2h = n * 4 + 8 * n_struct + n * 12 + 72 * n_struct

    # ---------------- max over ranks
    times = torch.tensor([total_ms, e2e_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    total_ms, e2e_ms = times.tolist()

    if rank == 0:
        atoms_total = (n_batch if sharded else n * world) * args.steps
        value = atoms_total / (total_ms / 1e3)
        e2e_value = atoms_total / (e2e_ms / 1e3)
        e_r, e_a = stats1["last_radial_edges"], stats1["last_angular_edges"]
        top = max(kstats.items(), key=lambda kv: kv[1][0]) if kstats else None
        roof = None
        if top:
            name, (ms, count) = top
            per_launch_ms = ms / max(count, 1)
            nbytes = algorithmic_bytes(name, n, e_r, e_a, params)
            peak, peak_kind = measured_peak()
            traffic = ncu_traffic().get(name)
            if nbytes:
                achieved = nbytes / (per_launch_ms / 1e3) / 1e9
                roof = {"kernel": name, "bound": "hbm", "achieved": achieved, "peak": peak,
                        "peak_kind": peak_kind, "unit": "GB/s", "frac": achieved / peak,
                        "traffic": traffic, "algorithmic_bytes": nbytes,
                        "launch_ms": per_launch_ms}
        shares = {k: round(v[0] / max(sum(x[0] for x in kstats.values()), 1e-12), 4)
                  for k, v in sorted(kstats.items(), key=lambda kv: -kv[1][0])}
        cpu = None
        parity = None
        if world == 1 and not args.skip_cpu and wl["family"] == "nep":
            n_centers = min(args.cpu_atoms, n)
            dt, res = oracle_sample(wl, n_centers, 1)
            cpu = {"value": n_centers / dt, "unit": "atoms/s", "cores": 1, "kind": "port",
                   "sample": f"float64 numpy oracle, {n_centers} centre atoms of the "
                             f"{n}-atom structure (all their edges), one process"}
            if n_centers == n:
                # the oracle's float64 result for the whole structure against the engine's
                # last e2e outputs (same positions)
                e_ref, f_ref, w_ref = res[0]
                de = abs(float(host["energy"][0]) - float(e_ref)) / n
                df = float(np.max(np.abs(host["forces"].double().numpy() - f_ref)))
                dw = float(np.max(np.abs(host["virial"][0].numpy() - np.ravel(w_ref))))
                parity = {"vs": "float64 oracle, whole structure", "energy_eV_per_atom": de,
                          "forces_max_eV_per_A": df, "virial_max_eV": dw,
                          "virial_max_eV_per_atom": dw / n,
                          "tolerance": {"energy_eV_per_atom": 1e-6, "forces_eV_per_A": 1e-5,
                                        "virial_eV": 1e-5}}
        line = {
            "metric": METRIC, "value": value, "unit": "atoms/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_ms / args.steps,
            "higher_is_better": True, "scaling": "strong" if sharded else "weak",
            "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": wl["name"], "n_atoms": n_batch if sharded else n,
                       "radial_edges": e_r,
                       "angular_edges": e_a, "l2": "flushed (256 MiB write) between steps",
                       "parallelism": (f"structure shards x{world}" if sharded
                                       else f"replicas x{world}")},
            "e2e": {"value": e2e_value, "unit": "atoms/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "gpu_launches": int(launches),
            "roofline": roof,
            "kernel_shares": shares,
            "kernel_ms_per_step": (sum(v[0] for v in kstats.values()) / args.steps
                                   if kstats else None),
            "fp32": fp32_fraction(args.config, value / world, fp32_peak),
            "cpu_baseline": cpu,
            "parity": parity,
            "clocks": clock_info,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


# EQ message FLOPs per atom in the reference's form (forward + dX-only backward, two layers,
# MgO edge density): the fair count for the EQ edge kernels' roofline.
EQ_FLOP_PER_ATOM_MGO = 129e6
EQ_EDGE_KERNELS = ("k_eq_forward_edges", "k_eq_backward_centre", "k_eq_backward_pull")


def run_domains(args):
    """Config 4: one large MgO structure cut into spatial domains (rune_b200.domain).
    eq-domains: a fixed grid of domains with redundant ghost shells (one per message layer),
    taken round-robin by the ranks (one GPU evaluates them in sequence). eq-halo: one domain per
    rank with per-layer halo exchange over NCCL (HaloEvaluator); one GPU evaluates the whole
    structure as one domain whose ghosts are its own periodic images. Strong scaling: the
    total work is fixed."""
    import torch

    world, rank, local = dist_env()
    dist = init_dist(world, local)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    sys.path.insert(0, str(ROOT))
    from rune_b200.domain import DomainEvaluator, HaloEvaluator, domain_grid

    wl = workload(args.config, args)
    model, params = build_engine_model(wl, dev)
    engine = model.engine()
    n = len(wl["types"])
    cell = wl["cells"].reshape(3, 3)
    pbc = wl["pbc"][0]
    types = torch.as_tensor(wl["types"], dtype=torch.int32, device=dev)
    pos = torch.as_tensor(wl["positions"], dtype=torch.float64, device=dev)
    halo = args.config == "eq-halo"
    if halo:
        ev = HaloEvaluator(model)
        grid = domain_grid(world, cell)
    else:
        ev = DomainEvaluator(model, n_domains=args.domains)
        grid = ev._grid(cell)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        return ev.evaluate(pos, cell, pbc, types)

    fp32_peak = fp32_peak_tflops(dev) if rank == 0 else None
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    steps = args.steps if args.steps is not None else 3
    stats0 = engine.stats()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t_begin = time.time()
    total_ms = 0.0
    for k in range(steps):
        flush.fill_(float(k))
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        step()
        e.record(stream)
        e.synchronize()
        total_ms += s.elapsed_time(e)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clock_info = clocks.stop(t_begin, time.time())
    launches = engine.stats()["kernel_launches"] - stats0["kernel_launches"]
    locals_ = [ev.last_local] if halo else ev.last_locals
    local_atoms = [loc.shell_end[-1] for loc in locals_]
    centre_atoms = ([loc.n_owned for loc in locals_] if halo else
                    [loc.shell_end[min(1, len(loc.shell_end) - 1)] for loc in locals_])
    halo_rows = (int(ev.last_plan.recv_rows.numel()), int(ev.last_plan.send_rows.numel())) \
        if halo else None

    engine.reset_kernel_stats()
    engine.set_profiling(True)
    step()
    torch.cuda.synchronize()
    engine.set_profiling(False)
    kstats = engine.kernel_stats()

    # e2e: positions and types from pinned host memory, results back to the host
    pin_pos = torch.as_tensor(wl["positions"], dtype=torch.float64).pin_memory()
    pin_types = torch.as_tensor(wl["types"], dtype=torch.int32).pin_memory()
    n_out = locals_[0].n_owned if halo else n  # halo: this rank's owned atoms come back
    host_e = torch.empty(n_out, dtype=torch.float64).pin_memory()
    host_f = torch.empty((n_out, 3), dtype=torch.float64).pin_memory()
    host_w = torch.empty(10, dtype=torch.float64).pin_memory()
    e2e_ms = 0.0
    for k in range(steps):
        flush.fill_(2.0)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        res = ev.evaluate(pin_pos.to(dev, non_blocking=True), cell, pbc,
                          pin_types.to(dev, non_blocking=True))
        host_e.copy_(res["energies"], non_blocking=True)
        host_f.copy_(res["forces"], non_blocking=True)
        host_w[:9].copy_(res["virial"], non_blocking=True)
        host_w[9:].copy_(res["energy"].reshape(1), non_blocking=True)
        e.record(stream)
        e.synchronize()
        e2e_ms += s.elapsed_time(e)
    times = torch.tensor([total_ms, e2e_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    total_ms, e2e_ms = times.tolist()
    if rank == 0:
        value = n * steps / (total_ms / 1e3)
        cpu = None
        if world == 1 and not args.skip_cpu:
            v, sample = oracle_mobius_sample("eq", 2)  # MgO 2x2x2
            cpu = {"value": v, "unit": "atoms/s", "cores": 1, "kind": "port", "sample": sample}
        eq_ms = sum(kstats[k][0] for k in EQ_EDGE_KERNELS if k in kstats)
        roof = None
        if eq_ms > 0:
            # seconds-long steps: the sustained (power-capped) GEMM figure
            peak, peak_kind = measured_peak("bf16_tflops_sustained")
            owned = sum(loc.n_owned for loc in locals_)
            achieved = EQ_FLOP_PER_ATOM_MGO * owned / (eq_ms / 1e3) / 1e12
            # DRAM bytes of one step's forward and backward edge launches (both message layers),
            # scaled by owned centres from the ncu capture on MgO 10^3; the pull is not included
            tr = ncu_traffic()
            per_centre = [tr.get(k + "_per_centre") for k in EQ_EDGE_KERNELS[:2]]
            traffic = (2 * owned * sum(per_centre)
                       if None not in per_centre and len(EQ_EDGE_KERNELS) >= 2 else None)
            roof = {"kernel": "+".join(EQ_EDGE_KERNELS), "bound": "tensor",
                    "achieved": achieved, "peak": peak, "peak_kind": peak_kind,
                    "unit": "TFLOP/s", "frac": achieved / peak, "traffic": traffic,
                    "traffic_note": "DRAM bytes per step of k_eq_forward_edges + "
                                    "k_eq_backward_centre (2 layers), from the ncu capture on "
                                    "MgO 10^3 scaled by owned centres; the pull is not included",
                    "algorithmic_flop_per_atom": EQ_FLOP_PER_ATOM_MGO,
                    "note": "FP32 SIMT kernels; owned atoms of this rank's domain(s)"}
        shares = {k: round(v[0] / max(sum(x[0] for x in kstats.values()), 1e-12), 4)
                  for k, v in sorted(kstats.items(), key=lambda kv: -kv[1][0])}
        print(json.dumps({
            "metric": METRIC, "value": value, "unit": "atoms/s", "n_gpus": world,
            "steps": steps, "warmup": args.warmup, "ms_per_step": total_ms / steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": {"workload": wl["name"], "n_atoms": n, "domains": list(grid),
                       "domains_per_rank": len(locals_),
                       "local_atoms_rank0": local_atoms, "layer0_centres_rank0": centre_atoms,
                       "halo_ghost_rows_rank0": halo_rows[0] if halo else None,
                       "halo_sent_rows_rank0": halo_rows[1] if halo else None,
                       "l2": "inputs larger than L2; 256 MiB flush between steps",
                       "parallelism": (f"halo domains {grid[0]}x{grid[1]}x{grid[2]}, one per "
                                       f"rank, NCCL all-to-all exchanges per layer" if halo else
                                       f"spatial domains {grid[0]}x{grid[1]}x{grid[2]} over "
                                       f"{world} rank(s)")},
            "e2e": {"value": n * steps / (e2e_ms / 1e3), "unit": "atoms/s",
                    "h2d_bytes_per_step": n * 3 * 8 + n * 4,
                    "d2h_bytes_per_step": n_out * 8 + n_out * 24 + 80},
            "gpu_launches": int(launches),
            "roofline": roof,
            "kernel_shares": shares,
            "kernel_ms_per_step": sum(v[0] for v in kstats.values()),
            "fp32": fp32_fraction("eq-domains", value / world, fp32_peak),
            "cpu_baseline": cpu,
            "clocks": clock_info,
        }), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_md(args):
    """Config 5: velocity-Verlet NVE (dt 1 fs, skin 1 A), one step = one MD step; the timed
    steps run in one rune_md_nve call bracketed by CUDA events. The per-edge state of the EQ
    blocks (GBs) is far larger than L2, so no flush is needed between steps."""
    import torch

    world, rank, local = dist_env()
    dist = init_dist(world, local)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    sys.path.insert(0, str(ROOT))
    from rune_b200.md import NVE, maxwell_boltzmann

    wl = workload("md", args)
    model, params = build_engine_model(wl, dev)
    n = len(wl["types"])
    elements = model.params["elements"]
    from rune_b200.elements import atomic_masses, atomic_numbers

    masses = np.array([atomic_masses[atomic_numbers[elements[t]]] for t in wl["types"]])
    vel = maxwell_boltzmann(masses, 1000.0, seed=SEED)
    cell = wl["cells"][0].reshape(3, 3)
    md = NVE(model, wl["positions"], cell, [True] * 3, wl["types"], masses=masses,
             velocities=vel, dt=1.0, skin=1.0, device=dev)
    fp32_peak = fp32_peak_tflops(dev) if rank == 0 else None
    md.run(args.warmup)
    steps = args.steps if args.steps is not None else 5
    engine = model.engine()
    stats0 = engine.stats()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t_begin = time.time()
    stream = torch.cuda.current_stream(dev)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(stream)
    out = md.run(steps)
    e.record(stream)
    e.synchronize()
    total_ms = s.elapsed_time(e)
    t_end = time.time()
    clock_info = clocks.stop(t_begin, t_end)
    launches = engine.stats()["kernel_launches"] - stats0["kernel_launches"]
    # e2e through the public API: state from host arrays (copied in by NVE), the same number of
    # steps, final positions back to the host (energies come back inside the call)
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record(stream)
    md2 = NVE(model, wl["positions"], cell, [True] * 3, wl["types"], masses=masses,
              velocities=vel, dt=1.0, skin=1.0, device=dev)
    md2.run(steps)
    final_host = md2.positions.cpu()
    e2.record(stream)
    e2.synchronize()
    e2e_ms = s2.elapsed_time(e2)
    del final_host
    times = torch.tensor([total_ms, e2e_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    total_ms, e2e_ms = times.tolist()
    if rank == 0:
        value = n * steps * world / (total_ms / 1e3)
        cpu = None
        if world == 1 and not args.skip_cpu:
            v, sample = oracle_mobius_sample("md", 2)
            cpu = {"value": v, "unit": "atom-steps/s", "cores": 1, "kind": "port",
                   "sample": sample + "; one force evaluation per MD step"}
        tot = out["total"] / n
        drift = float(np.polyfit(np.arange(len(tot)) * 1e-3, tot, 1)[0]) if len(tot) > 2 else None
        print(json.dumps({
            "metric": MD_METRIC, "value": value,
            "unit": "atom-steps/s", "n_gpus": world, "steps": steps, "warmup": args.warmup,
            "ms_per_step": total_ms / steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": wl["name"], "n_atoms": n, "dt_fs": 1.0, "skin_A": 1.0,
                       "temperature_K": 1000.0, "rebuilds": out["rebuilds"],
                       "energy_drift_eV_per_atom_per_ps": drift,
                       "l2": "per-edge state larger than L2", "parallelism": f"replicas x{world}"},
            "e2e": {"value": n * steps * world / (e2e_ms / 1e3), "unit": "atom-steps/s",
                    "h2d_bytes_per_step": n * (24 + 24 + 8 + 4) / steps,
                    "d2h_bytes_per_step": (n * 24 + (steps + 1) * 16) / steps},
            "gpu_launches": int(launches), "roofline": None,
            "fp32": fp32_fraction("md", value / world, fp32_peak), "cpu_baseline": cpu,
            "clocks": clock_info}))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None,
                    help="timed steps (default: enough for about one second, at least 20)")
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="engine", choices=["engine", "reference", "native"],
                    help="native: the reference's FP64 GPU evaluator (Möbius configs)")
    ap.add_argument("--config", default="eq-halo",
                    help="eq-halo (default, config 4 strong scaling), nep (config 2), local, mp, "
                         "eq, eq-domains, md")
    ap.add_argument("--cpu-atoms", type=int, default=32000,
                    help="cpu_baseline: centre atoms of the one-process oracle sample "
                         "(default: the whole structure, several seconds)")
    ap.add_argument("--reference-atoms", type=int, default=32000,
                    help="reference arm: centre atoms per step (default: the whole structure)")
    ap.add_argument("--skip-cpu", action="store_true")
    ap.add_argument("--structures", type=int, default=4096, help="config mp: structure count")
    ap.add_argument("--eq-cells", type=int, default=20, help="config eq: MgO cells per axis")
    ap.add_argument("--md-cells", type=int, default=30, help="config md: Si cells per axis")
    ap.add_argument("--eq-domain-cells", type=int, default=50,
                    help="config eq-domains: MgO cells per axis")
    ap.add_argument("--domains", type=int, default=8, help="config eq-domains: domain count")
    ap.add_argument("--eq-halo-cells", type=int, default=36,
                    help="config eq-halo: MgO cells per axis (one domain per rank)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    if args.impl == "native":
        return run_native(args)
    if args.config == "md":
        return run_md(args)
    if args.config in ("eq-domains", "eq-halo"):
        return run_domains(args)
    return run_engine(args)


if __name__ == "__main__":
    sys.exit(main())
