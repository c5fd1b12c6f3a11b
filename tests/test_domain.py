"""Spatial domain decomposition (rune_b200.domain, rune_engine_compute_domain).

CPU: the partition's invariants (every atom owned once; every neighbour that a shell's atoms
need is present one shell further out, at the right image position), the grid choice, and the
whole evaluator (partition + scatter + reduction) with a pair potential that follows the
engine's domain contract, against the same potential on the periodic structure, on one rank
and on two gloo ranks. GPU: the engine's domain call, for every model family, against its
periodic evaluation of the same structure (the two differ only in summation order)."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from rune_b200.domain import DomainEvaluator, domain_grid, partition, shell_radii

from .helpers import GOLDEN, load_params, load_state


def _structure(n=180, seed=5, cell=None, dmin=1.6):
    """Random atoms in a triclinic cell with a minimum pair distance (periodic)."""
    rng = np.random.default_rng(seed)
    if cell is None:
        cell = np.array([[11.0, 0.0, 0.0], [2.1, 10.5, 0.0], [-1.3, 1.7, 12.0]])
    inv = np.linalg.inv(cell)
    pos = []
    while len(pos) < n:
        x = rng.random(3) @ cell
        ok = True
        for p in pos:
            d = x - p
            d = d - np.round(d @ inv) @ cell
            if d @ d < dmin * dmin:
                ok = False
                break
        if ok:
            pos.append(x)
    pos = np.array(pos) + rng.normal(0.0, 3.0, size=(1, 3))  # not wrapped into the cell
    types = rng.integers(0, 2, size=n)
    return pos, cell, types


@pytest.mark.parametrize("grid", [(2, 1, 1), (2, 2, 2), (1, 3, 2)])
def test_partition_owns_every_atom_once_and_nests_shells(grid):
    pos, cell, _ = _structure()
    radii = [3.0, 6.0, 9.5]
    pos_t = torch.as_tensor(pos)
    owners = np.zeros(len(pos), int)
    for d in np.ndindex(*grid):
        loc = partition(pos_t, cell, [True] * 3, grid, d, radii)
        atoms = loc.atoms.numpy()
        owners[atoms[:loc.n_owned]] += 1
        assert len(loc.shell_end) == len(radii) + 1 and loc.shell_end[-1] == len(atoms)
        assert list(loc.shell_end) == sorted(loc.shell_end)
        x = loc.positions.numpy() + loc.origin
        # every local atom is an image of its global atom
        frac = (x - pos[atoms]) @ np.linalg.inv(cell)
        np.testing.assert_allclose(frac, np.round(frac), atol=1e-9)
        # neighbours within the shell width of atoms in shells <= k are local, in shells <= k + 1
        shell = np.searchsorted(loc.shell_end, np.arange(len(atoms)), side="right")
        for k, w in ((0, 3.0), (1, 3.0), (2, 3.5)):
            inner = np.nonzero(shell <= k)[0]
            for a in inner:
                d = x - x[a]
                # candidates: every image of every atom near x[a]
                for j in range(len(pos)):
                    base = pos[j] - x[a]
                    f = base @ np.linalg.inv(cell)
                    for s in np.ndindex(3, 3, 3):
                        v = base + (np.round(-f) + np.array(s) - 1) @ cell
                        r = np.linalg.norm(v)
                        if r >= w or r < 1e-9:
                            continue
                        match = np.nonzero((atoms == j) &
                                           (np.linalg.norm(d - v, axis=1) < 1e-8))[0]
                        assert len(match) == 1, (d, j, v)
                        assert shell[match[0]] <= k + 1
            if k == 0:
                break  # the full check on the owned shell; deeper shells below, sampled
        # sampled check of the deeper shells
        rng = np.random.default_rng(1)
        for k, w in ((1, 3.0), (2, 3.5)):
            inner = np.nonzero(shell == k)[0]
            for a in rng.choice(inner, size=min(5, len(inner)), replace=False):
                d = x - x[a]
                for j in range(len(pos)):
                    base = pos[j] - x[a]
                    f = base @ np.linalg.inv(cell)
                    for s in np.ndindex(3, 3, 3):
                        v = base + (np.round(-f) + np.array(s) - 1) @ cell
                        r = np.linalg.norm(v)
                        if r >= w or r < 1e-9:
                            continue
                        match = np.nonzero((atoms == j) &
                                           (np.linalg.norm(d - v, axis=1) < 1e-8))[0]
                        assert len(match) == 1 and shell[match[0]] <= k + 1
    np.testing.assert_array_equal(owners, 1)


def test_domain_grid_and_shell_radii():
    assert domain_grid(1) == (1, 1, 1)
    assert domain_grid(2) == (2, 1, 1)
    assert domain_grid(4) == (2, 2, 1)
    assert domain_grid(8) == (2, 2, 2)
    assert domain_grid(4, np.diag([10.0, 10.0, 40.0])) == (1, 1, 4)
    assert domain_grid(6, np.diag([20.0, 30.0, 10.0])) == (2, 3, 1)
    eq = dict(rcut_radial=6.0, rcut_angular=5.0, message_layers=2)
    assert shell_radii(eq, "mobius") == [6.0, 12.0, 18.0]
    assert shell_radii(dict(rcut_radial=3.0, rcut_angular=4.2, message_layers=2),
                       "mobius") == [3.0, 6.0, 10.2]
    assert shell_radii(dict(rcut_radial=6.0, rcut_angular=4.0), "nep") == [6.0]
    with pytest.raises(ValueError):
        partition(torch.zeros(2, 3, dtype=torch.float64), np.zeros((3, 3)), [True] * 3,
                  (1, 1, 1), (0, 0, 0), [3.0])


# ----------------------------------------------------------------------------- pair model
RC = 3.4


def _phi(r, a):
    """Smooth pair energy (eV) with a cutoff at RC."""
    x = torch.clamp(1.0 - r / RC, min=0.0)
    return a * x ** 3 * (1.0 + 2.0 * r)


def _pair_strength(ti, tj):
    return 0.3 + 0.2 * (ti + tj).double()


class _PairEngine:
    """The engine's domain contract for a pair potential E = sum over owned centres i of
    1/2 sum_j phi(r_ij): energy of owned atoms, its derivatives on every local atom, virial
    W = -sum over edges of g (x) r for the edges of owned centres."""

    device = torch.device("cpu")

    def compute_domain(self, types, positions, shell_end, cell, *, forces=True, virial=True):
        n_owned = int(shell_end[0])
        x = positions.clone().requires_grad_(True)
        t = torch.as_tensor(types)
        d = x[None, :, :] - x[:, None, :]                 # d[i, j] = x_j - x_i
        r = torch.sqrt((d * d).sum(-1) + torch.eye(len(x), dtype=x.dtype) * 1e6)
        mask = (r < RC) & (torch.arange(len(x))[:, None] < n_owned)
        e_pair = 0.5 * _phi(r, _pair_strength(t[:, None], t[None, :])) * mask
        energies = e_pair.sum(1)
        energy = energies.sum()
        g_r, = torch.autograd.grad(energy, r, retain_graph=True)
        grad, = torch.autograd.grad(energy, x)
        unit = d / r[..., None]
        g = (g_r * mask)[..., None] * unit               # dE / d(r_ij vector)
        w = -(g[..., :, None] * d[..., None, :]).sum((0, 1)).reshape(1, 9)
        return {"energy": energy.detach().reshape(1), "energies": energies.detach().float(),
                "forces": (-grad).float(), "virial": w.detach()}


class _PairModel:
    family = "nep"
    params = {"rcut_radial": RC, "rcut_angular": 2.0}

    def __init__(self):
        self._engine = _PairEngine()

    def engine(self):
        return self._engine


def _periodic_pair(pos, cell, types):
    """The pair potential on the periodic structure (brute force over images)."""
    x = torch.as_tensor(pos).clone().requires_grad_(True)
    t = torch.as_tensor(types)
    cell_t = torch.as_tensor(cell)
    energies = torch.zeros(len(pos), dtype=torch.float64)
    w = torch.zeros(9, dtype=torch.float64)
    terms = []
    for s in np.ndindex(5, 5, 5):
        shift = (torch.as_tensor(np.array(s) - 2.0)) @ cell_t
        d = x[None, :, :] + shift - x[:, None, :]
        home = not any(v != 2 for v in s)
        eye = torch.eye(len(pos), dtype=torch.float64)
        r = torch.sqrt((d * d).sum(-1) + (eye * 1e6 if home else 0.0))
        mask = r < RC
        e_pair = 0.5 * _phi(r, _pair_strength(t[:, None], t[None, :])) * mask
        terms.append((e_pair, r, d, mask))
        energies = energies + e_pair.sum(1)
    energy = energies.sum()
    grads = torch.autograd.grad(energy, [x] + [term[1] for term in terms])
    for (e_pair, r, d, mask), g_r in zip(terms, grads[1:]):
        g = (g_r * mask)[..., None] * d / r[..., None]
        w = w - (g[..., :, None] * d[..., None, :]).sum((0, 1)).reshape(9)
    return {"energy": energy.detach(), "energies": energies.detach(), "forces": -grads[0],
            "virial": w.detach()}


def _check_pair(got, ref):
    assert abs(float(got["energy"]) - float(ref["energy"])) < 1e-9
    np.testing.assert_allclose(got["energies"].numpy(), ref["energies"].numpy(), atol=1e-6)
    np.testing.assert_allclose(got["forces"].numpy(), ref["forces"].numpy(), atol=1e-5)
    np.testing.assert_allclose(got["virial"].numpy(), ref["virial"].numpy(), atol=1e-6)


@pytest.mark.parametrize("grid", [(1, 1, 1), (2, 1, 2), (2, 2, 2)])
def test_pair_model_domains_match_periodic(grid):
    pos, cell, types = _structure(n=120, seed=9)
    ref = _periodic_pair(pos, cell, types)
    got = DomainEvaluator(_PairModel(), grid=grid).evaluate(pos, cell, [True] * 3, types)
    _check_pair(got, ref)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        pos, cell, types = _structure(n=120, seed=9)
        ev = DomainEvaluator(_PairModel(), n_domains=4)
        assert ev.domains(cell) == [d for k, d in enumerate(np.ndindex(*domain_grid(4, cell)))
                                    if k % world == rank]
        got = ev.evaluate(pos, cell, [True] * 3, types)
        _check_pair(got, _periodic_pair(pos, cell, types))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(180)
def test_two_gloo_ranks_reduce_domains():
    mp.start_processes(_rank_main, args=(2, _free_port()), nprocs=2, join=True,
                       start_method="spawn")


# ----------------------------------------------------------------------------- engine (GPU)
DEV = "cuda"


def _model(name):
    g = np.load(GOLDEN / f"{name}.npz")
    params = load_params(g)
    if name.startswith("nep"):
        from rune_b200.nep.plugin import build_model
    else:
        from rune_b200.mobius.plugin import build_model
    model = build_model(params)
    model.load_state_dict({k: torch.as_tensor(v, dtype=torch.float32)
                           for k, v in load_state(g).items()}, strict=True)
    return model.to(DEV).eval()


def _fe_c(n=400, seed=3):
    """Fe / C atoms in a triclinic cell sized for the tiny models' 3.8 A cutoffs."""
    cell = np.array([[15.5, 0.0, 0.0], [1.2, 14.8, 0.0], [-0.9, 1.1, 16.0]])
    return _structure(n=n, seed=seed, cell=cell, dmin=1.5)


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["tiny_local", "tiny_scalar", "tiny_equivariant",
                                  "tiny_equivariant_zbl_ra", "tiny_equivariant_flexzbl",
                                  "tiny_equivariant_tail", "nep_fcc108"])
@pytest.mark.parametrize("grid", [(2, 1, 1), (2, 2, 2)])
def test_engine_domains_match_periodic(name, grid):
    model = _model(name)
    if name.startswith("nep"):
        # FCC 5x5x5 (a = 3.6 A, 500 atoms) with jitter, sheared into a triclinic cell
        rng = np.random.default_rng(4)
        basis = np.array([[0, 0, 0], [0, .5, .5], [.5, 0, .5], [.5, .5, 0]])
        grid_ = np.stack(np.meshgrid(*(np.arange(5),) * 3, indexing="ij"), -1).reshape(-1, 3)
        frac = ((grid_[:, None, :] + basis[None]).reshape(-1, 3)) / 5.0
        cell = np.array([[18.0, 0.0, 0.0], [0.9, 18.0, 0.0], [-0.6, 0.7, 18.0]])
        pos = frac @ cell + rng.normal(0.0, 0.1, size=(len(frac), 3))
        types = rng.integers(0, len(model.params["elements"]), size=len(pos))
    else:
        pos, cell, types = _fe_c()
    n = len(pos)
    ref = model.evaluate(torch.as_tensor(pos, device=DEV), cell.reshape(1, 9),
                         np.ones((1, 3), bool), torch.as_tensor(types, dtype=torch.int32,
                                                                 device=DEV))
    ev = DomainEvaluator(model, grid=grid)
    got = ev.evaluate(pos, cell, [True] * 3, types)
    torch.cuda.synchronize()
    assert abs(float(got["energy"]) - float(ref["energy"][0])) < 1e-6 * n
    np.testing.assert_allclose(got["energies"].cpu().numpy(),
                               ref["energies"].double().cpu().numpy(), atol=2e-6)
    np.testing.assert_allclose(got["forces"].cpu().numpy(),
                               ref["forces"].double().cpu().numpy(), atol=1e-5)
    np.testing.assert_allclose(got["virial"].cpu().numpy(),
                               ref["virial"][0].cpu().numpy(), atol=1e-5 * n)
    # layer prefixes: the local systems hold every shell
    radii = shell_radii(model.params, model.family)
    for loc in ev.last_locals:
        assert len(loc.shell_end) == len(radii) + 1
        assert loc.n_owned > 0 and loc.shell_end[-1] > loc.n_owned


@pytest.mark.gpu
def test_engine_domain_call_errors_and_energy_only():
    model = _model("tiny_equivariant")
    pos, cell, types = _fe_c(n=200)
    eng = model.engine()
    loc = partition(torch.as_tensor(pos, device=DEV), cell, [True] * 3, (2, 1, 1), (0, 0, 0),
                    shell_radii(model.params, "mobius"))
    typ = torch.as_tensor(types, dtype=torch.int32, device=DEV)[loc.atoms]
    with pytest.raises(ValueError, match="ghost shells"):
        eng.compute_domain(typ, loc.positions, loc.shell_end[:-1], loc.cell)
    bad = list(loc.shell_end)
    bad[-1] += 1
    with pytest.raises(ValueError, match="shell_end"):
        eng.compute_domain(typ, loc.positions, bad, loc.cell)
    full = eng.compute_domain(typ, loc.positions, loc.shell_end, loc.cell)
    e_only = eng.compute_domain(typ, loc.positions, loc.shell_end, loc.cell, forces=False,
                                virial=False)
    torch.cuda.synchronize()
    assert float(e_only["energy"][0]) == float(full["energy"][0])
    assert torch.all(full["energies"][loc.n_owned:] == 0)


# ----------------------------------------------------------------------------- halo exchange
class _HaloToyEngine:
    """The halo contract (rune_engine_compute_halo) for a model with one exchanged node state:
    h_i = sum_j phi(r_ij) over owned centres, then E = sum over owned i of
    0.4 h_i^2 + sum_j psi(r_ij) h_j, whose h_j of ghosts come from their owners (FILL), and
    whose adjoint dE/dh of ghost rows goes back to the owners (REDUCE) before the h stage's
    backward. Energies of owned atoms; forces on every local atom; virial of this rank's part
    (sum_i F_i (x) x_i, translation invariant per stage)."""

    device = torch.device("cpu")

    def compute_halo(self, types, positions, n_owned, cell, hook, *, forces=True,
                     virial=True):
        from rune_b200.runtime import library as L

        x = positions.clone().requires_grad_(True)
        t = torch.as_tensor(types)
        n = len(x)
        d = x[None, :, :] - x[:, None, :]
        r = torch.sqrt((d * d).sum(-1) + torch.eye(n, dtype=x.dtype) * 1e6)
        own = torch.arange(n) < n_owned
        m = (r < RC) & own[:, None]
        h_own = (_phi(r, _pair_strength(t[:, None], t[None, :])) * m).sum(1)[:n_owned]
        rows = torch.zeros(n, 1, dtype=torch.float32)
        rows[:n_owned, 0] = h_own.detach().float()
        hook(L.RUNE_HALO_FILL, rows)
        hf = rows[:, 0].double().clone().requires_grad_(True)
        e = 0.4 * hf ** 2 * own + (_phi(r, 0.7) * m * hf[None, :]).sum(1)
        energy = e.sum()
        g_h, g_x = torch.autograd.grad(energy, [hf, x], retain_graph=True)
        drows = g_h.float()[:, None].clone()
        hook(L.RUNE_HALO_REDUCE, drows)
        g_x2, = torch.autograd.grad(h_own, x, grad_outputs=drows[:n_owned, 0].double())
        f = -(g_x + g_x2)
        w = (f[:, :, None] * x.detach()[:, None, :]).sum(0).reshape(1, 9)
        return {"energy": energy.detach().reshape(1), "energies": e.detach().float(),
                "forces": f.float(), "virial": w}


class _HaloToyModel:
    family = "mobius"
    params = {"rcut_radial": RC, "rcut_angular": 2.0}

    def __init__(self):
        self._engine = _HaloToyEngine()

    def engine(self):
        return self._engine


def _periodic_toy(pos, cell, types):
    x = torch.as_tensor(pos).clone().requires_grad_(True)
    t = torch.as_tensor(types)
    cell_t = torch.as_tensor(cell)
    n = len(pos)
    terms = []
    for s in np.ndindex(5, 5, 5):
        shift = (torch.as_tensor(np.array(s) - 2.0)) @ cell_t
        d = x[None, :, :] + shift - x[:, None, :]
        home = not any(v != 2 for v in s)
        r = torch.sqrt((d * d).sum(-1) + (torch.eye(n, dtype=torch.float64) * 1e6 if home
                                          else 0.0))
        terms.append((d, r, r < RC))
    h = sum((_phi(r, _pair_strength(t[:, None], t[None, :])) * m).sum(1) for d, r, m in terms)
    e = 0.4 * h ** 2 + sum((_phi(r, 0.7) * m * h[None, :]).sum(1) for d, r, m in terms)
    energy = e.sum()
    grads = torch.autograd.grad(energy, [x] + [r for d, r, m in terms])
    w = torch.zeros(9, dtype=torch.float64)
    for (d, r, m), g_r in zip(terms, grads[1:]):
        g = (g_r * m)[..., None] * d / r[..., None]
        w = w - (g[..., :, None] * d[..., None, :]).sum((0, 1)).reshape(9)
    return {"energy": energy.detach(), "energies": e.detach(), "forces": -grads[0],
            "virial": w.detach()}


def _check_halo(got, ref):
    from rune_b200.domain import HaloEvaluator  # noqa: F401  (import path exercised)

    assert abs(float(got["energy"]) - float(ref["energy"])) < 1e-5, (got["energy"],
                                                                      ref["energy"])
    np.testing.assert_allclose(got["energies_all"].numpy(), ref["energies"].numpy(),
                               atol=2e-5)
    np.testing.assert_allclose(got["forces_all"].numpy(), ref["forces"].numpy(), atol=1e-4)
    np.testing.assert_allclose(got["virial"].numpy(), ref["virial"].numpy(), atol=1e-4)
    owned = got["owned"].numpy()
    np.testing.assert_allclose(got["forces"].double().numpy(), ref["forces"].numpy()[owned],
                               atol=1e-4)


def test_halo_one_rank_matches_periodic():
    """One domain: every ghost is a periodic image of an owned atom (owner = this rank)."""
    from rune_b200.domain import HaloEvaluator

    pos, cell, types = _structure(n=120, seed=9)
    got = HaloEvaluator(_HaloToyModel()).evaluate(pos, cell, [True] * 3, types, gather=True)
    _check_halo(got, _periodic_toy(pos, cell, types))


def test_halo_plan_fill_and_reduce_one_rank():
    """FILL copies owners into ghosts; REDUCE adds every ghost copy into its owner once (an
    owner with several images receives them all) and zeroes the ghosts."""
    from rune_b200.domain import HaloPlan

    atoms = torch.tensor([3, 0, 2, 0, 3, 3, 2])  # owned 3, 0, 2; ghosts: images of 0, 3, 3, 2
    owner = torch.zeros(4, dtype=torch.int64)
    plan = HaloPlan(atoms, 3, owner, 4)
    rows = torch.tensor([[1.0], [2.0], [3.0], [9.0], [9.0], [9.0], [9.0]])
    plan.fill(rows)
    np.testing.assert_array_equal(rows[:, 0].numpy(), [1, 2, 3, 2, 1, 1, 3])
    g = torch.tensor([[1.0], [10.0], [100.0], [1000.0], [2e4], [3e4], [4e5]])
    plan.reduce(g)
    np.testing.assert_array_equal(g[:, 0].numpy(), [1 + 2e4 + 3e4, 10 + 1000, 100 + 4e5,
                                                    0, 0, 0, 0])


def _halo_rank_main(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from rune_b200.domain import HaloEvaluator

        pos, cell, types = _structure(n=160, seed=4,
                                      cell=np.array([[14.0, 0.0, 0.0], [1.5, 13.0, 0.0],
                                                     [-1.0, 1.2, 12.5]]))
        got = HaloEvaluator(_HaloToyModel()).evaluate(pos, cell, [True] * 3, types,
                                                      gather=True)
        _check_halo(got, _periodic_toy(pos, cell, types))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
@pytest.mark.parametrize("world", [2, 4])
def test_halo_gloo_ranks_match_periodic(world):
    mp.start_processes(_halo_rank_main, args=(world, _free_port()), nprocs=world, join=True,
                       start_method="spawn")


# ----------------------------------------------------------------------------- halo (GPU)
def _check_engine_halo(got, ref, n):
    assert abs(float(got["energy"]) - float(ref["energy"][0])) < 1e-6 * n
    np.testing.assert_allclose(got["energies_all"].cpu().numpy(),
                               ref["energies"].double().cpu().numpy(), atol=2e-6)
    np.testing.assert_allclose(got["forces_all"].cpu().numpy(),
                               ref["forces"].double().cpu().numpy(), atol=1e-5)
    np.testing.assert_allclose(got["virial"].cpu().numpy(),
                               ref["virial"][0].cpu().numpy(), atol=1e-5 * n)


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["tiny_local", "tiny_equivariant", "tiny_equivariant_zbl_ra",
                                  "tiny_equivariant_tail"])
def test_engine_halo_one_domain_matches_periodic(name):
    """rune_engine_compute_halo with one domain: the ghosts are periodic images of owned atoms,
    so every exchange is this rank's own (FILL, REDUCE) and the result must equal the
    periodic evaluation."""
    from rune_b200.domain import HaloEvaluator

    model = _model(name)
    pos, cell, types = _fe_c()
    n = len(pos)
    ref = model.evaluate(torch.as_tensor(pos, device=DEV), cell.reshape(1, 9),
                         np.ones((1, 3), bool), torch.as_tensor(types, dtype=torch.int32,
                                                                 device=DEV))
    ev = HaloEvaluator(model)
    for _ in range(2):  # the second call reuses the rehearsed sizes
        got = ev.evaluate(pos, cell, [True] * 3, types, gather=True)
        torch.cuda.synchronize()
        _check_engine_halo(got, ref, n)
    assert ev.last_local.n_owned == n and ev.last_local.shell_end[-1] > n


@pytest.mark.gpu
def test_engine_halo_oam_eq_mgo_matches_periodic():
    """The repository EQ checkpoint on rocksalt MgO 4x4x4 (512 atoms), one domain."""
    from rune_b200.domain import HaloEvaluator
    from rune_b200.mobius.plugin import load_model
    from tests.helpers import WEIGHTS

    path = WEIGHTS / "mobius-oam-eq.pt"
    if not path.exists():
        pytest.skip("mobius-oam-eq.pt not present")
    model = load_model(path, device=DEV).eval()
    import bench

    pos, cell = bench.rocksalt_mgo(4)
    el = model.params["elements"]
    types = np.array([el.index(s) for s in (["Mg"] * 4 + ["O"] * 4) * (len(pos) // 8)])
    n = len(pos)
    ref = model.evaluate(torch.as_tensor(pos, device=DEV), cell.reshape(1, 9),
                         np.ones((1, 3), bool), torch.as_tensor(types, dtype=torch.int32,
                                                                 device=DEV))
    got = HaloEvaluator(model).evaluate(pos, cell, [True] * 3, types, gather=True)
    torch.cuda.synchronize()
    _check_engine_halo(got, ref, n)


def _engine_halo_rank(rank, world, port, name):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    from datetime import timedelta

    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from rune_b200.domain import HaloEvaluator

        global DEV
        DEV = f"cuda:{rank}"
        model = _model(name)
        pos, cell, types = _fe_c(n=500)
        n = len(pos)
        ref = model.evaluate(torch.as_tensor(pos, device=DEV), cell.reshape(1, 9),
                             np.ones((1, 3), bool),
                             torch.as_tensor(types, dtype=torch.int32, device=DEV))
        ev = HaloEvaluator(model)
        for _ in range(2):
            got = ev.evaluate(pos, cell, [True] * 3, types, gather=True)
            torch.cuda.synchronize()
            _check_engine_halo(got, ref, n)
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.timeout(600)
@pytest.mark.parametrize("name", ["tiny_equivariant", "tiny_local"])
def test_engine_halo_two_gpus_match_periodic(name):
    """Two ranks on two GPUs, NCCL exchanges: each rank owns half of the structure."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    mp.start_processes(_engine_halo_rank, args=(2, _free_port(), name), nprocs=2, join=True,
                       start_method="spawn")
