"""Spatial domain decomposition of one large periodic structure, one engine per GPU.

The reference evaluates a structure on one device (``Mobius.forward`` / ``NEP.forward``,
rune/mobius/model.py:307-393, rune/nep/model.py:87-170); its native evaluator leaves the
decomposition of large MD systems to GPUMD (rune/mobius/src/mobius.cu:334-402). Here a
structure too large for one GPU, or one spread over several, is cut into a grid of domains in
the cell's fractional coordinates. Each domain is evaluated as a local, non-periodic system:
its owned atoms, then ghost atoms (periodic images included) in shells by their distance from
the domain, one radial cutoff per message layer plus one descriptor cutoff
(``rune_engine_compute_domain``). The engine counts the energy of owned atoms only and returns
its derivatives with respect to every local atom, so the whole structure's forces are the sum,
over domains, of the local forces scattered to their global atoms, and the energy and virial
are sums over domains. Message layer l computes its centre kernels only over the shells whose
outputs later layers read, so the redundant work on ghosts shrinks layer by layer.

Distances to a domain are measured per axis, perpendicular to the domain's faces (the largest
over the three axes); every such distance changes by at most the length of a pair vector
between two atoms, which is what makes one cutoff per shell sufficient for triclinic cells too.

Domains go to ranks round-robin; with one rank the domains are evaluated one after another,
which bounds the device memory of a call by the largest domain. Results are reduced with one
all-reduce (float64) of [energy, virial, per-atom energies, forces].
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch


def shell_radii(params: dict, family: str) -> list[float]:
    """Outer radius of every ghost shell (A): one radial cutoff per message layer (message
    edges are the radial list's), then one max(radial, angular) cutoff for the descriptors."""
    rc_r, rc_a = float(params["rcut_radial"]), float(params["rcut_angular"])
    layers = int(params.get("message_layers", 0) or 0) if family == "mobius" else 0
    radii = [rc_r * (k + 1) for k in range(layers)]
    radii.append(rc_r * layers + max(rc_r, rc_a))
    return radii


def domain_grid(n_domains: int, cell=None) -> tuple[int, int, int]:
    """Domains per cell axis for `n_domains` (a product of three factors): the factorisation
    whose domains are closest to cubes for `cell` (the most even split when no cell is given;
    ties: more domains along earlier axes)."""
    if n_domains < 1:
        raise ValueError("the number of domains must be positive")
    lengths = np.ones(3) if cell is None else np.linalg.norm(np.asarray(cell, float).reshape(3, 3),
                                                             axis=1)
    best, best_score = None, None
    for gx in range(1, n_domains + 1):
        if n_domains % gx:
            continue
        for gy in range(1, n_domains // gx + 1):
            if (n_domains // gx) % gy:
                continue
            gz = n_domains // (gx * gy)
            side = lengths / np.array([gx, gy, gz])
            score = (float(side.max() / side.min()), -gx, -gy)
            if best_score is None or score < best_score:
                best, best_score = (gx, gy, gz), score
    return best


@dataclass
class LocalSystem:
    """One domain's local system, in the engine's order (owned atoms, then ghost shells)."""
    atoms: torch.Tensor       # int64 [n_local] global atom of every local atom
    positions: torch.Tensor   # float64 [n_local, 3] in the local frame (shifted by `origin`)
    shell_end: list           # cumulative counts, shell_end[0] = owned atoms
    cell: np.ndarray          # [9] binning box of the local frame
    origin: np.ndarray        # [3] local frame origin in the structure's frame

    @property
    def n_owned(self) -> int:
        return int(self.shell_end[0])


def _face_spacing(cell: np.ndarray) -> np.ndarray:
    """Distance between the two faces of the cell across each axis: volume / |b x c| etc."""
    vol = abs(float(np.linalg.det(cell)))
    return np.array([vol / np.linalg.norm(np.cross(cell[(k + 1) % 3], cell[(k + 2) % 3]))
                     for k in range(3)])


def wrapped_fractional(pos: torch.Tensor, cell, pbc):
    """Fractional coordinates wrapped into [0, 1) on periodic axes, and the wrapped Cartesian
    positions, of float64 `pos` [N, 3] (rows of `cell` are the cell vectors)."""
    cell_t = torch.as_tensor(np.asarray(cell, np.float64).reshape(3, 3), dtype=torch.float64,
                             device=pos.device)
    frac = pos @ torch.linalg.inv(cell_t)
    wrap = torch.zeros_like(frac)
    for k in range(3):
        if pbc[k]:
            wrap[:, k] = torch.floor(frac[:, k])
    frac = frac - wrap
    # f - floor(f) rounds to 1.0 for tiny negative f: such an atom belongs at 0
    top = frac >= 1.0
    frac = torch.where(top, frac - 1.0, frac)
    wrap = torch.where(top, wrap + 1.0, wrap)
    return frac, pos - wrap @ cell_t


def domain_owner(positions: torch.Tensor, cell, pbc, grid) -> torch.Tensor:
    """Row-major index of the domain that owns every atom (int64 [N]), by the same test as
    `partition`: lo <= wrapped fractional coordinate < hi with lo = index / grid (non-periodic
    axes: the outer domains extend to infinity)."""
    pbc = [bool(p) for p in np.asarray(pbc).reshape(3)]
    frac, _ = wrapped_fractional(positions.to(torch.float64), cell, pbc)
    idx = []
    for k in range(3):
        bounds = torch.as_tensor([m / grid[k] for m in range(1, grid[k])], dtype=torch.float64,
                                 device=positions.device)
        idx.append(torch.searchsorted(bounds, frac[:, k].contiguous(), right=True))
    return (idx[0] * grid[1] + idx[1]) * grid[2] + idx[2]


def partition(positions: torch.Tensor, cell, pbc, grid, index, radii) -> LocalSystem:
    """Local system of domain `index` (ix, iy, iz) of `grid` for a structure with float64
    `positions` [N, 3] (any device), 3x3 `cell` (rows are the cell vectors) and `pbc`.

    Owned atoms: wrapped fractional coordinates in [lo, hi) on every axis (non-periodic axes:
    the outer domains extend to infinity). Ghosts: every image (periodic axes) within the
    last shell radius of the domain that is not an owned atom itself; shell k holds distances
    up to radii[k - 1]. Order: shell, then global atom, then image."""
    dev = positions.device
    cell = np.asarray(cell, np.float64).reshape(3, 3)
    pbc = [bool(p) for p in np.asarray(pbc).reshape(3)]
    if abs(np.linalg.det(cell)) < 1e-12:
        raise ValueError("domain decomposition needs a cell with a volume")
    grid = [int(g) for g in grid]
    index = [int(i) for i in index]
    radii = [float(r) for r in radii]
    halo = radii[-1]
    h = _face_spacing(cell)
    cell_t = torch.as_tensor(cell, dtype=torch.float64, device=dev)
    pos = positions.to(torch.float64)
    frac, base = wrapped_fractional(pos, cell, pbc)
    lo = np.array([index[k] / grid[k] for k in range(3)])
    hi = np.array([(index[k] + 1) / grid[k] for k in range(3)])
    for k in range(3):
        if not pbc[k]:
            if index[k] == 0:
                lo[k] = -math.inf
            if index[k] == grid[k] - 1:
                hi[k] = math.inf
    reach = [int(math.ceil(halo / h[k])) + 1 if pbc[k] else 0 for k in range(3)]
    images = [(a, b, c) for a in range(-reach[0], reach[0] + 1)
              for b in range(-reach[1], reach[1] + 1) for c in range(-reach[2], reach[2] + 1)]
    n = pos.shape[0]
    lo_t = torch.as_tensor(lo, dtype=torch.float64, device=dev)
    hi_t = torch.as_tensor(hi, dtype=torch.float64, device=dev)
    h_t = torch.as_tensor(h, dtype=torch.float64, device=dev)
    radii_t = torch.as_tensor(radii, dtype=torch.float64, device=dev)
    atom_ids = torch.arange(n, device=dev, dtype=torch.int64)
    sel_atoms, sel_img, sel_shell = [], [], []
    for m, img in enumerate(images):
        f = frac + torch.as_tensor(img, dtype=torch.float64, device=dev)
        outside = torch.clamp(torch.maximum(lo_t - f, f - hi_t), min=0.0) * h_t
        dist = outside.max(dim=1).values
        owned = ((f >= lo_t) & (f < hi_t)).all(dim=1) if img == (0, 0, 0) else None
        keep = dist <= halo
        if owned is not None:
            keep = keep | owned
        idx = atom_ids[keep]
        if idx.numel() == 0:
            continue
        shell = torch.searchsorted(radii_t, dist[keep].contiguous(), right=False) + 1
        if owned is not None:
            shell = torch.where(owned[keep], torch.zeros_like(shell), shell)
        sel_atoms.append(idx)
        sel_img.append(torch.full_like(idx, m))
        sel_shell.append(shell)
    if sel_atoms:
        atoms = torch.cat(sel_atoms)
        img = torch.cat(sel_img)
        shell = torch.cat(sel_shell)
    else:
        atoms = img = shell = torch.zeros(0, dtype=torch.int64, device=dev)
    key = (shell * n + atoms) * len(images) + img
    order = torch.argsort(key)
    atoms, img, shell = atoms[order], img[order], shell[order]
    shifts = torch.as_tensor(images, dtype=torch.float64, device=dev)[img]
    local = base[atoms] + shifts @ cell_t
    counts = torch.bincount(shell, minlength=len(radii) + 1).cpu().numpy()
    shell_end = np.cumsum(counts).astype(np.int64).tolist()
    if local.shape[0]:
        lo_c = local.min(dim=0).values.cpu().numpy()
        hi_c = local.max(dim=0).values.cpu().numpy()
    else:
        lo_c = hi_c = np.zeros(3)
    origin = lo_c - 1.0
    box = np.diag(np.maximum(hi_c - lo_c + 2.0, 1.0)).reshape(9)
    local = local - torch.as_tensor(origin, dtype=torch.float64, device=dev)
    return LocalSystem(atoms, local.contiguous(), shell_end, box, origin)


def _rank_world(group):
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(group), dist.get_world_size(group)
    return 0, 1


class DomainEvaluator:
    """Energy, per-atom energies, forces and virial of one structure from a grid of domains.

    `model` is an engine model (``rune_b200.mobius`` / ``rune_b200.nep``) on this rank's GPU.
    `n_domains` (default: the world size) sets the grid (``domain_grid``); `grid` overrides
    it. Domains go to ranks round-robin; every rank returns the full reduced result."""

    def __init__(self, model, n_domains: int | None = None, grid=None, group=None):
        self.model = model
        self.group = group
        self.rank, self.world = _rank_world(group)
        self.n_domains = n_domains
        self.grid = tuple(grid) if grid is not None else None
        self.radii = shell_radii(model.params, model.family)
        self.last_locals: list[LocalSystem] = []

    def _grid(self, cell):
        if self.grid is not None:
            return self.grid
        return domain_grid(self.n_domains or self.world, cell)

    def domains(self, cell) -> list[tuple[int, int, int]]:
        """This rank's domains, (ix, iy, iz) in row-major domain order."""
        g = self._grid(cell)
        every = [(a, b, c) for a in range(g[0]) for b in range(g[1]) for c in range(g[2])]
        return [d for k, d in enumerate(every) if k % self.world == self.rank]

    def evaluate(self, positions, cell, pbc, types, *, forces=True, virial=True) -> dict:
        """positions [N, 3] and types [N] (tensors or arrays; moved to the model's device),
        cell 3x3, pbc [3]. Returns float64 device tensors: energy [], energies [N],
        forces [N, 3] (if requested), virial [9] (if requested)."""
        import torch.distributed as dist

        engine = self.model.engine()
        dev = (engine.device if isinstance(engine.device, torch.device)
               else torch.device("cuda", engine.device))
        pos = torch.as_tensor(positions).to(dev, torch.float64)
        typ = torch.as_tensor(types).to(dev, torch.int32)
        n = pos.shape[0]
        cell = np.asarray(cell, np.float64).reshape(3, 3)
        grid = self._grid(cell)
        # one float64 buffer for the reduction: energy, virial, energies, forces
        buf = torch.zeros(10 + 4 * n, dtype=torch.float64, device=dev)
        energies = buf[10:10 + n]
        force = buf[10 + n:].view(n, 3)
        self.last_locals = []
        for d in self.domains(cell):
            loc = partition(pos, cell, pbc, grid, d, self.radii)
            self.last_locals.append(loc)
            res = engine.compute_domain(typ[loc.atoms], loc.positions, loc.shell_end,
                                        loc.cell, forces=forces, virial=virial)
            buf[0] += res["energy"][0]
            if virial:
                buf[1:10] += res["virial"][0]
            owned = loc.atoms[:loc.n_owned]
            energies.index_add_(0, owned, res["energies"][:loc.n_owned].double())
            if forces:
                force.index_add_(0, loc.atoms, res["forces"].double())
        if self.world > 1:
            dist.all_reduce(buf, group=self.group)
        out = {"energy": buf[0], "energies": energies}
        if forces:
            out["forces"] = force
        if virial:
            out["virial"] = buf[1:10]
        return out


# --------------------------------------------------------------------------- halo exchange
class HaloPlan:
    """Which local rows go to which rank in one rank's local system (owned atoms, then ghosts).

    A ghost row is a copy of an atom owned by another domain (or a periodic image of one of this
    rank's own atoms). FILL: every ghost row receives its owner's row. REDUCE: every ghost row
    is added into its owner's row and then zeroed; an owner row that appears several times
    (several peers, several images) receives its additions one occurrence at a time, in a fixed
    order, so the sums are deterministic. Exchanges are ``all_to_all_single`` over `group`
    (NCCL on GPUs); with one rank they are local copies."""

    def __init__(self, atoms: torch.Tensor, n_owned: int, owner: torch.Tensor, n_global: int,
                 group=None):
        import torch.distributed as dist

        self.group = group
        self.rank, self.world = _rank_world(group)
        dev = atoms.device
        self.n_owned = int(n_owned)
        ghosts = atoms[self.n_owned:]
        g_owner = owner[ghosts]
        order = torch.sort(g_owner, stable=True).indices
        self.recv_rows = self.n_owned + order                 # ghost rows grouped by owner
        want = ghosts[order]                                   # their global atoms
        self.recv_counts = torch.bincount(g_owner, minlength=self.world).cpu().tolist()
        if self.world > 1:
            counts = torch.as_tensor(self.recv_counts, dtype=torch.int64, device=dev)
            peer_counts = torch.empty_like(counts)
            dist.all_to_all_single(peer_counts, counts, group=group)
            self.send_counts = peer_counts.cpu().tolist()
            asked = torch.empty(sum(self.send_counts), dtype=torch.int64, device=dev)
            dist.all_to_all_single(asked, want.contiguous(), self.send_counts, self.recv_counts,
                                   group=group)
        else:
            self.send_counts = list(self.recv_counts)
            asked = want
        local_of = torch.full((n_global,), -1, dtype=torch.int64, device=dev)
        local_of[atoms[:self.n_owned]] = torch.arange(self.n_owned, device=dev)
        self.send_rows = local_of[asked]
        if self.send_rows.numel() and int(self.send_rows.min()) < 0:
            raise RuntimeError("halo plan: a peer asked for an atom this rank does not own")
        # occurrence rank of every send row among equal rows (stable): REDUCE adds occurrence
        # 0 of every row, then occurrence 1, ..., each step with distinct target rows
        srt = torch.sort(self.send_rows, stable=True)
        first = torch.ones_like(srt.values, dtype=torch.bool)
        if srt.values.numel() > 1:
            first[1:] = srt.values[1:] != srt.values[:-1]
        start = torch.cummax(torch.where(first, torch.arange(len(first), device=dev),
                                         torch.zeros_like(srt.indices)), 0).values
        occ_sorted = torch.arange(len(first), device=dev) - start
        occ = torch.empty_like(occ_sorted)
        occ[srt.indices] = occ_sorted
        self.occ_groups = [torch.nonzero(occ == k).flatten()
                           for k in range(int(occ.max()) + 1 if occ.numel() else 0)]

    def _exchange(self, send, out_rows, in_counts, out_counts):
        import torch.distributed as dist

        recv = torch.empty((out_rows, send.shape[1]), dtype=send.dtype, device=send.device)
        if self.world > 1:
            dist.all_to_all_single(recv, send, out_counts, in_counts, group=self.group)
        else:
            recv.copy_(send)
        return recv

    def fill(self, rows: torch.Tensor):
        send = rows.index_select(0, self.send_rows)
        recv = self._exchange(send, self.recv_rows.numel(), self.send_counts, self.recv_counts)
        rows.index_copy_(0, self.recv_rows, recv)

    def reduce(self, rows: torch.Tensor):
        send = rows.index_select(0, self.recv_rows)
        recv = self._exchange(send, self.send_rows.numel(), self.recv_counts, self.send_counts)
        for grp in self.occ_groups:
            rows.index_add_(0, self.send_rows[grp], recv[grp])
        rows[self.n_owned:] = 0

    def hook(self, op: int, rows: torch.Tensor):
        from .runtime import library as L

        if op == L.RUNE_HALO_FILL:
            self.fill(rows)
        elif op == L.RUNE_HALO_REDUCE:
            self.reduce(rows)
        else:
            raise ValueError(f"unknown halo operation {op}")


class HaloEvaluator:
    """Energy, forces and virial of one structure with one domain per rank and per-layer halo
    exchange (``rune_engine_compute_halo``; Local and EQ Möbius models).

    Each rank's local system is its domain's owned atoms plus the ghosts within one
    max(radial, angular) cutoff; the engine evaluates only owned centres and asks for the ghost
    rows of every layer's node and direction states (FILL) and returns the ghost rows of their
    adjoints (REDUCE) through `HaloPlan`. After the call the ghost forces go to their owners
    (reverse force halo) and [energy, virial] is summed over ranks (one all-reduce of ten
    float64). No rank holds ghost work beyond the geometry of its boundary edges."""

    def __init__(self, model, group=None):
        self.model = model
        self.group = group
        self.rank, self.world = _rank_world(group)
        p = model.params
        self.radius = max(float(p["rcut_radial"]), float(p["rcut_angular"]))
        self.last_local: LocalSystem | None = None
        self.last_plan: HaloPlan | None = None

    def domain_index(self, grid):
        g = grid
        r = self.rank
        return (r // (g[1] * g[2]), (r // g[2]) % g[1], r % g[2])

    def evaluate(self, positions, cell, pbc, types, *, forces=True, virial=True,
                 gather=False) -> dict:
        """Returns float64 device tensors energy [], virial [9] (summed over ranks), and this
        rank's owned atoms: `owned` (global indices), `energies` and `forces` of them (float32);
        with gather=True also the whole structure's `energies_all` [N] and `forces_all`
        [N, 3] on every rank."""
        import torch.distributed as dist

        from .runtime import library as L

        engine = self.model.engine()
        dev = (engine.device if isinstance(engine.device, torch.device)
               else torch.device("cuda", engine.device))
        pos = torch.as_tensor(positions).to(dev, torch.float64)
        typ = torch.as_tensor(types).to(dev, torch.int32)
        n = pos.shape[0]
        cell = np.asarray(cell, np.float64).reshape(3, 3)
        pbc = [bool(p) for p in np.asarray(pbc).reshape(3)]
        grid = domain_grid(self.world, cell)
        loc = partition(pos, cell, pbc, grid, self.domain_index(grid), [self.radius])
        owner = domain_owner(pos, cell, pbc, grid)
        plan = HaloPlan(loc.atoms, loc.n_owned, owner, n, self.group)
        self.last_local, self.last_plan = loc, plan
        for _ in range(8):
            status, error = 0, None
            try:
                res = engine.compute_halo(typ[loc.atoms], loc.positions, loc.n_owned, loc.cell,
                                          plan.hook, forces=forces, virial=virial)
            except L.HaloRetry:
                status = 1
            except Exception as exc:  # every rank learns of it before raising
                status, error = 2, exc
            if self.world > 1:
                flag = torch.tensor([status], dtype=torch.int32, device=dev)
                dist.all_reduce(flag, op=dist.ReduceOp.MAX, group=self.group)
                status = int(flag.item())
            if status == 0:
                break
            if status == 2:
                raise error if error is not None else RuntimeError(
                    "halo evaluation failed on another rank")
        else:
            raise RuntimeError("halo evaluation: neighbour rows did not settle")
        if forces:
            plan.reduce(res["forces"])  # reverse force halo
        buf = torch.zeros(10, dtype=torch.float64, device=dev)
        buf[0] = res["energy"][0]
        if virial:
            buf[1:10] = res["virial"][0]
        if self.world > 1:
            dist.all_reduce(buf, group=self.group)
        k = loc.n_owned
        out = {"energy": buf[0], "owned": loc.atoms[:k], "energies": res["energies"][:k]}
        if forces:
            out["forces"] = res["forces"][:k]
        if virial:
            out["virial"] = buf[1:10]
        if gather:
            full = torch.zeros(4 * n, dtype=torch.float64, device=dev)
            full[:n].index_copy_(0, loc.atoms[:k], res["energies"][:k].double())
            if forces:
                full[n:].view(n, 3).index_copy_(0, loc.atoms[:k], res["forces"][:k].double())
            if self.world > 1:
                dist.all_reduce(full, group=self.group)
            out["energies_all"] = full[:n]
            if forces:
                out["forces_all"] = full[n:].view(n, 3)
        return out
