"""Python handle of one engine instance (one model on one CUDA device).

Inputs and outputs are torch CUDA tensors (device memory and streams only; every number is
computed by the CUDA library). The engine owns a float32 copy of the weights and a device
workspace; calls on one handle must not overlap.
"""

from __future__ import annotations

import ctypes
from ctypes import byref, c_double, c_float, c_int32, c_int64, c_uint8, c_void_p

import numpy as np
import torch

from .. import tables
from . import library as L


def _activation_code(name: str) -> int:
    key = str(name).strip().lower()
    if key not in L.RUNE_ACT:
        raise ValueError(f"Unsupported activation {name!r}")
    return L.RUNE_ACT[key]


def zbl_mode(config) -> tuple[int, float, float]:
    """(mode, rc_inner, rc_outer) from a reference zbl entry (rune/mobius/zbl.py:68-90)."""
    if config is None:
        return L.RUNE_ZBL_NONE, 0.0, 0.0
    if isinstance(config, dict):
        inner, outer = float(config["rc_inner"]), float(config["rc_outer"])
        flexible = bool(config.get("flexible", inner == 0.0 and outer == 0.0))
    else:
        inner, outer = map(float, config)
        flexible = inner == 0.0 and outer == 0.0
    return (L.RUNE_ZBL_FLEXIBLE if flexible else L.RUNE_ZBL_UNIVERSAL), inner, outer


def model_config(params: dict, family: str) -> L.ModelConfig:
    """Build the C config struct from resolved reference ``model_params``."""
    c = L.ModelConfig()
    p = params
    c.n_types = len(p["elements"])
    c.rc_radial = float(p["rcut_radial"])
    c.rc_angular = float(p["rcut_angular"])
    c.n_desc_radial = int(p["n_desc_radial"])
    c.n_desc_angular = int(p["n_desc_angular"])
    c.k_max_radial = int(p["k_max_radial"])
    c.k_max_angular = int(p["k_max_angular"])
    c.l_max = int(p["l_max"])
    c.has_q222 = int(p.get("has_q_222", int(p.get("l_max_4body", 2)) > 0))
    c.has_q1111 = int(p.get("has_q_1111", int(p.get("l_max_5body", 0)) > 0))
    c.has_q112 = int(p.get("has_q_112", 0))
    c.has_q123 = int(p.get("has_q_123", 0))
    c.has_q233 = int(p.get("has_q_233", 0))
    c.has_q134 = int(p.get("has_q_134", 0))
    c.max_neighbors_radial = int(p.get("max_neighbors_radial", 100))
    c.max_neighbors_angular = int(p.get("max_neighbors_angular", 30))
    c.norm_eps = float(p.get("norm_eps", 1e-8))
    mode, inner, outer = zbl_mode(p.get("zbl"))
    c.zbl_mode, c.zbl_rc_inner, c.zbl_rc_outer = mode, inner, outer
    if family == "nep":
        c.kind = L.RUNE_NEP
        c.nep_hidden = int(p["hidden_dims"][0])
        c.activation = L.RUNE_ACT["tanh"]
        return c
    layers = int(p.get("message_layers", 0))
    mode_name = p.get("message_mode", "scalar")
    c.kind = (L.RUNE_MOBIUS_LOCAL if layers == 0 else
              L.RUNE_MOBIUS_EQ if mode_name == "equivariant" else L.RUNE_MOBIUS_MP)
    c.hidden_dim = int(p["hidden_dim"])
    c.ffn_dim = int(p.get("ffn_dim", 2 * c.hidden_dim))
    c.blocks = int(p["blocks"])
    c.activation = _activation_code(p.get("activation", "silu"))
    c.message_layers = layers
    c.message_dim = int(p.get("message_dim", c.hidden_dim))
    c.pair_dim = int(p.get("pair_dim", 16))
    c.message_groups = int(p.get("message_groups", 8))
    c.vector_channels = int(p.get("vector_channels", 8))
    c.equivariant_channels = int(p.get("equivariant_channels", 0) or 0)
    c.equivariant_l_max = int(p.get("equivariant_l_max", 0) or 0)
    c.message_basis_size = int(p.get("message_basis_size", p["k_max_radial"]))
    c.message_cutoff = float(p.get("message_cutoff", p["rcut_radial"]))
    return c


def engine_tensors(state: dict, params: dict, family: str) -> dict[str, np.ndarray]:
    """float32 host arrays keyed as the engine expects (reference state_dict names)."""
    out = {}
    for key, value in state.items():
        arr = value.detach().to("cpu", torch.float32).contiguous().numpy()
        if family == "nep" and key.startswith("element_mlps."):
            _, element, rest = key.split(".", 2)
            key = f"element_mlps.{params['elements'].index(element)}.{rest}"
        out[key] = arr
    flags = tuple(int(params.get(k, 0)) for k in ("has_q_222", "has_q_1111", "has_q_112",
                                                  "has_q_123", "has_q_233", "has_q_134"))
    out["eq_scale"] = tables.orthonormal_scale(8).astype(np.float32)
    out["invariant_terms"] = tables.invariant_terms(
        int(params["l_max"]), flags, out["descriptor.angular.C3B"],
        out["descriptor.angular.C4B"], out["descriptor.angular.C5B"],
        out["descriptor.angular.C4B2"])
    return out


class _DeviceRows:
    """A float32 [rows, width] device array handed over by the engine (zero copy)."""

    def __init__(self, ptr, rows, width):
        self.__cuda_array_interface__ = {"shape": (rows, width), "typestr": "<f4",
                                         "data": (ptr, False), "version": 3, "strides": None}


def device_rows(ptr, rows, width, dev):
    """torch view of an engine array of `rows` x `width` float32 at device address `ptr`."""
    if rows == 0 or width == 0:
        return torch.empty((rows, width), dtype=torch.float32, device=dev)
    return torch.as_tensor(_DeviceRows(int(ptr), rows, width), device=dev)


class Engine:
    def __init__(self, config: L.ModelConfig, tensors: dict, device: int):
        self._lib = L.load_library()
        self.device = int(device)
        self.config = config
        handle = c_void_p()
        L.check(self._lib, self._lib.rune_engine_create(byref(config), self.device,
                                                         byref(handle)))
        self._h = handle
        try:
            for name, arr in tensors.items():
                arr = np.ascontiguousarray(arr, dtype=np.float32)
                ptr = arr.ctypes.data_as(ctypes.POINTER(c_float))
                L.check(self._lib, self._lib.rune_engine_set_tensor(
                    self._h, name.encode(), ptr, c_int64(arr.size)))
            L.check(self._lib, self._lib.rune_engine_finalize(self._h))
        except Exception:
            self.close()
            raise

    # ------------------------------------------------------------------ helpers
    def _stream(self, stream):
        if stream is None:
            stream = torch.cuda.current_stream(self.device)
        return c_void_p(stream.cuda_stream)

    def _dev(self):
        return torch.device("cuda", self.device)

    @staticmethod
    def _ptr(t):
        return c_void_p(t.data_ptr()) if t is not None else None

    # ------------------------------------------------------------------ MD
    def md_nve(self, types, positions, velocities, masses, cell, pbc, dt, n_steps, skin,
               forces=None, stream=None):
        """Velocity-Verlet NVE of one structure (rune_md_nve): positions / velocities (float64
        device tensors [N, 3]) are advanced in place. Returns energies [n_steps + 1, 2]
        (potential, kinetic; eV) and the number of candidate-list builds."""
        n = int(types.shape[0])
        for name, t, dt_ in (("positions", positions, torch.float64),
                             ("velocities", velocities, torch.float64),
                             ("masses", masses, torch.float64), ("types", types, torch.int32)):
            if t.dtype != dt_ or not t.is_contiguous() or t.device != self._dev():
                raise ValueError(f"{name} must be a contiguous {dt_} tensor on {self._dev()}")
        energies = np.zeros((n_steps + 1, 2), np.float64)
        rebuilds = c_int64(0)
        cell = np.ascontiguousarray(np.asarray(cell, np.float64).reshape(9))
        pbc = np.ascontiguousarray(np.asarray(pbc, bool).reshape(3).astype(np.uint8))
        L.check(self._lib, self._lib.rune_md_nve(
            self._h, n, self._ptr(types), self._ptr(positions), self._ptr(velocities),
            self._ptr(masses), cell.ctypes.data_as(ctypes.POINTER(ctypes.c_double)),
            pbc.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)), float(dt), int(n_steps),
            float(skin), energies.ctypes.data_as(ctypes.POINTER(ctypes.c_double)),
            self._ptr(forces), ctypes.byref(rebuilds), self._stream(stream)))
        return energies, int(rebuilds.value)

    # ------------------------------------------------------------------ compute
    def compute(self, types, positions, cells, pbc, atom_ptr, *, forces=True, virial=True,
                out=None, stream=None):
        """Device-built neighbour lists. types int32 [N] and positions float64 [N, 3] on this
        device; cells [B, 9] float64, pbc [B, 3] and atom_ptr [B + 1] on the host."""
        n = int(types.shape[0])
        cells = np.ascontiguousarray(np.asarray(cells, np.float64).reshape(-1, 9))
        pbc = np.ascontiguousarray(np.asarray(pbc, np.uint8).reshape(-1, 3))
        atom_ptr = np.ascontiguousarray(np.asarray(atom_ptr, np.int32).reshape(-1))
        b = cells.shape[0]
        if pbc.shape[0] != b or atom_ptr.shape[0] != b + 1:
            raise ValueError("cells, pbc and atom_ptr disagree on the number of structures")
        types = types.to(self._dev(), torch.int32).contiguous()
        positions = positions.to(self._dev(), torch.float64).contiguous()
        res = out if out is not None else self.allocate(n, b, forces, virial)
        flags = (L.RUNE_FORCES if forces else 0) | (L.RUNE_VIRIAL if virial else 0)
        status = self._lib.rune_engine_compute(
            self._h, n, b, self._ptr(types), self._ptr(positions),
            cells.ctypes.data_as(ctypes.POINTER(c_double)),
            pbc.ctypes.data_as(ctypes.POINTER(c_uint8)),
            atom_ptr.ctypes.data_as(ctypes.POINTER(c_int32)), flags,
            self._ptr(res["energies"]), self._ptr(res["energy"]),
            self._ptr(res.get("forces")), self._ptr(res.get("virial")), self._stream(stream))
        L.check(self._lib, status)
        return res

    def compute_domain(self, types, positions, shell_end, cell, *, forces=True, virial=True,
                       out=None, stream=None):
        """One rank's local system of a domain decomposition (rune_engine_compute_domain):
        owned atoms first, then ghost shells; shell_end [n_shells + 1] cumulative counts on the
        host; cell [9] a binning box. Energy of the owned atoms; forces and virial of that
        energy with respect to every local atom."""
        n = int(types.shape[0])
        shell_end = np.ascontiguousarray(np.asarray(shell_end, np.int32).reshape(-1))
        cell = np.ascontiguousarray(np.asarray(cell, np.float64).reshape(9))
        types = types.to(self._dev(), torch.int32).contiguous()
        positions = positions.to(self._dev(), torch.float64).contiguous()
        res = out if out is not None else self.allocate(n, 1, forces, virial)
        flags = (L.RUNE_FORCES if forces else 0) | (L.RUNE_VIRIAL if virial else 0)
        status = self._lib.rune_engine_compute_domain(
            self._h, n, int(shell_end.shape[0]) - 1,
            shell_end.ctypes.data_as(ctypes.POINTER(c_int32)), self._ptr(types),
            self._ptr(positions), cell.ctypes.data_as(ctypes.POINTER(c_double)), flags,
            self._ptr(res["energies"]), self._ptr(res["energy"]),
            self._ptr(res.get("forces")), self._ptr(res.get("virial")), self._stream(stream))
        L.check(self._lib, status)
        return res

    def compute_halo(self, types, positions, n_owned, cell, hook, *, forces=True, virial=True,
                     out=None, stream=None):
        """One rank's domain with per-layer halo exchange (rune_engine_compute_halo): owned atoms
        first, then one shell of ghosts; cell [9] a binning box. `hook(op, rows)` receives
        ``L.RUNE_HALO_FILL`` or ``L.RUNE_HALO_REDUCE`` and a float32 [n_atoms, width] view of the
        engine's array; it must fill the ghost rows from their owners (FILL) or add them into
        their owners and zero them (REDUCE), on the current stream. Raises ``L.HaloRetry`` when
        every rank must repeat the call."""
        n = int(types.shape[0])
        cell = np.ascontiguousarray(np.asarray(cell, np.float64).reshape(9))
        dev = self._dev()
        types = types.to(dev, torch.int32).contiguous()
        positions = positions.to(dev, torch.float64).contiguous()
        res = out if out is not None else self.allocate(n, 1, forces, virial)
        flags = (L.RUNE_FORCES if forces else 0) | (L.RUNE_VIRIAL if virial else 0)
        failure = []

        def trampoline(_ctx, op, rows, width, _stream):
            try:
                hook(int(op), device_rows(rows, n, int(width), dev))
                return 0
            except BaseException as exc:  # reported after the call returns
                failure.append(exc)
                return 1

        fn = L.HALO_FN(trampoline)
        status = self._lib.rune_engine_compute_halo(
            self._h, n, int(n_owned), self._ptr(types), self._ptr(positions),
            cell.ctypes.data_as(ctypes.POINTER(c_double)), flags, fn, None,
            self._ptr(res["energies"]), self._ptr(res["energy"]),
            self._ptr(res.get("forces")), self._ptr(res.get("virial")), self._stream(stream))
        if failure:
            raise failure[0]
        L.check(self._lib, status)
        return res

    def allocate(self, n, b, forces=True, virial=True):
        dev = self._dev()
        res = {"energies": torch.empty(n, dtype=torch.float32, device=dev),
               "energy": torch.empty(b, dtype=torch.float64, device=dev)}
        if forces:
            res["forces"] = torch.empty((n, 3), dtype=torch.float32, device=dev)
        if virial:
            res["virial"] = torch.empty((b, 9), dtype=torch.float64, device=dev)
        return res

    def compute_padded(self, types, positions, radial_neighbors, radial_offsets,
                       angular_neighbors, angular_offsets, atom_ptr, *, forces=True,
                       virial=True, stream=None):
        """The reference batch form: padded int64 neighbour rows (-1 = empty) and float32
        offsets, all on this device; atom_ptr on the host."""
        dev = self._dev()
        n = int(types.shape[0])
        atom_ptr = np.ascontiguousarray(np.asarray(atom_ptr, np.int32).reshape(-1))
        b = atom_ptr.shape[0] - 1
        types = types.to(dev, torch.int32).contiguous()
        positions = positions.to(dev, torch.float32).contiguous()
        rn = radial_neighbors.to(dev, torch.int64).contiguous()
        an = angular_neighbors.to(dev, torch.int64).contiguous()
        ro = radial_offsets.to(dev, torch.float32).contiguous()
        ao = angular_offsets.to(dev, torch.float32).contiguous()
        rw = int(rn.shape[1]) if rn.dim() == 2 else 0
        aw = int(an.shape[1]) if an.dim() == 2 else 0
        res = self.allocate(n, b, forces, virial)
        flags = (L.RUNE_FORCES if forces else 0) | (L.RUNE_VIRIAL if virial else 0)
        status = self._lib.rune_engine_compute_padded(
            self._h, n, b, self._ptr(types), self._ptr(positions), self._ptr(rn), rw,
            self._ptr(ro), self._ptr(an), aw, self._ptr(ao),
            atom_ptr.ctypes.data_as(ctypes.POINTER(c_int32)), flags,
            self._ptr(res["energies"]), self._ptr(res["energy"]),
            self._ptr(res.get("forces")), self._ptr(res.get("virial")), self._stream(stream))
        L.check(self._lib, status)
        return res

    def neighbor_pairs(self, which: str = "radial") -> np.ndarray:
        """(i, j, S0, S1, S2) rows of the last device-built list, engine order."""
        code = 0 if which == "radial" else 1
        count = c_int64()
        L.check(self._lib, self._lib.rune_engine_neighbor_pairs(self._h, code, None, 0,
                                                                  byref(count)))
        buf = np.zeros((max(count.value, 1), 5), dtype=np.int32)
        L.check(self._lib, self._lib.rune_engine_neighbor_pairs(
            self._h, code, buf.ctypes.data_as(ctypes.POINTER(c_int32)), count.value,
            byref(count)))
        return buf[:count.value].astype(np.int64)

    def stats(self) -> dict:
        s = L.Stats()
        L.check(self._lib, self._lib.rune_engine_stats(self._h, byref(s)))
        return {name: getattr(s, name) for name, _ in L.Stats._fields_}

    def set_wait_polls(self, polls: int):
        """Bound (mbarrier polls) of the EQ kernels' in-kernel waits; 0 makes every wait give up
        at once and the next EQ call raise RuntimeError. Default ``library.DEFAULT_WAIT_POLLS``."""
        L.check(self._lib, self._lib.rune_engine_set_wait_polls(self._h, int(polls)))

    def set_profiling(self, enabled: bool):
        """Bracket every kernel launch with CUDA events (per-kernel device time)."""
        L.check(self._lib, self._lib.rune_engine_set_profiling(self._h, int(bool(enabled))))

    def kernel_stats(self) -> dict:
        """{kernel name: (total ms, launches)} accumulated since the last reset."""
        out = {}
        buf = ctypes.create_string_buffer(128)
        ms = c_double()
        n = c_int64()
        index = 0
        while self._lib.rune_engine_kernel_stat(self._h, index, buf, 128, byref(ms),
                                                byref(n)) == L.RUNE_OK:
            out[buf.value.decode()] = (ms.value, n.value)
            index += 1
        return out

    def reset_kernel_stats(self):
        L.check(self._lib, self._lib.rune_engine_reset_kernel_stats(self._h))

    def close(self):
        if getattr(self, "_h", None) is not None and self._h.value:
            self._lib.rune_engine_destroy(self._h)
        self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
