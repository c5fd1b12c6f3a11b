"""Parameter containers that mirror the reference modules' state_dict layout, plus the glue
that hands the parameters to the CUDA engine.

The containers only hold parameters and buffers (with the reference names, shapes, dtypes and
initialisation order, so checkpoints load with ``strict=True`` and seeded random initialisation
matches); every forward computation goes through ``rune_b200.runtime.engine.Engine``.
"""

from __future__ import annotations

import numpy as np
import torch
import torch.nn as nn

from . import tables
from .elements import atomic_numbers
from .runtime.engine import Engine, engine_tensors, model_config


class RadialDescriptor(nn.Module):
    """c_table [T, T, n, K] (rune/mobius/descriptor.py:443-450)."""

    def __init__(self, n_types, n_desc, k_max, r_c):
        super().__init__()
        self.n_types, self.n_desc, self.k_max, self.r_c = n_types, n_desc, k_max, r_c
        self.c_table = nn.Parameter(torch.randn(n_types, n_types, n_desc, k_max))


class AngularDescriptor(nn.Module):
    """c_table and the float32 coefficient buffers (rune/mobius/descriptor.py:477-526)."""

    def __init__(self, n_types, n_desc, k_max, r_c, l_max, flags):
        super().__init__()
        self.n_types, self.n_desc, self.k_max, self.r_c = n_types, n_desc, k_max, r_c
        self.L_max = int(l_max)
        names = ("has_q_222", "has_q_1111", "has_q_112", "has_q_123", "has_q_233", "has_q_134")
        for name, value in zip(names, flags):
            setattr(self, name, int(value > 0))
        if (self.has_q_123 or self.has_q_233) and self.L_max < 3:
            raise ValueError("q_123 and q_233 require l_max >= 3.")
        if self.has_q_134 and self.L_max < 4:
            raise ValueError("q_134 requires l_max >= 4.")
        if (self.has_q_222 or self.has_q_112) and self.L_max < 2:
            raise ValueError("L_max must be >= 2 to include 4-body descriptors.")
        self.num_L = self.L_max + sum(int(v > 0) for v in flags)
        self.c_table = nn.Parameter(torch.randn(n_types, n_types, n_desc, k_max))
        self.register_buffer("C3B", torch.tensor(tables.C3B_VALUES, dtype=torch.float32))
        self.register_buffer("C4B", torch.tensor(tables.C4B_VALUES, dtype=torch.float32))
        self.register_buffer("C5B", torch.tensor(tables.C5B_VALUES, dtype=torch.float32))
        self.register_buffer("C4B2", torch.tensor(tables.C4B2_VALUES, dtype=torch.float32))
        for order, data in tables.z_tables().items():
            self.register_buffer(f"Z{order}", torch.tensor(data, dtype=torch.float32))

    @property
    def flags(self):
        return (self.has_q_222, self.has_q_1111, self.has_q_112, self.has_q_123,
                self.has_q_233, self.has_q_134)


class Descriptor(nn.Module):
    """Radial + angular descriptor parameters (rune/mobius/descriptor.py:765-800)."""

    def __init__(self, params):
        super().__init__()
        self.radial = RadialDescriptor(params["n_types"], params["n_desc_radial"],
                                       params["k_max_radial"], params["rcut_radial"])
        flags = (
            int(params.get("has_q_222", params.get("l_max_4body", 2) > 0)),
            int(params.get("has_q_1111", params.get("l_max_5body", 0) > 0)),
            int(params.get("has_q_112", 0)), int(params.get("has_q_123", 0)),
            int(params.get("has_q_233", 0)), int(params.get("has_q_134", 0)),
        )
        self.angular = AngularDescriptor(params["n_types"], params["n_desc_angular"],
                                         params["k_max_angular"], params["rcut_angular"],
                                         params["l_max"], flags)
        params["l_max_4body"] = 2 if flags[0] else 0
        params["l_max_5body"] = flags[1]
        for name, value in zip(("has_q_222", "has_q_1111", "has_q_112", "has_q_123",
                                "has_q_233", "has_q_134"), flags):
            params[name] = value


class ZBLRepulsion(nn.Module):
    """ZBL buffers (rune/mobius/zbl.py:20-66; flexible limits of rune/nep/zbl.py:44-66)."""

    UNIVERSAL = ((0.18175, 3.1998), (0.50986, 0.94229), (0.28022, 0.4029), (0.02817, 0.20162))

    def __init__(self, elements, config, *, max_pairs=None):
        super().__init__()
        self.n_elements = len(elements)
        if isinstance(config, dict):
            inner, outer = float(config["rc_inner"]), float(config["rc_outer"])
            flexible = bool(config.get("flexible", inner == 0.0 and outer == 0.0))
            parameters = config.get("parameters")
        else:
            if len(config) != 2:
                raise ValueError("zbl must be [rc_inner, rc_outer] or a mapping.")
            inner, outer = map(float, config)
            flexible = inner == 0.0 and outer == 0.0
            parameters = None
        if flexible and parameters is None:
            raise ValueError("Flexible ZBL requires ten parameters per element pair.")
        if not flexible and not (0.0 <= inner < outer):
            raise ValueError("Universal ZBL requires 0 <= rc_inner < rc_outer.")
        self.rc_inner, self.rc_outer, self.flexible = inner, outer, flexible
        self.register_buffer("atomic_numbers", torch.tensor(
            [atomic_numbers[e] for e in elements], dtype=torch.float32))
        self.register_buffer("universal_coefficients",
                             torch.tensor(self.UNIVERSAL, dtype=torch.float32))
        if flexible:
            expected = self.n_elements * (self.n_elements + 1) // 2
            if max_pairs is not None and expected > max_pairs:
                raise ValueError("GPUMD flexible ZBL supports at most 10 elements (550 parameters).")
            tensor = torch.as_tensor(parameters, dtype=torch.float32).reshape(-1, 10)
            if tensor.shape[0] != expected:
                raise ValueError(
                    f"Flexible ZBL expects {expected} pair rows, got {tensor.shape[0]}.")
            if not torch.isfinite(tensor).all():
                raise ValueError("Flexible ZBL parameters must all be finite.")
            if ((tensor[:, 0] < 0.0) | (tensor[:, 0] >= tensor[:, 1])).any():
                raise ValueError("Each flexible ZBL pair must satisfy 0 <= rc_inner < rc_outer.")
        else:
            tensor = torch.zeros((0, 10), dtype=torch.float32)
        self.register_buffer("pair_parameters", tensor)
        self.max_rc_outer = float(tensor[:, 1].max()) if flexible else self.rc_outer


def structure_pointer(n_atoms_per_structure) -> np.ndarray:
    counts = torch.as_tensor(n_atoms_per_structure).detach().to("cpu", torch.int64).reshape(-1)
    return np.concatenate([[0], np.cumsum(counts.numpy())]).astype(np.int32)


# Registrations of parameters, buffers and submodules anywhere in the process (attribute
# assignment included). Walking a model's module tree costs tens of microseconds per call, so
# the engine cache keeps its tensor list and walks again only after a registration.
_REGISTRATIONS = [0]


def _count_registration(*_args):
    _REGISTRATIONS[0] += 1


for _register in (nn.modules.module.register_module_parameter_registration_hook,
                  nn.modules.module.register_module_buffer_registration_hook,
                  nn.modules.module.register_module_module_registration_hook):
    _register(_count_registration)


class EngineModel(nn.Module):
    """Base: lazily builds (and rebuilds after parameter changes) the CUDA engine.

    The engine is reused while every parameter and buffer keeps its storage and its version
    counter (in-place edits, ``load_state_dict`` and ``.to`` all change one of the two); a
    replaced parameter, buffer or submodule makes the next call collect the tensors again."""

    family = "mobius"

    def _engine(self) -> Engine:
        cached = getattr(self, "_engine_cache", None)
        registrations = _REGISTRATIONS[0]
        if cached is not None and cached[2] == registrations:
            params = cached[3]
        else:
            params = list(self.parameters()) + list(self.buffers())
        if not params or params[0].device.type != "cuda":
            raise RuntimeError(
                "rune_b200 evaluates on CUDA devices only; move the model with .to('cuda') "
                "(there is no CPU path).")
        device = params[0].device
        key = (device.index, tuple((t.data_ptr(), t._version) for t in params))
        if cached is not None and cached[0] == key:
            if cached[2] != registrations:
                object.__setattr__(self, "_engine_cache", (key, cached[1], registrations, params))
            return cached[1]
        index = device.index if device.index is not None else torch.cuda.current_device()
        engine = Engine(model_config(self.params, self.family),
                        engine_tensors(self.state_dict(), self.params, self.family), index)
        object.__setattr__(self, "_engine_cache", (key, engine, registrations, params))
        return engine

    def engine(self) -> Engine:
        """The CUDA engine holding this model's current parameters."""
        return self._engine()

    def forward(self, batch: dict) -> dict:
        """Reference model contract (rune/mobius/model.py:307-393, rune/nep/model.py:87-155)."""
        compute_forces = bool(batch.get("compute_forces", True))
        compute_virial = bool(batch.get("compute_virial", True))
        engine = self._engine()
        dtype = next(self.parameters()).dtype
        atom_ptr = structure_pointer(batch["n_atoms_per_structure"])
        res = engine.compute_padded(
            batch["types"], batch["positions"], batch["radial_neighbors"],
            batch["radial_offsets"], batch["angular_neighbors"], batch["angular_offsets"],
            atom_ptr, forces=compute_forces, virial=compute_virial)
        out = {"energies": res["energies"].to(dtype), "energy": res["energy"].to(dtype)}
        if compute_forces:
            out["forces"] = res["forces"].to(dtype)
        if compute_virial:
            out["virial"] = res["virial"].to(dtype)
        return out

    def evaluate(self, positions, cells, pbc, types, n_atoms_per_structure=None, *,
                 compute_forces=True, compute_virial=True, stream=None):
        """Fast entry: device-built neighbour lists from positions / cell / pbc.

        positions [N, 3] (float64 preferred), cells [B, 3, 3], pbc [B, 3], types [N] type
        indices; n_atoms_per_structure [B] (default: one structure)."""
        engine = self._engine()
        cells = np.asarray(cells, np.float64).reshape(-1, 9)
        pbc = np.asarray(pbc, bool).reshape(-1, 3)
        if n_atoms_per_structure is None:
            n_atoms_per_structure = [int(types.shape[0])]
        atom_ptr = structure_pointer(n_atoms_per_structure)
        return engine.compute(torch.as_tensor(types), torch.as_tensor(positions), cells, pbc,
                              atom_ptr, forces=compute_forces, virial=compute_virial,
                              stream=stream)
