"""ASE Calculator for rune_b200 models (rune/mobius/interface/calculator.py:14-98 and its NEP copy).

The calculator keeps the reference signature and results (energy, free_energy, forces,
stress = -virial / volume in Voigt order). Instead of building padded neighbour lists on the
host (interface/batch.py), it hands positions, cell and pbc to the engine, which builds the
lists on the GPU. ASE is optional: without it a minimal stand-in base class provides the same
``calculate`` / ``get_*`` behaviour for objects with ``positions``, ``cell``, ``pbc`` and
``numbers``.
"""

from __future__ import annotations

import numpy as np
import torch

from .elements import atomic_numbers, chemical_symbols

try:  # pragma: no cover - depends on the environment
    from ase.calculators.calculator import Calculator as _Base
    from ase.calculators.calculator import PropertyNotImplementedError, all_changes

    HAVE_ASE = True
except ImportError:  # pragma: no cover
    HAVE_ASE = False

    class PropertyNotImplementedError(NotImplementedError):
        """Raised for a property the calculator does not provide (as in ASE)."""

    all_changes = ["positions", "numbers", "cell", "pbc", "initial_charges",
                   "initial_magmoms"]

    class _Base:
        """Minimal stand-in for ase.calculators.calculator.Calculator."""

        implemented_properties: list = []

        def __init__(self, **kwargs):
            self.atoms = None
            self.results = {}
            self.parameters = dict(kwargs)

        def calculate(self, atoms=None, properties=None, system_changes=all_changes):
            if atoms is not None:
                self.atoms = atoms

        def get_property(self, name, atoms=None, allow_calculation=True):
            if name not in self.implemented_properties:
                raise PropertyNotImplementedError(f"{name} property not implemented")
            self.calculate(atoms if atoms is not None else self.atoms, [name], all_changes)
            return self.results[name]

        def get_potential_energy(self, atoms=None, force_consistent=False):
            return self.get_property("energy", atoms)

        def get_forces(self, atoms=None):
            return self.get_property("forces", atoms)

        def get_stress(self, atoms=None):
            return self.get_property("stress", atoms)


def full_3x3_to_voigt_6_stress(stress):
    """Symmetrised Voigt form [xx, yy, zz, yz, xz, xy] (ase.stress convention)."""
    s = np.asarray(stress, dtype=np.float64).reshape(3, 3)
    return np.array([s[0, 0], s[1, 1], s[2, 2], 0.5 * (s[1, 2] + s[2, 1]),
                     0.5 * (s[0, 2] + s[2, 0]), 0.5 * (s[0, 1] + s[1, 0])])


def _volume(atoms, cell):
    if hasattr(atoms, "get_volume"):
        return float(atoms.get_volume())
    return float(abs(np.linalg.det(cell)))


class EngineCalculator(_Base):
    implemented_properties = ["energy", "free_energy", "forces", "stress"]
    family_label = "Möbius"

    def __init__(self, artifact, device="cuda", compute_stress: bool = True, **kwargs):
        super().__init__(**kwargs)
        self.device = torch.device(device) if device is not None else torch.device("cuda")
        self.model = self._load(artifact, self.device)
        self.model.eval()
        self.model.requires_grad_(False)
        self.compute_stress = bool(compute_stress)
        self.implemented_properties = ["energy", "free_energy", "forces"]
        if self.compute_stress:
            self.implemented_properties.append("stress")
        self.elements = list(self.model.params["elements"])
        self.z_to_type = {atomic_numbers[e]: t for t, e in enumerate(self.elements)}
        self._cached_numbers = None
        self._cached_types = None

    @staticmethod
    def _load(artifact, device):  # overridden per family
        raise NotImplementedError

    def _types(self, numbers) -> torch.Tensor:
        key = tuple(int(z) for z in numbers)
        if key == self._cached_numbers:
            return self._cached_types
        missing = sorted(set(key).difference(self.z_to_type))
        if missing:
            symbols = [chemical_symbols[z] if 0 <= z < len(chemical_symbols) else f"Z{z}"
                       for z in missing]
            raise ValueError(
                f"Atoms contain elements not supported by this {self.family_label} model: "
                f"{symbols}. Model elements (type-id order): {self.elements}.")
        self._cached_numbers = key
        self._cached_types = torch.tensor([self.z_to_type[z] for z in key], dtype=torch.int32,
                                          device=self.device)
        return self._cached_types

    def calculate(self, atoms=None, properties=None, system_changes=all_changes):
        properties = properties or ["energy"]
        super().calculate(atoms, properties, system_changes)
        atoms = atoms if atoms is not None else self.atoms
        if atoms is None:
            raise ValueError("Calculator requires an ASE Atoms object.")
        requested = set(properties)
        compute_forces = "forces" in requested
        compute_virial = "stress" in requested
        cell = np.asarray(getattr(atoms, "cell"), dtype=np.float64).reshape(3, 3)
        if compute_virial and not self.compute_stress:
            raise PropertyNotImplementedError(
                "Stress is disabled for this Calculator. "
                "Construct it with compute_stress=True for NPT or stress calculations.")
        volume = None
        if compute_virial:
            volume = _volume(atoms, cell)
            if volume <= 0:
                raise ValueError("Stress calculation requires a positive cell volume.")
        numbers = np.asarray(getattr(atoms, "numbers"))
        types = self._types(numbers)
        positions = torch.as_tensor(np.asarray(atoms.positions, dtype=np.float64),
                                    device=self.device)
        pbc = np.asarray(getattr(atoms, "pbc"), dtype=bool).reshape(1, 3)
        with torch.no_grad():
            res = self.model.evaluate(positions, cell.reshape(1, 9), pbc, types,
                                      compute_forces=compute_forces,
                                      compute_virial=compute_virial)
        energy = float(res["energy"][0].cpu())
        self.results = {"energy": energy, "free_energy": energy}
        if compute_forces:
            self.results["forces"] = res["forces"].cpu().numpy().astype(np.float64)
        if compute_virial:
            virial = res["virial"][0].cpu().numpy().reshape(3, 3)
            self.results["stress"] = full_3x3_to_voigt_6_stress(-virial / volume)
