"""Shared test helpers: fixture loading and error metrics."""

from __future__ import annotations

import ast
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"

_Z = {s: z for z, s in enumerate([
    "X", "H", "He", "Li", "Be", "B", "C", "N", "O", "F", "Ne", "Na", "Mg", "Al", "Si", "P",
    "S", "Cl", "Ar", "K", "Ca", "Sc", "Ti", "V", "Cr", "Mn", "Fe", "Co", "Ni", "Cu", "Zn",
    "Ga", "Ge", "As", "Se", "Br", "Kr", "Rb", "Sr", "Y", "Zr", "Nb", "Mo", "Tc", "Ru", "Rh",
    "Pd", "Ag", "Cd", "In", "Sn", "Sb", "Te", "I", "Xe", "Cs", "Ba", "La", "Ce", "Pr", "Nd",
    "Pm", "Sm", "Eu", "Gd", "Tb", "Dy", "Ho", "Er", "Tm", "Yb", "Lu", "Hf", "Ta", "W", "Re",
    "Os", "Ir", "Pt", "Au", "Hg", "Tl", "Pb", "Bi", "Po", "At", "Rn", "Fr", "Ra", "Ac", "Th",
    "Pa", "U", "Np", "Pu"])}


def load_params(g):
    return ast.literal_eval(str(g["params"]))


def load_state(g):
    return {k[len("param:"):]: np.asarray(g[k], dtype=np.float64) for k in g.files
            if k.startswith("param:")}


def z_of_type(params):
    return np.array([_Z[e] for e in params["elements"]], dtype=np.float64)


WEIGHTS = ROOT / "weights"


def oam_checkpoint(variant):
    """(params, float64 state) of a repository checkpoint, or None when it is not present."""
    path = WEIGHTS / f"mobius-oam-{variant}.pt"
    if not path.exists():
        return None
    import torch

    ckpt = torch.load(path, map_location="cpu", weights_only=False)
    state = {k: v.detach().double().numpy() for k, v in ckpt["model_state_dict"].items()}
    return ckpt["model_params"], state
