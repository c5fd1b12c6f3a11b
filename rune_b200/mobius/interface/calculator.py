"""Möbius ASE Calculator (rune/mobius/interface/calculator.py) on the rune_b200 engine."""

from __future__ import annotations

from ...interface import EngineCalculator, PropertyNotImplementedError  # noqa: F401
from ..plugin import load_model


class Calculator(EngineCalculator):
    family_label = "Möbius"

    @staticmethod
    def _load(artifact, device):
        return load_model(artifact, device=device)
