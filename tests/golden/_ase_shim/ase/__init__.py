"""Minimal stand-in for the parts of ASE that the RUNE reference imports at module load.

Used only by ``tests/golden/make_golden.py`` to import the reference PyTorch models in a
container without ASE. It provides the periodic table and ``complete_cell`` for full 3-D cells.
"""
