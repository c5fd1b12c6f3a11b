"""Test infrastructure: ctypes access to the reference's native FP64 Möbius evaluator.

``oracle/native/build.sh`` compiles the reference's own ``rune/mobius/src/*.cu`` (unmodified)
against stand-ins for the three GPUMD types it uses, into ``oracle/_ref/libmobius_native_ref.so``
(built by ``__graft_entry__.build()`` where a reference checkout is present; it travels with the
tree but stays out of git). This module loads it and runs ``Mobius::compute`` on one structure
(``oracle/native/ref_native.cu``). Only tests and bench.py's reference arm use it; it is the
checker, never the product.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

LIB = Path(__file__).resolve().parent / "_ref" / "libmobius_native_ref.so"
_lib = None


def available() -> bool:
    return LIB.exists()


def _load():
    global _lib
    if _lib is None:
        lib = ctypes.CDLL(str(LIB))
        lib.rn_last_error.restype = ctypes.c_char_p
        lib.rn_create.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.POINTER(ctypes.c_void_p)]
        lib.rn_destroy.argtypes = [ctypes.c_void_p]
        P = ctypes.c_void_p
        lib.rn_compute.argtypes = [P, ctypes.c_int, P, P, P, P, P, P, P, ctypes.c_int,
                                   ctypes.POINTER(ctypes.c_float)]
        _lib = lib
    return _lib


class NativeMobius:
    """``Mobius(model_path, n_atoms)`` of the reference's native evaluator."""

    def __init__(self, model_path, n_atoms):
        lib = _load()
        h = ctypes.c_void_p()
        if lib.rn_create(str(model_path).encode(), int(n_atoms), ctypes.byref(h)):
            raise RuntimeError(lib.rn_last_error().decode())
        self._h = h
        self.n = int(n_atoms)

    def compute(self, types, positions, cell, pbc=(True, True, True), reps=0):
        """Energies [n], forces [n, 3], virial [3, 3] (W_ab = -sum g_a r_b) and the mean device
        milliseconds of ``reps`` timed calls after one untimed call."""
        lib = _load()
        n = self.n
        t = np.ascontiguousarray(types, np.int32)
        p = np.ascontiguousarray(positions, np.float64)
        c = np.ascontiguousarray(np.asarray(cell, np.float64).reshape(9))
        b = np.ascontiguousarray(np.asarray(pbc, np.int32).reshape(3))
        e = np.zeros(n)
        f = np.zeros((n, 3))
        w = np.zeros(9)
        ms = ctypes.c_float(0.0)
        args = [a.ctypes.data for a in (t, p, c, b, e, f, w)]
        if lib.rn_compute(self._h, n, *args, int(reps), ctypes.byref(ms)):
            raise RuntimeError(lib.rn_last_error().decode())
        return {"energies": e, "energy": e.sum(), "forces": f, "virial": w.reshape(3, 3),
                "ms": float(ms.value)}

    def close(self):
        if self._h:
            _load().rn_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
