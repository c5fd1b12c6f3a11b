"""ctypes binding of the engine's C ABI (``include/rune_b200.h``).

The library is the only compute path: if it is missing or cannot be loaded, every model call
raises. Status codes map to the reference's exception classes (``ValueError`` for bad input and
neighbour overflow, ``RuntimeError`` for CUDA failures, ``MemoryError`` for allocation).
"""

from __future__ import annotations

import ctypes
import os
from ctypes import (POINTER, c_char_p, c_double, c_float, c_int, c_int32, c_int64, c_uint8,
                    c_uint32, c_void_p)
from pathlib import Path

from .build import LIB

RUNE_OK = 0
RUNE_ERR_INVALID = 1
RUNE_ERR_CUDA = 2
RUNE_ERR_NEIGHBOR_OVERFLOW = 3
RUNE_ERR_TYPE = 4
RUNE_ERR_OOM = 5
RUNE_ERR_STATE = 6
RUNE_ERR_RETRY = 7
DEFAULT_WAIT_POLLS = 4194304  # RUNE_DEFAULT_WAIT_POLLS
RUNE_HALO_FILL, RUNE_HALO_REDUCE = 0, 1
# rune_halo_fn: int (*)(void* ctx, int32 op, float* rows, int32 row_floats, void* stream)
HALO_FN = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p,
                           ctypes.c_int32, ctypes.c_void_p)

RUNE_NEP, RUNE_MOBIUS_LOCAL, RUNE_MOBIUS_MP, RUNE_MOBIUS_EQ = 0, 1, 2, 3
RUNE_ACT = {"tanh": 0, "silu": 1, "swish": 1, "gelu": 2}
RUNE_ZBL_NONE, RUNE_ZBL_UNIVERSAL, RUNE_ZBL_FLEXIBLE = 0, 1, 2
RUNE_FORCES, RUNE_VIRIAL = 1, 2

EXPORTED = [
    "rune_engine_create", "rune_engine_set_tensor", "rune_engine_finalize",
    "rune_engine_compute", "rune_engine_compute_padded", "rune_engine_compute_padded_static",
    "rune_engine_neighbor_pairs",
    "rune_engine_stats", "rune_engine_set_profiling", "rune_engine_kernel_stat",
    "rune_engine_set_wait_polls",
    "rune_engine_reset_kernel_stats", "rune_engine_destroy", "rune_last_error",
    "rune_md_nve", "rune_engine_compute_domain", "rune_engine_compute_halo",
    "rune_tc_selftest",
]


class RuneError(RuntimeError):
    """A failure reported by the CUDA engine."""


class HaloRetry(RuntimeError):
    """A halo call ended after every exchange with its neighbour rows regrown: every rank
    repeats the call."""


class ModelConfig(ctypes.Structure):
    _fields_ = [
        ("kind", c_int32), ("n_types", c_int32),
        ("rc_radial", c_double), ("rc_angular", c_double),
        ("n_desc_radial", c_int32), ("n_desc_angular", c_int32), ("k_max_radial", c_int32),
        ("k_max_angular", c_int32), ("l_max", c_int32),
        ("has_q222", c_int32), ("has_q1111", c_int32), ("has_q112", c_int32),
        ("has_q123", c_int32), ("has_q233", c_int32), ("has_q134", c_int32),
        ("max_neighbors_radial", c_int32), ("max_neighbors_angular", c_int32),
        ("nep_hidden", c_int32),
        ("hidden_dim", c_int32), ("ffn_dim", c_int32), ("blocks", c_int32),
        ("activation", c_int32), ("message_layers", c_int32), ("message_dim", c_int32),
        ("pair_dim", c_int32),
        ("message_groups", c_int32), ("vector_channels", c_int32),
        ("equivariant_channels", c_int32), ("equivariant_l_max", c_int32),
        ("message_basis_size", c_int32),
        ("message_cutoff", c_double), ("norm_eps", c_double),
        ("zbl_mode", c_int32),
        ("zbl_rc_inner", c_double), ("zbl_rc_outer", c_double),
    ]


class Stats(ctypes.Structure):
    _fields_ = [
        ("calls", c_int64), ("neighbor_builds", c_int64), ("last_edges", c_int64),
        ("last_radial_edges", c_int64), ("last_angular_edges", c_int64),
        ("workspace_bytes", c_int64), ("workspace_grows", c_int64),
        ("kernel_launches", c_int64), ("tensor_core_layers", c_int64),
    ]


_LIB = None


def library_path() -> Path:
    return LIB


def load_library(path: Path | None = None):
    """Load (once) and type the engine library. Raises ImportError when it is absent."""
    global _LIB
    if _LIB is not None and path is None:
        return _LIB
    target = Path(path) if path else Path(os.environ.get("RUNE_B200_LIBRARY", str(LIB)))
    if not target.exists():
        raise ImportError(
            f"rune_b200 CUDA library not found at {target}; build it with "
            "`python -m rune_b200.runtime.build` (nvcc, sm_100a). There is no CPU fallback.")
    lib = ctypes.CDLL(str(target))
    eng = c_void_p
    lib.rune_engine_create.argtypes = [POINTER(ModelConfig), c_int, POINTER(eng)]
    lib.rune_engine_set_tensor.argtypes = [eng, c_char_p, POINTER(c_float), c_int64]
    lib.rune_engine_finalize.argtypes = [eng]
    lib.rune_engine_compute.argtypes = [
        eng, c_int32, c_int32, c_void_p, c_void_p, POINTER(c_double), POINTER(c_uint8),
        POINTER(c_int32), c_int32, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]
    lib.rune_engine_compute_padded.argtypes = [
        eng, c_int32, c_int32, c_void_p, c_void_p, c_void_p, c_int32, c_void_p, c_void_p,
        c_int32, c_void_p, POINTER(c_int32), c_int32, c_void_p, c_void_p, c_void_p, c_void_p,
        c_void_p]
    lib.rune_engine_compute_padded_static.argtypes = lib.rune_engine_compute_padded.argtypes
    lib.rune_engine_compute_domain.argtypes = [
        eng, c_int32, c_int32, POINTER(c_int32), c_void_p, c_void_p, POINTER(c_double),
        c_int32, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]
    lib.rune_engine_neighbor_pairs.argtypes = [eng, c_int32, POINTER(c_int32), c_int64,
                                               POINTER(c_int64)]
    lib.rune_engine_stats.argtypes = [eng, POINTER(Stats)]
    lib.rune_engine_set_profiling.argtypes = [eng, c_int32]
    lib.rune_engine_set_wait_polls.argtypes = [eng, c_uint32]
    lib.rune_engine_kernel_stat.argtypes = [eng, c_int32, c_char_p, c_int32, POINTER(c_double),
                                            POINTER(c_int64)]
    lib.rune_engine_reset_kernel_stats.argtypes = [eng]
    lib.rune_engine_destroy.argtypes = [eng]
    lib.rune_engine_destroy.restype = None
    lib.rune_last_error.restype = c_char_p
    lib.rune_md_nve.argtypes = [
        eng, c_int32, c_void_p, c_void_p, c_void_p, c_void_p, POINTER(c_double),
        POINTER(c_uint8), c_double, c_int32, c_double, POINTER(c_double), c_void_p,
        POINTER(c_int64), c_void_p]
    lib.rune_engine_compute_halo.argtypes = [
        eng, c_int32, c_int32, c_void_p, c_void_p, POINTER(c_double), c_int32, HALO_FN,
        c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]
    lib.rune_tc_selftest.argtypes = [c_int32, c_int32, c_int32, POINTER(c_float),
                                     POINTER(c_float), POINTER(c_float), c_int32]
    for name in EXPORTED:
        if name not in ("rune_engine_destroy", "rune_last_error"):
            getattr(lib, name).restype = c_int
    if path is None:
        _LIB = lib
    return lib


def check(lib, status: int):
    if status == RUNE_OK:
        return
    message = (lib.rune_last_error() or b"").decode(errors="replace")
    if status in (RUNE_ERR_INVALID, RUNE_ERR_NEIGHBOR_OVERFLOW, RUNE_ERR_TYPE):
        raise ValueError(message)
    if status == RUNE_ERR_OOM:
        raise MemoryError(message)
    if status == RUNE_ERR_RETRY:
        raise HaloRetry(message)
    raise RuneError(f"rune_b200 error {status}: {message}")
