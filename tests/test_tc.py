"""The tcgen05 tensor-core GEMM (exact-integer products: power-of-two row / column scales, four
signed 7-bit digits per value, int32 accumulation in TMEM, one rounding of the float64
combination), called through the C ABI (rune_tc_selftest) on the layer shapes of the OAM models
(input projection 103 -> 256, FFN 256 <-> 512, EQ node / update layers 256 -> 640, 384 -> 192)
and on ragged ones, against a float64 product. Every output stays within 1e-6 of the sum of
|a b| (float32 rounding of the result included), and the errors carry no sign bias: their mean
is below 1e-8 of the sum of |a b| (a tf32 split accumulated in the tensor core's float32
accumulator rounds each step toward zero)."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from rune_b200.runtime import library as L

SHAPES = [(128, 128, 8), (512, 256, 103), (700, 512, 256), (512, 256, 512), (600, 640, 256),
          (1000, 192, 384), (513, 77, 13), (129, 300, 1)]


def _selftest(M, N, K, a, b):
    lib = L.load_library()
    c = np.zeros((M, N), np.float32)
    f = ctypes.POINTER(ctypes.c_float)
    status = lib.rune_tc_selftest(M, N, K, np.ascontiguousarray(a, np.float32).ctypes.data_as(f),
                                  np.ascontiguousarray(b, np.float32).ctypes.data_as(f),
                                  c.ctypes.data_as(f), 0)
    L.check(lib, status)
    return c


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", SHAPES)
def test_tc_gemm_is_float32_accurate(M, N, K):
    rng = np.random.default_rng(M * 7 + N * 3 + K)
    a = (rng.normal(size=(M, K)) * np.exp(rng.normal(size=(M, K)))).astype(np.float32)
    b = rng.normal(size=(K, N)).astype(np.float32)
    c = _selftest(M, N, K, a, b)
    ref = a.astype(np.float64) @ b.astype(np.float64)
    scale = np.abs(a.astype(np.float64)) @ np.abs(b.astype(np.float64))
    err = (c - ref) / scale
    rel = float(np.max(np.abs(err)))
    bias = float(abs(np.mean(err)))
    print(M, N, K, "max |c - ref| / sum|a b| =", rel, "mean =", bias)
    assert rel < 1e-6, rel
    assert bias < 1e-8, bias


@pytest.mark.gpu
def test_tc_gemm_rows_and_columns_are_not_mixed():
    """One nonzero in A and one in B select exactly one output element."""
    M, N, K = 300, 200, 24
    for m0, n0, k0 in ((0, 0, 0), (131, 5, 7), (299, 199, 23), (64, 128, 16)):
        a = np.zeros((M, K), np.float32)
        b = np.zeros((K, N), np.float32)
        a[m0, k0] = 1.5
        b[k0, n0] = -2.0
        c = _selftest(M, N, K, a, b)
        expect = np.zeros((M, N), np.float32)
        expect[m0, n0] = -3.0
        np.testing.assert_array_equal(c, expect)


def test_selftest_rejects_bad_sizes():
    lib = L.load_library()
    f = ctypes.POINTER(ctypes.c_float)
    buf = np.zeros(4, np.float32).ctypes.data_as(f)
    assert lib.rune_tc_selftest(0, 4, 4, buf, buf, buf, 0) == L.RUNE_ERR_INVALID
    assert lib.rune_tc_selftest(4, 4097, 4, buf, buf, buf, 0) == L.RUNE_ERR_INVALID
