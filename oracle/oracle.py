"""ctypes loader for the CPU oracle -- TEST INFRASTRUCTURE ONLY.

The oracle restates the reference CPU GEMM (gemm_dot_f32 / gemm_axpy_f32 /
gemm_avx2, src/momiru/tensor_light/execution/cpu.rs:2989-3098), the epilogue
activations relu / relu6 / silu / gelu_erf / gelu_tanh_approx (cpu.rs:2031-2168,
2214-2222) and the SplitMix64 input generators
(src/momiru/tensor_light/tensor.rs:1467-1500, 1809-1840) in C. Only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline leg import this module; the
product path never does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle_gemm.so")
_lib = None

EPI_NONE, EPI_BIAS, EPI_BIAS_RELU, EPI_RELU = 0, 1, 2, 3
EPI_RELU6, EPI_BIAS_RELU6, EPI_GELU_ERF, EPI_BIAS_GELU_ERF = 4, 5, 6, 7
EPI_GELU_TANH, EPI_BIAS_GELU_TANH, EPI_SILU, EPI_BIAS_SILU = 8, 9, 10, 11

_i64 = ctypes.c_int64
_vp = ctypes.c_void_p


def build(force: bool = False) -> str:
    """Compile the oracle with its Makefile (gcc, -ffp-contract=off)."""
    src = os.path.join(_HERE, "gemm_oracle.c")
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE, "liboracle_gemm.so"], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        l = ctypes.CDLL(_LIB_PATH)
        l.oracle_gemm.restype = ctypes.c_int
        l.oracle_gemm.argtypes = [_i64] * 4 + [_vp, _i64, _i64, _i64] * 2 + [_vp, _i64, _i64, _i64,
                                  _vp, ctypes.c_int, _vp, _i64, ctypes.c_int]
        l.oracle_gemm_f64.restype = ctypes.c_int
        l.oracle_gemm_f64.argtypes = [_i64] * 4 + [_vp, _i64, _i64, _i64] * 2 + [_vp, _vp, _i64]
        l.oracle_gemm_avx2_restated.restype = ctypes.c_int
        l.oracle_gemm_avx2_restated.argtypes = [_i64, _i64, _i64, _vp, _vp, _vp, _i64, _i64, ctypes.c_int]
        l.oracle_randu.argtypes = [_vp, _i64, ctypes.c_uint64, ctypes.c_float, ctypes.c_float]
        l.oracle_randn.argtypes = [_vp, _i64, ctypes.c_uint64, ctypes.c_float]
        l.oracle_splitmix64_words.argtypes = [ctypes.c_uint64, _vp, _i64]
        l.oracle_relu.argtypes = [_vp, _i64]
        l.oracle_activation.restype = ctypes.c_int
        l.oracle_activation.argtypes = [_vp, _i64, ctypes.c_int]
        l.oracle_selfcheck_kat.restype = ctypes.c_int
        _lib = l
    return _lib


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def randu(n: int, seed: int, lo: float = -1.0, hi: float = 1.0) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    lib().oracle_randu(_ptr(out), n, seed, lo, hi)
    return out


def randn(n: int, seed: int, sigma: float = 1.0) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    lib().oracle_randn(_ptr(out), n, seed, sigma)
    return out


def splitmix64_words(seed: int, n: int) -> np.ndarray:
    out = np.empty(n, dtype=np.uint64)
    lib().oracle_splitmix64_words(seed, _ptr(out), n)
    return out


def relu(x: np.ndarray) -> np.ndarray:
    y = np.ascontiguousarray(x, dtype=np.float32).copy()
    lib().oracle_relu(_ptr(y), y.size)
    return y


def activation(x: np.ndarray, epilogue: int) -> np.ndarray:
    """The epilogue's activation (its bias part ignored) applied elementwise."""
    y = np.ascontiguousarray(x, dtype=np.float32).copy()
    if lib().oracle_activation(_ptr(y), y.size, epilogue):
        raise ValueError(f"bad epilogue code {epilogue}")
    return y


def _strides3(view: np.ndarray, batched: bool):
    s = [st // 4 for st in view.strides]
    if batched:
        return s[0], s[1], s[2]
    return 0, s[0], s[1]


def matmul(a: np.ndarray, b: np.ndarray, bias: np.ndarray | None = None, epilogue: int = EPI_NONE,
           rows: np.ndarray | None = None, nthreads: int = 0) -> np.ndarray:
    """Reference-arithmetic matmul of f32 views a [.., M, K] and b [.., K, N].

    a and b are numpy views (any element strides, e.g. a.T); a rank-3 operand
    with batch 1, or a rank-2 operand against a rank-3 one, broadcasts. With
    `rows`, only those output rows are computed (returned compactly).
    """
    assert a.dtype == np.float32 and b.dtype == np.float32
    assert a.ndim in (2, 3) and b.ndim in (2, 3)
    batch = max(a.shape[0] if a.ndim == 3 else 1, b.shape[0] if b.ndim == 3 else 1)
    m, k = a.shape[-2:]
    k2, n = b.shape[-2:]
    assert k == k2
    a_sb, a_sm, a_sk = _strides3(a, a.ndim == 3 and a.shape[0] != 1)
    b_sb, b_sk, b_sn = _strides3(b, b.ndim == 3 and b.shape[0] != 1)
    out_rows = m if rows is None else len(rows)
    c = np.empty((batch, out_rows, n), dtype=np.float32)
    rows_arr = None if rows is None else np.ascontiguousarray(rows, dtype=np.int64)
    bias_arr = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    rc = lib().oracle_gemm(batch, m, n, k,
                           _ptr(a), a_sb, a_sm, a_sk,
                           _ptr(b), b_sb, b_sk, b_sn,
                           _ptr(c), out_rows * n, n, 1,
                           None if bias_arr is None else _ptr(bias_arr), epilogue,
                           None if rows_arr is None else _ptr(rows_arr), out_rows, nthreads)
    if rc:
        raise RuntimeError(f"oracle_gemm failed: {rc}")
    return c if (a.ndim == 3 or b.ndim == 3) else c[0]


def matmul_f64(a: np.ndarray, b: np.ndarray, rows: np.ndarray | None = None) -> np.ndarray:
    """fp64 comparator with the same indexing (error attribution only)."""
    batch = max(a.shape[0] if a.ndim == 3 else 1, b.shape[0] if b.ndim == 3 else 1)
    m, k = a.shape[-2:]
    n = b.shape[-1]
    a_sb, a_sm, a_sk = _strides3(a, a.ndim == 3 and a.shape[0] != 1)
    b_sb, b_sk, b_sn = _strides3(b, b.ndim == 3 and b.shape[0] != 1)
    out_rows = m if rows is None else len(rows)
    c = np.empty((batch, out_rows, n), dtype=np.float64)
    rows_arr = None if rows is None else np.ascontiguousarray(rows, dtype=np.int64)
    rc = lib().oracle_gemm_f64(batch, m, n, k, _ptr(a), a_sb, a_sm, a_sk, _ptr(b), b_sb, b_sk, b_sn,
                               _ptr(c), None if rows_arr is None else _ptr(rows_arr), out_rows)
    if rc:
        raise RuntimeError(f"oracle_gemm_f64 failed: {rc}")
    return c if (a.ndim == 3 or b.ndim == 3) else c[0]


def gemm_avx2_restated(a: np.ndarray, b: np.ndarray, row0: int = 0, row1: int | None = None,
                       nthreads: int = 0) -> np.ndarray:
    """gemm_avx2's loop structure (row-major contiguous A [M,K], B [K,N]);
    rows [row0,row1) of C are computed, the rest of the returned array is 0."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    m, k = a.shape
    n = b.shape[1]
    row1 = m if row1 is None else row1
    c = np.zeros((m, n), dtype=np.float32)
    rc = lib().oracle_gemm_avx2_restated(m, n, k, _ptr(a), _ptr(b), _ptr(c), row0, row1, nthreads)
    if rc:
        raise RuntimeError(f"oracle_gemm_avx2_restated failed: {rc}")
    return c


def selfcheck_kat() -> int:
    return lib().oracle_selfcheck_kat()
