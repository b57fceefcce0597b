"""The allocation-free entry point, mmr_gemm_run_noalloc, called through the C ABI.

It exists for callers that may not allocate device memory where they launch
(an allocator that owns all of HBM, a path that cannot absorb cudaMalloc's
device synchronisation, a caller with nowhere to keep a bound handle). Its
scratch is a fixed array inside the library, shared by every call on a device.
These tests compare it with the ordinary bind/run entry point on two calls in
a row -- the first with inf/NaN inputs, so the second proves the shared scratch
was cleared -- and with the oracle directly, over both transpose flags and a
batched product with a broadcast rhs (the allocation-free entry point is the
only caller of the one-CTA 3xTF32 kernel at large M, in every operand
layout), and check that an oversized problem is refused before launch.
This file is named to be collected last.
"""
import ctypes

import numpy as np
import pytest

from momiru_b200 import BoundGemm, DeviceBuffer, DeviceView, Epilogue, KernelMathMode, MatMulNode, rng
from momiru_b200 import _abi, execution

pytestmark = pytest.mark.gpu

STRICT_TOL = 1e-5  # the StrictFp32 tolerance used by the other GPU tests
NODE = MatMulNode(math_mode=KernelMathMode.StrictFp32, epilogue=Epilogue.BIAS_RELU)


def rel_frob(x, ref):
    x = np.asarray(x, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.linalg.norm(x - ref) / max(np.linalg.norm(ref), 1e-30))


def bound_path(a, b, bias, out_dims, node=NODE):
    out = DeviceView.empty(out_dims)
    with BoundGemm(node, a, b, out, bias) as g:
        g.replay()
        g.quiesce_or_abort(60)
    return out.to_host()


def noalloc_call(a, b, bias, out, stream, status, node=NODE):
    desc = execution._desc(node, a, b, out, bias, stream)
    return _abi.load().mmr_gemm_run_noalloc(ctypes.byref(desc), ctypes.cast(status.data_ptr(),
                                                                            ctypes.POINTER(ctypes.c_int32)))


@pytest.fixture(scope="module")
def oracle():
    from oracle import oracle as O
    O.build()
    return O


def test_noalloc_matches_bound_entry_point_on_two_calls(oracle):
    import torch
    m, k, n = 1000, 768, 1300      # ragged M and N: 8 x 6 = 48 output tiles
    a1 = rng.randn((m, k), 21)
    a1[17, 5] = np.inf             # first call: tiles with non-finite inputs
    a1[650, 600] = np.nan
    a2 = rng.randn((m, k), 22)     # second call: ordinary inputs
    b = rng.randn((k, n), 23)
    bias = rng.randn((n,), 24, 0.1)
    db, dbias = DeviceView.from_host(b), DeviceView.from_host(bias)
    stream = torch.cuda.current_stream().cuda_stream
    status = torch.full((1,), -1, dtype=torch.int32).pin_memory()

    for a_host in (a1, a2):
        da = DeviceView.from_host(a_host)
        want = bound_path(da, db, dbias, (m, n))
        out = DeviceView.from_host(np.full((m, n), 5.0, np.float32))
        assert noalloc_call(da, db, dbias, out, stream, status) == _abi.OK, _abi.last_error()
        torch.cuda.synchronize()
        assert int(status[0]) == 0
        got = out.to_host()
        assert np.array_equal(np.isnan(got), np.isnan(want))
        assert np.array_equal(np.isinf(got), np.isinf(want))
        fin = np.isfinite(want)
        assert rel_frob(got[fin], want[fin]) <= STRICT_TOL
        ref = oracle.matmul(a_host, b, bias=bias, epilogue=oracle.EPI_BIAS_RELU)
        assert np.array_equal(np.isnan(got), np.isnan(ref)) and np.array_equal(np.isinf(got), np.isinf(ref))
        assert rel_frob(got[np.isfinite(ref)], ref[np.isfinite(ref)]) <= STRICT_TOL
    assert np.isfinite(got).all()


@pytest.mark.parametrize("ta,tb", [(False, False), (True, False), (False, True), (True, True)])
def test_noalloc_transposed_operands_against_oracle_and_bound_path(oracle, ta, tb):
    """Both transpose flags (MN-major A, K-major B tiles through TMA), M large
    enough for many 128-row tiles, against the oracle and the bound path."""
    import torch
    m, k, n = 700, 320, 520
    a = rng.randn((k, m) if ta else (m, k), 31)
    b = rng.randn((n, k) if tb else (k, n), 32)
    bias = rng.randn((n,), 33, 0.1)
    node = MatMulNode(transpose_lhs=ta, transpose_rhs=tb, math_mode=KernelMathMode.StrictFp32,
                      epilogue=Epilogue.BIAS_RELU)
    ref = oracle.matmul(a.T if ta else a, b.T if tb else b, bias=bias, epilogue=oracle.EPI_BIAS_RELU)
    da, db, dbias = DeviceView.from_host(a), DeviceView.from_host(b), DeviceView.from_host(bias)
    want = bound_path(da, db, dbias, (m, n), node)
    stream = torch.cuda.current_stream().cuda_stream
    status = torch.full((1,), -1, dtype=torch.int32).pin_memory()
    for _ in range(2):
        out = DeviceView.from_host(np.full((m, n), 7.0, np.float32))
        assert noalloc_call(da, db, dbias, out, stream, status, node) == _abi.OK, _abi.last_error()
        torch.cuda.synchronize()
        assert int(status[0]) == 0
        got = out.to_host()
        assert rel_frob(got, ref) <= STRICT_TOL
        assert rel_frob(got, want) <= STRICT_TOL


def test_noalloc_batched_broadcast_rhs_against_oracle(oracle):
    """A batch of 6 lhs matrices against one broadcast rhs (rank 3 x rank 2)."""
    import torch
    bsz, m, k, n = 6, 200, 96, 300
    a = rng.randn((bsz, m, k), 34)
    b = rng.randn((k, n), 35)
    bias = rng.randn((n,), 36, 0.1)
    ref = oracle.matmul(a, b, bias=bias, epilogue=oracle.EPI_BIAS_RELU)
    da, db, dbias = DeviceView.from_host(a), DeviceView.from_host(b), DeviceView.from_host(bias)
    stream = torch.cuda.current_stream().cuda_stream
    status = torch.full((1,), -1, dtype=torch.int32).pin_memory()
    out = DeviceView.from_host(np.zeros((bsz, m, n), np.float32))
    assert noalloc_call(da, db, dbias, out, stream, status) == _abi.OK, _abi.last_error()
    torch.cuda.synchronize()
    assert int(status[0]) == 0
    assert rel_frob(out.to_host(), ref) <= STRICT_TOL
    assert rel_frob(out.to_host(), bound_path(da, db, dbias, (bsz, m, n))) <= STRICT_TOL


def test_noalloc_refuses_problems_beyond_its_scratch():
    # 64 x 129 x 1 tiles > MMR_NOALLOC_MAX_TILES; refused before any launch.
    m, n, k = 128 * 64, 256 * 129, 32
    G = 1 << 36
    a = DeviceView.contiguous(DeviceBuffer(G, 4 * m * k, 0), (m, k))
    b = DeviceView.contiguous(DeviceBuffer(2 * G, 4 * k * n, 0), (k, n))
    out = DeviceView.contiguous(DeviceBuffer(3 * G, 4 * m * n, 0), (m, n))
    desc = execution._desc(MatMulNode(), a, b, out, None, None)
    rc = _abi.load().mmr_gemm_run_noalloc(ctypes.byref(desc), None)
    assert rc == _abi.ERR_INVALID_SHAPE
    assert "at most" in _abi.last_error() and str(_abi.NOALLOC_MAX_TILES) in _abi.last_error()
    # and it runs only the StrictFp32 tcgen05 kernel
    desc = execution._desc(MatMulNode(math_mode=KernelMathMode.Tf32,
                                      accuracy=execution.AccuracyContract.AllowTf32),
                           DeviceView.contiguous(DeviceBuffer(G, 4 * 64 * 64, 0), (64, 64)),
                           DeviceView.contiguous(DeviceBuffer(2 * G, 4 * 64 * 64, 0), (64, 64)),
                           DeviceView.contiguous(DeviceBuffer(3 * G, 4 * 64 * 64, 0), (64, 64)), None, None)
    assert _abi.load().mmr_gemm_run_noalloc(ctypes.byref(desc), None) == _abi.ERR_UNSUPPORTED_MATH
