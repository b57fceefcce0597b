"""GPU parity of the skinny-M GEMV on the tensor cores (csrc/gemv_tc.cuh)
against the CPU oracle, through the C ABI.

The binder puts M >= 9 (StrictFp32) and M >= 2 (TF32) on this kernel when A
has a 16-byte row pitch; the tests check the launch record says so, then the
numbers: ragged N and K, every epilogue, and inf/NaN inputs, which the
StrictFp32 split turns into a whole-output recompute in the reference's
order (bit-identical to the oracle). Tolerances as in test_gemm_gpu.py.
"""
import numpy as np
import pytest

from momiru_b200 import BoundGemm, DeviceView, Epilogue, KernelMathMode, MatMulNode
from momiru_b200 import _abi, execution
from momiru_b200 import rng

pytestmark = pytest.mark.gpu

STRICT_TOL = 1e-5
TF32_TOL = 2e-3
STRICT = MatMulNode(math_mode=KernelMathMode.StrictFp32)
TF32 = MatMulNode(math_mode=KernelMathMode.Tf32, accuracy=execution.AccuracyContract.AllowTf32)


def rel_frob(x, ref):
    x = np.asarray(x, np.float64)
    ref = np.asarray(ref, np.float64)
    den = np.linalg.norm(ref)
    return float(np.linalg.norm(x - ref) / (den if den > 0 else 1.0))


def with_epilogue(base, epi):
    return MatMulNode(math_mode=base.math_mode, accuracy=base.accuracy, epilogue=epi)


def padded(arr):
    """Device copy whose rows are padded to 16 bytes, as the narrowed view
    (the TMA maps need 16-byte row pitches)."""
    rows, cols = arr.shape
    pc = (cols + 3) // 4 * 4
    phys = np.zeros((rows, pc), np.float32)
    phys[:, :cols] = arr
    return DeviceView.from_host(phys).narrow(1, 0, cols)


def run_tc(node_, a, b, bias=None, replays=1):
    """Bind (asserting the tensor-core GEMV was chosen), replay, quiesce; the
    output of every replay."""
    m, n = a.shape[0], b.shape[1]
    out = padded(np.zeros((m, n), np.float32))
    bv = DeviceView.from_host(bias) if bias is not None else None
    outs = []
    with BoundGemm(node_, padded(a), padded(b), out, bv) as g:
        rec = g.launch_record()
        assert g.family == "gemv" and rec.matrix_acceleration == _abi.ACCEL_TCGEN05, (m, n, node_.math_mode)
        for _ in range(replays):
            g.replay()
            g.quiesce_or_abort(60)
            outs.append(out.to_host())
    return outs[0] if replays == 1 else outs


@pytest.mark.parametrize("mode,m", [(STRICT, 9), (STRICT, 12), (STRICT, 16), (TF32, 2), (TF32, 5), (TF32, 16)])
@pytest.mark.parametrize("k,n", [(4096, 4096), (100, 130), (33, 260), (8192, 4100), (1, 128)])
def test_gemv_tc_ragged_bias_relu(oracle, mode, m, k, n):
    a = rng.randn((m, k), 31)
    b = rng.randn((k, n), 32)
    bias = rng.randn((n,), 33)
    ref = oracle.matmul(a, b, bias=bias, epilogue=oracle.EPI_BIAS_RELU)
    got = run_tc(with_epilogue(mode, Epilogue.BIAS_RELU), a, b, bias)
    tol = STRICT_TOL if mode is STRICT else TF32_TOL
    assert rel_frob(got, ref) <= tol


@pytest.mark.parametrize("epi", [Epilogue.NONE, Epilogue.BIAS, Epilogue.RELU, Epilogue.RELU6, Epilogue.BIAS_RELU6,
                                 Epilogue.GELU_ERF, Epilogue.BIAS_GELU_ERF, Epilogue.GELU_TANH,
                                 Epilogue.BIAS_GELU_TANH, Epilogue.SILU, Epilogue.BIAS_SILU])
def test_gemv_tc_every_epilogue(oracle, epi):
    a = rng.randn((16, 512), 34)
    b = rng.randn((512, 384), 35)
    bias = rng.randn((384,), 36, 0.5)
    ref = oracle.matmul(a, b, bias=bias, epilogue=int(epi))
    for mode in (STRICT, TF32):
        got = run_tc(with_epilogue(mode, epi), a, b, bias)
        assert rel_frob(got, ref) <= (STRICT_TOL if mode is STRICT else TF32_TOL), (epi, mode.math_mode)


def test_gemv_tc_strict_nonfinite_is_exact(oracle):
    """inf/NaN in A or B: the split would form inf * 0 in a cross term, so the
    whole output is recomputed in the reference's order, bit for bit."""
    a = rng.randn((16, 1000), 37)
    b = rng.randn((1000, 300), 38)
    a[3, 10] = np.inf
    a[7, 999] = np.nan
    b[500, 17] = -np.inf
    ref = oracle.matmul(a, b)
    # twice through one handle: the fix-up clears its flag after each run
    for got in run_tc(STRICT, a, b, replays=2):
        same = (got.view(np.uint32) == ref.view(np.uint32)) | (np.isnan(got) & np.isnan(ref))
        assert same.all()


def test_gemv_tc_tf32_nonfinite_propagates(oracle):
    a = rng.randn((8, 640), 40)
    b = rng.randn((640, 256), 41)
    a[2, 5] = np.nan
    b[100, 200] = np.inf
    ref = oracle.matmul(a, b)
    got = run_tc(TF32, a, b)
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    assert np.array_equal(np.isinf(got), np.isinf(ref))
    fin = np.isfinite(ref)
    assert rel_frob(got[fin], ref[fin]) <= TF32_TOL


def test_gemv_tc_replays_are_deterministic():
    """Fixed-order reduction over the K-slices: repeated runs are bit-identical."""
    a = DeviceView.from_host(rng.randn((16, 4096), 42))
    b = DeviceView.from_host(rng.randn((4096, 1024), 43))
    for mode in (STRICT, TF32):
        out = DeviceView.from_host(np.zeros((16, 1024), np.float32))
        with BoundGemm(mode, a, b, out) as g:
            g.replay()
            g.quiesce_or_abort(60)
            first = out.to_host()
            for _ in range(3):
                g.replay()
            g.quiesce_or_abort(60)
            assert np.array_equal(first.view(np.uint32), out.to_host().view(np.uint32)), mode.math_mode
