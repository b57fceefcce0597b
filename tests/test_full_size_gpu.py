"""Parity at the full sizes of the headline configurations, against the
oracle (the restated reference CPU GEMM), through the C ABI.

  C3   8192^3 + bias + ReLU: the whole output, StrictFp32 (<= 1e-5 relative
       Frobenius) and TF32 (<= 2e-3); the oracle runs once on every host core
       (the reference order is per element, so row-sharding it is bit-exact).
  C5a  the real batch of 512 x 1024^3: 16 batch entries spread over the whole
       range (first and last included), each in full; both modes.
  C4   4096 x 4096 x 11008 through the transposed-lhs and column-slice views:
       512 rows spread over the output; both modes.
"""
import os

import numpy as np
import pytest

from momiru_b200 import BoundGemm, DeviceView, Epilogue, KernelMathMode, MatMulNode
from momiru_b200 import execution, rng

pytestmark = pytest.mark.gpu

STRICT_TOL = 1e-5
TF32_TOL = 2e-3
STRICT = MatMulNode(math_mode=KernelMathMode.StrictFp32, epilogue=Epilogue.BIAS_RELU)
TF32 = MatMulNode(math_mode=KernelMathMode.Tf32, epilogue=Epilogue.BIAS_RELU,
                  accuracy=execution.AccuracyContract.AllowTf32)
CORES = os.cpu_count() or 1


def rel_frob(x, ref):
    x = np.asarray(x, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.linalg.norm(x - ref) / max(np.linalg.norm(ref), 1e-30))


def bound_run(node, a, b, out, bias=None):
    with BoundGemm(node, a, b, out, bias) as g:
        assert g.family == "tcgen05"
        g.replay()
        g.quiesce_or_abort(120)


def test_c3_whole_output_against_the_oracle(oracle):
    n = 8192
    a = rng.randu((n, n), 1)
    b = rng.randu((n, n), 2)
    bias = rng.randn((n,), 3, 0.1)
    ref = oracle.matmul(a, b, bias=bias, epilogue=oracle.EPI_BIAS_RELU, nthreads=CORES)
    da, db, dbias = DeviceView.from_host(a), DeviceView.from_host(b), DeviceView.from_host(bias)
    out = DeviceView.empty((n, n))
    for nd, tol in ((STRICT, STRICT_TOL), (TF32, TF32_TOL)):
        bound_run(nd, da, db, out, dbias)
        got = out.to_host()
        assert np.isfinite(got).all()
        err = rel_frob(got, ref)
        assert err <= tol, (nd.math_mode, err)
        # every row on its own is within the bar too (no tile or row is off)
        row_err = np.linalg.norm(got.astype(np.float64) - ref, axis=1) / np.maximum(
            np.linalg.norm(ref.astype(np.float64), axis=1), 1e-30)
        assert float(row_err.max()) <= 4 * tol, (nd.math_mode, float(row_err.max()))
        # ReLU writes +0, never -0, wherever the reference has 0
        assert not np.any(np.signbit(got))


def test_c5a_real_batch_512_sampled_entries(oracle):
    import torch
    bsz, n = 512, 1024
    a = oracle.randu(bsz * n * n, 1).reshape(bsz, n, n)
    b = oracle.randu(bsz * n * n, 2).reshape(bsz, n, n)
    da, db = DeviceView.from_host(a), DeviceView.from_host(b)
    out = DeviceView.empty((bsz, n, n))
    picks = sorted(set(np.linspace(0, bsz - 1, 16).astype(int).tolist()))
    refs = [oracle.matmul(a[i], b[i], nthreads=CORES) for i in picks]
    for node, tol in ((MatMulNode(math_mode=KernelMathMode.StrictFp32), STRICT_TOL),
                      (MatMulNode(math_mode=KernelMathMode.Tf32, accuracy=execution.AccuracyContract.AllowTf32),
                       TF32_TOL)):
        bound_run(node, da, db, out)
        got = out.torch_view()[picks].cpu().numpy()
        torch.cuda.synchronize()
        for j, i in enumerate(picks):
            assert rel_frob(got[j], refs[j]) <= tol, (node.math_mode, i)


def test_c4_full_size_512_rows(oracle):
    m, k, n, n_phys = 4096, 4096, 11008, 12288
    x = rng.randn((k, m), 1, 0.02)          # A = X^T
    w = rng.randn((k, n_phys), 2, 0.02)     # B = W[:, :n]
    rows = np.unique(np.linspace(0, m - 1, 512).astype(np.int64))
    ref = oracle.matmul(x.T, w[:, :n], rows=rows, nthreads=CORES)
    out = DeviceView.empty((m, n))
    dx, dw = DeviceView.from_host(x).transpose(), DeviceView.from_host(w).narrow(1, 0, n)
    for node, tol in ((MatMulNode(math_mode=KernelMathMode.StrictFp32), STRICT_TOL),
                      (MatMulNode(math_mode=KernelMathMode.Tf32, accuracy=execution.AccuracyContract.AllowTf32),
                       TF32_TOL)):
        bound_run(node, dx, dw, out)
        got = out.torch_view()[rows.tolist()].cpu().numpy()
        assert rel_frob(got, ref) <= tol, node.math_mode
