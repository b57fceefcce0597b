"""The MatMul node over operands in host memory (mmr_gemm_bind_host): copies
in, row-panel GEMMs and copies out overlapped on three streams. Parity against
the oracle through the C ABI; host row padding never written; replays see new
host inputs; pinned and pageable host memory both work."""
import numpy as np
import pytest

from momiru_b200 import Epilogue, HostGemm, KernelFamily, KernelMathMode, MatMulNode, execution
from momiru_b200 import rng

pytestmark = pytest.mark.gpu

STRICT_TOL = 1e-5
TF32_TOL = 2e-3


def rel_frob(x, ref):
    x = np.asarray(x, np.float64)
    ref = np.asarray(ref, np.float64)
    den = np.linalg.norm(ref)
    return float(np.linalg.norm(x - ref) / (den if den > 0 else 1.0))


def pinned(shape):
    import torch
    return torch.empty(shape, dtype=torch.float32, pin_memory=True).numpy()


def host(arr, pad=0, pin=True):
    """A host copy of `arr` whose rows carry `pad` extra columns, returned as
    the narrowed (logical) view."""
    arr = np.asarray(arr, np.float32)
    if arr.ndim == 1:
        out = pinned(arr.shape) if pin else np.empty(arr.shape, np.float32)
        out[...] = arr
        return out
    phys = pinned((arr.shape[0], arr.shape[1] + pad)) if pin else np.empty((arr.shape[0], arr.shape[1] + pad),
                                                                            np.float32)
    phys[...] = 7.0
    phys[:, :arr.shape[1]] = arr
    return phys[:, :arr.shape[1]]


@pytest.mark.parametrize("m,k,n,panels,mode,epi,trans_b,pad", [
    (1000, 300, 777, 3, "strict", Epilogue.BIAS_RELU, False, 5),
    (2304, 512, 1024, 4, "tf32", Epilogue.BIAS_GELU_ERF, False, 0),
    (256, 64, 128, 1, "strict", Epilogue.NONE, True, 3),
    (1537, 1000, 260, 0, "strict", Epilogue.SILU, True, 0),
    (5, 4096, 1024, 4, "strict", Epilogue.BIAS, False, 0),     # skinny: the GEMV family, one panel
])
def test_host_gemm_matches_oracle(oracle, m, k, n, panels, mode, epi, trans_b, pad):
    a = rng.randu((m, k), 51)
    b = rng.randu((k, n), 52)
    bias = rng.randn((n,), 53, 0.2)
    ref = oracle.matmul(a, b, bias=bias if epi.has_bias else None, epilogue=int(epi))
    node = MatMulNode(math_mode=KernelMathMode.StrictFp32 if mode == "strict" else KernelMathMode.Tf32,
                      accuracy=(execution.AccuracyContract.StrictFp32 if mode == "strict"
                                else execution.AccuracyContract.AllowTf32),
                      epilogue=epi, transpose_rhs=trans_b)
    ha = host(a, pad)
    hb = host(np.ascontiguousarray(b.T) if trans_b else b, pad)
    out = host(np.zeros((m, n), np.float32), pad + 2)
    with HostGemm(node, ha, hb, out, host(bias) if epi.has_bias else None, panels=panels) as g:
        g.replay()
        g.quiesce_or_abort(60)
        first = out.copy()
        g.replay()
        g.quiesce_or_abort(60)
        fam = g.family
    tol = STRICT_TOL if mode == "strict" else TF32_TOL
    assert rel_frob(first, ref) <= tol, (m, k, n, fam)
    assert np.array_equal(first.view(np.uint32), out.view(np.uint32))
    assert np.all(out.base[:, n:] == 7.0)  # the host rows' padding is never written
    assert fam == ("gemv" if m <= 16 else "tcgen05")


def test_host_gemm_replays_see_new_inputs_and_pageable_memory(oracle):
    m, k, n = 700, 256, 300
    a1, a2 = rng.randn((m, k), 61), rng.randn((m, k), 62)
    b = rng.randn((k, n), 63)
    ha = host(a1, pin=False)
    hb = host(b, pin=False)
    out = host(np.zeros((m, n), np.float32), 4, pin=False)
    with HostGemm(MatMulNode(), ha, hb, out, panels=2) as g:
        g.replay()
        g.quiesce_or_abort(60)
        assert rel_frob(out, oracle.matmul(a1, b)) <= STRICT_TOL
        ha[...] = a2
        g.replay()
        g.quiesce_or_abort(60)
        assert rel_frob(out, oracle.matmul(a2, b)) <= STRICT_TOL


def test_host_gemm_orders_with_the_callers_stream(oracle):
    """Work enqueued on the caller's stream after a replay sees its output."""
    import torch
    m, k, n = 512, 128, 256
    a = rng.randu((m, k), 71)
    b = rng.randu((k, n), 72)
    ha, hb, out = host(a), host(b), host(np.zeros((m, n), np.float32))
    s = torch.cuda.Stream()
    dev_copy = torch.empty((m, n), dtype=torch.float32, device="cuda:0")
    with HostGemm(MatMulNode(), ha, hb, out, panels=2, stream=s.cuda_stream) as g:
        g.replay()
        with torch.cuda.stream(s):
            dev_copy.copy_(torch.from_numpy(out), non_blocking=True)  # ordered after the copy-out
        s.synchronize()
        g.quiesce_or_abort(60)
    assert np.array_equal(dev_copy.cpu().numpy(), out)
    assert rel_frob(out, oracle.matmul(a, b)) <= STRICT_TOL


def test_host_gemm_exact_family_bit_identical(oracle):
    a = rng.randn((300, 77), 81)
    b = rng.randn((77, 45), 82)
    node = MatMulNode(math_mode=KernelMathMode.Exact, accuracy=execution.AccuracyContract.Exact,
                      family=KernelFamily.Simt, epilogue=Epilogue.RELU)
    out = host(np.zeros((300, 45), np.float32), 3)
    with HostGemm(node, host(a, 1), host(b), out, panels=2) as g:
        g.replay()
        g.quiesce_or_abort(60)
    ref = oracle.matmul(a, b, epilogue=oracle.EPI_RELU)
    assert np.array_equal(np.ascontiguousarray(out).view(np.uint32), ref.view(np.uint32))
