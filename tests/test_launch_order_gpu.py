"""Stream order under programmatic dependent launch.

Every kernel of the library is launched so that its prologue may overlap the
previous kernel's tail, and waits (griddepcontrol.wait) before its first
global access. These tests chain nodes of different families on one stream
with no synchronisation in between, where each node reads what the previous
one wrote (read after write) or overwrites what the previous one still reads
(write after read), and compare every result with the oracle.
"""
import numpy as np
import pytest

from momiru_b200 import (AccuracyContract, BoundGemm, DeviceView, Epilogue, KernelFamily, KernelMathMode,
                         MatMulNode)
from momiru_b200 import rng

pytestmark = pytest.mark.gpu

STRICT = MatMulNode(math_mode=KernelMathMode.StrictFp32)
TF32 = MatMulNode(math_mode=KernelMathMode.Tf32, accuracy=AccuracyContract.AllowTf32)
EXACT = MatMulNode(math_mode=KernelMathMode.Exact, accuracy=AccuracyContract.Exact)


@pytest.fixture(params=["default", "created"])
def stream(request):
    """The legacy default stream (None) or a created one shared by every node."""
    if request.param == "default":
        yield None
    else:
        import torch
        s = torch.cuda.Stream()
        yield s.cuda_stream
        s.synchronize()


def rel_frob(x, ref):
    x = np.asarray(x, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.linalg.norm(x - ref) / max(np.linalg.norm(ref), 1e-30))


def test_chain_read_after_write_across_families(oracle, stream):
    """X1 = X0 @ W1 (tcgen05), X2 = X1[:16] @ W2 (GEMV, tensor cores),
    X3 = X2 @ W3 (GEMV, CUDA cores), X4 = X3 @ W4 (exact CUDA cores),
    all queued back to back, five times over."""
    x0 = rng.randn((256, 512), 1, 0.5)
    w1 = rng.randn((512, 512), 2, 0.05)
    w2 = rng.randn((512, 256), 3, 0.05)
    w3 = rng.randn((256, 128), 4, 0.05)
    w4 = rng.randn((128, 64), 5, 0.05)
    d = {k: DeviceView.from_host(v) for k, v in (("x0", x0), ("w1", w1), ("w2", w2), ("w3", w3), ("w4", w4))}
    x1 = DeviceView.empty((256, 512))
    x2 = DeviceView.empty((16, 256))
    x3 = DeviceView.empty((16, 128))
    x4 = DeviceView.empty((16, 64))
    gs = [BoundGemm(MatMulNode(epilogue=Epilogue.RELU), d["x0"], d["w1"], x1, stream=stream),
          BoundGemm(STRICT, x1.narrow(0, 0, 16), d["w2"], x2, stream=stream),
          BoundGemm(STRICT, x2.narrow(0, 0, 1), d["w3"], x3.narrow(0, 0, 1), stream=stream),
          BoundGemm(EXACT, x3.narrow(0, 0, 1), d["w4"], x4.narrow(0, 0, 1), stream=stream)]
    assert [g.family for g in gs] == ["tcgen05", "gemv", "gemv", "simt"]
    try:
        for _ in range(5):
            for g in gs:
                g.replay()
        for g in gs:
            g.quiesce_or_abort(60)
        r1 = oracle.matmul(x0, w1, epilogue=oracle.EPI_RELU)
        r2 = oracle.matmul(r1[:16], w2)
        h1, h2 = x1.to_host(), x2.to_host()
        assert rel_frob(h1, r1) <= 1e-5
        assert rel_frob(h2, r2) <= 1e-5
        # the later links consume the device results, so check them against
        # the oracle applied to those
        r3 = oracle.matmul(h2[:1], w3)
        h3 = x3.to_host()[:1]
        assert rel_frob(h3, r3) <= 1e-5
        r4 = oracle.matmul(h3, w4)
        assert np.array_equal(x4.to_host()[:1].view(np.uint32), r4.view(np.uint32))
    finally:
        for g in gs:
            g.close()


@pytest.mark.parametrize("first,second", [(STRICT, STRICT), (TF32, STRICT), (STRICT, EXACT)])
def test_write_after_read(oracle, first, second, stream):
    """G1 reads X and writes Y; G2, queued right behind it, overwrites X.
    G1 must have finished reading X before G2 writes it."""
    x = rng.randn((512, 1024), 6)
    w = rng.randn((1024, 1024), 7, 0.03)
    z = rng.randn((512, 256), 8)
    v = rng.randn((256, 1024), 9, 0.05)
    dx = DeviceView.from_host(x)
    y = DeviceView.empty((512, 1024))
    g1 = BoundGemm(first, dx, DeviceView.from_host(w), y, stream=stream)
    g2 = BoundGemm(second, DeviceView.from_host(z), DeviceView.from_host(v), dx, stream=stream)
    try:
        g1.replay()
        g2.replay()
        g1.quiesce_or_abort(60)
        g2.quiesce_or_abort(60)
        tol = 1e-5 if first is STRICT else 2e-3
        assert rel_frob(y.to_host(), oracle.matmul(x, w)) <= tol
        assert rel_frob(dx.to_host(), oracle.matmul(z, v)) <= 1e-5
    finally:
        g1.close()
        g2.close()


def test_forced_families_back_to_back_on_one_output(oracle, stream):
    """Four nodes of different families write the same output in turn; the
    last one's result must be what remains (write after write)."""
    a = rng.randn((300, 200), 10)
    b = rng.randn((200, 160), 11)
    out = DeviceView.empty((300, 160))
    da, db = DeviceView.from_host(a), DeviceView.from_host(b)
    nodes = [MatMulNode(family=KernelFamily.Tcgen05), MatMulNode(family=KernelFamily.Simt,
                                                                 math_mode=KernelMathMode.Exact,
                                                                 accuracy=AccuracyContract.Exact),
             MatMulNode(family=KernelFamily.Tcgen05, epilogue=Epilogue.RELU),
             MatMulNode(family=KernelFamily.Simt, math_mode=KernelMathMode.Exact,
                        accuracy=AccuracyContract.Exact, epilogue=Epilogue.RELU)]
    gs = [BoundGemm(n, da, db, out, stream=stream) for n in nodes]
    try:
        for _ in range(3):
            for g in gs:
                g.replay()
        for g in gs:
            g.quiesce_or_abort(60)
        ref = oracle.matmul(a, b, epilogue=oracle.EPI_RELU)
        assert np.array_equal(out.to_host().view(np.uint32), ref.view(np.uint32))
    finally:
        for g in gs:
            g.close()
