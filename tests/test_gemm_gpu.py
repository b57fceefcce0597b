"""GPU parity of the f32 matmul hot path against the CPU oracle, through the C ABI.

Tolerances (relative Frobenius error against the oracle, the restated
reference CPU GEMM):
  StrictFp32 (3xTF32 on tcgen05, and the GEMV family)   <= 1e-5
  Tf32 (one TF32 pass)                                  <= 2e-3
  Exact (CUDA-core kernel in the reference's order)     bit-identical
"""
import numpy as np
import pytest

from momiru_b200 import (BoundGemm, DeviceBuffer, DeviceView, Epilogue, KernelFamily, KernelMathMode, MatMulNode,
                         PlanError, matmul, selftest_bounded_wait)
from momiru_b200 import _abi, execution
from momiru_b200 import rng

pytestmark = pytest.mark.gpu

STRICT_TOL = 1e-5
TF32_TOL = 2e-3
STRICT = MatMulNode(math_mode=KernelMathMode.StrictFp32)
TF32 = MatMulNode(math_mode=KernelMathMode.Tf32, accuracy=execution.AccuracyContract.AllowTf32)
EXACT = MatMulNode(math_mode=KernelMathMode.Exact, accuracy=execution.AccuracyContract.Exact)


def rel_frob(x, ref):
    x = np.asarray(x, np.float64)
    ref = np.asarray(ref, np.float64)
    den = np.linalg.norm(ref)
    return float(np.linalg.norm(x - ref) / (den if den > 0 else 1.0))


def node(base, **kw):
    d = dict(transpose_lhs=base.transpose_lhs, transpose_rhs=base.transpose_rhs, math_mode=base.math_mode,
             epilogue=base.epilogue, family=base.family, accuracy=base.accuracy)
    d.update(kw)
    return MatMulNode(**d)


def padded(arr, pad_to=4):
    """Device copy of a 2-D/3-D array whose rows are padded to a multiple of
    `pad_to` elements, returned as the narrowed (logical) view."""
    arr = np.ascontiguousarray(arr, np.float32)
    cols = arr.shape[-1]
    pc = (cols + pad_to - 1) // pad_to * pad_to
    phys = np.zeros(arr.shape[:-1] + (pc,), np.float32)
    phys[..., :cols] = arr
    v = DeviceView.from_host(phys)
    return v.narrow(-1, 0, cols)


def run(node_, a, b, bias=None, out_dims=None, family=None):
    """Bind, replay once, quiesce; the output rows are padded to 16 bytes."""
    if family is not None:
        node_ = node(node_, family=family)
    dims = out_dims or execution.output_dims(node_, a, b)
    out = padded(np.zeros(dims, np.float32)) if len(dims) >= 2 else DeviceView.empty(dims)
    with BoundGemm(node_, a, b, out, bias) as g:
        g.replay()
        g.quiesce_or_abort(60)
        fam = g.family
    return out.to_host(), fam


# ----------------------------------------------------------------- basics --
def test_bounded_wait_probe_returns_timeout_and_context_survives():
    assert selftest_bounded_wait(0, 0.02) == _abi.ERR_TIMEOUT
    a = DeviceView.from_host(np.eye(4, dtype=np.float32))
    out = matmul(a, a, node=EXACT)
    assert np.array_equal(out.to_host(), np.eye(4, dtype=np.float32))


@pytest.mark.parametrize("fam,mode", [(KernelFamily.Tcgen05, STRICT), (KernelFamily.Tcgen05, TF32),
                                      (KernelFamily.Simt, EXACT), (KernelFamily.Gemv, STRICT),
                                      (KernelFamily.Auto, STRICT)])
def test_reference_kat_every_family(oracle, fam, mode):
    # cpu.rs:827-846: [[1,2,3],[4,5,6]] @ [[7,8],[9,10],[11,12]] = [[58,64],[139,154]]
    a = np.array([[1, 2, 3], [4, 5, 6]], np.float32)
    b = np.array([[7, 8], [9, 10], [11, 12]], np.float32)
    want = np.array([[58, 64], [139, 154]], np.float32)
    if fam == KernelFamily.Gemv:
        b4 = np.zeros((3, 4), np.float32)
        b4[:, :2] = b
        got, f = run(mode, padded(a), DeviceView.from_host(b4), out_dims=(2, 4), family=fam)
        got = got[:, :2]
    else:
        got, f = run(mode, padded(a), padded(b), family=fam)
    assert np.array_equal(got, want), (f, got)


# ---------------------------------------------------------------- C1 512^3 --
@pytest.mark.parametrize("mode,tol", [(STRICT, STRICT_TOL), (TF32, TF32_TOL)])
def test_c1_square_512(oracle, mode, tol):
    a = rng.randu((512, 512), 1)
    b = rng.randu((512, 512), 2)
    ref = oracle.matmul(a, b)
    got, fam = run(mode, DeviceView.from_host(a), DeviceView.from_host(b))
    assert fam == "tcgen05"
    assert rel_frob(got, ref) <= tol


def test_c1_exact_is_bit_identical(oracle):
    a = rng.randu((512, 512), 1)
    b = rng.randu((512, 512), 2)
    ref = oracle.matmul(a, b)
    got, fam = run(EXACT, DeviceView.from_host(a), DeviceView.from_host(b))
    assert fam == "simt"
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_repeat_runs_are_bitwise_deterministic():
    a = DeviceView.from_host(rng.randu((384, 640), 3))
    b = DeviceView.from_host(rng.randu((640, 520), 4))
    out = DeviceView.empty((384, 520))
    with BoundGemm(STRICT, a, b, out) as g:
        g.replay()
        g.quiesce_or_abort()
        first = out.to_host()
        for _ in range(3):
            g.replay()
        g.quiesce_or_abort()
    assert np.array_equal(first.view(np.uint32), out.to_host().view(np.uint32))


# ------------------------------------------------- C2 batched + broadcast --
def test_c2_batched_broadcast(oracle):
    a = rng.randn((64, 256, 256), 1)
    b = rng.randn((256, 256), 2)
    ref = oracle.matmul(a, b)
    da, db = DeviceView.from_host(a), DeviceView.from_host(b)
    got, fam = run(STRICT, da, db)
    assert fam == "tcgen05" and rel_frob(got, ref) <= STRICT_TOL
    got, _ = run(TF32, da, db)
    assert rel_frob(got, ref) <= TF32_TOL
    got, fam = run(EXACT, da, db)
    assert fam == "simt" and np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_batched_broadcast_lhs_and_two_batch_axes(oracle):
    a = rng.randn((256, 64), 5)
    b = rng.randn((3, 64, 96), 6)
    ref = np.stack([oracle.matmul(a, b[i]) for i in range(3)])
    got, fam = run(STRICT, DeviceView.from_host(a), DeviceView.from_host(b))
    assert fam == "tcgen05" and rel_frob(got, ref) <= STRICT_TOL
    # [2,1,M,K] x [1,3,K,N] -> [2,3,M,N] cannot flatten to one batch axis: SIMT
    a4 = rng.randn((2, 1, 40, 24), 7)
    b4 = rng.randn((1, 3, 24, 36), 8)
    ref4 = np.stack([np.stack([oracle.matmul(a4[i, 0], b4[0, j]) for j in range(3)]) for i in range(2)])
    got4, fam = run(EXACT, DeviceView.from_host(a4), DeviceView.from_host(b4))
    assert np.array_equal(got4.view(np.uint32), ref4.view(np.uint32))


# ------------------------------------------------------ C3 fused epilogue --
@pytest.mark.parametrize("mode,tol", [(STRICT, STRICT_TOL), (TF32, TF32_TOL)])
@pytest.mark.parametrize("epi", [Epilogue.BIAS_RELU, Epilogue.BIAS, Epilogue.RELU])
def test_c3_epilogue_1024(oracle, mode, tol, epi):
    a = rng.randu((1024, 1024), 1)
    b = rng.randu((1024, 1024), 2)
    bias = rng.randn((1024,), 3, 0.1)
    oepi = {Epilogue.BIAS_RELU: oracle.EPI_BIAS_RELU, Epilogue.BIAS: oracle.EPI_BIAS, Epilogue.RELU: oracle.EPI_RELU}[epi]
    ref = oracle.matmul(a, b, bias=bias, epilogue=oepi)
    got, fam = run(node(mode, epilogue=epi), DeviceView.from_host(a), DeviceView.from_host(b),
                   DeviceView.from_host(bias))
    assert fam == "tcgen05" and rel_frob(got, ref) <= tol
    if epi != Epilogue.BIAS:
        # ReLU writes +0 (never -0) wherever the reference does.
        zeros = ref == 0
        assert np.all(got.view(np.uint32)[zeros & (got == 0)] == 0)
        assert not np.any(np.signbit(got))


def test_c3_full_size_row_sampled(oracle):
    """8192^3 + bias + ReLU: all rows computed on the GPU, 48 rows checked
    against the oracle, and a size-independent column-sum identity checked on
    the pre-activation product."""
    n = 8192
    a = rng.randu((n, n), 1)
    b = rng.randu((n, n), 2)
    bias = rng.randn((n,), 3, 0.1)
    da, db, dbias = DeviceView.from_host(a), DeviceView.from_host(b), DeviceView.from_host(bias)
    rows = np.random.default_rng(0).choice(n, 48, replace=False)
    ref = oracle.matmul(a, b, bias=bias, epilogue=oracle.EPI_BIAS_RELU, rows=rows)
    for mode, tol in ((STRICT, STRICT_TOL), (TF32, TF32_TOL)):
        got, fam = run(node(mode, epilogue=Epilogue.BIAS_RELU), da, db, dbias)
        assert fam == "tcgen05"
        assert np.isfinite(got).all()
        assert rel_frob(got[rows], ref) <= tol, mode
    # column sums: 1^T (A B) == (1^T A) B, in f64 on the host
    plain, _ = run(STRICT, da, db)
    lhs = plain.astype(np.float64).sum(axis=0)
    rhs = a.astype(np.float64).sum(axis=0) @ b.astype(np.float64)
    assert rel_frob(lhs, rhs) <= STRICT_TOL


# ----------------------------------------------------- C4 strided views --
def _c4(oracle, m, k, n, n_phys, rows=None):
    x = rng.randn((k, m), 1, 0.02)          # A = X^T
    w = rng.randn((k, n_phys), 2, 0.02)     # B = W[:, :n]
    dx, dw = DeviceView.from_host(x), DeviceView.from_host(w)
    ref = oracle.matmul(x.T, w[:, :n], rows=rows)
    return dx, dw, ref


def test_c4_strided_views_reduced(oracle):
    dx, dw, ref = _c4(oracle, 1024, 1024, 2752, 3072)
    for view_form in ("view", "flag"):
        lhs = dx.transpose() if view_form == "view" else dx
        nd = STRICT if view_form == "view" else node(STRICT, transpose_lhs=True)
        got, fam = run(nd, lhs, dw.narrow(1, 0, 2752))
        assert fam == "tcgen05" and rel_frob(got, ref) <= STRICT_TOL
    got, _ = run(TF32, dx.transpose(), dw.narrow(1, 0, 2752))
    assert rel_frob(got, ref) <= TF32_TOL


def test_k_major_rhs_via_transpose_flag(oracle):
    a = rng.randn((300, 200), 1)
    bt = rng.randn((260, 200), 2)           # B^T stored [N, K]
    ref = oracle.matmul(a, bt.T)
    got, fam = run(node(STRICT, transpose_rhs=True), DeviceView.from_host(a), DeviceView.from_host(bt))
    assert fam == "tcgen05" and rel_frob(got, ref) <= STRICT_TOL


# ------------------------------------------------------- C5a big batches --
def test_c5a_batched_reduced(oracle):
    a = rng.randu((8, 1024, 1024), 1)
    b = rng.randu((8, 1024, 1024), 2)
    got, fam = run(STRICT, DeviceView.from_host(a), DeviceView.from_host(b))
    assert fam == "tcgen05"
    for i in (0, 5, 7):
        assert rel_frob(got[i], oracle.matmul(a[i], b[i])) <= STRICT_TOL


# --------------------------------------------------------------- C5b GEMV --
@pytest.mark.parametrize("m", [1, 4, 16])
def test_c5b_gemv(oracle, m):
    a = rng.randn((m, 4096), 1)
    b = rng.randn((4096, 4096), 2)
    ref = oracle.matmul(a, b)
    got, fam = run(STRICT, DeviceView.from_host(a), DeviceView.from_host(b))
    assert fam == "gemv" and rel_frob(got, ref) <= STRICT_TOL


@pytest.mark.parametrize("m,k,n", [(3, 100, 64), (16, 8192, 260), (7, 1, 8), (1, 5000, 4)])
def test_gemv_ragged(oracle, m, k, n):
    a = rng.randn((m, k), 3)
    b = rng.randn((k, n), 4)
    bias = rng.randn((n,), 5)
    ref = oracle.matmul(a, b, bias=bias, epilogue=oracle.EPI_BIAS_RELU)
    got, fam = run(node(STRICT, epilogue=Epilogue.BIAS_RELU), DeviceView.from_host(a), DeviceView.from_host(b),
                   DeviceView.from_host(bias))
    assert fam == "gemv" and rel_frob(got, ref) <= STRICT_TOL


# ------------------------------------------------------------ edge cases --
@pytest.mark.parametrize("m,n,k", [(1, 1, 1), (7, 9, 5), (127, 129, 33), (129, 255, 257), (255, 257, 129),
                                   (128, 256, 32), (200, 300, 1000), (17, 520, 31)])
def test_tcgen05_ragged_tiles(oracle, m, n, k):
    a = rng.randn((m, k), m + 1)
    b = rng.randn((k, n), n + 2)
    ref = oracle.matmul(a, b)
    for mode, tol in ((STRICT, STRICT_TOL), (TF32, TF32_TOL)):
        got, fam = run(node(mode, family=KernelFamily.Tcgen05), padded(a), padded(b), out_dims=None)
        assert fam == "tcgen05"
        assert rel_frob(got, ref) <= tol, (m, n, k, mode.math_mode)
    got, fam = run(EXACT, DeviceView.from_host(a), DeviceView.from_host(b))
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("m,n,k,tmode", [
    (2304, 4096, 1000, "nn"),     # 144 tiles of 256x256
    (4352, 2500, 520, "tn"),      # 170 tiles; ragged N and K
    (3840, 1280, 4096, "nt"),     # 75 tiles: splits fall inside K chunks
    (8192, 1024, 2048, "nn"),     # the 8-way column shard of the 8192^2 output: 128 tiles
    (1536, 4864, 200, "tt"),      # 114 tiles, 13 k-blocks: tiles cut into three or more parts
])
def test_pair_kernel_split_tiles(oracle, m, n, k, tmode):
    """Shapes whose 256x256 tiles do not fill whole rounds of CTA pairs: the
    last tiles' k-blocks are split between pairs and summed by the tile's
    owner. Sampled rows against the oracle, both numeric modes, bias + ReLU,
    and a bitwise repeat."""
    a = rng.randu((m, k), m + 11)
    b = rng.randu((k, n), n + 12)
    bias = rng.randn((n,), 13, 0.1)
    rows = np.random.default_rng(m).choice(m, 96, replace=False)
    rows.sort()
    ref = oracle.matmul(a, b, bias=bias, epilogue=oracle.EPI_BIAS_RELU, rows=rows)
    # Operands as given (K-major) or as transposed views of the other layout.
    da = DeviceView.from_host(np.ascontiguousarray(a.T)).transpose() if tmode[0] == "t" else DeviceView.from_host(a)
    db = padded(np.ascontiguousarray(b.T)).transpose() if tmode[1] == "t" else padded(b)
    dbias = DeviceView.from_host(bias)
    for mode, tol in ((STRICT, STRICT_TOL), (TF32, TF32_TOL)):
        nd = node(mode, epilogue=Epilogue.BIAS_RELU, family=KernelFamily.Tcgen05)
        out = padded(np.zeros((m, n), np.float32))
        with BoundGemm(nd, da, db, out, dbias) as g:
            assert g.family == "tcgen05"
            g.replay()
            g.quiesce_or_abort(60)
            first = out.to_host()
            g.replay()
            g.replay()
            g.quiesce_or_abort(60)
            again = out.to_host()
        assert np.isfinite(first).all()
        assert rel_frob(first[rows], ref) <= tol, (m, n, k, mode.math_mode)
        assert np.array_equal(first.view(np.uint32), again.view(np.uint32))


def test_pair_kernel_small_output_long_k(oracle):
    """512 x 1024 output (8 pair tiles) with K = 8192: fewer tiles than CTA
    pairs, so each tile's k-blocks are split over several pairs (4 in 3xTF32,
    2 in TF32) and summed by the last part to arrive. Full output against the
    oracle, bias + ReLU, and a bitwise repeat."""
    m, n, k = 512, 1024, 8192
    a = rng.randu((m, k), 91)
    b = rng.randu((k, n), 92)
    bias = rng.randn((n,), 93, 0.1)
    ref = oracle.matmul(a, b, bias=bias, epilogue=oracle.EPI_BIAS_RELU)
    da, db, dbias = DeviceView.from_host(a), DeviceView.from_host(b), DeviceView.from_host(bias)
    for mode, tol in ((STRICT, STRICT_TOL), (TF32, TF32_TOL)):
        out = DeviceView.empty((m, n))
        with BoundGemm(node(mode, epilogue=Epilogue.BIAS_RELU, family=KernelFamily.Tcgen05), da, db, out, dbias) as g:
            g.replay()
            g.quiesce_or_abort(60)
            first = out.to_host()
            g.replay()
            g.quiesce_or_abort(60)
            again = out.to_host()
        assert rel_frob(first, ref) <= tol, mode.math_mode
        assert np.array_equal(first.view(np.uint32), again.view(np.uint32))


def test_pair_kernel_split_tiles_nonfinite(oracle):
    """inf/NaN inside tiles whose k-blocks are split between pairs: the exact
    fix-up recomputes those tiles whole."""
    m, n, k = 2304, 4096, 640
    a = rng.randn((m, k), 21)
    b = rng.randn((k, n), 22)
    a[1000, 600] = np.inf
    a[2000, 5] = np.nan
    b[300, 4000] = -np.inf
    rows = np.array([0, 999, 1000, 1001, 2000, 2303])
    ref = oracle.matmul(a, b, rows=rows)
    got, fam = run(node(STRICT, family=KernelFamily.Tcgen05), DeviceView.from_host(a), DeviceView.from_host(b))
    assert fam == "tcgen05"
    got = got[rows]
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    assert np.array_equal(np.isinf(got), np.isinf(ref))
    fin = np.isfinite(ref)
    assert rel_frob(got[fin], ref[fin]) <= STRICT_TOL


ACTIVATIONS = [Epilogue.RELU6, Epilogue.BIAS_RELU6, Epilogue.GELU_ERF, Epilogue.BIAS_GELU_ERF,
               Epilogue.GELU_TANH, Epilogue.BIAS_GELU_TANH, Epilogue.SILU, Epilogue.BIAS_SILU]


def _close_ulps(got, want, ulps, pre=None):
    """Elementwise: equal (NaN with NaN, signed zeros and infinities alike) or
    within `ulps` f32 units in the last place of the oracle's value. With
    `pre` (the pre-activation values) also within 2^-21 |pre|: GELU-tanh
    computes 0.5 x (1 + tanh(..)), and for x < 0 the sum cancels, so one or two
    ulp of difference between two tanhf implementations near -1 become that."""
    got = np.asarray(got, np.float32)
    want = np.asarray(want, np.float32)
    same = (got.view(np.uint32) == want.view(np.uint32)) | (np.isnan(got) & np.isnan(want))
    fin = np.isfinite(want) & np.isfinite(got)
    bound = ulps * np.spacing(np.abs(want)).astype(np.float64)
    if pre is not None:
        bound = np.maximum(bound, 2.0 ** -21 * np.abs(np.asarray(pre, np.float64)))
    near = fin & (np.abs(got.astype(np.float64) - want) <= bound)
    return bool(np.all(same | near))


@pytest.mark.parametrize("epi", ACTIVATIONS)
def test_activation_epilogues_every_family(oracle, epi):
    """MatMul -> [+bias] -> ReLU6 / GELU-erf / GELU-tanh / SiLU fused into each
    kernel family. tcgen05 and GEMV within their GEMM tolerance; the exact
    family bit-identical for ReLU6, within 1 f32 ulp for GELU-erf (the
    reference's own erfc approximation restated in f64; only its exp(-x^2)
    comes from a math library, CUDA's on the device and the host libm in the
    oracle) and within 4 f32 ulp for SiLU and GELU-tanh (CUDA's expf / tanhf
    against the host libm)."""
    has_bias = epi.has_bias
    cases = [
        (300, 96, 517, KernelFamily.Tcgen05),   # CTA pairs, ragged right edge
        (100, 200, 264, KernelFamily.Tcgen05),  # one-CTA kernel (M <= 128)
        (4, 512, 1024, KernelFamily.Gemv),
    ]
    for m, k, n, fam in cases:
        a = rng.randn((m, k), 41, 0.3)
        b = rng.randn((k, n), 42, 0.3)
        bias = rng.randn((n,), 43, 0.5)
        ref = oracle.matmul(a, b, bias=bias if has_bias else None, epilogue=int(epi))
        db = DeviceView.from_host(b) if fam == KernelFamily.Gemv else padded(b)
        modes = ((STRICT, STRICT_TOL), (TF32, TF32_TOL)) if fam == KernelFamily.Tcgen05 else ((STRICT, STRICT_TOL),)
        for mode, tol in modes:
            got, f = run(node(mode, epilogue=epi, family=fam), padded(a), db,
                         DeviceView.from_host(bias) if has_bias else None)
            assert f == fam.name.lower()
            assert rel_frob(got, ref) <= tol, (m, n, k, mode.math_mode)
    a = rng.randn((70, 33), 44, 0.5)
    b = rng.randn((33, 45), 45, 0.5)
    bias = rng.randn((45,), 46, 0.5)
    ref = oracle.matmul(a, b, bias=bias if has_bias else None, epilogue=int(epi))
    got, f = run(node(EXACT, epilogue=epi), DeviceView.from_host(a), DeviceView.from_host(b),
                 DeviceView.from_host(bias) if has_bias else None)
    assert f == "simt"
    if epi in (Epilogue.RELU6, Epilogue.BIAS_RELU6):
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    else:
        pre = oracle.matmul(a, b, bias=bias if has_bias else None,
                            epilogue=oracle.EPI_BIAS if has_bias else oracle.EPI_NONE)
        ulps = 1 if epi in (Epilogue.GELU_ERF, Epilogue.BIAS_GELU_ERF) else 4
        assert _close_ulps(got, ref, ulps, pre if epi in (Epilogue.GELU_TANH, Epilogue.BIAS_GELU_TANH) else None)


def test_gelu_erf_matches_reference_formula_across_its_ranges(oracle):
    """GELU-erf evaluated through the exact family with K = 1 (out = x * 1 = x
    exactly, then the activation), on values that cover every branch of the
    reference's erfc (|x|/sqrt 2 in [0, 1), [1, 8), [8, 27] and above 27),
    both signs, subnormals and zeros. At most 1 f32 ulp from the oracle
    everywhere (exp(-x^2) is the only library call: CUDA's against the host
    libm), and bit-identical on all but a handful of values."""
    mags = np.concatenate([np.geomspace(1e-38, 1e-30, 64), np.geomspace(1e-30, 1.0, 1024),
                           np.linspace(1.0, 45.0, 4096), np.array([1.4142135, 11.313708, 38.18377])])
    x = np.concatenate([mags, -mags, [0.0, -0.0, 1e-45, -1e-45]]).astype(np.float32)
    a = x.reshape(-1, 1)
    b = np.ones((1, 1), np.float32)
    ref = oracle.matmul(a, b, epilogue=int(Epilogue.GELU_ERF))
    got, f = run(node(EXACT, epilogue=Epilogue.GELU_ERF), DeviceView.from_host(a), DeviceView.from_host(b))
    assert f == "simt"
    assert _close_ulps(got, ref, 1)
    same = got.view(np.uint32) == ref.view(np.uint32)
    assert same.mean() >= 0.999, f"{int((~same).sum())} of {same.size} differ by one ulp"


def test_activation_epilogue_nonfinite_inputs(oracle):
    """A -inf in A: GELU-erf sends -inf to -0 and +inf to +inf; NaN stays NaN
    (3xTF32 tiles with non-finite inputs are recomputed exactly)."""
    a = rng.randn((256, 64), 47)
    b = rng.randn((64, 256), 48)
    a[5, 3] = -np.inf
    a[200, 10] = np.nan
    bias = rng.randn((256,), 49, 0.1)
    for epi in (Epilogue.BIAS_GELU_ERF, Epilogue.BIAS_SILU, Epilogue.BIAS_GELU_TANH):
        ref = oracle.matmul(a, b, bias=bias, epilogue=int(epi))
        for mode in (STRICT, TF32):
            got, _ = run(node(mode, epilogue=epi, family=KernelFamily.Tcgen05), DeviceView.from_host(a),
                         DeviceView.from_host(b), DeviceView.from_host(bias))
            assert np.array_equal(np.isnan(got), np.isnan(ref)), (epi, mode.math_mode)
            assert np.array_equal(np.isinf(got), np.isinf(ref))
            row = ref[5]
            neg0 = (row == 0) & np.signbit(row)
            assert neg0.any() and np.all(np.signbit(got[5][neg0]) & (got[5][neg0] == 0))


def test_output_pad_columns_untouched():
    """A ragged output tile is clipped: padding beyond N keeps its bytes."""
    a = DeviceView.from_host(rng.randn((130, 64), 1))
    b = padded(rng.randn((64, 70), 2))
    phys = DeviceView.from_host(np.full((130, 72), 7.0, np.float32))
    out = phys.narrow(1, 0, 70)
    with BoundGemm(STRICT, a, b, out) as g:
        g.replay()
        g.quiesce_or_abort()
    host = phys.to_host()
    assert np.all(host[:, 70:] == 7.0)


def test_k_zero_and_empty(oracle):
    a = DeviceView.contiguous(DeviceBuffer.allocate(4, 0), (5, 0))
    b = DeviceView.contiguous(DeviceBuffer.allocate(4, 0), (0, 3))
    bias = DeviceView.from_host(np.array([-1.0, 0.0, 2.0], np.float32))
    out = DeviceView.from_host(np.full((5, 3), 9.0, np.float32))
    with BoundGemm(node(STRICT, epilogue=Epilogue.BIAS_RELU), a, b, out, bias) as g:
        g.replay()
        g.quiesce_or_abort()
    want = np.tile(np.array([0.0, 0.0, 2.0], np.float32), (5, 1))
    got = out.to_host()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    # empty output: a no-op bind and replay
    e = DeviceView.contiguous(DeviceBuffer.allocate(4, 0), (0, 3))
    with BoundGemm(STRICT, DeviceView.contiguous(DeviceBuffer.allocate(4, 0), (0, 4)),
                   DeviceView.from_host(np.ones((4, 3), np.float32)), e) as g:
        g.replay()
        g.quiesce_or_abort()


def test_nan_and_inf_propagate(oracle):
    a = rng.randn((256, 128), 1)
    b = rng.randn((128, 256), 2)
    a[3, 7] = np.nan
    a[10, 0] = np.inf
    b[5, 9] = -np.inf
    ref = oracle.matmul(a, b)
    for mode in (STRICT, TF32):
        got, _ = run(mode, DeviceView.from_host(a), DeviceView.from_host(b))
        assert np.array_equal(np.isnan(got), np.isnan(ref)), mode.math_mode
        fin = np.isfinite(ref)
        assert np.array_equal(np.isinf(got), np.isinf(ref))
        assert rel_frob(got[fin], ref[fin]) <= (STRICT_TOL if mode is STRICT else TF32_TOL)
    got, _ = run(EXACT, DeviceView.from_host(a), DeviceView.from_host(b))
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    ok = ~np.isnan(ref)
    assert np.array_equal(got[ok].view(np.uint32), ref[ok].view(np.uint32))


def test_nonfinite_bookkeeping_resets_between_runs(oracle):
    """A replay with inf/NaN inputs, then finite inputs in the same buffers:
    the second result is the ordinary 3xTF32 one, within tolerance."""
    a = rng.randn((384, 256), 1)
    b = rng.randn((256, 512), 2)
    bad = a.copy()
    bad[100, 3] = np.inf
    bad[300, 9] = np.nan
    da, db = DeviceView.from_host(bad), DeviceView.from_host(b)
    out = DeviceView.empty((384, 512))
    with BoundGemm(STRICT, da, db, out) as g:
        g.replay()
        g.quiesce_or_abort()
        first = out.to_host()
        ref_bad = oracle.matmul(bad, b)
        assert np.array_equal(np.isnan(first), np.isnan(ref_bad))
        assert np.array_equal(np.isinf(first), np.isinf(ref_bad))
        da.copy_from_host(a)
        g.replay()
        g.quiesce_or_abort()
        g.replay()
        g.quiesce_or_abort()
        second = out.to_host()
    assert np.isfinite(second).all()
    assert rel_frob(second, oracle.matmul(a, b)) <= STRICT_TOL


def test_vector_operands(oracle):
    a = rng.randn((300,), 1)
    b = rng.randn((300, 40), 2)
    ref = oracle.matmul(a.reshape(1, 300), b).reshape(40)
    got, _ = run(STRICT, DeviceView.from_host(a), DeviceView.from_host(b))
    assert got.shape == (40,) and rel_frob(got, ref) <= STRICT_TOL
    bv = rng.randn((300,), 3)
    ref = oracle.matmul(b.T.copy(), bv.reshape(300, 1)).reshape(40)
    got, _ = run(EXACT, DeviceView.from_host(b.T.copy()), DeviceView.from_host(bv))
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_bind_rejects_host_memory_and_wrong_device():
    host = np.zeros((64, 64), np.float32)
    hv = DeviceView.contiguous(DeviceBuffer(host.ctypes.data, host.nbytes, 0), (64, 64))
    dv = DeviceView.from_host(np.ones((64, 64), np.float32))
    with pytest.raises(execution.UnsupportedDevice):
        BoundGemm(STRICT, hv, dv, DeviceView.empty((64, 64)))
    with pytest.raises(execution.UnsafeAliasing):
        BoundGemm(STRICT, dv, dv, dv)


def test_tf32_operands_are_truncated_by_the_tensor_core(oracle):
    """Records how the tensor core reads f32 operands in kind::tf32: the TF32
    result of raw inputs equals the TF32 result of inputs whose low 13
    mantissa bits were cleared on the host (truncation), so the 3xTF32 split
    hi = x & ~0x1FFF is the value the hardware multiplies."""
    a = rng.randn((256, 256), 11)
    b = rng.randn((256, 256), 12)
    mask = np.uint32(0xFFFFE000)
    at = (a.view(np.uint32) & mask).view(np.float32)
    bt = (b.view(np.uint32) & mask).view(np.float32)
    raw, _ = run(TF32, DeviceView.from_host(a), DeviceView.from_host(b))
    trunc, _ = run(TF32, DeviceView.from_host(at), DeviceView.from_host(bt))
    assert np.array_equal(raw.view(np.uint32), trunc.view(np.uint32))


# ------------------------------------------- ranks 0 and 5-8, signed views --
def _batched_oracle(oracle, a, b, bias=None, epilogue=0):
    """The oracle over NumPy-broadcast batch axes, one 2-D product per entry."""
    shape = np.broadcast_shapes(a.shape[:-2], b.shape[:-2])
    out = np.empty(shape + (a.shape[-2], b.shape[-1]), np.float32)
    ab = np.broadcast_to(a, shape + a.shape[-2:])
    bb = np.broadcast_to(b, shape + b.shape[-2:])
    for idx in np.ndindex(*shape):
        out[idx] = oracle.matmul(np.ascontiguousarray(ab[idx]), np.ascontiguousarray(bb[idx]), bias=bias,
                                 epilogue=epilogue)
    return out


def test_vector_dot_has_a_rank0_output_bit_exact(oracle):
    """[K] . [K] -> a rank-0 output (validation.rs:2355-2361), in the
    reference's exact order, in both the Exact and the default StrictFp32
    node (which binds the exact CUDA-core family for this shape)."""
    a = rng.randn((4096,), 51)
    b = rng.randn((4096,), 52)
    ref = oracle.matmul(a.reshape(1, -1), b.reshape(-1, 1))[0, 0]
    for nd in (EXACT, STRICT):
        out = DeviceView.empty(())
        with BoundGemm(nd, DeviceView.from_host(a), DeviceView.from_host(b), out) as g:
            assert g.family == "simt"
            g.replay()
            g.quiesce_or_abort(30)
        got = out.to_host()
        assert got.shape == ()
        assert got.view(np.uint32) == np.float32(ref).view(np.uint32)


@pytest.mark.parametrize("lhs,rhs,fam", [
    ((2, 1, 3, 1, 2, 1, 16, 24), (1, 2, 1, 2, 1, 2, 24, 20), "simt"),  # rank 8, broadcast on alternate axes
    ((2, 3, 4, 64, 32), (2, 3, 4, 32, 48), "tcgen05"),                  # rank 5: batch axes merge into one
    ((1, 2, 1, 3, 40, 36), (36, 72), "tcgen05"),                        # rank 6 x rank 2: rhs broadcast
])
def test_batched_ranks_up_to_eight(oracle, lhs, rhs, fam):
    a = rng.randn(lhs, 53, 0.5)
    b = rng.randn(rhs, 54, 0.5)
    ref = _batched_oracle(oracle, a, b)
    got, f = run(STRICT, DeviceView.from_host(a), DeviceView.from_host(b))
    assert f == fam
    assert got.shape == ref.shape
    assert rel_frob(got, ref) <= STRICT_TOL
    got, f = run(EXACT, DeviceView.from_host(a), DeviceView.from_host(b))
    assert f == "simt" and np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_negative_strides_run_on_the_exact_family(oracle):
    """A reversed-rows lhs view and a reversed-columns rhs view (signed
    strides, as the reference's signed views give): admitted on the SIMT
    family, bit-identical to the oracle on the logical matrices; the
    tensor-core family refuses them."""
    m, k, n = 70, 48, 90
    a = rng.randn((m, k), 55)
    b = rng.randn((k, n), 56)
    bias = rng.randn((n,), 57, 0.1)
    ra = DeviceView.from_host(np.ascontiguousarray(a[::-1]))
    rb = DeviceView.from_host(np.ascontiguousarray(b[:, ::-1]))
    av = DeviceView(ra.buffer, (m, k), (-k, 1), (m - 1) * k)
    bv = DeviceView(rb.buffer, (k, n), (n, -1), n - 1)
    ref = oracle.matmul(a, b, bias=bias, epilogue=oracle.EPI_BIAS_RELU)
    for nd in (EXACT, STRICT):
        got, f = run(node(nd, epilogue=Epilogue.BIAS_RELU), av, bv, DeviceView.from_host(bias))
        assert f == "simt"
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    with pytest.raises(execution.UnsupportedFamily):
        run(node(STRICT, family=KernelFamily.Tcgen05), av, bv)


def test_strided_bias_binds_the_exact_family(oracle):
    """A bias read with stride 2: the tensor-core epilogue reads the bias
    contiguously, so the node binds the SIMT family, which is exact."""
    m, k, n = 300, 64, 200
    a = rng.randn((m, k), 58)
    b = rng.randn((k, n), 59)
    bias2 = rng.randn((2 * n,), 60, 0.1)
    bb = DeviceView.from_host(bias2)
    bias_view = DeviceView(bb.buffer, (n,), (2,), 0)
    ref = oracle.matmul(a, b, bias=np.ascontiguousarray(bias2[::2]), epilogue=oracle.EPI_BIAS)
    got, f = run(node(STRICT, epilogue=Epilogue.BIAS), DeviceView.from_host(a), padded(b), bias_view)
    assert f == "simt"
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_bind_frozen_takes_exactly_the_planned_launch(oracle):
    """A plan's frozen launch record (here the host-derived one) binds and
    runs; the same record with one field changed is refused at bind with
    PlanMismatch and nothing is bound."""
    import torch
    from momiru_b200 import plan_launch
    from momiru_b200.execution import PlanMismatch
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    a = rng.randu((600, 384), 61)
    b = rng.randu((384, 520), 62)
    bias = rng.randn((520,), 63, 0.1)
    da, db, dbias = DeviceView.from_host(a), padded(b), DeviceView.from_host(bias)
    out = padded(np.zeros((600, 520), np.float32))
    nd = node(STRICT, epilogue=Epilogue.BIAS_RELU)
    rec = plan_launch(nd, da, db, out, dbias, sm_count=sms)
    with BoundGemm(nd, da, db, out, dbias, frozen=rec) as g:
        assert g.launch_record().as_dict() == rec.as_dict()
        g.replay()
        g.quiesce_or_abort(30)
    ref = oracle.matmul(a, b, bias=bias, epilogue=oracle.EPI_BIAS_RELU)
    assert rel_frob(out.to_host(), ref) <= STRICT_TOL
    for field, value in (("tile_k", rec.tile_k * 2), ("pipeline_stages", rec.pipeline_stages + 1),
                         ("stream_k_slices", rec.stream_k_slices + 1)):
        other = _abi.MmrLaunchRecord.from_buffer_copy(rec)
        setattr(other, field, value)
        with pytest.raises(PlanMismatch, match=field):
            BoundGemm(nd, da, db, out, dbias, frozen=other)
