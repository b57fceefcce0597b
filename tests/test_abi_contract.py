"""The C ABI on the host: the library loads, exports every declared symbol,
and its bind-time contract (validation.rs:2300-2398 shape/broadcast rules,
layout admission, aliasing, math contract, family choice) behaves as the
reference's validator does. No GPU: mmr_gemm_validate touches no device."""
import ctypes
import os
import re

import numpy as np
import pytest

from momiru_b200 import (AccuracyContract, Epilogue, KernelFamily, KernelMathMode, MatMulNode, PlanError, validate)
from momiru_b200 import _abi, execution
from momiru_b200.tensor import DeviceBuffer, DeviceView

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
G = 1 << 36


def fake(dims, slot, pad_cols=None):
    """A contiguous view over a fake device address (never dereferenced)."""
    dims = tuple(dims)
    if pad_cols:
        phys = dims[:-1] + (pad_cols,)
        buf = DeviceBuffer(slot * G, 4 * int(np.prod(phys)), 0)
        return DeviceView.contiguous(buf, phys).narrow(-1, 0, dims[-1])
    return DeviceView.contiguous(DeviceBuffer(slot * G, 4 * max(1, int(np.prod(dims))), 0), dims)


def test_library_exports_every_declared_symbol(cuda_lib):
    with open(os.path.join(ROOT, "include", "momiru_gemm.h")) as f:
        header = f.read()
    declared = set(re.findall(r"MMR_API\s+(?:int32_t|const char \*)\s*(mmr_\w+)\s*\(", header))
    assert declared, "no declarations parsed"
    assert declared == set(_abi.EXPORTED)
    for name in declared:
        assert hasattr(cuda_lib, name), name
    assert b"sm_100a" in cuda_lib.mmr_version()


def test_configs_pick_expected_families():
    # C1 512^3
    assert validate(MatMulNode(), fake((512, 512), 1), fake((512, 512), 2), fake((512, 512), 3))["family"] == 1
    # C2 batched with B broadcast
    info = validate(MatMulNode(), fake((64, 256, 256), 1), fake((256, 256), 2), fake((64, 256, 256), 3))
    assert info["family"] == 1 and info["batch"] == 64 and info["bytes"] == 4 * (64 * 256 * 256 * 2 + 256 * 256)
    # C3 with fused bias+ReLU
    n = MatMulNode(epilogue=Epilogue.BIAS_RELU)
    info = validate(n, fake((8192, 8192), 1), fake((8192, 8192), 2), fake((8192, 8192), 3), fake((8192,), 4))
    assert info["family"] == 1 and info["flops"] == 2 * 8192 ** 3
    # C4 zero-copy strided views
    x, w = fake((4096, 4096), 1), fake((4096, 12288), 2)
    info = validate(MatMulNode(), x.transpose(), w.narrow(1, 0, 11008), fake((4096, 11008), 3))
    assert info["family"] == 1 and info["a_mn_major"] == 1 and info["b_mn_major"] == 1
    # the same via the node's transpose flag on the physical buffer
    info = validate(MatMulNode(transpose_lhs=True), x, w.narrow(1, 0, 11008), fake((4096, 11008), 3))
    assert info["family"] == 1 and info["a_mn_major"] == 1
    # C5a
    assert validate(MatMulNode(), fake((512, 1024, 1024), 1), fake((512, 1024, 1024), 2),
                    fake((512, 1024, 1024), 3))["batch"] == 512
    # C5b -> GEMV
    for m in (1, 4, 16):
        assert validate(MatMulNode(), fake((m, 4096), 1), fake((4096, 4096), 2), fake((m, 4096), 3))["family"] == 2
    # Exact always runs the reference order on CUDA cores
    assert validate(MatMulNode(math_mode=KernelMathMode.Exact), fake((512, 512), 1), fake((512, 512), 2),
                    fake((512, 512), 3))["family"] == 3


def test_unaligned_layouts_fall_back_to_simt_or_reject_forced_family():
    a, b, c = fake((5, 7), 1), fake((7, 3), 2), fake((5, 3), 3)
    assert validate(MatMulNode(), a, b, c)["family"] == 3
    with pytest.raises(execution.UnsupportedFamily):
        validate(MatMulNode(family=KernelFamily.Tcgen05), a, b, c)
    with pytest.raises(execution.InvalidAccuracyContract):
        validate(MatMulNode(math_mode=KernelMathMode.Exact, family=KernelFamily.Gemv), a, b, c)
    # padded rows make the same logical shapes TMA-admissible
    a, b, c = fake((5, 7), 1, pad_cols=8), fake((7, 3), 2, pad_cols=4), fake((5, 3), 3, pad_cols=4)
    # M <= 16 with 16-byte rows streams B through the GEMV family (TMA
    # zero-fills the ragged N edge); the tcgen05 family is admissible too
    assert validate(MatMulNode(), a, b, c)["family"] == 2
    assert validate(MatMulNode(family=KernelFamily.Tcgen05), a, b, c)["family"] == 1


@pytest.mark.parametrize("lhs,rhs,out,ok", [
    ((3, 4), (4, 5), (3, 5), True),
    ((4,), (4, 5), (5,), True),              # rank-1 lhs: promoted dim removed
    ((3, 4), (4,), (3,), True),              # rank-1 rhs
    ((4,), (4,), (), True),                  # dot -> rank-0 scalar (validation.rs:2355-2361)
    ((4,), (4,), (1,), False),               # ... and not a rank-1 [1]
    ((2, 1, 3, 2, 5, 4), (3, 1, 4, 6), (2, 1, 3, 2, 5, 6), True),      # rank 6 x rank 4
    ((2, 1, 2, 1, 2, 1, 3, 4), (2, 1, 2, 1, 2, 4, 5), (2, 2, 2, 2, 2, 2, 3, 5), True),  # rank 8 x rank 7
    ((2, 1, 2, 1, 2, 1, 3, 4), (3, 1, 2, 1, 2, 1, 4, 5), (3, 1, 2, 1, 2, 1, 3, 5), False),  # 2 vs 3
    ((2, 3, 4), (4, 5), (2, 3, 5), True),    # broadcast rhs
    ((1, 3, 4), (6, 4, 5), (6, 3, 5), True),  # 1 vs 6 -> 6
    ((0, 3, 4), (1, 4, 5), (0, 3, 5), True),  # 0 vs 1 -> 0 (not max)
    ((2, 3, 4), (3, 4, 5), (2, 3, 5), False),  # 2 vs 3
    ((3, 4), (5, 6), (3, 6), False),         # K mismatch
    ((3, 4), (4, 5), (3, 6), False),         # wrong N
    ((3, 4), (4, 5), (1, 3, 5), False),      # wrong rank
])
def test_shape_contract(lhs, rhs, out, ok):
    args = (MatMulNode(), fake(lhs, 1), fake(rhs, 2), fake(out, 3))
    if ok:
        validate(*args)
    else:
        with pytest.raises(execution.InvalidShape):
            validate(*args)


def test_transpose_flags_and_rank1():
    validate(MatMulNode(transpose_lhs=True, transpose_rhs=True), fake((4, 3), 1), fake((5, 4), 2), fake((3, 5), 3))
    with pytest.raises(execution.InvalidShape):
        validate(MatMulNode(transpose_lhs=True), fake((4,), 1), fake((4, 5), 2), fake((5,), 3))


def test_aliasing_bounds_alignment_device():
    a = fake((64, 64), 1)
    with pytest.raises(execution.UnsafeAliasing):
        validate(MatMulNode(), a, fake((64, 64), 2), a)
    # an output view inside the rhs buffer
    big = fake((64, 128), 2)
    with pytest.raises(execution.UnsafeAliasing):
        validate(MatMulNode(), a, big.narrow(1, 0, 64), big.narrow(1, 64, 64))
    # view larger than its buffer
    buf = DeviceBuffer(5 * G, 4 * 100, 0)
    v = DeviceView(buf, (10, 11), (11, 1), 0)
    with pytest.raises(execution.OutOfBounds):
        validate(MatMulNode(), v, fake((11, 3), 2), fake((10, 3), 3))
    # misaligned base offset (bytes not a multiple of 4 cannot be expressed by
    # element offsets, so use a raw ABI descriptor)
    d = execution._desc(MatMulNode(), a, fake((64, 64), 2), fake((64, 64), 3), None, None)
    d.lhs.base_offset_bytes = 2
    info = _abi.MmrGemmInfo()
    import ctypes
    assert _abi.load().mmr_gemm_validate(ctypes.byref(d), ctypes.byref(info)) == _abi.ERR_UNSUPPORTED_LAYOUT
    # device ordinal mismatch
    other = DeviceView.contiguous(DeviceBuffer(6 * G, 4 * 64 * 64, 1), (64, 64))
    with pytest.raises(execution.UnsupportedDevice):
        validate(MatMulNode(), a, other, fake((64, 64), 3))
    # negative strides (a reversed view) are admitted on the SIMT family only
    neg = DeviceView(DeviceBuffer(7 * G, 4 * 64 * 64, 0), (64, 64), (64, -1), 63)
    assert validate(MatMulNode(), a, neg, fake((64, 64), 3))["family"] == _abi.FAMILY_SIMT
    with pytest.raises(execution.UnsupportedFamily):
        validate(MatMulNode(family=KernelFamily.Tcgen05), a, neg, fake((64, 64), 3))
    # ... and must stay inside the buffer: element [0, 63] would be 1 before it
    before = DeviceView(DeviceBuffer(7 * G, 4 * 64 * 64, 0), (64, 64), (64, -1), 62)
    with pytest.raises(execution.OutOfBounds):
        validate(MatMulNode(), a, before, fake((64, 64), 3))


def test_bias_contract():
    n = MatMulNode(epilogue=Epilogue.BIAS)
    validate(n, fake((8, 4), 1), fake((4, 16), 2), fake((8, 16), 3), fake((16,), 4))
    # a strided bias view: not the tensor-core family (its epilogue reads the
    # bias contiguously), the SIMT family takes it
    sb = DeviceView(DeviceBuffer(8 * G, 4 * 32, 0), (16,), (2,), 0)
    views = (fake((300, 64), 1), fake((64, 16), 2), fake((300, 16), 3))
    assert validate(n, *views, sb)["family"] == _abi.FAMILY_SIMT
    with pytest.raises(execution.UnsupportedFamily):
        validate(MatMulNode(epilogue=Epilogue.BIAS, family=KernelFamily.Tcgen05), *views, sb)
    with pytest.raises(execution.InvalidShape):
        validate(n, fake((8, 4), 1), fake((4, 16), 2), fake((8, 16), 3), fake((8,), 4))


def test_activation_epilogues_contract():
    """Every MMR_EPI_* code binds on every family; the odd codes from RELU6 on
    need a bias of N, the even ones take none; codes past BIAS_SILU are refused."""
    views = (fake((300, 64), 1), fake((64, 520), 2), fake((300, 520), 3))
    for e in Epilogue:
        bias = fake((520,), 4) if e.has_bias else None
        for fam, mode, acc in ((KernelFamily.Auto, KernelMathMode.StrictFp32, AccuracyContract.StrictFp32),
                               (KernelFamily.Simt, KernelMathMode.Exact, AccuracyContract.Exact)):
            validate(MatMulNode(epilogue=e, family=fam, math_mode=mode, accuracy=acc), *views, bias)
        if e.has_bias:
            with pytest.raises(PlanError):
                validate(MatMulNode(epilogue=e), *views, None)
    gv = (fake((4, 4096), 1), fake((4096, 4096), 2), fake((4, 4096), 3))
    assert validate(MatMulNode(epilogue=Epilogue.BIAS_GELU_ERF), *gv, fake((4096,), 4))["family"] == 2
    assert [e for e in Epilogue if e.has_bias] == [Epilogue.BIAS, Epilogue.BIAS_RELU, Epilogue.BIAS_RELU6,
                                                   Epilogue.BIAS_GELU_ERF, Epilogue.BIAS_GELU_TANH, Epilogue.BIAS_SILU]
    lib = _abi.load()
    d = execution._desc(MatMulNode(), *views, None, None)
    d.epilogue = 12
    info = _abi.MmrGemmInfo()
    assert lib.mmr_gemm_validate(ctypes.byref(d), ctypes.byref(info)) == _abi.ERR_INVALID_ARGUMENT


def test_host_entry_checks_arguments_before_any_device_work():
    """mmr_gemm_bind_host: host-side argument checks (rank, transpose_lhs,
    epilogue, bias, views inside their buffers, unit column stride) come
    before any device call."""
    lib = _abi.load()

    def desc(a, b, c, bias=None, **kw):
        d = _abi.MmrMatmulDesc()
        d.lhs, d.rhs, d.out = (execution._host_view(x, 0) for x in (a, b, c))
        if bias is not None:
            d.bias = execution._host_view(bias, 0)
        for k, v in kw.items():
            setattr(d, k, v)
        return d

    a, b, c = np.zeros((8, 4), np.float32), np.zeros((4, 16), np.float32), np.zeros((8, 16), np.float32)
    h = ctypes.c_void_p()
    bind = lambda d: lib.mmr_gemm_bind_host(ctypes.byref(d), 0, ctypes.byref(h))
    assert bind(desc(a, b, c, transpose_lhs=1)) == _abi.ERR_UNSUPPORTED_LAYOUT
    d = desc(a, b, c)
    d.lhs.rank = 3
    assert bind(d) == _abi.ERR_UNSUPPORTED_LAYOUT
    assert bind(desc(a, b, c, epilogue=12)) == _abi.ERR_INVALID_ARGUMENT
    assert bind(desc(a, b, c, epilogue=int(Epilogue.BIAS_SILU))) == _abi.ERR_INVALID_SHAPE  # no bias view
    d = desc(a, b, c)
    d.out.bytes = 4 * 100
    assert bind(d) == _abi.ERR_INVALID_SHAPE
    d = desc(a, b, c)
    d.rhs.strides[1] = 2
    assert bind(d) == _abi.ERR_UNSUPPORTED_LAYOUT
    assert lib.mmr_gemm_bind_host(ctypes.byref(desc(a, b, c)), 65, ctypes.byref(h)) == _abi.ERR_INVALID_ARGUMENT
    assert not h.value
    import torch
    if not torch.cuda.is_available():
        assert bind(desc(a, b, c)) == _abi.ERR_UNSUPPORTED_DEVICE


def test_math_contract_mirrors_reference():
    # validation.rs:3579-3640
    MatMulNode(math_mode=KernelMathMode.Tf32, accuracy=AccuracyContract.AllowTf32)
    MatMulNode(math_mode=KernelMathMode.StrictFp32, accuracy=AccuracyContract.AllowTf32)
    MatMulNode(math_mode=KernelMathMode.Exact, accuracy=AccuracyContract.Exact)
    with pytest.raises(PlanError):
        MatMulNode(math_mode=KernelMathMode.Tf32, accuracy=AccuracyContract.StrictFp32)
    with pytest.raises(PlanError):
        MatMulNode(math_mode=KernelMathMode.StrictFp32, accuracy=AccuracyContract.Exact)


def test_output_dims_helper():
    from momiru_b200 import output_dims
    assert output_dims(MatMulNode(), fake((2, 3, 4), 1), fake((4, 5), 2)) == (2, 3, 5)
    assert output_dims(MatMulNode(transpose_lhs=True), fake((4, 3), 1), fake((4, 5), 2)) == (3, 5)
    assert output_dims(MatMulNode(), fake((4,), 1), fake((4,), 2)) == ()


def test_view_ops():
    v = fake((4, 6), 1)
    t = v.transpose()
    assert t.dims == (6, 4) and t.strides == (1, 6)
    n = v.narrow(1, 2, 3)
    assert n.dims == (4, 3) and n.offset == 2
    s = v.slice([(1, 4, 2), None])
    assert s.dims == (2, 6) and s.strides == (12, 1) and s.offset == 6
    assert v.is_row_major_contiguous() and not t.is_row_major_contiguous()


def _numpy_matmul_dims(lhs, rhs, tl, tr):
    """The node's stated semantics, NumPy matmul with the transpose flags
    applied to the matrix axes; None where NumPy refuses (or a flag is set on
    a rank-1 operand, which the reference rejects)."""
    if (tl and len(lhs) == 1) or (tr and len(rhs) == 1):
        return None
    a = np.empty(lhs, np.float32)
    b = np.empty(rhs, np.float32)
    if tl:
        a = np.swapaxes(a, -1, -2)
    if tr:
        b = np.swapaxes(b, -1, -2)
    try:
        return np.matmul(a, b).shape
    except ValueError:
        return None


def test_shape_contract_matches_numpy_matmul_on_random_shapes():
    """Random ranks 1-8, extents 0-3 (0 and 1 included, so both broadcast
    rules and empty batches occur), transpose flags: the validator accepts
    exactly the shapes NumPy matmul accepts and only with NumPy's output dims
    (a vector-vector product included, whose output is rank 0)."""
    from hypothesis import given, settings, strategies as st
    dims = st.lists(st.integers(0, 3), min_size=1, max_size=8)

    @settings(max_examples=600, deadline=None, derandomize=True)
    @given(dims, dims, st.booleans(), st.booleans(), st.integers(0, 2))
    def check(lhs, rhs, tl, tr, bump):
        want = _numpy_matmul_dims(tuple(lhs), tuple(rhs), tl, tr)
        node = MatMulNode(transpose_lhs=tl, transpose_rhs=tr)
        if want is None:
            out = tuple(max(1, x) for x in lhs[:-1] + rhs[-1:])
            with pytest.raises(PlanError):
                validate(node, fake(lhs, 1), fake(rhs, 2), fake(out or (1,), 3))
            return
        validate(node, fake(lhs, 1), fake(rhs, 2), fake(want, 3))
        assert execution.output_dims(node, fake(lhs, 1), fake(rhs, 2)) == tuple(want)
        if bump and want:  # any other output extent is refused
            wrong = list(want)
            wrong[bump % len(wrong)] += 1
            with pytest.raises(PlanError):
                validate(node, fake(lhs, 1), fake(rhs, 2), fake(tuple(wrong), 3))

    check()


# ------------------------------------------------ frozen launch records --
def test_plan_launch_records_the_bound_launch_for_each_family():
    """The record bind would freeze, derived on the host for a 148-SM device:
    the 8192^3 node on CTA pairs (cluster 2, 256x256 tiles, 512 TMEM
    columns, TMA), the skinny-M node on the GEMV family (8-CTA clusters,
    split K), an exact node on the SIMT family (a grid, no TMA, no TMEM)."""
    from momiru_b200 import check_launch_record, plan_launch
    r = plan_launch(MatMulNode(epilogue=Epilogue.BIAS_RELU), fake((8192, 8192), 1), fake((8192, 8192), 2),
                    fake((8192, 8192), 3), fake((8192,), 4))
    assert r.family == _abi.FAMILY_TCGEN05 and r.matrix_acceleration == _abi.ACCEL_TCGEN05
    assert tuple(r.cluster) == (2, 1, 1) and r.cluster_launch == 1 and r.grid[0] == 148
    assert (r.tile_m, r.tile_n) == (256, 256) and r.tmem_columns_per_cta == 512 and r.tmem_accumulator_stages == 2
    assert r.async_copy == _abi.ASYNC_COPY_TMA and r.tensor_maps == 3 and r.producer_warps == 1
    assert r.partition == _abi.PARTITION_STREAM_K and r.stream_k_slices > 0 and r.persistent_ctas_per_sm == 1
    check_launch_record(r)
    tf32 = MatMulNode(math_mode=KernelMathMode.Tf32, accuracy=AccuracyContract.AllowTf32)
    g = plan_launch(tf32, fake((16, 4096), 1), fake((4096, 4096), 2), fake((16, 4096), 3))
    # skinny M, TF32: on the tensor cores, 4-CTA clusters over K, 128 x 16 swap-AB tiles, two
    # interleaved 16-column accumulators per chunk buffer (64 TMEM columns), 11 stages
    assert g.family == _abi.FAMILY_GEMV and tuple(g.cluster) == (1, 4, 1) and g.partition == _abi.PARTITION_SPLIT_K
    assert g.use_distributed_shared_memory == 1 and g.matrix_acceleration == _abi.ACCEL_TCGEN05
    assert (g.tile_m, g.tile_n, g.tile_k, g.tmem_columns_per_cta, g.tensor_maps) == (16, 128, 32, 64, 2)
    assert g.pipeline_stages == 11
    check_launch_record(g)
    # StrictFp32 at M = 16: tensor cores too, with lo(B) in TMEM (256 columns), 4 stages
    s = plan_launch(MatMulNode(), fake((16, 4096), 1), fake((4096, 4096), 2), fake((16, 4096), 3))
    assert s.family == _abi.FAMILY_GEMV and tuple(s.cluster) == (1, 4, 1) and s.tmem_columns_per_cta == 256
    assert s.matrix_acceleration == _abi.ACCEL_TCGEN05 and s.pipeline_stages == 4
    check_launch_record(s)
    # StrictFp32 at M <= 8, TF32 at M = 1, or an A without a 16-byte row pitch: the CUDA-core GEMV
    # (8-CTA clusters, no TMEM)
    for node, m in ((MatMulNode(), 8), (MatMulNode(), 1), (tf32, 1)):
        c = plan_launch(node, fake((m, 4096), 1), fake((4096, 4096), 2), fake((m, 4096), 3))
        assert c.family == _abi.FAMILY_GEMV and tuple(c.cluster) == (1, 8, 1) and c.tmem_columns_per_cta == 0
        assert c.matrix_acceleration == _abi.ACCEL_NONE
        check_launch_record(c)
    c = plan_launch(tf32, fake((5, 4095), 1, pad_cols=4097), fake((4095, 4096), 2), fake((5, 4096), 3))
    assert c.family == _abi.FAMILY_GEMV and tuple(c.cluster) == (1, 8, 1) and c.tmem_columns_per_cta == 0
    check_launch_record(c)
    e = plan_launch(MatMulNode(math_mode=KernelMathMode.Exact, accuracy=AccuracyContract.Exact), fake((100, 64), 1),
                    fake((64, 200), 2), fake((100, 200), 3))
    assert e.family == _abi.FAMILY_SIMT and e.async_copy == _abi.ASYNC_COPY_NONE and tuple(e.grid) == (4, 2, 1)
    check_launch_record(e)
    # small output with a long K: tiles split along K over several pairs
    s = plan_launch(MatMulNode(), fake((1024, 8192), 1), fake((8192, 1024), 2), fake((1024, 1024), 3))
    assert s.split_k > 1 and s.grid[0] == 2 * 16 * s.split_k
    # 512^3 (four pair tiles, K = 512): K is not split below 512 (3xTF32) or 1024 (TF32)
    for node in (MatMulNode(), tf32):
        s = plan_launch(node, fake((512, 512), 1), fake((512, 512), 2), fake((512, 512), 3))
        assert s.split_k == 1 and s.grid[0] == 2 * 4


def test_check_launch_record_enforces_the_gpu_validator_rules():
    """validation.rs:5846-5911 on the record: tcgen05 needs TMEM, TMEM columns
    a power of two and a multiple of 32 up to 512, TMA needs tensor maps,
    clusters up to 8 and launched as clusters, shared memory within 227 KB."""
    from momiru_b200 import check_launch_record, plan_launch
    from momiru_b200.execution import PlanMismatch
    base = plan_launch(MatMulNode(), fake((4096, 4096), 1), fake((4096, 4096), 2), fake((4096, 4096), 3))
    check_launch_record(base)

    def broken(**kw):
        r = _abi.MmrLaunchRecord.from_buffer_copy(base)
        for k, v in kw.items():
            if isinstance(v, tuple):
                getattr(r, k)[:] = v
            else:
                setattr(r, k, v)
        with pytest.raises(PlanMismatch):
            check_launch_record(r)

    broken(tmem_columns_per_cta=0, tmem_accumulator_stages=0)   # tcgen05 without TMEM
    broken(tmem_columns_per_cta=384)                            # not a power of two
    broken(tmem_columns_per_cta=1024)                           # above 512
    broken(tmem_columns_per_cta=16)                             # below the 32-column unit
    broken(tensor_maps=0)                                       # TMA without maps
    broken(cluster=(16, 1, 1))                                  # non-portable cluster
    broken(cluster_launch=0)                                    # cluster dims without a cluster launch
    broken(dynamic_shared_bytes=240 * 1024)                     # above 227 KB
    broken(warps_per_block=3)                                   # inconsistent with the block
    broken(matrix_acceleration=4)                               # wgmma is not an sm_100a path
    broken(split_k=0)
