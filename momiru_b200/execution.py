"""Frozen GPU MatMul node: validate, bind once, replay, quiesce.

Host-side mirror of the reference's execution contract for this one node:
  * the node:      Operation::MatMul{transpose_lhs, transpose_rhs}
                   (src/momiru/tensor_light/execution/ir.rs:1468-1473), with an
                   optional fused Add(bias)/Relu epilogue (the reference's
                   FusedStaticDataflow node, plan.rs:1080-1106)
  * math contract: validate_node_math_contract (validation.rs:3579-3640);
                   StrictFp32 runs as 3xTF32, Tf32 as one TF32 pass, Exact in
                   the reference's own per-element order
  * bind/replay:   Backend::bind_resources / BoundBackend::execute_gpu_node /
                   quiesce_or_abort (runtime.rs:879-988)
Every call goes through the C ABI (include/momiru_gemm.h); errors come back as
typed exceptions carrying the ABI status code, never as a silent fallback.
"""
from __future__ import annotations

import ctypes
import enum
from dataclasses import dataclass

from . import _abi
from .tensor import DeviceView


class AccuracyContract(enum.IntEnum):
    """ir.rs:541-553, same order."""
    Exact = 0
    StrictFp32 = 1
    AllowAlgebraic = 2
    AllowFastMath = 3
    AllowTf32 = 4
    AllowFp16Accumulate = 5
    AllowBf16Accumulate = 6
    QuantizedExactScale = 7
    TargetVerified = 8


class KernelMathMode(enum.IntEnum):
    """The subset of ir.rs:559-569 this GPU node executes."""
    Exact = 0
    StrictFp32 = 1
    Tf32 = 4


_MATH_TO_ABI = {KernelMathMode.StrictFp32: _abi.MATH_STRICT_FP32, KernelMathMode.Tf32: _abi.MATH_TF32,
                KernelMathMode.Exact: _abi.MATH_EXACT}


class Epilogue(enum.IntEnum):
    """MatMul -> optional Add(bias[N]) -> optional activation, one fused node.
    The activations are the reference CPU provider's elementwise kernels
    (cpu.rs:2158-2168 ReLU/ReLU6/SiLU, 2117-2129 GELU-erf, 2214-2222 GELU-tanh)."""
    NONE = _abi.EPI_NONE
    BIAS = _abi.EPI_BIAS
    BIAS_RELU = _abi.EPI_BIAS_RELU
    RELU = _abi.EPI_RELU
    RELU6 = _abi.EPI_RELU6
    BIAS_RELU6 = _abi.EPI_BIAS_RELU6
    GELU_ERF = _abi.EPI_GELU_ERF
    BIAS_GELU_ERF = _abi.EPI_BIAS_GELU_ERF
    GELU_TANH = _abi.EPI_GELU_TANH
    BIAS_GELU_TANH = _abi.EPI_BIAS_GELU_TANH
    SILU = _abi.EPI_SILU
    BIAS_SILU = _abi.EPI_BIAS_SILU

    @property
    def has_bias(self) -> bool:
        return self in (Epilogue.BIAS, Epilogue.BIAS_RELU) or (self >= Epilogue.RELU6 and self & 1 == 1)


class KernelFamily(enum.IntEnum):
    Auto = _abi.FAMILY_AUTO
    Tcgen05 = _abi.FAMILY_TCGEN05
    Gemv = _abi.FAMILY_GEMV
    Simt = _abi.FAMILY_SIMT


# ------------------------------------------------------------------ errors --
class PlanError(Exception):
    code = -1

    def __init__(self, message: str, code: int | None = None):
        super().__init__(message)
        if code is not None:
            self.code = code


class InvalidArgument(PlanError): code = _abi.ERR_INVALID_ARGUMENT
class InvalidShape(PlanError): code = _abi.ERR_INVALID_SHAPE
class UnsupportedLayout(PlanError): code = _abi.ERR_UNSUPPORTED_LAYOUT
class UnsafeAliasing(PlanError): code = _abi.ERR_UNSAFE_ALIASING
class InvalidAccuracyContract(PlanError): code = _abi.ERR_UNSUPPORTED_MATH
class UnsupportedDevice(PlanError): code = _abi.ERR_UNSUPPORTED_DEVICE
class OutOfBounds(PlanError): code = _abi.ERR_OUT_OF_BOUNDS
class CudaError(PlanError): code = _abi.ERR_CUDA
class PeerAccessError(PlanError): code = _abi.ERR_PEER_ACCESS
class QuiescenceTimeout(PlanError): code = _abi.ERR_TIMEOUT
class DeviceErrorFlag(PlanError): code = _abi.ERR_DEVICE_FAULT_FLAG
class UnsupportedFamily(PlanError): code = _abi.ERR_UNSUPPORTED_FAMILY
class PlanMismatch(PlanError): code = _abi.ERR_PLAN_MISMATCH


_BY_CODE = {c.code: c for c in (InvalidArgument, InvalidShape, UnsupportedLayout, UnsafeAliasing,
                                InvalidAccuracyContract, UnsupportedDevice, OutOfBounds, CudaError, PeerAccessError,
                                QuiescenceTimeout, DeviceErrorFlag, UnsupportedFamily, PlanMismatch)}


def _check(rc: int) -> None:
    if rc != _abi.OK:
        cls = _BY_CODE.get(rc, PlanError)
        raise cls(_abi.last_error(), rc)


# -------------------------------------------------------------------- node --
@dataclass(frozen=True)
class MatMulNode:
    transpose_lhs: bool = False
    transpose_rhs: bool = False
    math_mode: KernelMathMode = KernelMathMode.StrictFp32
    epilogue: Epilogue = Epilogue.NONE
    family: KernelFamily = KernelFamily.Auto
    accuracy: AccuracyContract = AccuracyContract.StrictFp32  # of the output tensor

    def __post_init__(self):
        validate_node_math_contract(self.math_mode, self.accuracy)


def validate_node_math_contract(mode: KernelMathMode, accuracy: AccuracyContract) -> None:
    """validation.rs:3579-3640 for the modes this node runs."""
    A = AccuracyContract
    if mode == KernelMathMode.Exact:
        ok = True
    elif mode == KernelMathMode.StrictFp32:
        ok = accuracy in (A.StrictFp32, A.AllowAlgebraic, A.AllowFastMath, A.AllowTf32, A.AllowFp16Accumulate,
                          A.AllowBf16Accumulate, A.TargetVerified)
    elif mode == KernelMathMode.Tf32:
        ok = accuracy in (A.AllowTf32, A.AllowFastMath, A.TargetVerified)
    else:
        ok = False
    if not ok:
        raise InvalidAccuracyContract(f"math mode {mode.name} is not permitted by accuracy {accuracy.name}",
                                      _abi.ERR_UNSUPPORTED_MATH)


def _desc(node: MatMulNode, lhs: DeviceView, rhs: DeviceView, out: DeviceView, bias: DeviceView | None,
          stream: int | None) -> _abi.MmrMatmulDesc:
    d = _abi.MmrMatmulDesc()
    d.lhs = lhs.to_abi()
    d.rhs = rhs.to_abi()
    d.out = out.to_abi()
    if bias is not None:
        d.bias = bias.to_abi()
    d.transpose_lhs = int(node.transpose_lhs)
    d.transpose_rhs = int(node.transpose_rhs)
    d.math_mode = _MATH_TO_ABI[node.math_mode]
    d.epilogue = int(node.epilogue)
    d.family = int(node.family)
    d.device_ordinal = out.buffer.device_ordinal
    d.stream = stream or None
    return d


def validate(node: MatMulNode, lhs: DeviceView, rhs: DeviceView, out: DeviceView,
             bias: DeviceView | None = None) -> dict:
    """Host-only contract check and family choice (no GPU needed)."""
    lib = _abi.load()
    info = _abi.MmrGemmInfo()
    _check(lib.mmr_gemm_validate(ctypes.byref(_desc(node, lhs, rhs, out, bias, None)), ctypes.byref(info)))
    return info.as_dict()


def plan_launch(node: MatMulNode, lhs: DeviceView, rhs: DeviceView, out: DeviceView,
                bias: DeviceView | None = None, sm_count: int = 148) -> _abi.MmrLaunchRecord:
    """The launch record bind would freeze for this node on a device with
    `sm_count` SMs (host only): what a plan's GpuKernelPlan carries for it."""
    rec = _abi.MmrLaunchRecord()
    _check(_abi.load().mmr_gemm_plan_launch(ctypes.byref(_desc(node, lhs, rhs, out, bias, None)), sm_count,
                                            ctypes.byref(rec)))
    return rec


def check_launch_record(rec: _abi.MmrLaunchRecord) -> None:
    """The GPU validator's rules on a frozen launch record (host only)."""
    _check(_abi.load().mmr_check_launch_record(ctypes.byref(rec)))


class BoundGemm:
    """A bound GPU MatMul node (BoundBackend for one frozen node).

    With `frozen` (an MmrLaunchRecord from the plan), the node binds only to
    exactly that launch; any difference raises PlanMismatch."""

    def __init__(self, node: MatMulNode, lhs: DeviceView, rhs: DeviceView, out: DeviceView,
                 bias: DeviceView | None = None, stream: int | None = None,
                 frozen: _abi.MmrLaunchRecord | None = None):
        self._lib = _abi.load()
        self.node = node
        # Keep the views (and so their buffers) alive for the handle's lifetime.
        self._views = (lhs, rhs, out, bias)
        self._handle = ctypes.c_void_p()
        desc = _desc(node, lhs, rhs, out, bias, stream)
        if frozen is None:
            _check(self._lib.mmr_gemm_bind(ctypes.byref(desc), ctypes.byref(self._handle)))
        else:
            _check(self._lib.mmr_gemm_bind_frozen(ctypes.byref(desc), ctypes.byref(frozen),
                                                  ctypes.byref(self._handle)))
        info = _abi.MmrGemmInfo()
        _check(self._lib.mmr_gemm_query(self._handle, ctypes.byref(info)))
        self.info = info.as_dict()

    @property
    def family(self) -> str:
        return _abi.FAMILY_NAMES[self.info["family"]]

    def launch_record(self) -> _abi.MmrLaunchRecord:
        rec = _abi.MmrLaunchRecord()
        _check(self._lib.mmr_gemm_launch_record(self._handle, ctypes.byref(rec)))
        return rec

    def replay(self, stream: int | None = None) -> None:
        if not self._handle:
            raise InvalidArgument("handle closed")
        if stream is None:
            _check(self._lib.mmr_gemm_run(self._handle))
        else:
            _check(self._lib.mmr_gemm_run_on(self._handle, ctypes.c_void_p(stream)))

    def quiesce_or_abort(self, timeout_s: float = 30.0) -> None:
        _check(self._lib.mmr_gemm_quiesce(self._handle, int(timeout_s * 1e9)))

    def close(self) -> None:
        if self._handle:
            rc = self._lib.mmr_gemm_destroy(self._handle)
            self._handle = ctypes.c_void_p()
            _check(rc)

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            if self._handle:
                self._lib.mmr_gemm_destroy(self._handle)
        except Exception:
            pass


def _host_view(arr, device_ordinal: int) -> _abi.MmrView:
    """An MmrView over a host f32 numpy array (row-major rows, any row pitch)."""
    import numpy as np
    if not isinstance(arr, np.ndarray) or arr.dtype != np.float32:
        raise InvalidArgument("host operands are float32 numpy arrays", _abi.ERR_INVALID_ARGUMENT)
    if arr.ndim not in (1, 2) or (arr.size and arr.strides[-1] != 4):
        raise UnsupportedLayout("host operands are rank 1-2 with unit column stride", _abi.ERR_UNSUPPORTED_LAYOUT)
    v = _abi.MmrView()
    v.address = arr.ctypes.data
    v.bytes = 4 * max(arr.size, 1) if arr.ndim == 1 else 4 * (
        ((arr.shape[0] - 1) * (arr.strides[0] // 4) + arr.shape[1]) if arr.size else 0)
    v.base_offset_bytes = 0
    v.rank = arr.ndim
    v.device_ordinal = device_ordinal
    for i, d in enumerate(arr.shape):
        v.dims[i] = d
        v.strides[i] = arr.strides[i] // 4 if arr.size else (arr.shape[1] if i == 0 and arr.ndim == 2 else 1)
    v.allocation_id = 0  # host operands are copied to buffers of the handle's own
    return v


class HostGemm:
    """The MatMul node over operands in HOST memory, as the reference's own
    CPU provider is called (cpu.rs:651-654 binds host buffers only).

    Binds mmr_gemm_bind_host: each replay copies rhs and bias to the device,
    then streams lhs by row panels (``panels``; 0 = one per 512 rows, at most
    16), each panel's GEMM starting as soon as its
    rows have landed and its output rows copied back while later panels copy
    in and compute. Arrays should live in pinned memory (e.g.
    ``torch.empty(..., pin_memory=True).numpy()``) for the copies to overlap.
    ``out`` may be a column-narrowed view of a wider array: only its logical
    columns are written.
    """

    def __init__(self, node: MatMulNode, lhs, rhs, out, bias=None, panels: int = 0, device_ordinal: int = 0,
                 stream: int | None = None):
        self._lib = _abi.load()
        self.node = node
        self._arrays = (lhs, rhs, out, bias)
        d = _abi.MmrMatmulDesc()
        d.lhs = _host_view(lhs, device_ordinal)
        d.rhs = _host_view(rhs, device_ordinal)
        d.out = _host_view(out, device_ordinal)
        if bias is not None:
            d.bias = _host_view(bias, device_ordinal)
        d.transpose_lhs = int(node.transpose_lhs)
        d.transpose_rhs = int(node.transpose_rhs)
        d.math_mode = _MATH_TO_ABI[node.math_mode]
        d.epilogue = int(node.epilogue)
        d.family = int(node.family)
        d.device_ordinal = device_ordinal
        d.stream = stream or None
        self._handle = ctypes.c_void_p()
        _check(self._lib.mmr_gemm_bind_host(ctypes.byref(d), int(panels), ctypes.byref(self._handle)))
        info = _abi.MmrGemmInfo()
        _check(self._lib.mmr_gemm_query(self._handle, ctypes.byref(info)))
        self.info = info.as_dict()

    @property
    def family(self) -> str:
        return _abi.FAMILY_NAMES[self.info["family"]]

    def replay(self, stream: int | None = None) -> None:
        if not self._handle:
            raise InvalidArgument("handle closed")
        if stream is None:
            _check(self._lib.mmr_gemm_run(self._handle))
        else:
            _check(self._lib.mmr_gemm_run_on(self._handle, ctypes.c_void_p(stream)))

    def quiesce_or_abort(self, timeout_s: float = 60.0) -> None:
        _check(self._lib.mmr_gemm_quiesce(self._handle, int(timeout_s * 1e9)))

    def close(self) -> None:
        if self._handle:
            rc = self._lib.mmr_gemm_destroy(self._handle)
            self._handle = ctypes.c_void_p()
            _check(rc)

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            if self._handle:
                self._lib.mmr_gemm_destroy(self._handle)
        except Exception:
            pass


def output_dims(node: MatMulNode, lhs: DeviceView, rhs: DeviceView) -> tuple:
    """Output shape by the MatMul contract (validation.rs:2300-2398)."""
    lv, rv = lhs.rank == 1, rhs.rank == 1
    if lv:
        m, k = 1, lhs.dims[0]
    else:
        r, c = lhs.dims[-2:]
        m, k = (c, r) if node.transpose_lhs else (r, c)
    if rv:
        n = 1
    else:
        r, c = rhs.dims[-2:]
        n = r if node.transpose_rhs else c
    lb = () if lv else tuple(lhs.dims[:-2])
    rb = () if rv else tuple(rhs.dims[:-2])
    br = max(len(lb), len(rb))
    lb = (1,) * (br - len(lb)) + lb
    rb = (1,) * (br - len(rb)) + rb
    batch = []
    for a, b in zip(lb, rb):
        if a == b or b == 1:
            batch.append(a)
        elif a == 1:
            batch.append(b)
        else:
            raise InvalidShape(f"batch extents {a} and {b} do not broadcast", _abi.ERR_INVALID_SHAPE)
    out = list(batch)
    if not lv:
        out.append(m)
    if not rv:
        out.append(n)
    return tuple(out)


def matmul(lhs: DeviceView, rhs: DeviceView, bias: DeviceView | None = None, node: MatMulNode | None = None,
           out: DeviceView | None = None, stream: int | None = None, timeout_s: float = 60.0) -> DeviceView:
    """One-shot convenience: bind, replay once, quiesce, release."""
    node = node or MatMulNode()
    if out is None:
        dims = output_dims(node, lhs, rhs)
        out = DeviceView.empty(dims, lhs.buffer.device_ordinal)
    with BoundGemm(node, lhs, rhs, out, bias, stream) as g:
        g.replay()
        g.quiesce_or_abort(timeout_s)
    return out


def selftest_bounded_wait(device_ordinal: int = 0, limit_s: float = 0.05) -> int:
    """Run the device bounded-wait probe; returns the ABI status (TIMEOUT = healthy)."""
    return _abi.load().mmr_selftest_bounded_wait(device_ordinal, int(limit_s * 1e9))


def shard_columns(n: int, nranks: int, rank: int, align: int = 256) -> tuple:
    lib = _abi.load()
    c0, c1 = ctypes.c_int64(), ctypes.c_int64()
    _check(lib.mmr_shard_columns(n, nranks, rank, align, ctypes.byref(c0), ctypes.byref(c1)))
    return c0.value, c1.value
