"""ctypes bindings of the C ABI declared in include/momiru_gemm.h.

The shared library is built in-tree (momiru_b200/lib/libmomiru_gemm.so) by
momiru_b200/build.py. There is no fallback: if the library is missing the
import of the execution layer fails loudly.
"""
from __future__ import annotations

import ctypes
import os

MAX_RANK = 8

# status codes
OK = 0
ERR_INVALID_ARGUMENT = 1
ERR_INVALID_SHAPE = 2
ERR_UNSUPPORTED_LAYOUT = 3
ERR_UNSAFE_ALIASING = 4
ERR_UNSUPPORTED_MATH = 5
ERR_UNSUPPORTED_DEVICE = 6
ERR_OUT_OF_BOUNDS = 7
ERR_CUDA = 8
ERR_PEER_ACCESS = 9
ERR_TIMEOUT = 10
ERR_DEVICE_FAULT_FLAG = 11
ERR_UNSUPPORTED_FAMILY = 12
ERR_PLAN_MISMATCH = 13

MATH_STRICT_FP32, MATH_TF32, MATH_EXACT = 0, 1, 2
EPI_NONE, EPI_BIAS, EPI_BIAS_RELU, EPI_RELU = 0, 1, 2, 3
EPI_RELU6, EPI_BIAS_RELU6, EPI_GELU_ERF, EPI_BIAS_GELU_ERF = 4, 5, 6, 7
EPI_GELU_TANH, EPI_BIAS_GELU_TANH, EPI_SILU, EPI_BIAS_SILU = 8, 9, 10, 11
FAMILY_AUTO, FAMILY_TCGEN05, FAMILY_GEMV, FAMILY_SIMT = 0, 1, 2, 3
FAMILY_NAMES = {FAMILY_AUTO: "auto", FAMILY_TCGEN05: "tcgen05", FAMILY_GEMV: "gemv", FAMILY_SIMT: "simt"}

EXPORTED = [
    "mmr_gemm_validate", "mmr_gemm_bind", "mmr_gemm_run", "mmr_gemm_run_on", "mmr_gemm_quiesce",
    "mmr_gemm_destroy", "mmr_gemm_query", "mmr_last_error", "mmr_version",
    "mmr_selftest_bounded_wait", "mmr_shard_columns", "mmr_gemm_run_noalloc",
    "mmr_ipc_export", "mmr_ipc_import", "mmr_ipc_release", "mmr_sharded_gemm_bind", "mmr_gemm_bind_host",
    "mmr_shard_local_desc", "mmr_gemm_plan_launch", "mmr_gemm_launch_record", "mmr_check_launch_record",
    "mmr_gemm_bind_frozen",
]
ACCEL_NONE, ACCEL_TCGEN05 = 0, 5
ASYNC_COPY_NONE, ASYNC_COPY_TMA = 0, 4
PARTITION_GRID, PARTITION_SPLIT_K, PARTITION_STREAM_K, PARTITION_PERSISTENT_CTA = 0, 1, 2, 3
NOALLOC_SCRATCH_BYTES = 64 * 1024
NOALLOC_MAX_TILES = 8189


class MmrView(ctypes.Structure):
    _fields_ = [
        ("address", ctypes.c_uint64),
        ("bytes", ctypes.c_uint64),
        ("base_offset_bytes", ctypes.c_uint64),
        ("rank", ctypes.c_int32),
        ("device_ordinal", ctypes.c_int32),
        ("dims", ctypes.c_int64 * MAX_RANK),
        ("strides", ctypes.c_int64 * MAX_RANK),
        ("allocation_id", ctypes.c_uint64),
    ]


class MmrMatmulDesc(ctypes.Structure):
    _fields_ = [
        ("lhs", MmrView),
        ("rhs", MmrView),
        ("out", MmrView),
        ("bias", MmrView),
        ("transpose_lhs", ctypes.c_int32),
        ("transpose_rhs", ctypes.c_int32),
        ("math_mode", ctypes.c_int32),
        ("epilogue", ctypes.c_int32),
        ("family", ctypes.c_int32),
        ("device_ordinal", ctypes.c_int32),
        ("stream", ctypes.c_void_p),
    ]


class MmrGemmInfo(ctypes.Structure):
    _fields_ = [
        ("family", ctypes.c_int32),
        ("math_mode", ctypes.c_int32),
        ("batch", ctypes.c_int64),
        ("m", ctypes.c_int64),
        ("n", ctypes.c_int64),
        ("k", ctypes.c_int64),
        ("a_mn_major", ctypes.c_int32),
        ("b_mn_major", ctypes.c_int32),
        ("grid", ctypes.c_int32),
        ("block", ctypes.c_int32),
        ("cluster", ctypes.c_int32),
        ("smem_bytes", ctypes.c_int32),
        ("tile_m", ctypes.c_int32),
        ("tile_n", ctypes.c_int32),
        ("tile_k", ctypes.c_int32),
        ("stages", ctypes.c_int32),
        ("tiles", ctypes.c_int64),
        ("flops", ctypes.c_double),
        ("bytes", ctypes.c_double),
    ]

    def as_dict(self) -> dict:
        return {name: getattr(self, name) for name, _ in self._fields_}


class MmrLaunchRecord(ctypes.Structure):
    """mmr_launch_record: the GpuKernelPlan fields the library freezes."""
    _fields_ = [
        ("family", ctypes.c_int32),
        ("math_mode", ctypes.c_int32),
        ("grid", ctypes.c_int32 * 3),
        ("block", ctypes.c_int32 * 3),
        ("cluster", ctypes.c_int32 * 3),
        ("dynamic_shared_bytes", ctypes.c_int32),
        ("tmem_columns_per_cta", ctypes.c_int32),
        ("tmem_accumulator_stages", ctypes.c_int32),
        ("tile_m", ctypes.c_int32),
        ("tile_n", ctypes.c_int32),
        ("tile_k", ctypes.c_int32),
        ("pipeline_stages", ctypes.c_int32),
        ("warps_per_block", ctypes.c_int32),
        ("producer_warps", ctypes.c_int32),
        ("consumer_warps", ctypes.c_int32),
        ("matrix_acceleration", ctypes.c_int32),
        ("async_copy", ctypes.c_int32),
        ("tensor_maps", ctypes.c_int32),
        ("partition", ctypes.c_int32),
        ("split_k", ctypes.c_int32),
        ("stream_k_slices", ctypes.c_int32),
        ("persistent_ctas_per_sm", ctypes.c_int32),
        ("cluster_launch", ctypes.c_int32),
        ("use_distributed_shared_memory", ctypes.c_int32),
    ]

    def as_dict(self) -> dict:
        out = {}
        for name, typ in self._fields_:
            v = getattr(self, name)
            out[name] = tuple(v) if hasattr(typ, "_length_") else v
        return out


class MmrIpcHandle(ctypes.Structure):
    _fields_ = [("bytes", ctypes.c_uint8 * 64), ("offset", ctypes.c_uint64)]


class MmrShardedDesc(ctypes.Structure):
    _fields_ = [
        ("local", MmrMatmulDesc),
        ("rank", ctypes.c_int32),
        ("nranks", ctypes.c_int32),
        ("peer_out", ctypes.c_uint64 * 8),
        ("peer_signal", ctypes.c_uint64 * 8),
        ("signal", ctypes.c_uint64),
    ]


HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libmomiru_gemm.so")
_lib = None


def load() -> ctypes.CDLL:
    """Load the in-tree library (build it first with momiru_b200.build)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"momiru_b200: CUDA library not built ({LIB_PATH} missing); run `python -m momiru_b200.build`")
    lib = ctypes.CDLL(LIB_PATH)
    P = ctypes.POINTER
    h = ctypes.c_void_p
    lib.mmr_gemm_validate.argtypes = [P(MmrMatmulDesc), P(MmrGemmInfo)]
    lib.mmr_gemm_bind.argtypes = [P(MmrMatmulDesc), P(h)]
    lib.mmr_gemm_run.argtypes = [h]
    lib.mmr_gemm_run_on.argtypes = [h, ctypes.c_void_p]
    lib.mmr_gemm_quiesce.argtypes = [h, ctypes.c_uint64]
    lib.mmr_gemm_destroy.argtypes = [h]
    lib.mmr_gemm_query.argtypes = [h, P(MmrGemmInfo)]
    lib.mmr_last_error.restype = ctypes.c_char_p
    lib.mmr_version.restype = ctypes.c_char_p
    lib.mmr_selftest_bounded_wait.argtypes = [ctypes.c_int32, ctypes.c_uint64]
    lib.mmr_gemm_run_noalloc.argtypes = [P(MmrMatmulDesc), P(ctypes.c_int32)]
    lib.mmr_ipc_export.argtypes = [ctypes.c_uint64, P(MmrIpcHandle)]
    lib.mmr_ipc_import.argtypes = [P(MmrIpcHandle), ctypes.c_int32, P(ctypes.c_uint64)]
    lib.mmr_ipc_release.argtypes = [ctypes.c_uint64, P(MmrIpcHandle)]
    lib.mmr_sharded_gemm_bind.argtypes = [P(MmrShardedDesc), P(h)]
    lib.mmr_gemm_bind_host.argtypes = [P(MmrMatmulDesc), ctypes.c_int32, P(h)]
    lib.mmr_gemm_plan_launch.argtypes = [P(MmrMatmulDesc), ctypes.c_int32, P(MmrLaunchRecord)]
    lib.mmr_gemm_launch_record.argtypes = [h, P(MmrLaunchRecord)]
    lib.mmr_check_launch_record.argtypes = [P(MmrLaunchRecord)]
    lib.mmr_gemm_bind_frozen.argtypes = [P(MmrMatmulDesc), P(MmrLaunchRecord), P(h)]
    lib.mmr_shard_local_desc.argtypes = [P(MmrMatmulDesc), ctypes.c_int32, ctypes.c_int32, P(MmrMatmulDesc),
                                         P(ctypes.c_int64), P(ctypes.c_int64), P(ctypes.c_uint64)]
    lib.mmr_shard_columns.argtypes = [ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                      P(ctypes.c_int64), P(ctypes.c_int64)]
    for name in EXPORTED:
        fn = getattr(lib, name)
        if name not in ("mmr_last_error", "mmr_version"):
            fn.restype = ctypes.c_int32
    _lib = lib
    return lib


def last_error() -> str:
    return load().mmr_last_error().decode(errors="replace")
