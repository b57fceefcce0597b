"""momiru_b200 -- B200 (sm_100a) f32 matmul hot path for Momiru's frozen-plan GEMM node.

The compute path is the in-tree CUDA library (csrc/, built by build.py) behind
the C ABI in include/momiru_gemm.h; this package is the host-side mirror of
the reference's node / bind / replay / quiesce interface.
"""
from .execution import (AccuracyContract, BoundGemm, Epilogue, HostGemm, KernelFamily,
                        KernelMathMode, MatMulNode, PlanError, check_launch_record, matmul, output_dims,
                        plan_launch, selftest_bounded_wait, shard_columns, validate)
from .tensor import DeviceBuffer, DeviceView

__all__ = [
    "AccuracyContract", "BoundGemm", "DeviceBuffer", "DeviceView", "Epilogue", "HostGemm",
    "KernelFamily",
    "KernelMathMode", "MatMulNode", "PlanError", "check_launch_record", "matmul", "output_dims", "plan_launch",
    "selftest_bounded_wait", "shard_columns", "validate",
]
