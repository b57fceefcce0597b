//! Validator extension for GPU MatMul nodes, and the conversion of a frozen
//! `GpuKernelPlan` (plan.rs:941-1026) to the library's launch record.
//!
//! The reference's validator rejects the CPU-only GEMM families on a GPU
//! placement (validation.rs:5500-5516) and admits fusion only for
//! `FusedStaticDataflow`, `TargetNative` or `VendorExact`
//! (validation.rs:4036-4050). A GPU MatMul node of this backend is frozen as
//! `KernelFamily::TargetNative` with an `ArtifactKind::Cubin` artifact
//! (target.rs:714-716) built from `libmomiru_gemm`, or as
//! `FusedStaticDataflow` when it carries the bias / activation epilogue; the
//! record's matrix acceleration names the library family (tcgen05, or none for
//! the GEMV and exact CUDA-core families).
//!
//! NOT COMPILED HERE (no Rust toolchain in the build image).

use super::{ffi, GpuGemmError};
use crate::tensor_light::execution::ir::Operation;
use crate::tensor_light::execution::plan::{
    AsyncCopyKind, FrozenNode, GpuKernelPlan, GpuPartitionKind, KernelFamily, MatrixAcceleration,
};

/// Structural admission of a GPU MatMul node (the rules this backend adds to
/// the plan validator's GPU branch).
pub fn check_gpu_matmul_kernel(node: &FrozenNode, kernel: &GpuKernelPlan) -> Result<(), GpuGemmError> {
    if !matches!(node.operation, Operation::MatMul { .. }) {
        return Err(GpuGemmError::UnsupportedOperation);
    }
    match kernel.family {
        KernelFamily::TargetNative => {
            if !node.fused_operations.is_empty() {
                // a fused epilogue is frozen as FusedStaticDataflow
                return Err(GpuGemmError::UnsupportedOperation);
            }
        }
        KernelFamily::FusedStaticDataflow => {
            if node.fused_operations.is_empty() {
                return Err(GpuGemmError::UnsupportedOperation);
            }
        }
        _ => return Err(GpuGemmError::UnsupportedOperation),
    }
    // The library runs tcgen05 (with TMA) or no tensor-core path; multicast
    // TMA is never frozen for it.
    if !matches!(kernel.matrix_acceleration, MatrixAcceleration::Tcgen05 | MatrixAcceleration::None) {
        return Err(GpuGemmError::UnsupportedOperation);
    }
    if !matches!(kernel.async_copy, AsyncCopyKind::Tma | AsyncCopyKind::None) {
        return Err(GpuGemmError::UnsupportedOperation);
    }
    // The GPU validator's TMEM / tcgen05 rules, checked here on the record the
    // library will be held to (validation.rs:5846-5911): the library repeats
    // them in mmr_check_launch_record.
    let rec = launch_record_of(kernel);
    super::status(unsafe { ffi::mmr_check_launch_record(&rec) })
}

/// Library family a frozen kernel names: tcgen05 acceleration is the
/// tensor-core family; otherwise a TMA split-K cluster launch is the GEMV
/// family and a plain grid the exact CUDA-core family.
pub fn family_of(kernel: &GpuKernelPlan) -> Result<i32, GpuGemmError> {
    Ok(match (kernel.matrix_acceleration, kernel.async_copy, kernel.partition) {
        (MatrixAcceleration::Tcgen05, AsyncCopyKind::Tma, _) => ffi::MMR_FAMILY_TCGEN05,
        (MatrixAcceleration::None, AsyncCopyKind::Tma, GpuPartitionKind::SplitK) => ffi::MMR_FAMILY_GEMV,
        (MatrixAcceleration::None, AsyncCopyKind::None, GpuPartitionKind::Grid) => ffi::MMR_FAMILY_SIMT,
        _ => return Err(GpuGemmError::UnsupportedOperation),
    })
}

/// The fields of a frozen `GpuKernelPlan` the library decides, in its launch
/// record (enum discriminants are the reference's own: MatrixAcceleration,
/// AsyncCopyKind and GpuPartitionKind are `#[repr(u8)]` enums whose order the
/// C header's MMR_ACCEL_* / MMR_ASYNC_COPY_* / MMR_PARTITION_* values follow).
pub fn launch_record_of(kernel: &GpuKernelPlan) -> ffi::mmr_launch_record {
    ffi::mmr_launch_record {
        family: family_of(kernel).unwrap_or(ffi::MMR_FAMILY_AUTO),
        math_mode: match kernel.math_mode {
            crate::tensor_light::execution::ir::KernelMathMode::StrictFp32 => ffi::MMR_MATH_STRICT_FP32,
            crate::tensor_light::execution::ir::KernelMathMode::Tf32 => ffi::MMR_MATH_TF32,
            _ => ffi::MMR_MATH_EXACT,
        },
        grid: [kernel.grid.x as i32, kernel.grid.y as i32, kernel.grid.z as i32],
        block: [kernel.block.x as i32, kernel.block.y as i32, kernel.block.z as i32],
        cluster: [kernel.cluster.x as i32, kernel.cluster.y as i32, kernel.cluster.z as i32],
        dynamic_shared_bytes: kernel.dynamic_shared_bytes as i32,
        tmem_columns_per_cta: i32::from(kernel.tmem_columns_per_cta),
        tmem_accumulator_stages: i32::from(kernel.tmem_accumulator_stages),
        tile_m: i32::from(kernel.tile_m),
        tile_n: i32::from(kernel.tile_n),
        tile_k: i32::from(kernel.tile_k),
        pipeline_stages: i32::from(kernel.pipeline_stages),
        warps_per_block: i32::from(kernel.warps_per_block),
        producer_warps: i32::from(kernel.producer_warps),
        consumer_warps: i32::from(kernel.consumer_warps),
        matrix_acceleration: kernel.matrix_acceleration as u8 as i32,
        async_copy: kernel.async_copy as u8 as i32,
        tensor_maps: kernel.tensor_maps.len() as i32,
        partition: kernel.partition as u8 as i32,
        split_k: i32::from(kernel.split_k.max(1)),
        stream_k_slices: i32::from(kernel.stream_k_slices),
        persistent_ctas_per_sm: i32::from(kernel.persistent_ctas_per_sm),
        cluster_launch: i32::from(kernel.cluster_launch),
        use_distributed_shared_memory: i32::from(kernel.use_distributed_shared_memory),
    }
}

/// Offline side: the record the specializer freezes into the plan for a node
/// (its `GpuKernelPlan` fields are filled from it). Host only; `sm_count` is
/// the target's (148 on B200).
pub fn plan_launch(desc: &ffi::mmr_matmul_desc, sm_count: i32) -> Result<ffi::mmr_launch_record, GpuGemmError> {
    let mut rec = ffi::mmr_launch_record::default();
    super::status(unsafe { ffi::mmr_gemm_plan_launch(desc, sm_count, &mut rec) })?;
    Ok(rec)
}
