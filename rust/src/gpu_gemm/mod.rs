//! GPU backend for frozen MatMul nodes on B200 (sm_100a).
//!
//! This is the Rust side of the drop-in: it implements the reference
//! runtime's `Backend` / `BoundBackend` traits
//! (src/momiru/tensor_light/execution/runtime.rs:879-988) for plans whose
//! nodes are GPU-placed f32 `Operation::MatMul` nodes (ir.rs:1468-1473),
//! optionally fused with `Elementwise Add` of a broadcast bias and one
//! activation (a `FusedStaticDataflow` node, plan.rs:1080-1106), and calls the
//! CUDA library through its C ABI (`ffi`, include/momiru_gemm.h).
//!
//! * `bind_resources` resolves every storage to a device view (dims, signed
//!   strides, byte base offset inside a `BufferHandle::Device`), lowers each
//!   node to an `mmr_matmul_desc`, converts the node's frozen `GpuKernelPlan`
//!   to an `mmr_launch_record` and binds with `mmr_gemm_bind_frozen`, which
//!   refuses any launch other than the frozen one. All TMA descriptors,
//!   workspaces and events are created here; nothing is enqueued.
//! * `execute_gpu_node` is one `mmr_gemm_run`: a prebuilt launch, no
//!   allocation, planning or descriptor encoding.
//! * `quiesce_or_abort` waits (bounded) on every bound node and aborts the
//!   process when completion cannot be proven, as the trait requires.
//!
//! NOT COMPILED HERE: the image this library was built in has no Rust
//! toolchain (no rustc / cargo). The file is written against the reference's
//! published types; `INTEGRATION.md` lists the two lines that register the
//! module and the `build.rs` step (`build_gpu.rs`) that builds and links the
//! CUDA library.

pub mod collective;
pub mod ffi;
pub mod validate;

use core::ptr;
use std::sync::OnceLock;

use crate::tensor_light::execution::ir::{ElementwiseKind, KernelMathMode, LayoutKind, Operation, TensorSpec};
use crate::tensor_light::execution::plan::{
    FrozenExecutionPlan, FrozenNode, GpuKernelPlan, Placement, ScheduleItem, TensorStoragePlan,
};
use crate::tensor_light::execution::runtime::{
    Backend, BoundBackend, BufferHandle, CpuGpuSlice, CpuKernelPlan, GpuGraphSegmentPlan, HostBoundaryClass,
    RuntimeCapabilityBinding, StorageBinding, SyncPlan, TransferBatchPlan, TransferPlan,
};
use crate::tensor_light::tensor::{DType, MAX_RANK};

/// Errors of the GPU MatMul backend (the analogue of `CpuNativeError`,
/// cpu.rs:290-306); `Native` carries an `MMR_ERR_*` status of the library.
#[derive(Clone, Copy, Debug, PartialEq, Eq)]
pub enum GpuGemmError {
    NotConfigured,
    InvalidCapabilities,
    UnsupportedDevice,
    UnsupportedMemory,
    UnsupportedOperation,
    UnsupportedLayout,
    InvalidNode,
    MissingBinding,
    InvalidShape,
    Native { status: i32 },
}

fn status(rc: i32) -> Result<(), GpuGemmError> {
    if rc == ffi::MMR_OK { Ok(()) } else { Err(GpuGemmError::Native { status: rc }) }
}

/// Capabilities installed once by the embedding runtime (device ordinal, SM
/// count and the hardware identity the plan was specialised for).
#[derive(Clone, Copy)]
pub struct InstalledGpu {
    pub capabilities: RuntimeCapabilityBinding,
    pub device_ordinal: u16,
    pub sm_count: i32,
    /// cudaStream_t every node of this backend runs on (null: legacy stream).
    pub stream: *mut core::ffi::c_void,
}
unsafe impl Send for InstalledGpu {}
unsafe impl Sync for InstalledGpu {}

pub static INSTALLED_GPU: OnceLock<InstalledGpu> = OnceLock::new();

pub struct GpuGemmBackend;

/// Nodes bound by frozen node id (no runtime map, as the CPU provider does).
pub struct BoundGpuGemm {
    handles: Vec<*mut ffi::mmr_gemm_handle>,
}

impl Drop for BoundGpuGemm {
    fn drop(&mut self) {
        self.quiesce_or_abort();
        for h in self.handles.drain(..) {
            if !h.is_null() {
                // SAFETY: quiesced above; each handle is released exactly once.
                unsafe { ffi::mmr_gemm_destroy(h) };
            }
        }
    }
}

const QUIESCE_LIMIT_NS: u64 = 10_000_000_000;

unsafe impl BoundBackend for BoundGpuGemm {
    type Error = GpuGemmError;

    fn execute_cpu_node(&mut self, _: &'static FrozenNode, _: &'static CpuKernelPlan) -> Result<(), Self::Error> {
        Err(GpuGemmError::UnsupportedDevice)
    }

    #[inline]
    fn execute_gpu_node(&mut self, node: &'static FrozenNode, _kernel: &'static GpuKernelPlan) -> Result<(), Self::Error> {
        let h = *self.handles.get(node.id as usize).ok_or(GpuGemmError::InvalidNode)?;
        if h.is_null() {
            return Err(GpuGemmError::InvalidNode);
        }
        // SAFETY: bound by bind_resources against the frozen launch record;
        // BoundExecution keeps every borrowed buffer alive until quiescence.
        status(unsafe { ffi::mmr_gemm_run(h) })
    }

    fn launch_cpu_slice(&mut self, _: &'static FrozenNode, _: u16, _: &'static CpuGpuSlice, _: &'static CpuKernelPlan) -> Result<(), Self::Error> {
        Err(GpuGemmError::UnsupportedOperation)
    }
    fn launch_gpu_slice(&mut self, _: &'static FrozenNode, _: u16, _: &'static CpuGpuSlice, _: &'static GpuKernelPlan) -> Result<(), Self::Error> {
        Err(GpuGemmError::UnsupportedOperation)
    }
    fn complete_cpu_gpu_slice(&mut self, _: &'static FrozenNode, _: u16, _: &'static CpuGpuSlice) -> Result<(), Self::Error> {
        Err(GpuGemmError::UnsupportedOperation)
    }
    fn execute_gpu_graph_segment(&mut self, _: &'static GpuGraphSegmentPlan) -> Result<(), Self::Error> {
        Err(GpuGemmError::UnsupportedOperation)
    }
    fn execute_transfer(&mut self, _: &'static TransferPlan) -> Result<(), Self::Error> {
        Err(GpuGemmError::UnsupportedOperation)
    }
    fn execute_host_readback(&mut self, _: &'static TransferPlan, _: HostBoundaryClass) -> Result<(), Self::Error> {
        Err(GpuGemmError::UnsupportedOperation)
    }
    fn execute_transfer_batch(&mut self, _: &'static TransferBatchPlan) -> Result<(), Self::Error> {
        Err(GpuGemmError::UnsupportedOperation)
    }
    fn execute_sync(&mut self, _: &'static SyncPlan) -> Result<(), Self::Error> {
        Err(GpuGemmError::UnsupportedOperation)
    }

    /// Every node's last launch is awaited with a bounded host poll (and its
    /// device error word read). A node that cannot be proven complete aborts
    /// the process: borrowed buffers must never be released under live work.
    fn quiesce_or_abort(&mut self) {
        for &h in &self.handles {
            if !h.is_null() && unsafe { ffi::mmr_gemm_quiesce(h, QUIESCE_LIMIT_NS) } != ffi::MMR_OK {
                std::process::abort();
            }
        }
    }
}

unsafe impl Backend for GpuGemmBackend {
    type Bound = BoundGpuGemm;
    type Error = GpuGemmError;

    fn bind_capabilities() -> Result<RuntimeCapabilityBinding, Self::Error> {
        INSTALLED_GPU.get().map(|g| g.capabilities).ok_or(GpuGemmError::NotConfigured)
    }

    unsafe fn bind_resources(
        plan: &'static FrozenExecutionPlan,
        capabilities: RuntimeCapabilityBinding,
        bindings: &[StorageBinding<'_>],
    ) -> Result<Self::Bound, Self::Error> {
        let gpu = INSTALLED_GPU.get().ok_or(GpuGemmError::NotConfigured)?;
        if gpu.capabilities != capabilities || !capabilities.matches_plan(plan) {
            return Err(GpuGemmError::InvalidCapabilities);
        }
        // Transfers, events and graph segments belong to a fuller GPU runtime.
        if !plan.transfers.is_empty() || !plan.transfer_batches.is_empty() || !plan.gpu_graph_segments.is_empty() {
            return Err(GpuGemmError::UnsupportedOperation);
        }
        let mut bound = BoundGpuGemm { handles: vec![ptr::null_mut(); plan.nodes.len()] };
        for node in plan.nodes {
            if node.placement != Placement::Gpu {
                return Err(GpuGemmError::UnsupportedDevice);
            }
            let idx = node.id as usize;
            if idx >= bound.handles.len() || !bound.handles[idx].is_null() {
                return Err(GpuGemmError::InvalidNode);
            }
            let kernel = node.gpu.ok_or(GpuGemmError::UnsupportedOperation)?;
            validate::check_gpu_matmul_kernel(node, kernel)?;
            let desc = lower_matmul_node(plan, node, kernel, bindings, gpu)?;
            let frozen = validate::launch_record_of(kernel);
            let mut h = ptr::null_mut();
            status(ffi::mmr_gemm_bind_frozen(&desc, &frozen, &mut h))?;
            bound.handles[idx] = h;
        }
        // No schedule item may name a node this backend did not bind.
        for item in plan.schedule {
            if let ScheduleItem::Node(id) = item {
                if bound.handles.get(*id as usize).map_or(true, |h| h.is_null()) {
                    return Err(GpuGemmError::InvalidNode);
                }
            }
        }
        Ok(bound)
    }
}

/// A storage's device view: the frozen tensor's dims and physical strides
/// (signed, in elements) at its byte base offset inside the bound device
/// buffer (cpu.rs:613-714 restated for `BufferHandle::Device`; the library
/// re-checks bounds, alignment, device ordinal and aliasing at bind).
fn device_view(
    plan: &FrozenExecutionPlan,
    storage_id: u32,
    bindings: &[StorageBinding<'_>],
    gpu: &InstalledGpu,
) -> Result<(ffi::mmr_view, &'static TensorSpec), GpuGemmError> {
    let storage: &TensorStoragePlan = plan.storages.get(storage_id as usize)
        .filter(|s| s.id == storage_id)
        .ok_or(GpuGemmError::MissingBinding)?;
    let tensor: &'static TensorSpec = plan.tensors.iter().find(|t| t.id == storage.tensor)
        .ok_or(GpuGemmError::InvalidShape)?;
    if tensor.dtype != DType::F32 {
        return Err(GpuGemmError::UnsupportedLayout);
    }
    let layout = storage.physical_layout;
    if !matches!(layout.kind, LayoutKind::RowMajorContiguous | LayoutKind::ColumnMajorContiguous | LayoutKind::Strided) {
        return Err(GpuGemmError::UnsupportedLayout);
    }
    let slot = plan.memory_slots.get(storage.slot as usize)
        .filter(|s| s.id == storage.slot)
        .ok_or(GpuGemmError::MissingBinding)?;
    // A read-only alias view takes its address from the root storage it aliases.
    let root = storage.external_alias_of.unwrap_or(storage_id);
    let binding = bindings.iter().find(|b| b.storage() == root).ok_or(GpuGemmError::MissingBinding)?;
    if binding.dtype() != DType::F32 {
        return Err(GpuGemmError::UnsupportedLayout);
    }
    let handle = match binding.buffer() {
        BufferHandle::Device(h) if h.device_ordinal == gpu.device_ordinal => h,
        BufferHandle::Device(_) => return Err(GpuGemmError::UnsupportedDevice),
        _ => return Err(GpuGemmError::UnsupportedMemory),
    };
    let rank = tensor.shape.rank();
    if rank > MAX_RANK {
        return Err(GpuGemmError::InvalidShape);
    }
    let mut v = ffi::mmr_view {
        address: handle.address,
        bytes: handle.bytes as u64,
        base_offset_bytes: slot.offset_bytes.checked_add(storage.base_offset_bytes).ok_or(GpuGemmError::InvalidShape)?
            as u64,
        rank: rank as i32,
        device_ordinal: i32::from(handle.device_ordinal),
        dims: [0; ffi::MMR_MAX_RANK],
        strides: [0; ffi::MMR_MAX_RANK],
        // The root storage identifies the allocation, so the library can
        // prove an output disjoint from inputs bound to other allocations.
        allocation_id: u64::from(root) + 1,
    };
    for axis in 0..rank {
        v.dims[axis] = tensor.shape.dim(axis).ok_or(GpuGemmError::InvalidShape)? as i64;
        v.strides[axis] = layout.strides[axis] as i64;
    }
    Ok((v, tensor))
}

/// The fused epilogue a node carries: `MatMul`, then optionally `Elementwise
/// Add` of a rank-1 bias broadcast over the rows, then optionally one
/// activation the library fuses (plan.rs:1080-1106 fused steps).
fn epilogue_of(node: &FrozenNode) -> Result<(i32, Option<u32>), GpuGemmError> {
    let steps = node.fused_operations;
    if steps.is_empty() {
        return Ok((ffi::MMR_EPI_NONE, None));
    }
    if !matches!(steps[0].operation, Operation::MatMul { .. }) {
        return Err(GpuGemmError::UnsupportedOperation);
    }
    let mut bias = None;
    let mut rest = &steps[1..];
    if let Some(step) = rest.first() {
        if let Operation::Elementwise { kind: ElementwiseKind::Add, arity: 2, .. } = step.operation {
            // inputs: [matmul result, bias]; the bias is the non-chained input
            bias = Some(*step.inputs.get(1).ok_or(GpuGemmError::UnsupportedOperation)?);
            rest = &rest[1..];
        }
    }
    let act = match rest {
        [] => None,
        [step] => match step.operation {
            Operation::Elementwise { kind, arity: 1, .. } => Some(kind),
            _ => return Err(GpuGemmError::UnsupportedOperation),
        },
        _ => return Err(GpuGemmError::UnsupportedOperation),
    };
    let code = match (bias.is_some(), act) {
        (false, None) => ffi::MMR_EPI_NONE,
        (true, None) => ffi::MMR_EPI_BIAS,
        (true, Some(ElementwiseKind::Relu)) => ffi::MMR_EPI_BIAS_RELU,
        (false, Some(ElementwiseKind::Relu)) => ffi::MMR_EPI_RELU,
        (false, Some(ElementwiseKind::Relu6)) => ffi::MMR_EPI_RELU6,
        (true, Some(ElementwiseKind::Relu6)) => ffi::MMR_EPI_BIAS_RELU6,
        (false, Some(ElementwiseKind::GeluErfExact)) => ffi::MMR_EPI_GELU_ERF,
        (true, Some(ElementwiseKind::GeluErfExact)) => ffi::MMR_EPI_BIAS_GELU_ERF,
        (false, Some(ElementwiseKind::GeluTanhApprox)) => ffi::MMR_EPI_GELU_TANH,
        (true, Some(ElementwiseKind::GeluTanhApprox)) => ffi::MMR_EPI_BIAS_GELU_TANH,
        (false, Some(ElementwiseKind::Silu)) => ffi::MMR_EPI_SILU,
        (true, Some(ElementwiseKind::Silu)) => ffi::MMR_EPI_BIAS_SILU,
        _ => return Err(GpuGemmError::UnsupportedOperation),
    };
    Ok((code, bias))
}

fn storage_of(plan: &FrozenExecutionPlan, tensor: u32) -> Result<u32, GpuGemmError> {
    plan.storages.iter().find(|s| s.tensor == tensor).map(|s| s.id).ok_or(GpuGemmError::MissingBinding)
}

/// Lowers one frozen GPU node to the library's node descriptor.
fn lower_matmul_node(
    plan: &FrozenExecutionPlan,
    node: &'static FrozenNode,
    kernel: &'static GpuKernelPlan,
    bindings: &[StorageBinding<'_>],
    gpu: &InstalledGpu,
) -> Result<ffi::mmr_matmul_desc, GpuGemmError> {
    let (transpose_lhs, transpose_rhs) = match node.operation {
        Operation::MatMul { transpose_lhs, transpose_rhs } => (transpose_lhs, transpose_rhs),
        _ => return Err(GpuGemmError::UnsupportedOperation),
    };
    let (epilogue, bias_tensor) = epilogue_of(node)?;
    let (lhs, _) = device_view(plan, storage_of(plan, node.inputs[0])?, bindings, gpu)?;
    let (rhs, _) = device_view(plan, storage_of(plan, node.inputs[1])?, bindings, gpu)?;
    let out_tensor = *node.outputs.first().ok_or(GpuGemmError::InvalidNode)?;
    let (out, out_spec) = device_view(plan, storage_of(plan, out_tensor)?, bindings, gpu)?;
    let bias = match bias_tensor {
        Some(t) => device_view(plan, storage_of(plan, t)?, bindings, gpu)?.0,
        None => ffi::mmr_view::default(),
    };
    let math_mode = match kernel.math_mode {
        KernelMathMode::StrictFp32 => ffi::MMR_MATH_STRICT_FP32,
        KernelMathMode::Tf32 => ffi::MMR_MATH_TF32,
        KernelMathMode::Exact => ffi::MMR_MATH_EXACT,
        _ => return Err(GpuGemmError::UnsupportedOperation),
    };
    // The output tensor's accuracy contract must admit the frozen math mode
    // (validate_node_math_contract, validation.rs:3579-3640); the plan
    // validator has checked it, and the library repeats the check.
    let _ = out_spec.accuracy;
    Ok(ffi::mmr_matmul_desc {
        lhs,
        rhs,
        out,
        bias,
        transpose_lhs: i32::from(transpose_lhs),
        transpose_rhs: i32::from(transpose_rhs),
        math_mode,
        epilogue,
        family: validate::family_of(kernel)?,
        device_ordinal: i32::from(gpu.device_ordinal),
        stream: gpu.stream,
    })
}
