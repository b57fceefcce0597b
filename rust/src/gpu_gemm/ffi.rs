//! Raw bindings of `include/momiru_gemm.h`, the C ABI of the B200 matmul
//! library (`libmomiru_gemm`). Every struct is `#[repr(C)]` with the header's
//! field order; every function returns an `i32` status (0 = OK).
//!
//! NOT COMPILED HERE: the image this library was built in has no Rust
//! toolchain. The layouts are the header's; `tests/test_abi_contract.py`
//! checks the same layouts from Python (ctypes) against the built library.

#![allow(non_camel_case_types)]

use core::ffi::{c_char, c_void};

pub const MMR_MAX_RANK: usize = 8;

pub const MMR_OK: i32 = 0;
pub const MMR_ERR_INVALID_ARGUMENT: i32 = 1;
pub const MMR_ERR_INVALID_SHAPE: i32 = 2;
pub const MMR_ERR_UNSUPPORTED_LAYOUT: i32 = 3;
pub const MMR_ERR_UNSAFE_ALIASING: i32 = 4;
pub const MMR_ERR_UNSUPPORTED_MATH: i32 = 5;
pub const MMR_ERR_UNSUPPORTED_DEVICE: i32 = 6;
pub const MMR_ERR_OUT_OF_BOUNDS: i32 = 7;
pub const MMR_ERR_CUDA: i32 = 8;
pub const MMR_ERR_PEER_ACCESS: i32 = 9;
pub const MMR_ERR_TIMEOUT: i32 = 10;
pub const MMR_ERR_DEVICE_FAULT_FLAG: i32 = 11;
pub const MMR_ERR_UNSUPPORTED_FAMILY: i32 = 12;
pub const MMR_ERR_PLAN_MISMATCH: i32 = 13;

pub const MMR_MATH_STRICT_FP32: i32 = 0;
pub const MMR_MATH_TF32: i32 = 1;
pub const MMR_MATH_EXACT: i32 = 2;

pub const MMR_EPI_NONE: i32 = 0;
pub const MMR_EPI_BIAS: i32 = 1;
pub const MMR_EPI_BIAS_RELU: i32 = 2;
pub const MMR_EPI_RELU: i32 = 3;
pub const MMR_EPI_RELU6: i32 = 4;
pub const MMR_EPI_BIAS_RELU6: i32 = 5;
pub const MMR_EPI_GELU_ERF: i32 = 6;
pub const MMR_EPI_BIAS_GELU_ERF: i32 = 7;
pub const MMR_EPI_GELU_TANH: i32 = 8;
pub const MMR_EPI_BIAS_GELU_TANH: i32 = 9;
pub const MMR_EPI_SILU: i32 = 10;
pub const MMR_EPI_BIAS_SILU: i32 = 11;

pub const MMR_FAMILY_AUTO: i32 = 0;
pub const MMR_FAMILY_TCGEN05: i32 = 1;
pub const MMR_FAMILY_GEMV: i32 = 2;
pub const MMR_FAMILY_SIMT: i32 = 3;

#[repr(C)]
#[derive(Clone, Copy, Default)]
pub struct mmr_view {
    pub address: u64,
    pub bytes: u64,
    pub base_offset_bytes: u64,
    pub rank: i32,
    pub device_ordinal: i32,
    pub dims: [i64; MMR_MAX_RANK],
    pub strides: [i64; MMR_MAX_RANK],
    pub allocation_id: u64,
}

#[repr(C)]
#[derive(Clone, Copy)]
pub struct mmr_matmul_desc {
    pub lhs: mmr_view,
    pub rhs: mmr_view,
    pub out: mmr_view,
    pub bias: mmr_view,
    pub transpose_lhs: i32,
    pub transpose_rhs: i32,
    pub math_mode: i32,
    pub epilogue: i32,
    pub family: i32,
    pub device_ordinal: i32,
    pub stream: *mut c_void,
}

#[repr(C)]
#[derive(Clone, Copy, Default)]
pub struct mmr_gemm_info {
    pub family: i32,
    pub math_mode: i32,
    pub batch: i64,
    pub m: i64,
    pub n: i64,
    pub k: i64,
    pub a_mn_major: i32,
    pub b_mn_major: i32,
    pub grid: i32,
    pub block: i32,
    pub cluster: i32,
    pub smem_bytes: i32,
    pub tile_m: i32,
    pub tile_n: i32,
    pub tile_k: i32,
    pub stages: i32,
    pub tiles: i64,
    pub flops: f64,
    pub bytes: f64,
}

pub const MMR_ACCEL_NONE: i32 = 0;
pub const MMR_ACCEL_TCGEN05: i32 = 5;
pub const MMR_ASYNC_COPY_NONE: i32 = 0;
pub const MMR_ASYNC_COPY_TMA: i32 = 4;
pub const MMR_PARTITION_GRID: i32 = 0;
pub const MMR_PARTITION_SPLIT_K: i32 = 1;
pub const MMR_PARTITION_STREAM_K: i32 = 2;
pub const MMR_PARTITION_PERSISTENT_CTA: i32 = 3;

#[repr(C)]
#[derive(Clone, Copy, Default, PartialEq, Eq, Debug)]
pub struct mmr_launch_record {
    pub family: i32,
    pub math_mode: i32,
    pub grid: [i32; 3],
    pub block: [i32; 3],
    pub cluster: [i32; 3],
    pub dynamic_shared_bytes: i32,
    pub tmem_columns_per_cta: i32,
    pub tmem_accumulator_stages: i32,
    pub tile_m: i32,
    pub tile_n: i32,
    pub tile_k: i32,
    pub pipeline_stages: i32,
    pub warps_per_block: i32,
    pub producer_warps: i32,
    pub consumer_warps: i32,
    pub matrix_acceleration: i32,
    pub async_copy: i32,
    pub tensor_maps: i32,
    pub partition: i32,
    pub split_k: i32,
    pub stream_k_slices: i32,
    pub persistent_ctas_per_sm: i32,
    pub cluster_launch: i32,
    pub use_distributed_shared_memory: i32,
}

#[repr(C)]
#[derive(Clone, Copy)]
pub struct mmr_ipc_handle {
    pub bytes: [u8; 64],
    pub offset: u64,
}

#[repr(C)]
#[derive(Clone, Copy)]
pub struct mmr_sharded_desc {
    pub local: mmr_matmul_desc,
    pub rank: i32,
    pub nranks: i32,
    pub peer_out: [u64; 8],
    pub peer_signal: [u64; 8],
    pub signal: u64,
}

/// Opaque bound node.
#[repr(C)]
pub struct mmr_gemm_handle {
    _private: [u8; 0],
}

#[link(name = "momiru_gemm")]
extern "C" {
    pub fn mmr_gemm_validate(desc: *const mmr_matmul_desc, info: *mut mmr_gemm_info) -> i32;
    pub fn mmr_gemm_bind(desc: *const mmr_matmul_desc, out: *mut *mut mmr_gemm_handle) -> i32;
    pub fn mmr_gemm_bind_frozen(
        desc: *const mmr_matmul_desc,
        frozen: *const mmr_launch_record,
        out: *mut *mut mmr_gemm_handle,
    ) -> i32;
    pub fn mmr_gemm_plan_launch(desc: *const mmr_matmul_desc, sm_count: i32, out: *mut mmr_launch_record) -> i32;
    pub fn mmr_gemm_launch_record(h: *const mmr_gemm_handle, out: *mut mmr_launch_record) -> i32;
    pub fn mmr_check_launch_record(rec: *const mmr_launch_record) -> i32;
    pub fn mmr_gemm_run(h: *mut mmr_gemm_handle) -> i32;
    pub fn mmr_gemm_run_on(h: *mut mmr_gemm_handle, stream: *mut c_void) -> i32;
    pub fn mmr_gemm_quiesce(h: *mut mmr_gemm_handle, timeout_ns: u64) -> i32;
    pub fn mmr_gemm_destroy(h: *mut mmr_gemm_handle) -> i32;
    pub fn mmr_gemm_query(h: *const mmr_gemm_handle, info: *mut mmr_gemm_info) -> i32;
    pub fn mmr_last_error() -> *const c_char;
    pub fn mmr_version() -> *const c_char;
    pub fn mmr_shard_columns(n: i64, nranks: i32, rank: i32, align: i32, col0: *mut i64, col1: *mut i64) -> i32;
    pub fn mmr_shard_local_desc(
        whole: *const mmr_matmul_desc,
        rank: i32,
        nranks: i32,
        local: *mut mmr_matmul_desc,
        col0: *mut i64,
        col1: *mut i64,
        out_offset_bytes: *mut u64,
    ) -> i32;
    pub fn mmr_ipc_export(address: u64, out: *mut mmr_ipc_handle) -> i32;
    pub fn mmr_ipc_import(h: *const mmr_ipc_handle, device_ordinal: i32, address_out: *mut u64) -> i32;
    pub fn mmr_ipc_release(address: u64, h: *const mmr_ipc_handle) -> i32;
    pub fn mmr_sharded_gemm_bind(desc: *const mmr_sharded_desc, out: *mut *mut mmr_gemm_handle) -> i32;
}
