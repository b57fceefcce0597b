/*
 * momiru_gemm.h -- C ABI of the B200 (sm_100a) f32 matmul hot path.
 *
 * This is the drop-in boundary a GPU backend of Momiru's frozen-plan runtime
 * binds. In the reference, a frozen GEMM node reaches a backend through two
 * traits (src/momiru/tensor_light/execution/runtime.rs):
 *
 *   Backend::bind_resources            runtime.rs:954-988   -> mmr_gemm_bind
 *   BoundBackend::execute_gpu_node     runtime.rs:886-890   -> mmr_gemm_run
 *   BoundBackend::quiesce_or_abort     runtime.rs:944-946   -> mmr_gemm_quiesce
 *   (drop of the bound backend)                            -> mmr_gemm_destroy
 *
 * and the node itself is Operation::MatMul{transpose_lhs, transpose_rhs}
 * (src/momiru/tensor_light/execution/ir.rs:1468-1473) whose shape and
 * broadcast contract is validation.rs:2300-2398. Device buffers follow
 * BufferHandle::Device{device_ordinal, address, bytes} (runtime.rs:297-301);
 * views follow Shape{dims, strides} plus a byte base offset
 * (tensor/shape.rs:130-206, plan.rs:1285-1307).
 *
 * Conventions:
 *   - Every entry point returns an int32 status (MMR_OK = 0). Nothing throws
 *     or aborts across this boundary. mmr_last_error() gives a message for the
 *     calling thread's last failure.
 *   - Caller owns every buffer. A bound handle keeps raw device addresses; the
 *     caller must keep the buffers alive until mmr_gemm_quiesce (or destroy)
 *     has returned MMR_OK after the last run.
 *   - Bind does all validation, kernel-family choice and TMA descriptor
 *     encoding. Run only enqueues the pre-built launch on the bound stream:
 *     no allocation, no planning, no descriptor encoding (runtime.rs:962-973).
 */
#ifndef MOMIRU_GEMM_H
#define MOMIRU_GEMM_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MMR_API __attribute__((visibility("default")))
#else
#define MMR_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes (CpuNativeError / PlanError analogues, cpu.rs:290-306) */
enum {
  MMR_OK = 0,
  MMR_ERR_INVALID_ARGUMENT = 1,   /* null pointer, bad enum value            */
  MMR_ERR_INVALID_SHAPE = 2,      /* MatMul shape/broadcast contract broken  */
  MMR_ERR_UNSUPPORTED_LAYOUT = 3, /* strides/offset/alignment not admissible */
  MMR_ERR_UNSAFE_ALIASING = 4,    /* output overlaps an input                */
  MMR_ERR_UNSUPPORTED_MATH = 5,   /* math mode vs accuracy contract mismatch */
  MMR_ERR_UNSUPPORTED_DEVICE = 6, /* ordinal mismatch / not an sm_100 device  */
  MMR_ERR_OUT_OF_BOUNDS = 7,      /* a view does not fit its bound buffer    */
  MMR_ERR_CUDA = 8,               /* a CUDA runtime/driver call failed       */
  MMR_ERR_PEER_ACCESS = 9,        /* a buffer could not be shared with or
                                     mapped from another rank's process      */
  MMR_ERR_TIMEOUT = 10,           /* bounded wait expired (host or device)   */
  MMR_ERR_DEVICE_FAULT_FLAG = 11, /* a kernel reported an error word         */
  MMR_ERR_UNSUPPORTED_FAMILY = 12, /* forced kernel family cannot run this   */
  MMR_ERR_PLAN_MISMATCH = 13       /* a frozen launch record breaks a rule or
                                      differs from what this library binds     */
};

/* ---- numeric mode (KernelMathMode, ir.rs:559-569; gated by the output's
 *      AccuracyContract, validation.rs:3579-3640) */
enum {
  MMR_MATH_STRICT_FP32 = 0, /* 3xTF32 split on tcgen05; rel-Frobenius <= 1e-5 */
  MMR_MATH_TF32 = 1,        /* one TF32 pass; needs AllowTf32; <= 2e-3        */
  MMR_MATH_EXACT = 2        /* bit-exact with the reference CPU GEMM order   */
};

/* ---- fused epilogue: MatMul -> Add(bias[N] broadcast) -> activation,
 *      expressed in the reference as a FusedStaticDataflow node
 *      (plan.rs:1080-1106); the activations are the reference CPU provider's
 *      elementwise kernels (cpu.rs:2117-2168 and 2214-2222): ReLU, ReLU6,
 *      GELU (erf, exact), GELU (tanh approximation), SiLU */
enum {
  MMR_EPI_NONE = 0,
  MMR_EPI_BIAS = 1,
  MMR_EPI_BIAS_RELU = 2,
  MMR_EPI_RELU = 3,
  MMR_EPI_RELU6 = 4,
  MMR_EPI_BIAS_RELU6 = 5,
  MMR_EPI_GELU_ERF = 6,
  MMR_EPI_BIAS_GELU_ERF = 7,
  MMR_EPI_GELU_TANH = 8,
  MMR_EPI_BIAS_GELU_TANH = 9,
  MMR_EPI_SILU = 10,
  MMR_EPI_BIAS_SILU = 11
};

/* ---- kernel family (KernelFamily, plan.rs:326-431); AUTO lets bind choose */
enum {
  MMR_FAMILY_AUTO = 0,
  MMR_FAMILY_TCGEN05 = 1, /* TMA + tcgen05/TMEM tensor-core GEMM              */
  MMR_FAMILY_GEMV = 2,    /* skinny-M (M <= 16) HBM-streaming kernel          */
  MMR_FAMILY_SIMT = 3     /* CUDA-core kernel, any strides; bit-exact order  */
};

#define MMR_MAX_RANK 8 /* the reference tensor ranks: MIN_RANK 0 .. MAX_RANK 8 (tensor.rs:148-149) */

/* A strided f32 view of a device buffer (Shape{dims,strides} + base offset).
 * Strides are in elements and signed (a negative stride walks an axis
 * backwards, as the reference's signed views do); the tensor-core and GEMV
 * families need non-negative ones, the SIMT family takes any. */
typedef struct mmr_view {
  uint64_t address;           /* device address of the bound buffer          */
  uint64_t bytes;             /* bytes of the bound buffer from `address`     */
  uint64_t base_offset_bytes; /* byte offset of element [0,..,0]              */
  int32_t rank;               /* 1..MMR_MAX_RANK; 0 = a scalar output (vector
                                 x vector), or an absent bias                 */
  int32_t device_ordinal;
  int64_t dims[MMR_MAX_RANK];
  int64_t strides[MMR_MAX_RANK];
  uint64_t allocation_id;     /* identity of the owning allocation; 0 = unknown */
} mmr_view;

/* The frozen GEMM node plus its storage bindings. */
typedef struct mmr_matmul_desc {
  mmr_view lhs, rhs, out;
  mmr_view bias;              /* rank 1 [N] when the epilogue adds a bias     */
  int32_t transpose_lhs;
  int32_t transpose_rhs;
  int32_t math_mode;          /* MMR_MATH_*                                   */
  int32_t epilogue;           /* MMR_EPI_*                                    */
  int32_t family;             /* MMR_FAMILY_*                                 */
  int32_t device_ordinal;
  void *stream;               /* cudaStream_t; NULL = legacy default stream  */
} mmr_matmul_desc;

/* What bind decided (for logging and tests). */
typedef struct mmr_gemm_info {
  int32_t family;             /* chosen MMR_FAMILY_*                          */
  int32_t math_mode;
  int64_t batch, m, n, k;
  int32_t a_mn_major;         /* 1: A tile is M-contiguous (transposed view)  */
  int32_t b_mn_major;         /* 1: B tile is N-contiguous (row-major B)      */
  int32_t grid, block, cluster;
  int32_t smem_bytes;
  int32_t tile_m, tile_n, tile_k, stages;
  int64_t tiles;
  double flops;               /* 2*batch*M*N*K                                */
  double bytes;               /* algorithmic HBM bytes (A + B + C [+ bias])   */
} mmr_gemm_info;

typedef struct mmr_gemm_handle mmr_gemm_handle;

/* ---- the frozen launch record ----------------------------------------------
 * The fields of the reference's frozen GpuKernelPlan (plan.rs:941-1026) that
 * this library decides for a node: launch shape, tiling, pipeline, TMEM and
 * partition. Enum values follow the reference's enums: matrix_acceleration
 * is MatrixAcceleration (0 None, 5 Tcgen05; plan.rs:757-772), async_copy is
 * AsyncCopyKind (0 None, 4 Tma; plan.rs:629-639), partition is
 * GpuPartitionKind (0 Grid, 1 SplitK, 2 StreamK, 3 PersistentCta;
 * plan.rs:776-783). A plan that freezes a GPU MatMul node carries this record;
 * mmr_gemm_bind_frozen binds the node only if the record obeys the GPU
 * validator's rules (validation.rs:5630-5700, 5846-5911) and equals what the
 * library launches, so no kernel, tile or schedule is substituted at bind. */
enum { MMR_ACCEL_NONE = 0, MMR_ACCEL_TCGEN05 = 5 };
enum { MMR_ASYNC_COPY_NONE = 0, MMR_ASYNC_COPY_TMA = 4 };
enum { MMR_PARTITION_GRID = 0, MMR_PARTITION_SPLIT_K = 1, MMR_PARTITION_STREAM_K = 2,
       MMR_PARTITION_PERSISTENT_CTA = 3 };

typedef struct mmr_launch_record {
  int32_t family;                  /* MMR_FAMILY_* the node binds              */
  int32_t math_mode;               /* MMR_MATH_*                               */
  int32_t grid[3], block[3], cluster[3];
  int32_t dynamic_shared_bytes;
  int32_t tmem_columns_per_cta;    /* 0: no tensor memory                      */
  int32_t tmem_accumulator_stages;
  int32_t tile_m, tile_n, tile_k;
  int32_t pipeline_stages;
  int32_t warps_per_block, producer_warps, consumer_warps;
  int32_t matrix_acceleration;     /* MMR_ACCEL_*                              */
  int32_t async_copy;              /* MMR_ASYNC_COPY_*                         */
  int32_t tensor_maps;             /* TMA descriptors encoded at bind          */
  int32_t partition;               /* MMR_PARTITION_*                          */
  int32_t split_k;                 /* K parts per output tile (1 = unsplit)    */
  int32_t stream_k_slices;         /* output tiles split stream-K style        */
  int32_t persistent_ctas_per_sm;  /* 0: not persistent                        */
  int32_t cluster_launch;          /* 1: launched as thread-block clusters     */
  int32_t use_distributed_shared_memory;
} mmr_launch_record;

/* Host-only, touches no GPU: the record mmr_gemm_bind would freeze for `desc`
 * on a device with `sm_count` SMs (148 on B200). */
MMR_API int32_t mmr_gemm_plan_launch(const mmr_matmul_desc *desc, int32_t sm_count, mmr_launch_record *out);

/* The record a bound handle launches with. */
MMR_API int32_t mmr_gemm_launch_record(const mmr_gemm_handle *h, mmr_launch_record *out);

/* Host-only: the GPU validator's rules on a frozen record alone -- tcgen05
 * needs tensor memory; TMEM columns a power of two, a multiple of the
 * 32-column allocation unit and at most 512; accumulator stages with TMEM;
 * TMA needs tensor maps; clusters within 8 CTAs and launched as clusters;
 * shared memory within 227 KB; block and warp counts consistent.
 * MMR_ERR_PLAN_MISMATCH names the rule broken. */
MMR_API int32_t mmr_check_launch_record(const mmr_launch_record *rec);

/* Bind as mmr_gemm_bind does, but only to the launch `frozen` describes: the
 * record must pass mmr_check_launch_record and equal, field by field, what
 * this library binds for the node on this device; otherwise nothing is bound
 * and MMR_ERR_PLAN_MISMATCH names the first differing field. */
MMR_API int32_t mmr_gemm_bind_frozen(const mmr_matmul_desc *desc, const mmr_launch_record *frozen,
                                     mmr_gemm_handle **out);

/* Host-only validation of the MatMul contract and layout admission; touches no
 * GPU. Fills `info` (may be NULL). validation.rs:2300-2398, cpu.rs:613-714,
 * runtime.rs:618-811. */
MMR_API int32_t mmr_gemm_validate(const mmr_matmul_desc *desc, mmr_gemm_info *info);

/* Bind: validate, choose the kernel family, encode TMA descriptors, create the
 * completion event. Enqueues no work. runtime.rs:954-988. */
MMR_API int32_t mmr_gemm_bind(const mmr_matmul_desc *desc, mmr_gemm_handle **out);

/* Replay: enqueue the bound kernel on the bound stream. runtime.rs:886-890. */
MMR_API int32_t mmr_gemm_run(mmr_gemm_handle *h);

/* Replay on another stream (same device). */
MMR_API int32_t mmr_gemm_run_on(mmr_gemm_handle *h, void *stream);

/* Establish completion of every run on this handle, polling with a host
 * deadline; also reads the device error word. runtime.rs:944-946. */
MMR_API int32_t mmr_gemm_quiesce(mmr_gemm_handle *h, uint64_t timeout_ns);

/* Release the handle (waits for completion first, bounded by 10 s). */
MMR_API int32_t mmr_gemm_destroy(mmr_gemm_handle *h);

MMR_API int32_t mmr_gemm_query(const mmr_gemm_handle *h, mmr_gemm_info *info);

/* Message for the calling thread's last non-OK status. */
MMR_API const char *mmr_last_error(void);

/* Library version string and build flags. */
MMR_API const char *mmr_version(void);

/* ---- device-side bounded-wait self test (failure-detection path) ---------
 * Launches one CTA that waits on an mbarrier nobody arrives at, with a limit
 * of `limit_ns`; the kernel gives up, records MMR_ERR_TIMEOUT in its error
 * word and returns, leaving the context usable. Returns the status the host
 * read back (MMR_ERR_TIMEOUT is the expected, healthy answer). */
MMR_API int32_t mmr_selftest_bounded_wait(int32_t device_ordinal, uint64_t limit_ns);

/* ---- one-shot launch that allocates nothing --------------------------------
 * No counterpart in the reference: the reference's CPU provider never touches
 * device memory. This is for callers that cannot call cudaMalloc at the point
 * where they launch -- a serving runtime whose allocator owns every byte of
 * HBM and forbids other allocations, code that must not pay cudaMalloc's
 * implicit device synchronisation, or a caller that has no place to keep a
 * bound handle. mmr_gemm_bind allocates a small scratch area (the kernel's
 * error word and its bookkeeping for inf/NaN tiles); this entry point uses a
 * fixed array compiled into the library instead, so it makes no device
 * allocation at all. Each GPU that loads the library holds that array
 * (MMR_NOALLOC_SCRATCH_BYTES) until the process exits.
 *
 * It validates `desc` exactly as mmr_gemm_bind does, then enqueues the
 * StrictFp32 (3xTF32) tcgen05 kernel and its inf/NaN fix-up on desc->stream.
 * Only math_mode MMR_MATH_STRICT_FP32 with a TMA-admissible layout is
 * accepted, and at most MMR_NOALLOC_MAX_TILES output tiles of 128 x 256
 * (batch included; 8192 x 8192 needs 2048). Larger problems are rejected with
 * MMR_ERR_INVALID_SHAPE before anything is launched.
 *
 * The first call on a device looks up the array's device address and sets the
 * kernel's shared-memory limit for that device; make that first call before
 * any stream capture begins. All calls on a device share the one array: calls
 * whose work may overlap on the GPU (different streams with no ordering
 * between them) race on it and must be serialised by the caller. The array
 * keeps the last call's contents; each call clears the parts that must start
 * at zero before its kernels run.
 *
 * `status_out` (optional: NULL, or pinned host memory -- cudaHostAlloc or
 * cudaHostRegister -- that the caller keeps alive until the stream has passed
 * this call's work) receives 0, or the kernel's device error code when a
 * bounded wait expired. It is written by an asynchronous device-to-host copy
 * enqueued on desc->stream after the kernels, so it holds the status only once
 * the stream has reached that point.
 * Returns MMR_OK when the work was enqueued. */
#define MMR_NOALLOC_SCRATCH_BYTES (64 * 1024)
#define MMR_NOALLOC_MAX_TILES 8189
MMR_API int32_t mmr_gemm_run_noalloc(const mmr_matmul_desc *desc, int32_t *status_out);

/* ---- column-block sharding -------------------------------------------------
 * Column range [col0, col1) of rank `rank` when N output columns are dealt to
 * `nranks` ranks in whole units of `align` columns (the output-tile width).
 * Pure host arithmetic. */
MMR_API int32_t mmr_shard_columns(int64_t n, int32_t nranks, int32_t rank, int32_t align,
                                  int64_t *col0, int64_t *col1);

/* ---- device memory shared between the processes of one node ----------------
 * One process drives one GPU; a rank maps its peers' buffers through CUDA IPC.
 * `offset` is the address's distance from the start of its allocation, so
 * buffers handed out by a caching allocator can be shared. */
typedef struct mmr_ipc_handle {
  uint8_t bytes[64];          /* cudaIpcMemHandle_t of the allocation         */
  uint64_t offset;            /* address - allocation base                    */
} mmr_ipc_handle;

MMR_API int32_t mmr_ipc_export(uint64_t address, mmr_ipc_handle *out);
/* Maps a peer's buffer into this process (on `device_ordinal`, which must be
 * current-capable of peer access to the exporter). */
MMR_API int32_t mmr_ipc_import(const mmr_ipc_handle *h, int32_t device_ordinal, uint64_t *address_out);
MMR_API int32_t mmr_ipc_release(uint64_t address, const mmr_ipc_handle *h);

/* ---- column-block sharded GEMM with the output replicated on every rank ----
 * Rank r of `nranks` computes out[:, c0:c1] = epilogue(lhs @ rhs[:, c0:c1])
 * for its column block (mmr_shard_columns, 256-column units) and every
 * finished output tile is stored, by the GEMM's own epilogue, into the
 * output replica of every rank over NVLink (peer stores). This is the
 * all-gather of the reference IR's CollectiveKind::AllGather
 * (src/momiru/tensor_light/execution/ir.rs:1140-1154), which the reference
 * IR rejects today (ir.rs:1773-1779), fused into the GEMM. After the GEMM a
 * one-block kernel publishes this rank's completion into every peer's signal
 * array and waits (bounded; MMR_ERR_TIMEOUT via quiesce) until every peer
 * has published, so a completed run means every replica is whole.
 * `local` describes the full lhs, rhs, bias and this rank's full output
 * replica; all ranks use the same shapes and the same output layout. */
typedef struct mmr_sharded_desc {
  mmr_matmul_desc local;
  int32_t rank, nranks;       /* nranks <= 8                                  */
  uint64_t peer_out[8];       /* rank i's output replica, mapped here         */
  uint64_t peer_signal[8];    /* rank i's signal array (nranks u64), mapped   */
  uint64_t signal;            /* this rank's signal array (zero-initialised)  */
} mmr_sharded_desc;

MMR_API int32_t mmr_sharded_gemm_bind(const mmr_sharded_desc *desc, mmr_gemm_handle **out);

/* Host-only, touches no GPU: the node rank `rank` of `nranks` binds inside
 * mmr_sharded_gemm_bind. `whole` is validated as a whole; `local` is `whole`
 * narrowed to the rank's column block [col0, col1) (rhs columns, bias
 * entries, out columns, as zero-copy views), and `out_offset_bytes` is where
 * that block starts in every replica (its byte offset from the output
 * buffer's address), which is where the rank's epilogue stores its tiles in
 * each peer's replica. The data-plane counterpart of the AllGather the
 * reference IR names (ir.rs:1140-1154) for a column-sharded MatMul. */
MMR_API int32_t mmr_shard_local_desc(const mmr_matmul_desc *whole, int32_t rank, int32_t nranks,
                                     mmr_matmul_desc *local, int64_t *col0, int64_t *col1,
                                     uint64_t *out_offset_bytes);

/* ---- operands in host memory. The reference's CPU provider binds host
 * buffers only (cpu.rs:651-654), so its callers hold their matrices in host
 * memory; this binds the same node over HOST views (`address` = host
 * pointer) on device `device_ordinal`. Each run copies rhs and bias in,
 * then lhs by row panels (`panels` of them, multiples of 256 rows; 0 = one
 * per 512 rows, at most 16),
 * runs the bound device GEMM of each panel as soon as its rows have landed
 * and copies its output rows back while later panels still copy in and
 * compute: three streams chained by events, ordered after earlier work on
 * `desc->stream` (or the stream given to mmr_gemm_run_on) and before later
 * work on it, and after the handle's previous run whichever stream that was
 * on (the device staging buffers belong to the handle). Only the logical columns are
 * copied, so padding in host rows is never written. Host buffers should be
 * pinned (cudaHostAlloc / cudaHostRegister) for the copies to overlap.
 * Operands: rank 2, row-major with unit column stride; transpose_lhs = 0
 * (lhs is streamed by rows; transpose_rhs is allowed). Device buffers are
 * allocated here (16-byte row pitch), and the returned handle runs, waits
 * and is freed with mmr_gemm_run / mmr_gemm_quiesce / mmr_gemm_destroy. */
MMR_API int32_t mmr_gemm_bind_host(const mmr_matmul_desc *host_desc, int32_t panels, mmr_gemm_handle **out);

#ifdef __cplusplus
}
#endif

#endif /* MOMIRU_GEMM_H */
