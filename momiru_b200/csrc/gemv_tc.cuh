// gemv_tc.cuh -- skinny-M (M <= 16) f32 matmul on the tensor cores, swap-AB.
//
// y[m, n] = epilogue(sum_k A[m, k] * B[k, n]) for a row-major B that is read
// from HBM exactly once (the GEMV family's work; measured in GB/s). The
// CUDA-core GEMV (gemv.cuh) spends its time in the packed multiply-adds at
// M = 16 (8 flop per byte of B); here the tensor core does them:
//   D[n, m] (+)= B^T[n, k] * A^T[k, m]
// with the 128 columns of a B strip as the MMA's M (an MN-major operand:
// B's rows are n-contiguous) and the up-to-16 rows of A as its N (a K-major
// operand), kind::tf32, 128 x 16 x 8 per instruction; TF32 is that one pass.
// StrictFp32 runs the error-corrected split hi(B)*hi(A) + hi(B)*lo(A) +
// lo(B)*hi(A) in two instructions per k-step, so that the 16 KiB B tile is
// read from shared memory once by the tensor core:
//   * 128 x 32 x 8: the raw B tile (its hi part) times [hi(A) | lo(A)], the
//     A panel and its low parts stacked as 32 K-major rows;
//   * 128 x 16 x 8 with A from TMEM: lo(B), which the split warps compute and
//     store to TMEM (one 32-column slot per ring stage), times hi(A).
// Both accumulate into the same 32 TMEM columns; the epilogue adds column
// m and column 16 + m.
//
// Launch: grid.x = ceil(N / 128) strips, grid.y = GT_KSPLIT K-slices; the
// K-slices of a strip are one cluster (1 x GT_KSPLIT x 1) and add their
// partial sums through distributed shared memory in a fixed order (each CTA
// pushes to the owner of each output row group).
// Warps: 0-3 epilogue (TMEM lane quarters = the strip's 128 columns),
// 4 TMA producer, 5 MMA issuer, 6-13 split (StrictFp32 only).
// Each stage carries 32 rows of K: the B tile (32 x 128, 4 atoms of 32
// columns in the 128-byte swizzle with 32-byte atoms) and the matching A
// panel (16 x 32, K-major, 128-byte swizzle), so no A slice is staged up
// front; TMA zero-fills rows of A beyond M and K beyond the tensor. In
// StrictFp32 the panel's low parts follow it in the same layout.
// K is accumulated in chunks in two TMEM buffers and the chunks are summed
// with round-to-nearest adds (the tensor core's own accumulation is not RN),
// as in the GEMM. Inputs with inf/NaN (StrictFp32): the split warps raise a
// flag in their CTA, the CTAs of a strip pass it to one another with their
// partial sums (together they see all of A and the strip's columns of B), and
// then each owner computes its outputs again in the reference's exact order
// instead of adding the partials. Every wait is bounded.
#pragma once
#include <cooperative_groups.h>
#include <stdint.h>

#include "epilogue.cuh"
#include "ptx.cuh"

namespace mmr {

constexpr int GT_COLS = 128;                         // B columns per strip (MMA M)
constexpr int GT_MN = 16;                            // A rows, padded (MMA N)
constexpr int GT_BK = 32;                            // K rows per stage
constexpr int GT_KSPLIT = 4;                         // K-slices per strip (cluster size)
// Ring depth. TF32: as many stages as fit beside the receive buffer, about
// 200 KB of B in flight per CTA (one CTA per SM). StrictFp32 is bound by the
// MMA issue (two instructions per k-step), not by the bytes in flight; four
// stages keep it fed and leave room for two CTAs per SM.
__host__ __device__ constexpr int gt_stages(int mode) { return mode ? 4 : 11; }
// K per TMEM accumulation chunk; chunks are summed with RN adds. The tensor
// core's own f32 accumulation is not round-to-nearest (about one unit in the
// last place per instruction, of either sign); with the two issuers below,
// each with its own accumulator, a 256-wide chunk adds 16 instructions per
// accumulator.
constexpr int GT_CHUNK = 256;
constexpr int GT_B_BYTES = GT_BK * GT_COLS * 4;      // 16 KiB
constexpr int GT_A_BYTES = GT_MN * GT_BK * 4;        // 2 KiB
constexpr int GT_LOAD_BYTES = GT_B_BYTES + GT_A_BYTES;  // what TMA brings per stage
// A ring stage: B tile | A panel | (StrictFp32) the A panel's low parts.
__host__ __device__ constexpr int gt_stage_bytes(int mode) { return GT_LOAD_BYTES + (mode ? GT_A_BYTES : 0); }
// StrictFp32 split warps: GT_SPLIT_GROUPS groups of 8, taking stages in
// turn (one group keeps ahead of the MMA issuer).
constexpr int GT_EPI_WARPS = 4, GT_PRODUCER_WARP = 4, GT_MMA_WARP0 = 5, GT_ISSUERS = 2, GT_SPLIT_WARP0 = 7;
constexpr int GT_SPLIT_GROUP_WARPS = 8, GT_SPLIT_GROUPS = 1;
__host__ __device__ constexpr int gt_threads(int mode) {
  return 32 * (GT_SPLIT_WARP0 + (mode ? GT_SPLIT_GROUPS * GT_SPLIT_GROUP_WARPS : 0));
}
constexpr int GT_PART_BYTES = GT_MN * GT_COLS * 4;   // the CTA's partial sums [m][n]
// MMA issue: GT_ISSUERS warps, issuer j taking the stages s = j mod
// GT_ISSUERS of each chunk into an accumulator of its own. An MMA that adds
// into the accumulator of the one before it waits for that one to finish, and
// a 128 x 16 (or x 32) instruction is short next to that latency; two chains
// keep two in flight. TMEM: for each of two chunk buffers, one accumulator
// per issuer of GT_MN columns (TF32) or 2 * GT_MN (StrictFp32: [hi(A) | lo(A)]
// products); then, StrictFp32 only, lo(B) of each ring stage in GT_BK
// columns (lane = strip column, column = k).
constexpr int GT_ACC_BUFS = 2 * GT_ISSUERS;  // buffer (chunk parity, issuer)
__host__ __device__ constexpr int gt_acc_cols(int mode) { return mode ? 2 * GT_MN : GT_MN; }
constexpr int GT_LO_COL0 = GT_ACC_BUFS * 2 * GT_MN;
__host__ __device__ constexpr int gt_pow2_cols(int c) { return c <= 32 ? 32 : c <= 64 ? 64 : c <= 128 ? 128 : c <= 256 ? 256 : 512; }
__host__ __device__ constexpr int gt_tmem_cols(int mode) {
  return gt_pow2_cols(mode ? GT_LO_COL0 + gt_stages(1) * GT_BK : GT_ACC_BUFS * GT_MN);
}
static_assert(GT_ACC_BUFS * gt_acc_cols(0) <= gt_tmem_cols(0), "TF32 accumulators exceed the TMEM allocation");
static_assert(GT_LO_COL0 + gt_stages(1) * GT_BK <= 512, "lo(B) ring exceeds TMEM");
static_assert(GT_LOAD_BYTES % 1024 == 0 && GT_A_BYTES % 1024 == 0, "stages and panels keep 1024-byte alignment");

// Dynamic shared memory: the ring, the partial-sum tile, barriers; +1024 to
// align the base to 1024 bytes.
constexpr int GT_BAR_BYTES = 512;
__host__ __device__ constexpr int gt_smem_bytes(int mode) {
  return gt_stages(mode) * gt_stage_bytes(mode) + GT_PART_BYTES + GT_BAR_BYTES + 1024;
}
static_assert((3 * 11 + 2 * GT_ACC_BUFS + GT_ISSUERS + 1) * 8 + 8 <= GT_BAR_BYTES, "barrier area");
static_assert(gt_smem_bytes(0) <= 227 * 1024 && gt_smem_bytes(1) <= 227 * 1024, "shared memory");

struct GemvTcParams {
  int m, n, k;
  int kslice;                 // K per slice, a multiple of GT_BK
  float* c; long long c_m;    // C row stride; column stride 1
  const float* bias;
  int epilogue;
  int* err;
  unsigned long long timeout_ns;
  // StrictFp32: the operands again, for the exact recompute of a strip
  // whose inputs hold inf or NaN (A is K-contiguous).
  const float* a; long long a_m;
  const float* b; long long b_k;
};

// MMA instruction descriptor geometry: B tile = MN-major A operand (32-column
// atoms of GT_BK rows: LBO = atom stride, SBO = 4-row groups, +1024 B per
// 8-row k-step); A panel = K-major B operand (128-byte rows, 8-row groups
// 1024 B apart, +32 B per k-step).
constexpr uint32_t GT_ATOM_BYTES = GT_BK * 128u;

template <int MODE>
__global__ void __launch_bounds__(gt_threads(MODE), 1)
    mmr_gemv_tc_kernel(const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmA,
                       const GemvTcParams p) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  constexpr int S = gt_stages(MODE);
  constexpr int kStagesPerChunk = GT_CHUNK / GT_BK;
  extern __shared__ uint8_t gt_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(gt_raw) + 1023) & ~uintptr_t(1023));
  constexpr int kStage = gt_stage_bytes(MODE);
  uint8_t* ops = smem;                                         // [S][B tile | A panel | lo(A)]
  float* part = reinterpret_cast<float*>(smem + S * kStage);   // receive buffer [GT_KSPLIT][kPer]
  uint64_t* bars = reinterpret_cast<uint64_t*>(part + GT_MN * GT_COLS);
  uint64_t* full = bars;             // [S] TMA -> split / MMA
  uint64_t* split_done = bars + S;   // [S] split -> MMA (StrictFp32)
  uint64_t* empty = bars + 2 * S;    // [S] MMA -> producer
  constexpr int kAcc = GT_ACC_BUFS;
  uint64_t* acc_full = bars + 3 * S;     // [kAcc] MMA -> epilogue
  uint64_t* acc_empty = acc_full + kAcc; // [kAcc] epilogue -> MMA
  uint64_t* drain = acc_full + 2 * kAcc;  // [GT_ISSUERS]
  uint64_t* recv = drain + GT_ISSUERS;    // GT_KSPLIT arrivals: every K-slice's partial is in `part`
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(recv + 1);
  uint32_t* nonfinite_seen = tmem_slot + 1;  // StrictFp32: an input of this strip held inf/NaN

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rank = static_cast<int>(cluster.block_rank());  // K-slice index
  const int col0 = blockIdx.x * GT_COLS;
  const int k_lo = rank * p.kslice;
  const int k_hi = min(p.k, k_lo + p.kslice);
  const int nstages = k_hi > k_lo ? (k_hi - k_lo + GT_BK - 1) / GT_BK : 0;
  const int nchunks = (nstages + kStagesPerChunk - 1) / kStagesPerChunk;
  const WaitCtl ctl{p.err, p.timeout_ns};

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&split_done[s], GT_SPLIT_GROUP_WARPS);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < kAcc; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], GT_EPI_WARPS);
    }
    for (int j = 0; j < GT_ISSUERS; ++j) mbar_init(&drain[j], 1);
    mbar_init(recv, GT_KSPLIT);
    *nonfinite_seen = 0u;
    fence_mbar_init();
  }
  if (warp == GT_PRODUCER_WARP && lane == 0) {
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmA);
  }
  if (warp == GT_MMA_WARP0) {
    tmem_alloc(tmem_slot, gt_tmem_cols(MODE));
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  cluster_arrive_release();  // the receive barrier is ready; waited on before the first push
  griddep_wait();
  griddep_release();

  // Epilogue threads: the GT_MN sums of strip column warp * 32 + lane.
  float sum[GT_MN];
#pragma unroll
  for (int i = 0; i < GT_MN; ++i) sum[i] = 0.0f;
  if (warp < GT_EPI_WARPS) {
    // ------------------------------------------------------------ epilogue
    // Thread (warp, lane) owns column n = warp * 32 + lane of the strip (TMEM
    // lane) and its GT_MN sums; each K-chunk is added with RN adds.
    // Chunk c: issuer j's accumulator in buffer (c mod 2, j), added in
    // issuer order; an issuer with no stage in the last chunk is skipped by
    // both sides.
    for (int c = 0; c < nchunks; ++c) {
      const int c_end = min(nstages, (c + 1) * kStagesPerChunk);
      const uint32_t acc_phase = static_cast<uint32_t>(c >> 1) & 1u;
      float v[GT_MN];
      bool ok = true;
#pragma unroll
      for (int j = 0; j < GT_ISSUERS; ++j) {
        if (c * kStagesPerChunk + j >= c_end) break;
        const int acc = (c & 1) * GT_ISSUERS + j;
        if (!mbar_wait(&acc_full[acc], acc_phase, ctl, kDevTimeoutAcc)) { ok = false; break; }
        tc_fence_after();
        // StrictFp32: columns m and GT_MN + m hold the [hi(A) | lo(A)] products
        constexpr int kGroups = gt_acc_cols(MODE) / GT_MN;
        const uint32_t t = tmem_base + (static_cast<uint32_t>(warp * 32) << 16) + static_cast<uint32_t>(acc * gt_acc_cols(MODE));
        uint32_t r[kGroups][16];
#pragma unroll
        for (int g = 0; g < kGroups; ++g) tmem_ld_32x32b_x16(t + g * GT_MN, r[g]);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < GT_MN; ++i) {
          float x = __uint_as_float(r[0][i]);
#pragma unroll
          for (int g = 1; g < kGroups; ++g) x = __fadd_rn(x, __uint_as_float(r[g][i]));
          v[i] = j == 0 ? x : __fadd_rn(v[i], x);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[acc]);
      }
      if (!ok) break;
#pragma unroll
      for (int i = 0; i < GT_MN; ++i) sum[i] = __fadd_rn(sum[i], v[i]);
    }
  } else if (warp == GT_PRODUCER_WARP) {
    // ---------------------------------------------------------- producer
    if (lane == 0) {
      int issued = 0;
      for (int s = 0; s < nstages; ++s) {
        const int slot = s % S;
        const uint32_t phase = static_cast<uint32_t>(s / S) & 1u;
        if (!mbar_wait(&empty[slot], phase ^ 1u, ctl, kDevTimeoutEmpty)) break;
        uint8_t* st = ops + slot * kStage;
        const int k0 = k_lo + s * GT_BK;
        mbar_arrive_expect_tx(&full[slot], GT_LOAD_BYTES);
#pragma unroll
        for (int i = 0; i < GT_COLS / 32; ++i) tma_load_3d(st + i * GT_ATOM_BYTES, &tmB, &full[slot], col0 + 32 * i, k0, 0);
        tma_load_3d(st + GT_B_BYTES, &tmA, &full[slot], k0, 0, 0);
        ++issued;
      }
      // Every issued load must have landed before the CTA may exit.
      for (int s = issued > S ? issued - S : 0; s < issued; ++s) {
        const uint32_t a = smem_u32(&full[s % S]);
        const uint32_t phase = static_cast<uint32_t>(s / S) & 1u;
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(a, phase)) {
          if (globaltimer_ns() - t0 > p.timeout_ns) { atomicCAS(p.err, 0, kDevTimeoutDrain); break; }
        }
      }
    }
  } else if (warp < GT_MMA_WARP0 + GT_ISSUERS) {
    // ------------------------------------------------------- MMA issuers
    const int jw = warp - GT_MMA_WARP0;  // this issuer takes stages s = jw mod GT_ISSUERS
    if (lane == 0) {
      // B tile (MN-major) x the A panel, or x [A panel | lo(A)] in StrictFp32
      constexpr uint32_t idesc = idesc_tf32(GT_COLS, gt_acc_cols(MODE), true, false);
      // lo(B) from TMEM (K-major) x the A panel
      constexpr uint32_t idesc_ts = idesc_tf32(GT_COLS, GT_MN, false, false);
      const uint64_t a_desc0 = smem_desc(smem_u32(ops), GT_ATOM_BYTES, 512u, 1u);        // B tile, MN-major
      const uint64_t b_desc0 = smem_desc(smem_u32(ops) + GT_B_BYTES, 16u, 1024u, 2u);    // A panel, K-major
      constexpr uint64_t kStageStep = kStage >> 4;
      uint64_t* const ready = MODE ? split_done : full;
      bool ok = true, issued_any = false;
      for (int c = 0; ok && c < nchunks; ++c) {
        const int s_end = min(nstages, (c + 1) * kStagesPerChunk);
        if (c * kStagesPerChunk + jw >= s_end) break;  // no stage of this chunk (only the last can lack one)
        const int acc = (c & 1) * GT_ISSUERS + jw;
        const uint32_t acc_phase = static_cast<uint32_t>(c >> 1) & 1u;
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1u, ctl, kDevTimeoutAcc)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * gt_acc_cols(MODE));
        uint32_t accumulate = 0u;
        for (int s = c * kStagesPerChunk + jw; s < s_end; s += GT_ISSUERS) {
          const int stage = s % S;
          const uint32_t phase = static_cast<uint32_t>(s / S) & 1u;
          if (!mbar_wait(&ready[stage], phase, ctl, MODE ? kDevTimeoutXform : kDevTimeoutFull)) { ok = false; break; }
          tc_fence_after();
          const uint64_t so = static_cast<uint64_t>(stage) * kStageStep;
#pragma unroll
          for (int kk = 0; kk < GT_BK / 8; ++kk) {
            const uint64_t ad = a_desc0 + so + kk * (1024u >> 4);
            const uint64_t bd = b_desc0 + so + kk * (32u >> 4);
            umma_tf32(d_tmem, ad, bd, idesc, accumulate);  // hi(B) x hi(A) [| lo(A)]
            if (MODE) {                                    // lo(B) x hi(A)
              const uint32_t lo_b = tmem_base + static_cast<uint32_t>(GT_LO_COL0 + stage * GT_BK + kk * 8);
              umma_tf32_ts(d_tmem, lo_b, bd, idesc_ts, 1u);
            }
            accumulate = 1u;
          }
          issued_any = true;
          umma_commit(&empty[stage]);
        }
        if (!ok) break;
        umma_commit(&acc_full[acc]);
      }
      if (issued_any) {
        // Every MMA of this issuer must have finished before TMEM is freed.
        umma_commit(&drain[jw]);
        const uint32_t a = smem_u32(&drain[jw]);
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(a, 0u)) {
          if (globaltimer_ns() - t0 > p.timeout_ns) { atomicCAS(p.err, 0, kDevTimeoutDrain); break; }
        }
      }
    }
  } else if (MODE) {
    // ------------------------------------------------------- split warps
    // lo = x - hi (the tensor core reads the raw value as hi). lo(B) goes to
    // the stage's TMEM slot: warp (quarter q, half h) takes strip columns
    // 32q..32q+31 (its TMEM lane quarter; thread = column) and K rows
    // 16h..16h+15 of the stage (16 columns); group g takes the stages
    // s = g mod GT_SPLIT_GROUPS. lo(A) goes to shared memory right after the
    // A panel. inf/NaN raises the fix-up flag.
    const int sw = warp - GT_SPLIT_WARP0;
    const int group = sw / GT_SPLIT_GROUP_WARPS;
    const int quarter = warp & 3, half = (sw % GT_SPLIT_GROUP_WARPS) >> 2;
    const int tid = (sw % GT_SPLIT_GROUP_WARPS) * 32 + lane;  // thread within the group
    const uint32_t t_lane = static_cast<uint32_t>(quarter * 32) << 16;
    bool nonfinite = false;
    // lo is exact in f32 but has up to 13 significant bits; it is rounded
    // to the nearest TF32 value here (half away from zero on the magnitude)
    // rather than left to the tensor core's truncation.
    auto split1 = [&nonfinite](uint32_t u) -> uint32_t {
      const bool nf = (u & 0x7F800000u) == 0x7F800000u;
      nonfinite |= nf;
      const uint32_t lo = __float_as_uint(__fsub_rn(__uint_as_float(u), __uint_as_float(u & 0xFFFFE000u)));
      return nf ? 0u : (lo + 0x1000u) & 0xFFFFE000u;
    };
    for (int s = group; s < nstages; s += GT_SPLIT_GROUPS) {
      const int slot = s % S;
      const uint32_t phase = static_cast<uint32_t>(s / S) & 1u;
      if (!mbar_wait(&full[slot], phase, ctl, kDevTimeoutFull)) break;
      tc_fence_after();
      uint8_t* st = ops + slot * kStage;
      // Element (k, c) of a 32 x 32 atom of the B tile sits at byte
      // k * 128 + (4c XOR 32 * (k mod 4)) (128-byte swizzle of 32-byte units);
      // one k across the warp's 32 columns is one 128-byte row.
      const uint8_t* atom = st + quarter * GT_ATOM_BYTES;
      uint32_t lo[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int k = half * 16 + j;
        lo[j] = *reinterpret_cast<const uint32_t*>(atom + k * 128 + ((lane * 4) ^ ((k & 3) << 5)));
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) lo[j] = split1(lo[j]);
      tmem_st_32x32b_x16(tmem_base + t_lane + static_cast<uint32_t>(GT_LO_COL0 + slot * GT_BK + half * 16), lo);
      if (tid < GT_A_BYTES / 16) {
        const uint4 v = reinterpret_cast<const uint4*>(st + GT_B_BYTES)[tid];
        uint4 l;
        l.x = split1(v.x);
        l.y = split1(v.y);
        l.z = split1(v.z);
        l.w = split1(v.w);
        reinterpret_cast<uint4*>(st + GT_B_BYTES + GT_A_BYTES)[tid] = l;
      }
      tmem_st_wait();
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&split_done[slot]);
    }
    if (__any_sync(0xffffffffu, nonfinite) && lane == 0) atomicOr(nonfinite_seen, 1u);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == GT_MMA_WARP0) {
    tc_fence_after();
    tmem_dealloc(tmem_base, gt_tmem_cols(MODE));
  }

  // Cluster reduction: CTA r owns rows 4r..4r+3 of the strip's GT_MN x
  // GT_COLS outputs (kPer of them); every CTA stores its partial of them
  // into r's receive buffer, slot = its own rank, through distributed shared
  // memory and arrives on r's barrier; r adds slots 0..GT_KSPLIT-1 in order.
  // No CTA exits before every peer's pushes to it have landed, so no
  // cluster-wide barrier is needed at the end.
  constexpr int kPer = GT_MN * GT_COLS / GT_KSPLIT;
  constexpr int kRowsPer = GT_MN / GT_KSPLIT;
  static_assert(GT_MN % GT_KSPLIT == 0, "owner rows");
  cluster_wait_acquire();  // every peer's receive barrier is initialised
  if (warp < GT_EPI_WARPS) {
    const int n = warp * 32 + lane;
#pragma unroll
    for (int i = 0; i < GT_MN; ++i)
      cluster.map_shared_rank(part, i / kRowsPer)[rank * kPer + (i % kRowsPer) * GT_COLS + n] = sum[i];
  }
  __syncthreads();
  if (threadIdx.x < GT_KSPLIT) {
    // this CTA's inf/NaN flag travels with its partials (the arrive releases both)
    if (MODE && *nonfinite_seen) atomicOr(cluster.map_shared_rank(nonfinite_seen, threadIdx.x), 1u);
    mbar_arrive_release_cluster(mapa_shared(smem_u32(recv), threadIdx.x));
  }
  if (!mbar_wait_acquire_cluster(recv, 0u, ctl, kDevTimeoutReduce)) return;
  const bool add_bias = epi_has_bias(p.epilogue);
  const int act = epi_act(p.epilogue);
  // StrictFp32 with inf/NaN in the strip's inputs: the split products can
  // differ from the reference (inf * 0 = NaN in a cross term), so each owned
  // output is computed again in the reference's order, s = s + a * b with
  // the product and the sum rounded, k increasing.
  const bool exact = MODE && *reinterpret_cast<volatile uint32_t*>(nonfinite_seen) != 0u;
  for (int j = threadIdx.x; j < kPer; j += blockDim.x) {
    const int idx = rank * kPer + j;
    const int mm = idx / GT_COLS, cc = col0 + (idx - mm * GT_COLS);
    float v = 0.0f;
    if (exact) {
      if (mm >= p.m || cc >= p.n) continue;
      const float* a = p.a + mm * p.a_m;
      for (int kk = 0; kk < p.k; ++kk) v = __fadd_rn(v, __fmul_rn(a[kk], p.b[kk * p.b_k + cc]));
    } else {
#pragma unroll
      for (int q = 0; q < GT_KSPLIT; ++q) v = __fadd_rn(v, part[q * kPer + j]);
    }
    if (mm < p.m && cc < p.n) {
      if (add_bias) v = __fadd_rn(v, p.bias[cc]);
      p.c[mm * p.c_m + cc] = act_apply(act, v);
    }
  }
}

}  // namespace mmr
