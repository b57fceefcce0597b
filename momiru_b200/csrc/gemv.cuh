// gemv.cuh -- skinny-M (M <= 16) f32 matmul that streams B from HBM once.
//
// y[m, n] = epilogue(sum_k A[m, k] * B[k, n]) for a row-major B. The work is
// HBM-bound (B is read exactly once, 4*K*N bytes), so the kernel is measured in
// GB/s. Launch:
//   grid.x  = ceil(N / 128) column strips of 128 columns
//   grid.y  = GV_KSPLIT K-slices; the GV_KSPLIT CTAs of a strip form one
//             thread-block cluster (dims 1 x GV_KSPLIT x 1)
//   block   = 8 consumer warps + 1 producer warp
// The producer thread streams the CTA's B slice through a gv_stages(MT)-deep
// shared-memory ring with TMA (32 rows x 128 columns, 16 KiB per stage), so
// the bytes in flight do not depend on registers; the consumer warps take 4
// rows of each stage (lane = 4 columns) and accumulate M x 4 partial sums.
// Partials are reduced in a fixed order -- warps through shared memory (the
// idle ring), then the cluster's CTAs: CTA r owns 1/GV_KSPLIT of the strip's
// outputs, every CTA stores its partial of them into r's receive buffer
// (slot = its own rank) through distributed shared memory and arrives on r's
// barrier, and r adds the slots in rank order -- so results are
// deterministic, without atomics, a global scratch buffer or a cluster-wide
// barrier at the end.
// Waits are bounded like the GEMM's.
#pragma once
#include <cooperative_groups.h>
#include <stdint.h>

#include "epilogue.cuh"
#include "ptx.cuh"

namespace mmr {

constexpr int GV_CONSUMER_WARPS = 8;
constexpr int GV_THREADS = 32 * (GV_CONSUMER_WARPS + 1);
constexpr int GV_COLS = 128;
constexpr int GV_ROWS = 32;                             // B rows per stage
constexpr int GV_STAGE_BYTES = GV_ROWS * GV_COLS * 4;   // 16 KiB
// Ring depth: six stages for M <= 4 (the A slice is small), four for larger
// M, so that two CTAs fit on an SM at every M.
__host__ __device__ constexpr int gv_stages(int mt) { return mt <= 4 ? 6 : 4; }
constexpr int GV_KSPLIT = 8;
constexpr int GV_MAX_M = 16;
constexpr int GV_MAX_KSLICE = 1024;  // K <= GV_KSPLIT * GV_MAX_KSLICE = 8192

struct GemvParams {
  int m, n, k;
  int kslice;  // ceil(K / GV_KSPLIT) rounded up to GV_ROWS
  const float* a; long long a_m, a_k;
  float* c; long long c_m;        // C row stride; column stride 1
  const float* bias;
  int epilogue;
  int* err;
  unsigned long long timeout_ns;
};

// Dynamic shared memory: the stage ring (reused afterwards for the per-warp
// partials [8][MT][128]), the A slice [kslice][MT] (transposed), the receive
// buffer [GV_KSPLIT][MT * 128 / GV_KSPLIT] that cluster peers write, the
// ring's barriers and the receive barrier.
__host__ __device__ constexpr int gemv_ring_bytes(int mt) {
  return (gv_stages(mt) * GV_STAGE_BYTES > GV_CONSUMER_WARPS * mt * GV_COLS * 4)
             ? gv_stages(mt) * GV_STAGE_BYTES
             : GV_CONSUMER_WARPS * mt * GV_COLS * 4;
}
__host__ __device__ constexpr int gemv_smem_bytes(int mt, int kslice) {
  return gemv_ring_bytes(mt) + mt * kslice * 4 + mt * GV_COLS * 4 + (2 * gv_stages(mt) + 1) * 8 + 1024;
}

// Packed pairs of f32 (low half = first element) and the sm_100 packed
// fused multiply-add, d = a * b + c per element, each rounded once.
__device__ __forceinline__ unsigned long long pack_f32x2(float lo, float hi) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void unpack_f32x2(unsigned long long v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ unsigned long long fma_f32x2(unsigned long long a, unsigned long long b,
                                                        unsigned long long c) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

template <int MT>
__global__ void __launch_bounds__(GV_THREADS, 2) mmr_gemv_cluster_kernel(const __grid_constant__ CUtensorMap tmB,
                                                                  const GemvParams p) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  constexpr int kStages = gv_stages(MT);
  extern __shared__ uint8_t gv_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(gv_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = base;                                                  // [stages][32][128] f32
  float* red = reinterpret_cast<float*>(base);                           // aliases the ring afterwards
  float* As = reinterpret_cast<float*>(base + gemv_ring_bytes(MT));      // [kslice][MT]
  float* part = As + MT * p.kslice;                                      // [GV_KSPLIT][per]
  uint64_t* full = reinterpret_cast<uint64_t*>(part + MT * GV_COLS);
  uint64_t* empty = full + kStages;
  uint64_t* recv = empty + kStages;  // GV_KSPLIT arrivals: every K-slice's partial is in `part`

  const int rank = static_cast<int>(cluster.block_rank());  // K-slice index
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int col0 = blockIdx.x * GV_COLS;
  const int k_lo = rank * p.kslice;
  const int k_hi = min(p.k, k_lo + p.kslice);
  const int nstages = k_hi > k_lo ? (k_hi - k_lo + GV_ROWS - 1) / GV_ROWS : 0;
  const WaitCtl ctl{p.err, p.timeout_ns};

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], GV_CONSUMER_WARPS);
    }
    mbar_init(recv, GV_KSPLIT);
    fence_mbar_init();
  }
  // the tensor map is a kernel parameter: fetch it before waiting on the
  // previous kernel
  if (warp == GV_CONSUMER_WARPS && lane == 0) tma_prefetch_desc(&tmB);
  __syncthreads();
  cluster_arrive_release();  // the receive barrier is ready; waited on before the first push
  griddep_wait();
  griddep_release();

  if (warp == GV_CONSUMER_WARPS) {
    // ---------------------------------------------------------- producer
    if (lane == 0) {
      int issued = 0;
      for (int s = 0; s < nstages; ++s) {
        const int slot = s % kStages;
        const uint32_t phase = static_cast<uint32_t>(s / kStages) & 1u;
        if (!mbar_wait(&empty[slot], phase ^ 1u, ctl, kDevTimeoutEmpty)) break;
        mbar_arrive_expect_tx(&full[slot], GV_STAGE_BYTES);
        tma_load_3d(ring + slot * GV_STAGE_BYTES, &tmB, &full[slot], col0, k_lo + s * GV_ROWS, 0);
        ++issued;
      }
      // Every issued load must land before the ring is reused or the CTA
      // exits (already true on the normal path).
      for (int s = issued > kStages ? issued - kStages : 0; s < issued; ++s) {
        const uint32_t a = smem_u32(&full[s % kStages]);
        const uint32_t phase = static_cast<uint32_t>(s / kStages) & 1u;
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(a, phase)) {
          if (globaltimer_ns() - t0 > p.timeout_ns) { atomicCAS(p.err, 0, kDevTimeoutDrain); break; }
        }
      }
    }
  } else {
    // A slice into shared memory while the first stages are in flight; the
    // loads are independent, so issue them back to back (16-byte vectors when
    // A's rows are K-contiguous and aligned).
    // Stored transposed, As[kk][mm], so that one B row's M multipliers are
    // contiguous and arrive as MT/4 broadcast 16-byte loads.
    const bool vec = p.a_k == 1 && (p.a_m & 3) == 0 && (k_lo & 3) == 0 &&
                     (reinterpret_cast<uintptr_t>(p.a) & 15u) == 0;
    if (vec) {
      // Consecutive lanes take consecutive rows m of A at the same k (the
      // warp still reads whole 32-byte sectors of each row), so their
      // transposed stores land in consecutive words: 2-way bank conflicts at
      // MT = 16 instead of 32-way with lanes along k.
      const int q4 = p.kslice >> 2;  // kslice is a multiple of 32
#pragma unroll 4
      for (int idx = threadIdx.x; idx < MT * q4; idx += GV_CONSUMER_WARPS * 32) {
        const int mm = idx % MT, kk = (idx / MT) * 4;
        const int gk = k_lo + kk;
        float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (mm < p.m) {
          if (gk + 3 < k_hi) {
            v = __ldg(reinterpret_cast<const float4*>(p.a + mm * p.a_m + gk));
          } else {
            if (gk < k_hi) v.x = p.a[mm * p.a_m + gk];
            if (gk + 1 < k_hi) v.y = p.a[mm * p.a_m + gk + 1];
            if (gk + 2 < k_hi) v.z = p.a[mm * p.a_m + gk + 2];
          }
        }
        As[(kk + 0) * MT + mm] = v.x;
        As[(kk + 1) * MT + mm] = v.y;
        As[(kk + 2) * MT + mm] = v.z;
        As[(kk + 3) * MT + mm] = v.w;
      }
    } else {
#pragma unroll 8
      for (int idx = threadIdx.x; idx < MT * p.kslice; idx += GV_CONSUMER_WARPS * 32) {
        const int mm = idx % MT, kk = idx / MT;  // consecutive lanes: consecutive words of As
        const int gk = k_lo + kk;
        As[kk * MT + mm] = (mm < p.m && gk < k_hi) ? p.a[mm * p.a_m + gk * p.a_k] : 0.0f;
      }
    }
    asm volatile("bar.sync 1, %0;" ::"n"(GV_CONSUMER_WARPS * 32) : "memory");  // consumers only
  }

  float acc[MT][4];
#pragma unroll
  for (int i = 0; i < MT; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.0f;

  if (warp < GV_CONSUMER_WARPS) {
    // ---------------------------------------------------------- consumers
    // For MT >= 2 the sums of rows m, m+1 (adjacent in the transposed A
    // slice) share one packed f32x2 FMA: the same per-element fused
    // multiply-add in the same order as scalar fmaf, at half the issue slots.
    constexpr int MP = MT >= 2 ? MT / 2 : 1;
    unsigned long long acc2[MP][4];
#pragma unroll
    for (int i = 0; i < MP; ++i) acc2[i][0] = acc2[i][1] = acc2[i][2] = acc2[i][3] = 0ull;
    for (int s = 0; s < nstages; ++s) {
      const int slot = s % kStages;
      const uint32_t phase = static_cast<uint32_t>(s / kStages) & 1u;
      if (!mbar_wait(&full[slot], phase, ctl, kDevTimeoutFull)) break;
      const uint8_t* st = ring + slot * GV_STAGE_BYTES + warp * 4 * (GV_COLS * 4) + lane * 16;
      const int kk0 = s * GV_ROWS + warp * 4;  // row offset within the slice
      const float* a0 = As + kk0 * MT;
      // This warp's four B rows go to registers and the slot is handed back
      // before the multiply-adds, so a slot is held for four shared loads,
      // not for the arithmetic: the whole ring stays in flight from HBM.
      float4 brow[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) brow[r] = *reinterpret_cast<const float4*>(st + r * (GV_COLS * 4));
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        if (k_lo + kk0 + r < k_hi) {
          const float4 bv = brow[r];
          if constexpr (MT >= 2) {
            const unsigned long long bd[4] = {pack_f32x2(bv.x, bv.x), pack_f32x2(bv.y, bv.y),
                                              pack_f32x2(bv.z, bv.z), pack_f32x2(bv.w, bv.w)};
            unsigned long long ap[MP];
            if constexpr (MT >= 4) {
#pragma unroll
              for (int i = 0; i < MT; i += 4) {
                const float4 a4 = *reinterpret_cast<const float4*>(a0 + r * MT + i);
                ap[i / 2] = pack_f32x2(a4.x, a4.y);
                ap[i / 2 + 1] = pack_f32x2(a4.z, a4.w);
              }
            } else {
              const float2 a2 = *reinterpret_cast<const float2*>(a0 + r * MT);
              ap[0] = pack_f32x2(a2.x, a2.y);
            }
#pragma unroll
            for (int i = 0; i < MP; ++i)
#pragma unroll
              for (int j = 0; j < 4; ++j) acc2[i][j] = fma_f32x2(ap[i], bd[j], acc2[i][j]);
          } else {
            const float av = a0[r * MT];
            acc[0][0] = fmaf(av, bv.x, acc[0][0]);
            acc[0][1] = fmaf(av, bv.y, acc[0][1]);
            acc[0][2] = fmaf(av, bv.z, acc[0][2]);
            acc[0][3] = fmaf(av, bv.w, acc[0][3]);
          }
        }
      }
    }
    if constexpr (MT >= 2) {
#pragma unroll
      for (int i = 0; i < MP; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) unpack_f32x2(acc2[i][j], acc[2 * i][j], acc[2 * i + 1][j]);
    }
  }
  __syncthreads();  // the ring is idle from here on: reuse it for partials

  if (warp < GV_CONSUMER_WARPS) {
#pragma unroll
    for (int i = 0; i < MT; ++i)
      *reinterpret_cast<float4*>(red + (warp * MT + i) * GV_COLS + lane * 4) =
          make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
  }
  __syncthreads();
  // CTA partial (fixed warp order 0..7), pushed to its owner: element idx of
  // the MT x 128 tile belongs to CTA idx / per and lands in slot `rank`.
  constexpr int per = MT * GV_COLS / GV_KSPLIT;
  static_assert(MT * GV_COLS % GV_KSPLIT == 0, "owner slices");
  cluster_wait_acquire();  // every peer's receive barrier is initialised
  for (int idx = threadIdx.x; idx < MT * GV_COLS; idx += GV_THREADS) {
    float sum = 0.0f;
#pragma unroll
    for (int w = 0; w < GV_CONSUMER_WARPS; ++w) sum += red[w * MT * GV_COLS + idx];
    cluster.map_shared_rank(part, idx / per)[rank * per + idx % per] = sum;
  }
  __syncthreads();
  if (threadIdx.x < GV_KSPLIT) mbar_arrive_release_cluster(mapa_shared(smem_u32(recv), threadIdx.x));

  // This CTA's share of the strip's outputs: slots 0..GV_KSPLIT-1 in order.
  // The CTA does not exit before every peer's pushes have landed here.
  if (!mbar_wait_acquire_cluster(recv, 0u, ctl, kDevTimeoutReduce)) return;
  const bool add_bias = epi_has_bias(p.epilogue);
  const int act = epi_act(p.epilogue);
  for (int j = threadIdx.x; j < per; j += GV_THREADS) {
    const int idx = rank * per + j;
    float sum = 0.0f;
#pragma unroll
    for (int q = 0; q < GV_KSPLIT; ++q) sum += part[q * per + j];
    const int mm = idx / GV_COLS, cc = col0 + (idx - mm * GV_COLS);
    if (mm < p.m && cc < p.n) {
      if (add_bias) sum = __fadd_rn(sum, p.bias[cc]);
      sum = act_apply(act, sum);
      p.c[mm * p.c_m + cc] = sum;
    }
  }
}

}  // namespace mmr
