// gemv.cuh -- skinny-M (M <= 16) f32 matmul that streams B from HBM once.
//
// y[m, n] = epilogue(sum_k A[m, k] * B[k, n]) for a row-major (N-contiguous)
// B. The work is HBM-bound (B is read exactly once, 4*K*N bytes), so the
// kernel is judged in GB/s, not FLOP/s. Layout of the launch:
//   grid.x  = ceil(N / 128) column blocks of 128 columns (32 lanes x float4)
//   grid.y  = GV_KSPLIT K-slices, one thread-block cluster of GV_KSPLIT CTAs
//             per column block (cluster dims 1 x GV_KSPLIT x 1)
//   8 warps per CTA split the CTA's K-slice again.
// Partial sums are reduced in a fixed order -- warps through shared memory,
// then the cluster's CTAs through distributed shared memory -- so results are
// deterministic run to run, without atomics or a global scratch buffer.
#pragma once
#include <cooperative_groups.h>
#include <stdint.h>

namespace mmr {

constexpr int GV_THREADS = 256;
constexpr int GV_WARPS = GV_THREADS / 32;
constexpr int GV_COLS = 128;
constexpr int GV_KSPLIT = 8;
constexpr int GV_MAX_M = 16;
constexpr int GV_MAX_KSLICE = 1024;  // K <= GV_KSPLIT * GV_MAX_KSLICE = 8192

struct GemvParams {
  int m, n, k;
  int kslice;  // ceil(K / GV_KSPLIT), a multiple of GV_WARPS
  const float* a; long long a_m, a_k;
  const float* b; long long b_k;  // B row stride (elements); column stride 1
  float* c; long long c_m;        // C row stride; column stride 1
  const float* bias;
  int epilogue;
};

// Dynamic shared memory: A slice [MT][kslice], per-warp partials
// [GV_WARPS][MT][128], and the CTA partial [MT][128] that cluster peers read.
__host__ __device__ constexpr int gemv_smem_bytes(int mt, int kslice) {
  return (mt * kslice + GV_WARPS * mt * GV_COLS + mt * GV_COLS) * 4;
}

template <int MT>
__global__ void __launch_bounds__(GV_THREADS) gemv_cluster_kernel(const GemvParams p) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  extern __shared__ float4 gv_smem4[];
  float* smem = reinterpret_cast<float*>(gv_smem4);
  float* As = smem;                                   // [MT][kslice]
  float* red = smem + MT * p.kslice;                  // [warp][MT][128]
  float* part = red + GV_WARPS * MT * GV_COLS;        // [MT][128]

  const int rank = static_cast<int>(cluster.block_rank());  // K-slice index
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int col0 = blockIdx.x * GV_COLS;
  const int k_lo = rank * p.kslice;
  const int k_hi = min(p.k, k_lo + p.kslice);

  for (int idx = threadIdx.x; idx < MT * p.kslice; idx += GV_THREADS) {
    const int mm = idx / p.kslice, kk = idx - mm * p.kslice;
    const int gk = k_lo + kk;
    As[idx] = (mm < p.m && gk < k_hi) ? p.a[mm * p.a_m + gk * p.a_k] : 0.0f;
  }
  __syncthreads();

  float acc[MT][4];
#pragma unroll
  for (int i = 0; i < MT; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.0f;

  const int wk = p.kslice / GV_WARPS;  // rows per warp
  const int wk_lo = k_lo + warp * wk;
  const int wk_hi = min(k_hi, wk_lo + wk);
  const int col = col0 + lane * 4;
  if (col < p.n) {
    const float* bcol = p.b + col;
    int k = wk_lo;
    for (; k + 8 <= wk_hi; k += 8) {
      float4 bv[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) bv[u] = __ldg(reinterpret_cast<const float4*>(bcol + (long long)(k + u) * p.b_k));
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const float* arow = As + (k + u - k_lo);
#pragma unroll
        for (int i = 0; i < MT; ++i) {
          const float av = arow[i * p.kslice];
          acc[i][0] = fmaf(av, bv[u].x, acc[i][0]);
          acc[i][1] = fmaf(av, bv[u].y, acc[i][1]);
          acc[i][2] = fmaf(av, bv[u].z, acc[i][2]);
          acc[i][3] = fmaf(av, bv[u].w, acc[i][3]);
        }
      }
    }
    for (; k < wk_hi; ++k) {
      const float4 bv = __ldg(reinterpret_cast<const float4*>(bcol + (long long)k * p.b_k));
      const float* arow = As + (k - k_lo);
#pragma unroll
      for (int i = 0; i < MT; ++i) {
        const float av = arow[i * p.kslice];
        acc[i][0] = fmaf(av, bv.x, acc[i][0]);
        acc[i][1] = fmaf(av, bv.y, acc[i][1]);
        acc[i][2] = fmaf(av, bv.z, acc[i][2]);
        acc[i][3] = fmaf(av, bv.w, acc[i][3]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < MT; ++i)
    *reinterpret_cast<float4*>(red + (warp * MT + i) * GV_COLS + lane * 4) =
        make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
  __syncthreads();

  // CTA partial: fixed warp order 0..7.
  for (int idx = threadIdx.x; idx < MT * GV_COLS; idx += GV_THREADS) {
    float s = 0.0f;
#pragma unroll
    for (int w = 0; w < GV_WARPS; ++w) s += red[w * MT * GV_COLS + idx];
    part[idx] = s;
  }
  cluster.sync();

  // Cluster reduction through DSMEM: CTA `rank` finalises a 1/GV_KSPLIT slice
  // of this column block's MT x 128 outputs, summing ranks 0..7 in order.
  const int per = (MT * GV_COLS + GV_KSPLIT - 1) / GV_KSPLIT;
  const bool add_bias = (p.epilogue == 1 || p.epilogue == 2);
  const bool relu = (p.epilogue == 2 || p.epilogue == 3);
  for (int j = threadIdx.x; j < per; j += GV_THREADS) {
    const int idx = rank * per + j;
    if (idx >= MT * GV_COLS) break;
    float s = 0.0f;
#pragma unroll
    for (int q = 0; q < GV_KSPLIT; ++q) s += cluster.map_shared_rank(part, q)[idx];
    const int mm = idx / GV_COLS, cc = col0 + (idx - mm * GV_COLS);
    if (mm < p.m && cc < p.n) {
      if (add_bias) s = __fadd_rn(s, p.bias[cc]);
      if (relu) s = (s != s) ? s : (s > 0.0f ? s : 0.0f);
      p.c[mm * p.c_m + cc] = s;
    }
  }
  cluster.sync();  // keep this CTA's `part` alive until every peer has read it
}

}  // namespace mmr
