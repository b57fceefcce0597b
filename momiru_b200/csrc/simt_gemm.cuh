// simt_gemm.cuh -- CUDA-core f32 GEMM in the reference's exact arithmetic.
//
// Every output element is s = +0; for p = 0..K-1: s = s + (a*b), with the
// product and the sum each rounded to f32 (__fmul_rn / __fadd_rn, no FMA) and
// p increasing -- the per-element order of gemm_dot_f32 / gemm_axpy_f32 /
// gemm_avx2 (src/momiru/tensor_light/execution/cpu.rs:2989-3098). Results are
// therefore bit-identical to the reference except for NaN payloads. Handles any
// element strides (negative ones too: reversed views), up to six batch axes
// with broadcast (stride 0), K = 0 (+0 then the epilogue), and every shape. It
// serves MMR_MATH_EXACT and the layouts TMA cannot describe.
#pragma once
#include <stdint.h>

#include "epilogue.cuh"
#include "ptx.cuh"

namespace mmr {

constexpr int SIMT_MAX_BATCH = 6;

struct SimtParams {
  int m, n, k;
  // Batch axes (outermost first); the flat batch index enumerates them in
  // row-major order. Strides are in elements, 0 on broadcast axes.
  int nb;
  int bdims[SIMT_MAX_BATCH];
  const float* a; long long a_bs[SIMT_MAX_BATCH], a_m, a_k;
  const float* b; long long b_bs[SIMT_MAX_BATCH], b_k, b_n;
  float* c; long long c_bs[SIMT_MAX_BATCH], c_m, c_n;
  const float* bias; long long bias_n;
  int epilogue;  // EPI_* (epilogue.cuh)
  // Replicas of C on other ranks (same element offsets), for the exact
  // recompute of a column-sharded GEMM's flagged tiles.
  int npeers;
  float* peer_c[7];
};

constexpr int SIMT_BM = 64, SIMT_BN = 64, SIMT_BK = 16;

// One 64x64 output block (rows m0.., cols n0.. of flat batch entry bz) in the
// reference's exact order, written through the epilogue. 256 threads.
__device__ __forceinline__ void simt_block_exact(const SimtParams& p, int m0, int n0, int bz,
                                                 float (*As)[SIMT_BM + 4], float (*Bs)[SIMT_BN + 4]) {
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  long long ao = 0, bo = 0, co = 0;
  for (int j = p.nb - 1, rem = bz; j >= 0; --j) {
    const int i = rem % p.bdims[j];
    rem /= p.bdims[j];
    ao += i * p.a_bs[j];
    bo += i * p.b_bs[j];
    co += i * p.c_bs[j];
  }
  const float* A = p.a + ao;
  const float* B = p.b + bo;
  float* C = p.c + co;

  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;

  for (int k0 = 0; k0 < p.k; k0 += SIMT_BK) {
    const int kmax = min(SIMT_BK, p.k - k0);
    for (int idx = threadIdx.x; idx < SIMT_BK * SIMT_BM; idx += 256) {
      const int kk = idx / SIMT_BM, mm = idx - kk * SIMT_BM;
      const int gm = m0 + mm, gk = k0 + kk;
      As[kk][mm] = (gm < p.m && kk < kmax) ? A[(long long)gm * p.a_m + (long long)gk * p.a_k] : 0.0f;
    }
    for (int idx = threadIdx.x; idx < SIMT_BK * SIMT_BN; idx += 256) {
      const int kk = idx / SIMT_BN, nn = idx - kk * SIMT_BN;
      const int gn = n0 + nn, gk = k0 + kk;
      Bs[kk][nn] = (gn < p.n && kk < kmax) ? B[(long long)gk * p.b_k + (long long)gn * p.b_n] : 0.0f;
    }
    __syncthreads();
    for (int kk = 0; kk < kmax; ++kk) {
      float av[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) av[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) bv[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(av[i], bv[j]));
    }
    __syncthreads();
  }

  const bool add_bias = epi_has_bias(p.epilogue);
  const int act = epi_act(p.epilogue);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int gm = m0 + ty * 4 + i;
    if (gm >= p.m) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int gn = n0 + tx * 4 + j;
      if (gn >= p.n) continue;
      float x = acc[i][j];
      if (add_bias) x = __fadd_rn(x, p.bias[(long long)gn * p.bias_n]);
      x = act_apply(act, x);
      C[(long long)gm * p.c_m + (long long)gn * p.c_n] = x;
      for (int q = 0; q < p.npeers; ++q)
        p.peer_c[q][co + gm * p.c_m + gn * p.c_n] = x;
    }
  }
}

__global__ void __launch_bounds__(256) mmr_simt_gemm_exact_kernel(const SimtParams p) {
  __shared__ float As[SIMT_BK][SIMT_BM + 4];
  __shared__ float Bs[SIMT_BK][SIMT_BN + 4];
  griddep_wait();
  griddep_release();
  simt_block_exact(p, blockIdx.y * SIMT_BM, blockIdx.x * SIMT_BN, blockIdx.z, As, Bs);
}

}  // namespace mmr
