// fixup.cuh -- exact recompute of the 3xTF32 tiles whose inputs hold inf or
// NaN (see tc_gemm.cuh): the tile list the split warps flagged is walked by
// 64x64 blocks of the CUDA-core kernel in the reference's exact order.
#pragma once
#include "simt_gemm.cuh"
#include "tc_gemm.cuh"

namespace mmr {

// Recomputes, in the reference's exact order, every output of the tiles the
// split warps flagged, then clears the bookkeeping for the next run (the last
// block to finish does it). With nothing flagged every block returns at once.
__global__ void __launch_bounds__(256) mmr_tc_nonfinite_fixup_kernel(const SimtParams sp, const TcParams p) {
  __shared__ float As[SIMT_BK][SIMT_BM + 4];
  __shared__ float Bs[SIMT_BK][SIMT_BN + 4];
  __shared__ bool last;
  griddep_wait();
  griddep_release();
  const unsigned int count = *reinterpret_cast<volatile unsigned int*>(&p.nf[0]);
  if (count == 0) return;
  const int kSub = (p.tile_m / SIMT_BM) * (TC_BN / SIMT_BN);
  for (unsigned int w = blockIdx.x; w < count * kSub; w += gridDim.x) {
    const int t = static_cast<int>(p.nf[2 + p.tiles_total + w / kSub]);
    const int sub = static_cast<int>(w % kSub);
    int mt, nt, bt;
    tc_tile_coords(p, t, mt, nt, bt);
    const int m0 = mt * p.tile_m + (sub / (TC_BN / SIMT_BN)) * SIMT_BM;
    const int n0 = nt * TC_BN + (sub % (TC_BN / SIMT_BN)) * SIMT_BN;
    simt_block_exact(sp, m0, n0, bt, As, Bs);
  }
  if (sp.npeers) __threadfence_system();
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last = (atomicAdd(&p.nf[1], 1u) == gridDim.x - 1);
  __syncthreads();
  if (last) {
    __threadfence();
    for (unsigned int i = threadIdx.x; i < count; i += blockDim.x) p.nf[2 + p.nf[2 + p.tiles_total + i]] = 0u;
    __syncthreads();
    if (threadIdx.x == 0) {
      p.nf[0] = 0u;
      p.nf[1] = 0u;
    }
  }
}

}  // namespace mmr
