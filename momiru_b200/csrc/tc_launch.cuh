// tc_launch.cuh -- launch and preparation of one tcgen05 kernel family
// (numeric mode x CTA shape) over the four operand-major combinations.
// Included by exactly one translation unit per family.
#pragma once
#include "launch.cuh"
#include "tc_gemm_2sm.cuh"
#include "tc_launch.h"

namespace mmr {

template <int MODE, bool PAIR, bool AMN, bool BMN>
cudaError_t tc_launch_one(const TcShape& sh, cudaStream_t s, const CUtensorMap& tm_a, const CUtensorMap& tm_b,
                          const CUtensorMap& tm_c, const TcParams& p) {
  if constexpr (PAIR) {
    return launch_kernel(mmr_tc_gemm_2sm_kernel<MODE, AMN, BMN>, sh.grid, sh.block, sh.smem, s, dim3(2, 1, 1), tm_a,
                         tm_b, tm_c, p);
  } else {
    return launch_kernel(mmr_tc_gemm_kernel<MODE, AMN, BMN>, sh.grid, sh.block, sh.smem, s, dim3(1, 1, 1), tm_a, tm_b,
                         tm_c, p);
  }
}

// setmaxnreg.inc waits until the block's launch registers (threads x compiled
// count) can cover the request, so a split larger than that would never
// proceed: such a build is refused here instead of launched.
template <int MODE, bool PAIR, bool AMN, bool BMN>
cudaError_t tc_prepare_one(int smem) {
  using Cfg1 = TcConfig<MODE>;
  using Cfg2 = Tc2Config<MODE>;
  constexpr int threads = PAIR ? Cfg2::kThreads : Cfg1::kThreads;
  constexpr int epi_regs = PAIR ? Cfg2::kEpiRegs : Cfg1::kEpiRegs;
  constexpr int other_regs = PAIR ? Cfg2::kOtherRegs : Cfg1::kOtherRegs;
  const void* fn;
  if constexpr (PAIR) fn = reinterpret_cast<const void*>(mmr_tc_gemm_2sm_kernel<MODE, AMN, BMN>);
  else fn = reinterpret_cast<const void*>(mmr_tc_gemm_kernel<MODE, AMN, BMN>);
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  cudaFuncAttributes fa;
  e = cudaFuncGetAttributes(&fa, fn);
  if (e != cudaSuccess) return e;
  const long need = 2L * 128 * epi_regs + long(threads - 256) * other_regs;
  if (long(fa.numRegs) * threads < need) return cudaErrorInvalidConfiguration;
  return cudaSuccess;
}

template <int MODE, bool PAIR>
cudaError_t tc_launch_family(bool a_mn, bool b_mn, const TcShape& sh, cudaStream_t s, const CUtensorMap& tm_a,
                             const CUtensorMap& tm_b, const CUtensorMap& tm_c, const TcParams& p) {
  if (a_mn) {
    return b_mn ? tc_launch_one<MODE, PAIR, true, true>(sh, s, tm_a, tm_b, tm_c, p)
                : tc_launch_one<MODE, PAIR, true, false>(sh, s, tm_a, tm_b, tm_c, p);
  }
  return b_mn ? tc_launch_one<MODE, PAIR, false, true>(sh, s, tm_a, tm_b, tm_c, p)
              : tc_launch_one<MODE, PAIR, false, false>(sh, s, tm_a, tm_b, tm_c, p);
}

template <int MODE, bool PAIR>
cudaError_t tc_prepare_family(bool a_mn, bool b_mn, int smem) {
  if (a_mn) return b_mn ? tc_prepare_one<MODE, PAIR, true, true>(smem) : tc_prepare_one<MODE, PAIR, true, false>(smem);
  return b_mn ? tc_prepare_one<MODE, PAIR, false, true>(smem) : tc_prepare_one<MODE, PAIR, false, false>(smem);
}

}  // namespace mmr
