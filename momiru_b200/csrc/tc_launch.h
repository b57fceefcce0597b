// tc_launch.h -- host-side entry points of the tcgen05 GEMM kernels.
//
// The kernels are instantiated in four translation units, one per numeric
// mode (3xTF32 / TF32) and CTA shape (one CTA per 128x256 tile / CTA pairs
// on 256x256 tiles), so that they compile in parallel; each unit covers the
// four operand-major combinations (A K- or M-contiguous, B K- or
// N-contiguous).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include "tc_gemm.cuh"

namespace mmr {

struct TcShape {
  dim3 grid, block;
  int smem;
};

// mode 1 = StrictFp32 (3xTF32), 0 = TF32; pair = CTA-pair kernel.
cudaError_t tc_launch(int mode, bool pair, bool a_mn, bool b_mn, const TcShape& sh, cudaStream_t s,
                      const CUtensorMap& tm_a, const CUtensorMap& tm_b, const CUtensorMap& tm_c, const TcParams& p);
// Shared-memory opt-in and the register-split check (cudaErrorInvalidConfiguration
// when the compiled register count cannot cover the kernel's setmaxnreg split).
cudaError_t tc_prepare(int mode, bool pair, bool a_mn, bool b_mn, int smem);

// The four units (tc_strict_1cta.cu, tc_tf32_1cta.cu, tc_strict_pair.cu, tc_tf32_pair.cu).
cudaError_t tc_launch_strict_1cta(bool a_mn, bool b_mn, const TcShape& sh, cudaStream_t s, const CUtensorMap& tm_a,
                                  const CUtensorMap& tm_b, const CUtensorMap& tm_c, const TcParams& p);
cudaError_t tc_launch_tf32_1cta(bool a_mn, bool b_mn, const TcShape& sh, cudaStream_t s, const CUtensorMap& tm_a,
                                const CUtensorMap& tm_b, const CUtensorMap& tm_c, const TcParams& p);
cudaError_t tc_launch_strict_pair(bool a_mn, bool b_mn, const TcShape& sh, cudaStream_t s, const CUtensorMap& tm_a,
                                  const CUtensorMap& tm_b, const CUtensorMap& tm_c, const TcParams& p);
cudaError_t tc_launch_tf32_pair(bool a_mn, bool b_mn, const TcShape& sh, cudaStream_t s, const CUtensorMap& tm_a,
                                const CUtensorMap& tm_b, const CUtensorMap& tm_c, const TcParams& p);
cudaError_t tc_prepare_strict_1cta(bool a_mn, bool b_mn, int smem);
cudaError_t tc_prepare_tf32_1cta(bool a_mn, bool b_mn, int smem);
cudaError_t tc_prepare_strict_pair(bool a_mn, bool b_mn, int smem);
cudaError_t tc_prepare_tf32_pair(bool a_mn, bool b_mn, int smem);

inline cudaError_t tc_launch(int mode, bool pair, bool a_mn, bool b_mn, const TcShape& sh, cudaStream_t s,
                             const CUtensorMap& tm_a, const CUtensorMap& tm_b, const CUtensorMap& tm_c,
                             const TcParams& p) {
  if (pair)
    return mode ? tc_launch_strict_pair(a_mn, b_mn, sh, s, tm_a, tm_b, tm_c, p)
                : tc_launch_tf32_pair(a_mn, b_mn, sh, s, tm_a, tm_b, tm_c, p);
  return mode ? tc_launch_strict_1cta(a_mn, b_mn, sh, s, tm_a, tm_b, tm_c, p)
              : tc_launch_tf32_1cta(a_mn, b_mn, sh, s, tm_a, tm_b, tm_c, p);
}

inline cudaError_t tc_prepare(int mode, bool pair, bool a_mn, bool b_mn, int smem) {
  if (pair) return mode ? tc_prepare_strict_pair(a_mn, b_mn, smem) : tc_prepare_tf32_pair(a_mn, b_mn, smem);
  return mode ? tc_prepare_strict_1cta(a_mn, b_mn, smem) : tc_prepare_tf32_1cta(a_mn, b_mn, smem);
}

}  // namespace mmr
