// tc_strict_pair.cu -- the StrictFp32 (3xTF32) tcgen05 kernels on CTA pairs (256x256 tiles).
#include "tc_launch.cuh"

namespace mmr {

cudaError_t tc_launch_strict_pair(bool a_mn, bool b_mn, const TcShape& sh, cudaStream_t s, const CUtensorMap& tm_a,
                                  const CUtensorMap& tm_b, const CUtensorMap& tm_c, const TcParams& p) {
  return tc_launch_family<1, true>(a_mn, b_mn, sh, s, tm_a, tm_b, tm_c, p);
}

cudaError_t tc_prepare_strict_pair(bool a_mn, bool b_mn, int smem) { return tc_prepare_family<1, true>(a_mn, b_mn, smem); }

}  // namespace mmr
