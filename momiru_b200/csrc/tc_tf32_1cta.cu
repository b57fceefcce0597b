// tc_tf32_1cta.cu -- the TF32 tcgen05 kernels on one CTA per 128x256 tile.
#include "tc_launch.cuh"

namespace mmr {

cudaError_t tc_launch_tf32_1cta(bool a_mn, bool b_mn, const TcShape& sh, cudaStream_t s, const CUtensorMap& tm_a,
                                const CUtensorMap& tm_b, const CUtensorMap& tm_c, const TcParams& p) {
  return tc_launch_family<0, false>(a_mn, b_mn, sh, s, tm_a, tm_b, tm_c, p);
}

cudaError_t tc_prepare_tf32_1cta(bool a_mn, bool b_mn, int smem) { return tc_prepare_family<0, false>(a_mn, b_mn, smem); }

}  // namespace mmr
