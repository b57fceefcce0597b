// epilogue.cuh -- the fused epilogue of the MatMul node:
//   out = act(acc + bias[col])    (bias optional, act one of the activations
// the reference CPU provider implements as elementwise f32 kernels).
//
// Activations, as the reference computes them (paths inside the reference):
//   relu       src/momiru/tensor_light/execution/cpu.rs:2158-2160
//              NaN kept, x > 0 kept, else +0
//   relu6      cpu.rs:2161-2163   NaN kept, x <= 0 -> +0, x >= 6 -> 6, else x
//   silu       cpu.rs:2166-2168 with sigmoid_value cpu.rs:2137-2144
//              -inf -> -0; else x * sigmoid(x), sigmoid split at 0 so that
//              exp never overflows; f32 arithmetic
//   gelu_tanh  cpu.rs:2214-2222   -inf -> -0, +inf -> +inf; else
//              0.5 x (1 + tanh(0.7978846 (x + 0.044715 x^3))) in f32
//   gelu_erf   cpu.rs:2117-2129   NaN / +-0 kept, -inf -> -0, +inf -> +inf;
//              else 0.5 x erfc(|x|/sqrt 2) for x < 0 and
//              0.5 x (2 - erfc(|x|/sqrt 2)) for x > 0, in f64, rounded to f32
// Products and sums are written with explicit round-to-nearest intrinsics so
// the compiler does not contract them into FMAs the reference does not use.
// expf / tanhf / erfc are CUDA's own library functions (the reference calls
// its platform's libm); their last-place differences are the only difference.
#pragma once
#include <cstdint>

namespace mmr {

// Epilogue codes (the ABI's MMR_EPI_* values).
enum : int {
  EPI_NONE = 0, EPI_BIAS = 1, EPI_BIAS_RELU = 2, EPI_RELU = 3,
  EPI_RELU6 = 4, EPI_BIAS_RELU6 = 5, EPI_GELU_ERF = 6, EPI_BIAS_GELU_ERF = 7,
  EPI_GELU_TANH = 8, EPI_BIAS_GELU_TANH = 9, EPI_SILU = 10, EPI_BIAS_SILU = 11,
  EPI_LAST = EPI_BIAS_SILU
};
enum : int { ACT_NONE = 0, ACT_RELU = 1, ACT_RELU6 = 2, ACT_GELU_ERF = 3, ACT_GELU_TANH = 4, ACT_SILU = 5 };

__host__ __device__ __forceinline__ bool epi_has_bias(int e) {
  return e == EPI_BIAS || e == EPI_BIAS_RELU || (e >= EPI_RELU6 && (e & 1));
}
__host__ __device__ __forceinline__ int epi_act(int e) {
  if (e == EPI_BIAS_RELU || e == EPI_RELU) return ACT_RELU;
  if (e >= EPI_RELU6) return ACT_RELU6 + (e - EPI_RELU6) / 2;
  return ACT_NONE;
}

__device__ __forceinline__ float act_relu(float x) { return (x != x) ? x : (x > 0.0f ? x : 0.0f); }

__device__ __forceinline__ float sigmoid_ref(float x) {
  if (x >= 0.0f) return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x)));
  const float e = expf(x);
  return __fdiv_rn(e, __fadd_rn(1.0f, e));
}

// The activations other than ReLU: called out of line, once per element, from
// epilogues that keep their accumulators in registers.
__device__ __noinline__ float act_other(int act, float x) {
  switch (act) {
    case ACT_RELU6:
      if (x != x) return x;
      if (x <= 0.0f) return 0.0f;
      return x >= 6.0f ? 6.0f : x;
    case ACT_SILU:
      if (x == -__int_as_float(0x7f800000)) return -0.0f;
      return __fmul_rn(x, sigmoid_ref(x));
    case ACT_GELU_TANH: {
      if (x == -__int_as_float(0x7f800000)) return -0.0f;
      if (x == __int_as_float(0x7f800000)) return x;
      const float cubic = __fmul_rn(__fmul_rn(x, x), x);
      const float t = tanhf(__fmul_rn(0.7978846f, __fadd_rn(x, __fmul_rn(0.044715f, cubic))));
      return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, t));
    }
    case ACT_GELU_ERF: {
      if (x != x || x == 0.0f) return x;
      if (x == -__int_as_float(0x7f800000)) return -0.0f;
      if (x == __int_as_float(0x7f800000)) return x;
      const double xd = static_cast<double>(x);
      const double ec = erfc(__ddiv_rn(fabs(xd), 1.4142135623730951));
      const double half_x = __dmul_rn(0.5, xd);
      return static_cast<float>(x < 0.0f ? __dmul_rn(half_x, ec) : __dmul_rn(half_x, __dsub_rn(2.0, ec)));
    }
    default:
      return x;
  }
}

__device__ __forceinline__ float act_apply(int act, float x) {
  if (act == ACT_NONE) return x;
  if (act == ACT_RELU) return act_relu(x);
  return act_other(act, x);
}

}  // namespace mmr
