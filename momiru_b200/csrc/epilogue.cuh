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
//              0.5 x (2 - erfc(|x|/sqrt 2)) for x > 0, in f64, rounded to f32,
//              with erfc the reference's own rational approximation
//              (erfc_nonnegative_f64, cpu.rs:2031-2099), restated below
// Products and sums are written with explicit round-to-nearest intrinsics so
// the compiler does not contract them into FMAs the reference does not use.
// The only library calls are the ones the reference makes to its platform's
// libm: expf (SiLU), tanhf (GELU-tanh) and the f64 exp inside erfc; CUDA's
// versions of those may differ from the host's in the last place.
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

// Horner evaluation in f64 as the reference writes it (horner and
// horner_leading_one, cpu.rs:2031-2046): r = r * x + c with the product and
// the sum rounded separately (the reference's Rust is never contracted to an
// FMA).
template <int N>
__device__ __forceinline__ double horner_rn(double x, const double (&c)[N]) {
  double r = c[0];
#pragma unroll
  for (int i = 1; i < N; ++i) r = __dadd_rn(__dmul_rn(r, x), c[i]);
  return r;
}
template <int N>
__device__ __forceinline__ double horner_one_rn(double x, const double (&c)[N]) {
  double r = __dadd_rn(x, c[0]);
#pragma unroll
  for (int i = 1; i < N; ++i) r = __dadd_rn(__dmul_rn(r, x), c[i]);
  return r;
}

// erfc of a finite nonnegative f64: the reference's erfc_nonnegative_f64
// (cpu.rs:2062-2099), the classical rational erf / erfc approximants on
// [0, 1), [1, 8) and [8, 27] with their published coefficients (the same
// constants as the reference, which the result depends on to the last bit),
// 0 above 27, and exp(-x^2) from the math library.
static __device__ __noinline__ double erfc_nonnegative(double x) {
  constexpr double T[5] = {9.60497373987051638749e0, 9.00260197203842689217e1, 2.23200534594684319226e3,
                           7.00332514112805075473e3, 5.55923013010394962768e4};
  constexpr double U[5] = {3.35617141647503099647e1, 5.21357949780152679795e2, 4.59432382970980127987e3,
                           2.26290000613890934246e4, 4.92673942608635921086e4};
  constexpr double P[9] = {2.46196981473530512524e-10, 5.64189564831068821977e-1, 7.46321056442269912687e0,
                           4.86371970985681366614e1,   1.96520832956077098242e2,  5.26445194995477358631e2,
                           9.34528527171957607540e2,   1.02755188689515710272e3,  5.57535335369399327526e2};
  constexpr double Q[8] = {1.32281951154744992508e1, 8.67072140885989742329e1, 3.54937778887819891062e2,
                           9.75708501743205489753e2, 1.82390916687909736289e3, 2.24633760818710981792e3,
                           1.65666309194161350182e3, 5.57535340817727675546e2};
  constexpr double R[6] = {5.64189583547755073984e-1, 1.27536670759978104416e0, 5.01905042251180477414e0,
                           6.16021097993053585195e0,  7.40974269950448939160e0, 2.97886665372100240670e0};
  constexpr double S[6] = {2.26052863220117276590e0, 9.39603524938001434673e0, 1.20489539808096656605e1,
                           1.70814450747565897222e1, 9.60896809063285878198e0, 3.36907645100081516050e0};
  if (x < 1.0) {
    const double x2 = __dmul_rn(x, x);
    // 1 - (x * T(x^2)) / U(x^2), left to right as the reference writes it
    return __dsub_rn(1.0, __ddiv_rn(__dmul_rn(x, horner_rn(x2, T)), horner_one_rn(x2, U)));
  }
  if (x > 27.0) return 0.0;
  const double fraction = x < 8.0 ? __ddiv_rn(horner_rn(x, P), horner_one_rn(x, Q))
                                  : __ddiv_rn(horner_rn(x, R), horner_one_rn(x, S));
  return __dmul_rn(exp(__dmul_rn(-x, x)), fraction);
}

// The activations other than ReLU: called out of line, once per element, from
// epilogues that keep their accumulators in registers.
static __device__ __noinline__ float act_other(int act, float x) {
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
      const double ec = erfc_nonnegative(__ddiv_rn(fabs(xd), 1.4142135623730951));
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
