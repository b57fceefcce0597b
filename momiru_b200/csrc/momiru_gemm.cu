// momiru_gemm.cu -- C ABI of the B200 f32 matmul hot path (include/momiru_gemm.h).
//
// Bind-time work (validation, kernel-family choice, TMA descriptor encoding,
// event creation) happens once in mmr_gemm_bind; mmr_gemm_run only enqueues
// the pre-built launch. This mirrors the reference runtime's split between
// Backend::bind_resources and BoundBackend::execute_gpu_node
// (src/momiru/tensor_light/execution/runtime.rs:879-988).
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "../../include/momiru_gemm.h"
#include "gemv.cuh"
#include "gemv_tc.cuh"
#include "launch.cuh"
#include "ptx.cuh"
#include "fixup.cuh"
#include "simt_gemm.cuh"
#include "tc_gemm_2sm.cuh"
#include "tc_launch.h"

namespace {

thread_local std::string g_last_error;

int32_t fail(int32_t code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

#define MMR_CUDA_TRY(expr)                                                                      \
  do {                                                                                          \
    cudaError_t e_ = (expr);                                                                    \
    if (e_ != cudaSuccess) return fail(MMR_ERR_CUDA, "%s: %s", #expr, cudaGetErrorString(e_)); \
  } while (0)

// Restores the caller's current device on scope exit.
struct DeviceGuard {
  int prev = -1;
  bool ok = false;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) == cudaSuccess && cudaSetDevice(dev) == cudaSuccess) ok = true;
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

// ------------------------------------------------------------- the plan --

// Batch axes a plan keeps after canonicalisation (a rank-8 view has six).
constexpr int kMaxBatch = MMR_MAX_RANK - 2;
static_assert(kMaxBatch == mmr::SIMT_MAX_BATCH, "the SIMT kernel indexes every batch axis a plan keeps");

// A logical matrix operand: element (batch index i[0..nb), row r, col c)
// lives at base + sum_j i[j]*s_b[j] + r*s_r + c*s_c (elements, signed;
// s_b[j] = 0 where the operand is broadcast over batch axis j).
struct Operand {
  uint64_t base = 0;  // device address of element [0,..,0]
  int64_t s_b[kMaxBatch] = {};
  int64_t s_r = 0, s_c = 0;
  uint64_t lo = 0, hi = 0;  // byte range touched (for aliasing checks)
  uint64_t alloc = 0;
};

struct Plan {
  // Batch axes of the output after canonicalisation: extent-1 axes dropped,
  // neighbours merged wherever every operand walks them as one axis.
  int nb = 0;
  int64_t bdims[kMaxBatch] = {};
  int64_t batch = 1;  // product of bdims
  int64_t m = 0, n = 0, k = 0;
  Operand a, b, c;
  uint64_t bias = 0;
  int64_t bias_s = 0;
  int32_t epilogue = MMR_EPI_NONE;
  int32_t math = MMR_MATH_STRICT_FP32;
  int32_t family = MMR_FAMILY_AUTO;
  int32_t device = 0;
  bool empty = false;  // nothing to compute (some output extent is zero)
};

// Smallest and largest element offset a view reaches (strides may be
// negative: a reversed axis); false when some extent is 0 (no element).
bool view_span(const mmr_view& v, int64_t* lo, int64_t* hi) {
  *lo = 0;
  *hi = 0;
  for (int i = 0; i < v.rank; ++i) {
    if (v.dims[i] == 0) return false;
    const int64_t reach = (v.dims[i] - 1) * v.strides[i];
    if (reach < 0) *lo += reach; else *hi += reach;
  }
  return true;
}

// Shape, alignment and bounds of one view (cpu.rs:613-714 restated for
// device views). Rank 0 (a scalar) is admitted where `allow_scalar` is set:
// the output of a vector-vector product (validation.rs:2355-2361).
int32_t check_view(const mmr_view& v, const char* name, int32_t device, bool allow_scalar = false) {
  const int min_rank = allow_scalar ? 0 : 1;
  if (v.rank < min_rank || v.rank > MMR_MAX_RANK)
    return fail(MMR_ERR_INVALID_SHAPE, "%s: rank %d outside %d..%d", name, v.rank, min_rank, MMR_MAX_RANK);
  for (int i = 0; i < v.rank; ++i) {
    if (v.dims[i] < 0) return fail(MMR_ERR_INVALID_SHAPE, "%s: negative extent on axis %d", name, i);
    if (v.dims[i] > (int64_t(1) << 31) - 1)
      return fail(MMR_ERR_INVALID_SHAPE, "%s: extent %lld on axis %d exceeds 2^31-1", name,
                  (long long)v.dims[i], i);
    if (v.strides[i] > (int64_t(1) << 40) || v.strides[i] < -(int64_t(1) << 40))
      return fail(MMR_ERR_UNSUPPORTED_LAYOUT, "%s: stride on axis %d beyond 2^40 elements", name, i);
  }
  if (v.base_offset_bytes % 4 != 0)
    return fail(MMR_ERR_UNSUPPORTED_LAYOUT, "%s: base offset %llu is not f32-aligned", name,
                (unsigned long long)v.base_offset_bytes);
  if (v.address % 4 != 0) return fail(MMR_ERR_UNSUPPORTED_LAYOUT, "%s: address is not f32-aligned", name);
  int64_t lo = 0, hi = 0;
  if (view_span(v, &lo, &hi)) {
    if (v.address == 0) return fail(MMR_ERR_INVALID_ARGUMENT, "%s: null address", name);
    const int64_t first = int64_t(v.base_offset_bytes / 4) + lo;
    if (first < 0)
      return fail(MMR_ERR_OUT_OF_BOUNDS, "%s: a negative stride reaches %lld elements before the buffer", name,
                  (long long)-first);
    const uint64_t need = v.base_offset_bytes + uint64_t(hi + 1) * 4u;
    if (need > v.bytes)
      return fail(MMR_ERR_OUT_OF_BOUNDS, "%s: view needs %llu bytes but the buffer has %llu", name,
                  (unsigned long long)need, (unsigned long long)v.bytes);
  }
  if (v.device_ordinal != device)
    return fail(MMR_ERR_UNSUPPORTED_DEVICE, "%s: device ordinal %d differs from the node's %d", name,
                v.device_ordinal, device);
  return MMR_OK;
}

// canonical_broadcast_extent (src/momiru/tensor_light/execution/ir.rs:247-252):
// equal -> that; 1 vs x -> x (so 0 vs 1 -> 0); otherwise incompatible.
bool broadcast_extent(int64_t l, int64_t r, int64_t* out) {
  if (l == r) { *out = l; return true; }
  if (l == 1) { *out = r; return true; }
  if (r == 1) { *out = l; return true; }
  return false;
}

void set_range(Operand& o, const mmr_view& v) {
  int64_t lo = 0, hi = 0;
  const uint64_t at = v.address + v.base_offset_bytes;
  if (view_span(v, &lo, &hi)) {
    o.lo = at + uint64_t(lo * 4);  // wraps correctly for lo < 0 (bounds checked)
    o.hi = at + uint64_t((hi + 1) * 4);
  } else {
    o.lo = o.hi = at;
  }
  o.alloc = v.allocation_id;
}

bool ranges_overlap(const Operand& x, const Operand& y) {
  if (x.lo == x.hi || y.lo == y.hi) return false;
  return x.lo < y.hi && y.lo < x.hi;
}

// The MatMul node's shape and broadcast contract, following
// validation.rs:2300-2398, plus the bind-time layout admission of
// cpu.rs:613-714 / runtime.rs:618-811 restated for device views.
int32_t build_plan(const mmr_matmul_desc* d, Plan* p) {
  if (!d) return fail(MMR_ERR_INVALID_ARGUMENT, "null descriptor");
  if (d->math_mode < MMR_MATH_STRICT_FP32 || d->math_mode > MMR_MATH_EXACT)
    return fail(MMR_ERR_INVALID_ARGUMENT, "unknown math mode %d", d->math_mode);
  if (d->epilogue < MMR_EPI_NONE || d->epilogue > MMR_EPI_BIAS_SILU)
    return fail(MMR_ERR_INVALID_ARGUMENT, "unknown epilogue %d", d->epilogue);
  if (d->family < MMR_FAMILY_AUTO || d->family > MMR_FAMILY_SIMT)
    return fail(MMR_ERR_INVALID_ARGUMENT, "unknown kernel family %d", d->family);
  p->epilogue = d->epilogue;
  p->math = d->math_mode;
  p->family = d->family;
  p->device = d->device_ordinal;

  const mmr_view &L = d->lhs, &R = d->rhs, &O = d->out;
  int32_t rc;
  if ((rc = check_view(L, "lhs", d->device_ordinal))) return rc;
  if ((rc = check_view(R, "rhs", d->device_ordinal))) return rc;
  if ((rc = check_view(O, "out", d->device_ordinal, true))) return rc;

  const int lr = L.rank, rr = R.rank;
  const bool ta = d->transpose_lhs != 0, tb = d->transpose_rhs != 0;
  if ((lr == 1 && ta) || (rr == 1 && tb))
    return fail(MMR_ERR_INVALID_SHAPE, "transpose flag on a rank-1 operand");
  const bool lv = lr == 1, rv = rr == 1;

  // Logical A [M,K] and B [K,N] with the promoted vector dims.
  int64_t m, k1, k2, n;
  Operand A, B, C;
  A.base = L.address + L.base_offset_bytes;
  B.base = R.address + R.base_offset_bytes;
  C.base = O.address + O.base_offset_bytes;
  if (lv) {
    m = 1; k1 = L.dims[0]; A.s_r = 0; A.s_c = L.strides[0];
  } else {
    const int64_t rows = L.dims[lr - 2], cols = L.dims[lr - 1];
    const int64_t sr = L.strides[lr - 2], sc = L.strides[lr - 1];
    if (ta) { m = cols; k1 = rows; A.s_r = sc; A.s_c = sr; }
    else    { m = rows; k1 = cols; A.s_r = sr; A.s_c = sc; }
  }
  if (rv) {
    k2 = R.dims[0]; n = 1; B.s_r = R.strides[0]; B.s_c = 0;
  } else {
    const int64_t rows = R.dims[rr - 2], cols = R.dims[rr - 1];
    const int64_t sr = R.strides[rr - 2], sc = R.strides[rr - 1];
    if (tb) { k2 = cols; n = rows; B.s_r = sc; B.s_c = sr; }
    else    { k2 = rows; n = cols; B.s_r = sr; B.s_c = sc; }
  }
  if (k1 != k2)
    return fail(MMR_ERR_INVALID_SHAPE, "contraction mismatch: lhs K=%lld, rhs K=%lld", (long long)k1,
                (long long)k2);
  const int lbr = lv ? 0 : lr - 2, rbr = rv ? 0 : rr - 2;
  const int br = std::max(lbr, rbr);
  const int mat_rank = (lv ? 0 : 1) + (rv ? 0 : 1);
  // The output's rank is exactly batch rank + matrix dims: a vector-vector
  // product has a rank-0 (scalar) output (validation.rs:2355-2361).
  if (O.rank != br + mat_rank)
    return fail(MMR_ERR_INVALID_SHAPE, "output rank %d, expected %d", O.rank, br + mat_rank);

  // Batch axes, right-aligned (NumPy broadcast), each checked against the
  // output; extent-1 axes index nothing and are dropped.
  int nb = 0;
  int64_t bdims[kMaxBatch];
  int64_t as_b[kMaxBatch], bs_b[kMaxBatch], cs_b[kMaxBatch];
  for (int b = 0; b < br; ++b) {
    const int li = b - (br - lbr), ri = b - (br - rbr);
    const int64_t ld = li >= 0 ? L.dims[li] : 1, rd = ri >= 0 ? R.dims[ri] : 1;
    int64_t e;
    if (!broadcast_extent(ld, rd, &e))
      return fail(MMR_ERR_INVALID_SHAPE, "batch axis %d: %lld vs %lld do not broadcast", b, (long long)ld,
                  (long long)rd);
    if (O.dims[b] != e)
      return fail(MMR_ERR_INVALID_SHAPE, "output batch axis %d is %lld, expected %lld", b,
                  (long long)O.dims[b], (long long)e);
    if (e == 1) continue;
    bdims[nb] = e;
    as_b[nb] = (li >= 0 && ld != 1) ? L.strides[li] : 0;
    bs_b[nb] = (ri >= 0 && rd != 1) ? R.strides[ri] : 0;
    cs_b[nb] = O.strides[b];
    ++nb;
  }
  // Merge neighbouring axes that every operand walks as one (outer stride =
  // inner stride x inner extent; broadcast axes have stride 0 on both).
  for (int j = nb - 2; j >= 0; --j) {
    const int64_t d1 = bdims[j + 1];
    if (as_b[j] == as_b[j + 1] * d1 && bs_b[j] == bs_b[j + 1] * d1 && cs_b[j] == cs_b[j + 1] * d1) {
      bdims[j] *= d1;
      as_b[j] = as_b[j + 1];
      bs_b[j] = bs_b[j + 1];
      cs_b[j] = cs_b[j + 1];
      for (int q = j + 1; q + 1 < nb; ++q) {
        bdims[q] = bdims[q + 1];
        as_b[q] = as_b[q + 1];
        bs_b[q] = bs_b[q + 1];
        cs_b[q] = cs_b[q + 1];
      }
      --nb;
    }
  }
  int64_t batch = 1;
  for (int j = 0; j < nb; ++j) {
    if (bdims[j] > 0 && batch > (int64_t(1) << 40) / bdims[j])
      return fail(MMR_ERR_INVALID_SHAPE, "batch of more than 2^40 matrices");
    batch *= bdims[j];
  }
  int oax = br;
  if (!lv) {
    if (O.dims[oax] != m)
      return fail(MMR_ERR_INVALID_SHAPE, "output rows %lld, expected %lld", (long long)O.dims[oax], (long long)m);
    C.s_r = O.strides[oax];
    ++oax;
  }
  if (!rv) {
    if (O.dims[oax] != n)
      return fail(MMR_ERR_INVALID_SHAPE, "output cols %lld, expected %lld", (long long)O.dims[oax], (long long)n);
    C.s_c = O.strides[oax];
  }
  if (lv && !rv) C.s_r = 0;
  if (rv && !lv) { C.s_r = O.strides[br]; C.s_c = 0; }
  for (int j = 0; j < nb; ++j) {
    A.s_b[j] = as_b[j];
    B.s_b[j] = bs_b[j];
    C.s_b[j] = cs_b[j];
  }
  set_range(A, L);
  set_range(B, R);
  set_range(C, O);

  // Aliasing: the output may not overlap an input (runtime.rs:540-551).
  if (ranges_overlap(C, A) || ranges_overlap(C, B))
    return fail(MMR_ERR_UNSAFE_ALIASING, "output storage overlaps an input");

  const bool needs_bias = mmr::epi_has_bias(d->epilogue);
  if (needs_bias) {
    const mmr_view& V = d->bias;
    if ((rc = check_view(V, "bias", d->device_ordinal))) return rc;
    if (V.rank != 1 || V.dims[0] != n)
      return fail(MMR_ERR_INVALID_SHAPE, "bias must be rank 1 with N=%lld entries", (long long)n);
    Operand bo;
    set_range(bo, V);
    if (ranges_overlap(C, bo)) return fail(MMR_ERR_UNSAFE_ALIASING, "output storage overlaps the bias");
    p->bias = V.address + V.base_offset_bytes;
    p->bias_s = V.strides[0];
  }

  p->nb = nb;
  for (int j = 0; j < nb; ++j) p->bdims[j] = bdims[j];
  p->batch = batch;
  p->m = m;
  p->n = n;
  p->k = k1;
  p->a = A;
  p->b = B;
  p->c = C;
  p->empty = (batch == 0 || m == 0 || n == 0);
  return MMR_OK;
}

// ---------------------------------------------------- family admission --

// One batch axis for TMA: the operand is either broadcast over the whole
// batch or indexed by the flattened (row-major) batch index with a single
// stride, i.e. its strides chain across every batch axis.
bool flat_batch(const Plan& p, const Operand& o, int64_t* stride, bool* batched) {
  bool any = false;
  for (int j = 0; j < p.nb; ++j) any |= o.s_b[j] != 0;
  *batched = any;
  *stride = 0;
  if (!any) return true;
  for (int j = 0; j + 1 < p.nb; ++j)
    if (o.s_b[j] != o.s_b[j + 1] * p.bdims[j + 1]) return false;
  *stride = o.s_b[p.nb - 1];
  return true;
}

struct TmaLayout {
  bool ok = false;
  bool a_mn = false, b_mn = false;
  bool a_batched = false, b_batched = false;
  int64_t a_sb = 0, b_sb = 0, c_sb = 0;
  const char* why = "";
};

TmaLayout tma_admission(const Plan& p) {
  TmaLayout t;
  auto aligned16 = [](uint64_t x) { return (x & 15u) == 0; };
  if (p.k <= 0) { t.why = "K = 0"; return t; }
  if (p.m > INT32_MAX || p.n > INT32_MAX || p.k > INT32_MAX) { t.why = "extent too large"; return t; }
  bool cb;
  if (!flat_batch(p, p.a, &t.a_sb, &t.a_batched) || !flat_batch(p, p.b, &t.b_sb, &t.b_batched) ||
      !flat_batch(p, p.c, &t.c_sb, &cb)) {
    t.why = "batch axes do not flatten to one strided axis";
    return t;
  }
  const int64_t batch = p.batch;
  if (batch > 1 && !cb) { t.why = "output broadcast over the batch"; return t; }
  if ((t.a_batched && t.a_sb <= 0) || (t.b_batched && t.b_sb <= 0) || (batch > 1 && t.c_sb <= 0)) {
    t.why = "a negative batch stride (TMA walks forward only)";
    return t;
  }
  if (p.bias && p.bias_s != 1) { t.why = "strided bias"; return t; }
  // A: K-contiguous (K-major) or M-contiguous (MN-major).
  if (p.a.s_c == 1 && (p.a.s_r % 4 == 0) && p.a.s_r > 0) t.a_mn = false;
  else if (p.a.s_r == 1 && (p.a.s_c % 4 == 0) && p.a.s_c > 0) t.a_mn = true;
  else { t.why = "lhs has no unit-stride matrix axis with a 16-byte-aligned other stride"; return t; }
  // B: N-contiguous (MN-major) or K-contiguous (K-major).
  if (p.b.s_c == 1 && (p.b.s_r % 4 == 0) && p.b.s_r > 0) t.b_mn = true;
  else if (p.b.s_r == 1 && (p.b.s_c % 4 == 0) && p.b.s_c > 0) t.b_mn = false;
  else { t.why = "rhs has no unit-stride matrix axis with a 16-byte-aligned other stride"; return t; }
  if (!(p.c.s_c == 1 && p.c.s_r % 4 == 0 && p.c.s_r > 0)) { t.why = "output is not row-major with 16-byte rows"; return t; }
  if (!aligned16(p.a.base) || !aligned16(p.b.base) || !aligned16(p.c.base)) {
    t.why = "operand base not 16-byte aligned";
    return t;
  }
  if ((t.a_batched && t.a_sb % 4) || (t.b_batched && t.b_sb % 4) || (batch > 1 && t.c_sb % 4)) {
    t.why = "batch stride not 16-byte aligned";
    return t;
  }
  t.ok = true;
  return t;
}

bool gemv_admission(const Plan& p, const char** why) {
  if (p.batch != 1) { *why = "batched"; return false; }
  if (p.a.s_r < 0 || p.a.s_c < 0 || p.c.s_r < 0 || p.c.s_c < 0) { *why = "negative strides"; return false; }
  if (p.m < 1 || p.m > mmr::GV_MAX_M) { *why = "M outside 1..16"; return false; }
  if (p.k < 1 || p.k > int64_t(mmr::GV_KSPLIT) * mmr::GV_MAX_KSLICE) { *why = "K outside 1..8192"; return false; }
  if (p.n > INT32_MAX) { *why = "N too large"; return false; }
  // B is streamed by TMA: N-contiguous rows with a 16-byte pitch and base.
  if (!(p.b.s_c == 1 && p.b.s_r % 4 == 0 && p.b.s_r > 0 && (p.b.base & 15u) == 0)) {
    *why = "rhs must be row-major with 16-byte rows";
    return false;
  }
  if (p.c.s_c != 1 && p.n > 1) { *why = "output columns not contiguous"; return false; }
  if (p.bias && p.bias_s != 1) { *why = "strided bias"; return false; }
  return true;
}

// The tensor-core GEMV also streams A through TMA, by 32-wide K panels of its
// (up to 16) rows: A must be K-contiguous with 16-byte-aligned rows and base.
// It replaces the CUDA-core GEMV where it is faster (B200, N = K = 4096):
// TF32 from M = 2 (about 4.6 TB/s at every M; the CUDA-core kernel's time
// grows with M), StrictFp32 above M = 8, where the CUDA-core kernel's
// multiply-adds (8 flop per byte of B at M = 16) outlast the split's two
// tensor-core instructions per k-step.
constexpr int kGemvTcMinMTf32 = 2, kGemvTcMinMStrict = 9;
bool gemv_tc_admission(const Plan& p) {
  if (p.m < (p.math == MMR_MATH_TF32 ? kGemvTcMinMTf32 : kGemvTcMinMStrict)) return false;
  if (p.a.s_c != 1 || (p.a.base & 15u) != 0) return false;
  if (p.m > 1 && (p.a.s_r <= 0 || p.a.s_r % 4 != 0)) return false;
  return true;
}

// --------------------------------------------------------- TMA encoding --

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// 3-D f32 tensor map {inner, outer, batch} with a 128-byte swizzle: 16-byte
// atoms for K-major operand tiles and the output, 32-byte atoms (the layout
// tcgen05 kind::tf32 reads MN-major operands in) when `atom32` is set.
int32_t encode_3d(CUtensorMap* tm, uint64_t base, uint64_t inner, uint64_t outer, uint64_t batch,
                  int64_t outer_stride_el, int64_t batch_stride_el, uint32_t box_inner, uint32_t box_outer,
                  const char* name, bool atom32 = false, bool no_swizzle = false) {
  // A 16-wide (64-byte) box of a K-major operand takes the 64-byte swizzle.
  const CUtensorMapSwizzle swz = no_swizzle ? CU_TENSOR_MAP_SWIZZLE_NONE
                                 : atom32   ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B
                                 : box_inner * 4 == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B;
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(MMR_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  if (batch < 1) batch = 1;
  uint64_t bstride = uint64_t(batch_stride_el) * 4u;
  if (batch == 1 || bstride == 0) {
    // Unused axis (extent 1): any legal stride.
    bstride = ((uint64_t(outer_stride_el) * 4u * std::max<uint64_t>(outer, 1)) + 15u) & ~uint64_t(15);
    if (bstride == 0) bstride = 16;
  }
  cuuint64_t dims[3] = {inner, outer, batch};
  cuuint64_t strides[2] = {uint64_t(outer_stride_el) * 4u, bstride};
  cuuint32_t box[3] = {box_inner, box_outer, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, reinterpret_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(MMR_ERR_UNSUPPORTED_LAYOUT, "%s: cuTensorMapEncodeTiled failed (%d): dims {%llu,%llu,%llu}", name,
                int(r), (unsigned long long)inner, (unsigned long long)outer, (unsigned long long)batch);
  return MMR_OK;
}

}  // namespace

namespace {

// Every launch decision bind freezes for a node, derived on the host from the
// plan and the device's SM count alone (no CUDA call): the fields of the
// reference's frozen GpuKernelPlan (plan.rs:941-1026) that this library owns.
struct Launch {
  int32_t family = MMR_FAMILY_AUTO;
  int mode = 0;         // tcgen05: 1 = 3xTF32, 0 = TF32
  bool pair = false;    // tcgen05 on CTA pairs
  uint32_t bk = 0;      // k-block width
  int tile_m = 0, tile_n = 0, tile_k = 0;
  int64_t tiles = 0;
  int k_blocks = 0, chunk_kb = 0;
  int64_t npairs = 0;   // CTA pairs launched (pair kernel)
  int64_t split = 1;    // K parts per tile when there are fewer tiles than pairs
  int sk_tiles = 0;     // trailing tiles split stream-K style
  dim3 grid, block;
  int smem = 0;
  int cluster_x = 1, cluster_y = 1;
  int stages = 0, warps = 0, producer_warps = 0, consumer_warps = 0;
  int tmem_columns = 0, tmem_acc_stages = 0;
  int gv_mt = 0, kslice = 0;
  bool gemv_tc = false;  // GEMV on the tensor cores (swap-AB), else on CUDA cores
  int tensor_maps = 0;
};

}  // namespace

// ----------------------------------------------------------------- handle --

struct mmr_gemm_handle {
  Plan plan;
  mmr_gemm_info info{};
  int device = 0;
  cudaStream_t stream = nullptr;
  int family = MMR_FAMILY_AUTO;
  // tcgen05
  CUtensorMap tmA, tmB, tmC;
  mmr::TcParams tcp{};
  bool a_mn = false, b_mn = false;
  int mode = 0;
  bool pair = false;  // StrictFp32 on CTA pairs (cta_group::2)
  // gemv
  mmr::GemvParams gvp{};
  int gv_mt = 16;
  // gemv on the tensor cores
  bool gemv_tc = false;
  mmr::GemvTcParams gtp{};
  CUtensorMap tmA_gv;
  // simt
  mmr::SimtParams sp{};
  dim3 grid, block;
  int smem = 0;
  int* d_err = nullptr;
  int* h_err = nullptr;  // pinned host copy of the error word
  unsigned int* d_nf = nullptr;  // 3xTF32 non-finite bookkeeping
  float* d_ws = nullptr;         // stream-K partial sums (CTA pairs)
  unsigned int* d_ws_count = nullptr;
  size_t ws_count_bytes = 0;
  int sms = 148;
  Launch launch;  // the frozen launch decisions (mmr_gemm_launch_record)
  // column-sharded GEMM with replicated output
  bool sharded = false;
  int rank = 0, nranks = 1;
  unsigned long long* peer_signal[8] = {};
  unsigned long long* signal = nullptr;
  unsigned long long epoch = 0;
  CUtensorMap* d_peer_tm = nullptr;  // the peers' replica tensor maps (device memory)
  cudaEvent_t done = nullptr, err_ev = nullptr;
  bool ran = false;
  uint64_t wait_timeout_ns = 2000000000ull;
  // operands in host memory (mmr_gemm_bind_host): a device GEMM per row panel
  struct Copy2D {
    char* host = nullptr;
    size_t host_pitch = 0;
    char* dev = nullptr;
    size_t dev_pitch = 0;
    size_t width = 0;  // bytes of one row's logical columns
    size_t rows = 0;
  };
  bool host = false;
  Copy2D h_lhs, h_rhs, h_out, h_bias;
  void* dbuf[4] = {};
  std::vector<mmr_gemm_handle*> panel;
  std::vector<int64_t> panel_row;  // panel i covers rows [panel_row[i], panel_row[i + 1])
  cudaStream_t s_in = nullptr, s_comp = nullptr, s_out = nullptr;
  cudaEvent_t ev_start = nullptr, ev_rhs = nullptr;
  std::vector<cudaEvent_t> ev_lhs, ev_gemm;
};

namespace {

// The three tensor maps of a tcgen05 launch: operand boxes are one k-block
// wide (bk = 32 or 16 f32) and 128 (A) / b_rows (B: 256 for one CTA, 128 for
// each CTA of a pair) long, or 32-wide MN atoms; the output box is 32 x 32.
int32_t encode_tc_maps(mmr_gemm_handle* h, const Plan& p, const TmaLayout& t, int64_t batch, uint32_t bk,
                       uint32_t b_rows = mmr::TC_BN) {
  int32_t e;
  const uint32_t panel_k = std::min(bk, 32u);  // K-major boxes are one 32-wide (128-byte) panel at most
  if (!t.a_mn) e = encode_3d(&h->tmA, p.a.base, p.k, p.m, t.a_batched ? batch : 1, p.a.s_r, t.a_sb, panel_k, mmr::TC_BM, "lhs");
  else e = encode_3d(&h->tmA, p.a.base, p.m, p.k, t.a_batched ? batch : 1, p.a.s_c, t.a_sb, 32, bk, "lhs", true);
  if (e) return e;
  if (t.b_mn) e = encode_3d(&h->tmB, p.b.base, p.n, p.k, t.b_batched ? batch : 1, p.b.s_r, t.b_sb, 32, bk, "rhs", true);
  else e = encode_3d(&h->tmB, p.b.base, p.k, p.n, t.b_batched ? batch : 1, p.b.s_c, t.b_sb, panel_k, b_rows, "rhs");
  if (e) return e;
  return encode_3d(&h->tmC, p.c.base, p.n, p.m, batch, p.c.s_r, t.c_sb, 32, 32, "out");
}

template <int MT>
cudaError_t launch_gemv_mt(const mmr_gemm_handle* h, cudaStream_t s) {
  return mmr::launch_kernel(mmr::mmr_gemv_cluster_kernel<MT>, h->grid, h->block, h->smem, s,
                            dim3(1, mmr::GV_KSPLIT, 1), h->tmB, h->gvp);
}

template <int MT>
cudaError_t prepare_gemv_mt(int smem) {
  cudaError_t e = cudaFuncSetAttribute(mmr::mmr_gemv_cluster_kernel<MT>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(mmr::mmr_gemv_cluster_kernel<MT>, cudaFuncAttributeNonPortableClusterSizeAllowed, 0);
}

cudaError_t launch_gemv_tc(const mmr_gemm_handle* h, cudaStream_t s) {
  const dim3 cluster(1, mmr::GT_KSPLIT, 1);
  if (h->mode) return mmr::launch_kernel(mmr::mmr_gemv_tc_kernel<1>, h->grid, h->block, h->smem, s, cluster, h->tmB, h->tmA_gv, h->gtp);
  return mmr::launch_kernel(mmr::mmr_gemv_tc_kernel<0>, h->grid, h->block, h->smem, s, cluster, h->tmB, h->tmA_gv, h->gtp);
}

cudaError_t launch_gemv(const mmr_gemm_handle* h, cudaStream_t s) {
  switch (h->gv_mt) {
    case 1: return launch_gemv_mt<1>(h, s);
    case 2: return launch_gemv_mt<2>(h, s);
    case 4: return launch_gemv_mt<4>(h, s);
    case 8: return launch_gemv_mt<8>(h, s);
    default: return launch_gemv_mt<16>(h, s);
  }
}
cudaError_t prepare_gemv(int mt, int smem) {
  switch (mt) {
    case 1: return prepare_gemv_mt<1>(smem);
    case 2: return prepare_gemv_mt<2>(smem);
    case 4: return prepare_gemv_mt<4>(smem);
    case 8: return prepare_gemv_mt<8>(smem);
    default: return prepare_gemv_mt<16>(smem);
  }
}

void fill_simt_params(const Plan& p, mmr::SimtParams* sp) {
  mmr::SimtParams& s = *sp;
  s.m = int(p.m);
  s.n = int(p.n);
  s.k = int(p.k);
  s.nb = p.nb;
  for (int j = 0; j < mmr::SIMT_MAX_BATCH; ++j) {
    s.bdims[j] = j < p.nb ? int(p.bdims[j]) : 1;
    s.a_bs[j] = j < p.nb ? p.a.s_b[j] : 0;
    s.b_bs[j] = j < p.nb ? p.b.s_b[j] : 0;
    s.c_bs[j] = j < p.nb ? p.c.s_b[j] : 0;
  }
  s.a = reinterpret_cast<const float*>(p.a.base);
  s.a_m = p.a.s_r; s.a_k = p.a.s_c;
  s.b = reinterpret_cast<const float*>(p.b.base);
  s.b_k = p.b.s_r; s.b_n = p.b.s_c;
  s.c = reinterpret_cast<float*>(p.c.base);
  s.c_m = p.c.s_r; s.c_n = p.c.s_c;
  s.bias = reinterpret_cast<const float*>(p.bias);
  s.bias_n = p.bias_s;
  s.epilogue = p.epilogue;
}

void fill_info_common(const Plan& p, mmr_gemm_info* info) {
  info->math_mode = p.math;
  info->batch = p.batch;
  info->m = p.m;
  info->n = p.n;
  info->k = p.k;
  info->flops = 2.0 * double(info->batch) * double(p.m) * double(p.n) * double(p.k);
}

// Algorithmic HBM bytes: every operand element read once, C written once.
double algorithmic_bytes(const Plan& p, bool a_batched, bool b_batched) {
  const double batch = double(p.batch);
  const double a = double(p.m) * double(p.k) * (a_batched ? batch : 1.0);
  const double b = double(p.k) * double(p.n) * (b_batched ? batch : 1.0);
  const double c = double(p.m) * double(p.n) * batch;
  const double bias = p.bias ? double(p.n) : 0.0;
  return 4.0 * (a + b + c + bias);
}

int32_t choose_family(const Plan& p, const TmaLayout& t, int32_t* family) {
  const char* gemv_why = "";
  const bool gemv_ok = p.math != MMR_MATH_EXACT && gemv_admission(p, &gemv_why);
  if (p.family == MMR_FAMILY_AUTO) {
    if (p.math == MMR_MATH_EXACT) *family = MMR_FAMILY_SIMT;
    else if (gemv_ok) *family = MMR_FAMILY_GEMV;
    else if (t.ok) *family = MMR_FAMILY_TCGEN05;
    else *family = MMR_FAMILY_SIMT;
    return MMR_OK;
  }
  if (p.family == MMR_FAMILY_TCGEN05) {
    if (p.math == MMR_MATH_EXACT)
      return fail(MMR_ERR_UNSUPPORTED_MATH, "the tcgen05 family cannot give the bit-exact reference order");
    if (!t.ok) return fail(MMR_ERR_UNSUPPORTED_FAMILY, "tcgen05 family not admissible: %s", t.why);
  } else if (p.family == MMR_FAMILY_GEMV) {
    if (p.math == MMR_MATH_EXACT)
      return fail(MMR_ERR_UNSUPPORTED_MATH, "the GEMV family splits K and cannot give the bit-exact order");
    if (!gemv_ok) return fail(MMR_ERR_UNSUPPORTED_FAMILY, "GEMV family not admissible: %s", gemv_why);
  }
  *family = p.family;
  return MMR_OK;
}

int32_t derive_launch(const Plan& p, const TmaLayout& t, int32_t fam, int sms, Launch* out) {
  Launch L;
  L.family = fam;
  const int64_t batch = p.batch;
  if (p.empty) {
    *out = L;
    return MMR_OK;
  }
  if (fam == MMR_FAMILY_TCGEN05) {
    L.mode = (p.math == MMR_MATH_STRICT_FP32) ? 1 : 0;
    // Both modes run on CTA pairs (256-row tiles) unless M fits one 128-row tile.
    L.pair = p.m > mmr::TC_BM;
    L.bk = L.pair ? (L.mode ? mmr::Tc2Config<1>::kBK : mmr::Tc2Config<0>::kBK)
                  : (L.mode ? mmr::TcConfig<1>::kBK : mmr::TcConfig<0>::kBK);
    L.tile_m = L.pair ? 2 * mmr::TC_BM : mmr::TC_BM;
    L.tile_n = mmr::TC_BN;
    L.tile_k = int(L.bk);
    const int64_t tiles_m = (p.m + L.tile_m - 1) / L.tile_m, tiles_n = (p.n + mmr::TC_BN - 1) / mmr::TC_BN;
    L.tiles = tiles_m * tiles_n * batch;
    if (L.tiles > INT32_MAX) return fail(MMR_ERR_INVALID_SHAPE, "too many output tiles");
    L.k_blocks = int((p.k + L.bk - 1) / L.bk);
    // StrictFp32 sums K in chunks of 256 with round-to-nearest adds; one TF32
    // pass keeps a single chain per tile.
    L.chunk_kb = L.mode ? int(256 / L.bk) : L.k_blocks;
    L.tensor_maps = 3;
    L.tmem_columns = 512;
    L.tmem_acc_stages = 2;
    L.producer_warps = 1;
    if (L.pair) {
      L.smem = L.mode ? mmr::Tc2Config<1>::kSmemBytes : mmr::Tc2Config<0>::kSmemBytes;
      // Fewer tiles than pairs and a long K: split each tile along K over
      // several pairs, stream-K style, in parts of at least 512 K (3xTF32)
      // or 1024 K (TF32). Measured on B200 with parts of 2048 / 512 / 256 /
      // 64 K (3xTF32): 512^2 x 4096 76 / 40.5 / 44.2 / 46.1 us, 256^2 x
      // 16384 82 / 61 / 83 / 100 us; TF32 1024^2 x 8192 60 / 45 us at
      // 4096 / 1024 K. Each part parks a 256 KB partial tile in L2 and the
      // last one reads them all back, which is what shorter parts lose on.
      const int64_t min_part_k = L.mode ? 512 : 1024;
      L.split = L.tiles < sms / 2
                    ? std::max<int64_t>(1, std::min<int64_t>((sms / 2) / L.tiles, p.k / min_part_k))
                    : 1;
      L.npairs = std::min<int64_t>(L.tiles, sms / 2) * L.split;
      L.grid = dim3(unsigned(2 * L.npairs));
      // Whole rounds of tiles stay round-robin. When the tiles do not fill
      // the last round, that round is split stream-K; when it is less than
      // half full, the round before it is split too, so that no tile is cut
      // into more pieces than about three pairs.
      const int64_t rem = L.tiles % L.npairs;
      L.sk_tiles = L.npairs > L.tiles ? int(L.tiles) : rem == 0 ? 0 : int(2 * rem >= L.npairs ? rem : L.npairs + rem);
      L.block = dim3(L.mode ? mmr::Tc2Config<1>::kThreads : mmr::Tc2Config<0>::kThreads);
      L.cluster_x = 2;
      L.stages = L.mode ? mmr::Tc2Config<1>::kStages : mmr::Tc2Config<0>::kStages;
    } else {
      L.smem = L.mode ? mmr::TcConfig<1>::kSmemBytes : mmr::TcConfig<0>::kSmemBytes;
      L.grid = dim3(unsigned(std::min<int64_t>(L.tiles, sms)));
      L.block = dim3(L.mode ? mmr::TcConfig<1>::kThreads : mmr::TcConfig<0>::kThreads);
      L.stages = L.mode ? mmr::TcConfig<1>::kStages : mmr::TcConfig<0>::kStages;
    }
    L.warps = int(L.block.x / 32);
    L.consumer_warps = L.warps - 2;  // epilogue (+ split) warps beside the producer and the MMA issuer
  } else if (fam == MMR_FAMILY_GEMV && gemv_tc_admission(p)) {
    // Tensor cores: 128-column strips x GT_KSPLIT K-slices (one cluster per
    // strip), 32-row stages of B with the matching A panel.
    L.gemv_tc = true;
    L.mode = (p.math == MMR_MATH_STRICT_FP32) ? 1 : 0;
    const int64_t kslice = (p.k + mmr::GT_KSPLIT - 1) / mmr::GT_KSPLIT;
    L.kslice = int((kslice + mmr::GT_BK - 1) / mmr::GT_BK * mmr::GT_BK);
    L.smem = mmr::gt_smem_bytes(L.mode);
    L.grid = dim3(unsigned((p.n + mmr::GT_COLS - 1) / mmr::GT_COLS), mmr::GT_KSPLIT, 1);
    L.block = dim3(mmr::gt_threads(L.mode));
    L.cluster_y = mmr::GT_KSPLIT;
    L.stages = mmr::gt_stages(L.mode);
    L.warps = int(L.block.x / 32);
    L.producer_warps = 1;
    L.consumer_warps = L.warps - 2;
    L.tile_m = mmr::GT_MN;
    L.tile_n = mmr::GT_COLS;
    L.tile_k = mmr::GT_BK;
    L.tmem_columns = mmr::gt_tmem_cols(L.mode);
    L.tmem_acc_stages = 2;
    L.tensor_maps = 2;
  } else if (fam == MMR_FAMILY_GEMV) {
    int kslice = int((p.k + mmr::GV_KSPLIT - 1) / mmr::GV_KSPLIT);
    L.kslice = (kslice + mmr::GV_ROWS - 1) / mmr::GV_ROWS * mmr::GV_ROWS;
    L.gv_mt = p.m <= 1 ? 1 : p.m <= 2 ? 2 : p.m <= 4 ? 4 : p.m <= 8 ? 8 : 16;
    L.smem = mmr::gemv_smem_bytes(L.gv_mt, L.kslice);
    L.grid = dim3(unsigned((p.n + mmr::GV_COLS - 1) / mmr::GV_COLS), mmr::GV_KSPLIT, 1);
    L.block = dim3(mmr::GV_THREADS);
    L.cluster_y = mmr::GV_KSPLIT;
    L.stages = mmr::gv_stages(L.gv_mt);
    L.warps = mmr::GV_THREADS / 32;
    L.producer_warps = 1;
    L.consumer_warps = L.warps - 1;
    L.tile_m = L.gv_mt;
    L.tile_n = mmr::GV_COLS;
    L.tile_k = L.kslice;
    L.tensor_maps = 1;
  } else {
    if (batch > 65535) return fail(MMR_ERR_INVALID_SHAPE, "batch too large for the SIMT family");
    L.grid = dim3(unsigned((p.n + mmr::SIMT_BN - 1) / mmr::SIMT_BN), unsigned((p.m + mmr::SIMT_BM - 1) / mmr::SIMT_BM),
                  unsigned(batch));
    if (L.grid.y > 65535) return fail(MMR_ERR_INVALID_SHAPE, "M too large for the SIMT family");
    L.block = dim3(256);
    L.tile_m = mmr::SIMT_BM;
    L.tile_n = mmr::SIMT_BN;
    L.tile_k = mmr::SIMT_BK;
    L.warps = 8;
    L.consumer_warps = 8;
    L.stages = 1;
  }
  *out = L;
  return MMR_OK;
}

void to_record(const Launch& L, int32_t math, mmr_launch_record* r) {
  memset(r, 0, sizeof *r);
  r->family = L.family;
  r->math_mode = math;
  r->grid[0] = int32_t(L.grid.x);
  r->grid[1] = int32_t(L.grid.y);
  r->grid[2] = int32_t(L.grid.z);
  r->block[0] = int32_t(L.block.x);
  r->block[1] = int32_t(L.block.y);
  r->block[2] = int32_t(L.block.z);
  r->cluster[0] = L.cluster_x;
  r->cluster[1] = L.cluster_y;
  r->cluster[2] = 1;
  r->dynamic_shared_bytes = L.smem;
  r->tmem_columns_per_cta = L.tmem_columns;
  r->tmem_accumulator_stages = L.tmem_acc_stages;
  r->tile_m = L.tile_m;
  r->tile_n = L.tile_n;
  r->tile_k = L.tile_k;
  r->pipeline_stages = L.stages;
  r->warps_per_block = L.warps;
  r->producer_warps = L.producer_warps;
  r->consumer_warps = L.consumer_warps;
  const bool tc = L.family == MMR_FAMILY_TCGEN05;
  r->matrix_acceleration = (tc || L.gemv_tc) ? MMR_ACCEL_TCGEN05 : MMR_ACCEL_NONE;
  r->async_copy = L.tensor_maps > 0 ? MMR_ASYNC_COPY_TMA : MMR_ASYNC_COPY_NONE;
  r->tensor_maps = L.tensor_maps;
  if (tc) {
    r->partition = L.sk_tiles > 0 ? MMR_PARTITION_STREAM_K : MMR_PARTITION_PERSISTENT_CTA;
    r->split_k = int32_t(L.split);
    r->stream_k_slices = L.sk_tiles;
    r->persistent_ctas_per_sm = 1;
  } else if (L.family == MMR_FAMILY_GEMV) {
    r->partition = MMR_PARTITION_SPLIT_K;  // K over the CTAs of a cluster, reduced in DSMEM
    r->split_k = L.gemv_tc ? mmr::GT_KSPLIT : mmr::GV_KSPLIT;
    r->use_distributed_shared_memory = 1;
  } else {
    r->partition = MMR_PARTITION_GRID;
    r->split_k = 1;
  }
  r->cluster_launch = (L.cluster_x * L.cluster_y > 1) ? 1 : 0;
}

// The GPU validator's rules on a frozen record (validation.rs:5630-5700,
// 5846-5911, restated for the fields this record carries; B200 limits:
// 512 TMEM columns per CTA in units of 32, 227 KB of shared memory per block,
// portable clusters of at most 8 CTAs).
int32_t check_record_rules(const mmr_launch_record& r) {
  auto bad = [](const char* why) { return fail(MMR_ERR_PLAN_MISMATCH, "frozen launch record: %s", why); };
  if (r.family < MMR_FAMILY_TCGEN05 || r.family > MMR_FAMILY_SIMT) return bad("family is not a bound kernel family");
  if (r.math_mode < MMR_MATH_STRICT_FP32 || r.math_mode > MMR_MATH_EXACT) return bad("unknown math mode");
  for (int i = 0; i < 3; ++i)
    if (r.grid[i] < 0 || r.block[i] < 1 || r.cluster[i] < 1) return bad("grid, block and cluster extents");
  const long threads = long(r.block[0]) * r.block[1] * r.block[2];
  if (threads > 1024) return bad("more than 1024 threads per block");
  if (r.warps_per_block != (threads + 31) / 32) return bad("warps_per_block differs from the block size");
  if (r.producer_warps < 0 || r.consumer_warps < 0 || r.producer_warps + r.consumer_warps > r.warps_per_block)
    return bad("producer and consumer warps exceed the block");
  if (r.dynamic_shared_bytes < 0 || r.dynamic_shared_bytes > 232448) return bad("dynamic shared memory above 227 KB");
  const int cl = r.cluster[0] * r.cluster[1] * r.cluster[2];
  if (cl > 8) return bad("cluster of more than 8 CTAs (non-portable)");
  if ((cl > 1) != (r.cluster_launch != 0)) return bad("cluster dims and cluster_launch disagree");
  for (int i = 0; i < 3; ++i)
    if (r.cluster[i] > 1 && r.grid[i] % r.cluster[i] != 0) return bad("grid is not a whole number of clusters");
  const bool uses_tmem = r.tmem_columns_per_cta > 0 || r.tmem_accumulator_stages > 0;
  if (uses_tmem) {
    if (r.tmem_columns_per_cta <= 0 || r.tmem_accumulator_stages <= 0 || r.tmem_columns_per_cta > 512)
      return bad("TMEM columns must be 1..512 with at least one accumulator stage");
    if (r.tmem_columns_per_cta % 32 != 0 || (r.tmem_columns_per_cta & (r.tmem_columns_per_cta - 1)) != 0)
      return bad("TMEM columns must be a power of two and a multiple of 32");
  }
  if (r.matrix_acceleration == MMR_ACCEL_TCGEN05 && !uses_tmem) return bad("tcgen05 without tensor memory");
  if (r.matrix_acceleration != MMR_ACCEL_TCGEN05 && r.matrix_acceleration != MMR_ACCEL_NONE)
    return bad("matrix acceleration other than none or tcgen05");
  if (r.async_copy == MMR_ASYNC_COPY_TMA && r.tensor_maps < 1) return bad("TMA without tensor maps");
  if (r.async_copy != MMR_ASYNC_COPY_TMA && r.tensor_maps != 0) return bad("tensor maps without TMA");
  if (r.async_copy != MMR_ASYNC_COPY_TMA && r.async_copy != MMR_ASYNC_COPY_NONE)
    return bad("async copy other than none or TMA");
  if (r.partition < MMR_PARTITION_GRID || r.partition > MMR_PARTITION_PERSISTENT_CTA) return bad("unknown partition");
  if (r.split_k < 1 || r.stream_k_slices < 0) return bad("split_k below 1 or negative stream-K slices");
  if (r.tile_m < 1 || r.tile_n < 1 || r.tile_k < 1 || r.pipeline_stages < 1) return bad("tile or stage count below 1");
  return MMR_OK;
}

int32_t fill_validate_info(const Plan& p, mmr_gemm_info* info) {
  TmaLayout t = tma_admission(p);
  int32_t fam = MMR_FAMILY_AUTO;
  int32_t rc = choose_family(p, t, &fam);
  if (rc) return rc;
  if (info) {
    memset(info, 0, sizeof *info);
    fill_info_common(p, info);
    info->family = fam;
    info->a_mn_major = t.a_mn;
    info->b_mn_major = t.b_mn;
    info->bytes = algorithmic_bytes(p, fam == MMR_FAMILY_TCGEN05 ? t.a_batched : true,
                                    fam == MMR_FAMILY_TCGEN05 ? t.b_batched : true);
  }
  return MMR_OK;
}

}  // namespace

// ------------------------------------------------------------------- ABI --

// ------------------------------------------------------------------------
// Scratch for mmr_gemm_run_noalloc: a fixed array in the library image, so
// that entry point never allocates device memory. Layout (32-bit words):
//   [0] device error word, [1..3] unused,
//   [4] inf/NaN tile count, [5] fix-up blocks done,
//   [6, 6+T) per-tile flags, [6+T, 6+2T) flagged tile list (T = output tiles).
// Host code must not use the array's name as a pointer: it stands for a host
// shadow, not a device address. The device address comes from
// cudaGetSymbolAddress, once per device, with that device current.
constexpr int kNoAllocWords = MMR_NOALLOC_SCRATCH_BYTES / 4;
static_assert(6 + 2 * MMR_NOALLOC_MAX_TILES <= kNoAllocWords, "scratch too small for the stated tile limit");
static __device__ __align__(256) unsigned int g_noalloc_scratch[kNoAllocWords];

namespace {

struct NoAllocDevice {
  bool ready = false;
  unsigned int* scratch = nullptr;  // device address of g_noalloc_scratch
  int sms = 0;
};
constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
NoAllocDevice g_noalloc_dev[kNoAllocMaxDevices];

// First use on a device (that device current): resolve the array's device
// address and prepare the four 3xTF32 kernel variants (shared-memory opt-in and
// the register-split check). Allocates nothing.
int32_t noalloc_setup(int dev, NoAllocDevice** out) {
  if (dev < 0 || dev >= kNoAllocMaxDevices)
    return fail(MMR_ERR_UNSUPPORTED_DEVICE, "device ordinal %d outside 0..%d", dev, kNoAllocMaxDevices - 1);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  NoAllocDevice& d = g_noalloc_dev[dev];
  if (!d.ready) {
    void* ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess) return fail(MMR_ERR_CUDA, "cudaGetSymbolAddress(scratch): %s", cudaGetErrorString(e));
    int sms = 0;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return fail(MMR_ERR_CUDA, "cudaDeviceGetAttribute: %s", cudaGetErrorString(e));
    const int smem = mmr::TcConfig<1>::kSmemBytes;
    for (int amn = 0; amn < 2; ++amn)
      for (int bmn = 0; bmn < 2; ++bmn) {
        e = mmr::tc_prepare(1, false, amn, bmn, smem);
        if (e != cudaSuccess)
          return fail(MMR_ERR_CUDA, "preparing the 3xTF32 kernel: %s", cudaGetErrorString(e));
      }
    d.scratch = static_cast<unsigned int*>(ptr);
    d.sms = sms;
    d.ready = true;
  }
  *out = &d;
  return MMR_OK;
}

}  // namespace

static_assert(int(mmr::EPI_LAST) == int(MMR_EPI_BIAS_SILU) && int(mmr::EPI_BIAS_GELU_ERF) == int(MMR_EPI_BIAS_GELU_ERF),
              "device epilogue codes follow the ABI");

extern "C" {

const char* mmr_last_error(void) { return g_last_error.c_str(); }

const char* mmr_version(void) {
  return "momiru_b200 0.1.0 (sm_100a; tcgen05 tf32/3xtf32, gemv-cluster, simt-exact)";
}

int32_t mmr_gemm_validate(const mmr_matmul_desc* desc, mmr_gemm_info* info) {
  Plan p;
  int32_t rc = build_plan(desc, &p);
  if (rc) return rc;
  return fill_validate_info(p, info);
}

int32_t mmr_gemm_bind(const mmr_matmul_desc* desc, mmr_gemm_handle** out) {
  if (!out) return fail(MMR_ERR_INVALID_ARGUMENT, "null output handle pointer");
  *out = nullptr;
  Plan p;
  int32_t rc = build_plan(desc, &p);
  if (rc) return rc;

  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0)
    return fail(MMR_ERR_UNSUPPORTED_DEVICE, "no CUDA device is visible");
  if (p.device < 0 || p.device >= ndev)
    return fail(MMR_ERR_UNSUPPORTED_DEVICE, "device ordinal %d outside 0..%d", p.device, ndev - 1);
  DeviceGuard guard(p.device);
  if (!guard.ok) return fail(MMR_ERR_CUDA, "cudaSetDevice(%d) failed", p.device);
  int major = 0, minor = 0, sms = 0;
  MMR_CUDA_TRY(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, p.device));
  MMR_CUDA_TRY(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, p.device));
  MMR_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, p.device));
  if (major != 10 || minor != 0)
    return fail(MMR_ERR_UNSUPPORTED_DEVICE, "device %d is sm_%d%d; this library is built for sm_100a", p.device,
                major, minor);
  // Every bound address must be device memory of this ordinal.
  const uint64_t addrs[4] = {desc->lhs.address, desc->rhs.address, desc->out.address,
                             mmr::epi_has_bias(desc->epilogue) ? desc->bias.address : 0};
  for (uint64_t a : addrs) {
    if (!a) continue;
    cudaPointerAttributes pa;
    if (cudaPointerGetAttributes(&pa, reinterpret_cast<void*>(a)) != cudaSuccess) {
      cudaGetLastError();
      return fail(MMR_ERR_UNSUPPORTED_DEVICE, "address 0x%llx is not known to CUDA", (unsigned long long)a);
    }
    if (pa.type != cudaMemoryTypeDevice && pa.type != cudaMemoryTypeManaged)
      return fail(MMR_ERR_UNSUPPORTED_DEVICE, "address 0x%llx is not device memory", (unsigned long long)a);
    if (pa.device != p.device)
      return fail(MMR_ERR_UNSUPPORTED_DEVICE, "address 0x%llx lives on device %d, not %d", (unsigned long long)a,
                  pa.device, p.device);
  }

  TmaLayout t = tma_admission(p);
  int32_t fam = MMR_FAMILY_AUTO;
  if ((rc = choose_family(p, t, &fam))) return rc;

  mmr_gemm_handle* h = new mmr_gemm_handle();
  h->plan = p;
  h->device = p.device;
  h->stream = reinterpret_cast<cudaStream_t>(desc->stream);
  h->family = fam;
  fill_info_common(p, &h->info);
  h->info.family = fam;

  auto cleanup = [&](int32_t code) {
    mmr_gemm_destroy(h);
    return code;
  };
  if (cudaMalloc(&h->d_err, sizeof(int)) != cudaSuccess) return cleanup(fail(MMR_ERR_CUDA, "cudaMalloc(error word) failed"));
  if (cudaMemset(h->d_err, 0, sizeof(int)) != cudaSuccess) return cleanup(fail(MMR_ERR_CUDA, "cudaMemset failed"));
  if (cudaHostAlloc(&h->h_err, sizeof(int), cudaHostAllocDefault) != cudaSuccess)
    return cleanup(fail(MMR_ERR_CUDA, "cudaHostAlloc failed"));
  *h->h_err = 0;
  if (cudaEventCreateWithFlags(&h->done, cudaEventDisableTiming) != cudaSuccess ||
      cudaEventCreateWithFlags(&h->err_ev, cudaEventDisableTiming) != cudaSuccess)
    return cleanup(fail(MMR_ERR_CUDA, "cudaEventCreate failed"));

  if (p.empty) {
    h->info.bytes = 0;
    *out = h;
    return MMR_OK;
  }

  const int64_t batch = p.batch;
  Launch L;
  if ((rc = derive_launch(p, t, fam, sms, &L))) return cleanup(rc);
  h->launch = L;
  h->grid = L.grid;
  h->block = L.block;
  h->smem = L.smem;
  h->sms = sms;
  if (fam == MMR_FAMILY_TCGEN05) {
    h->mode = L.mode;
    h->pair = L.pair;
    h->a_mn = t.a_mn;
    h->b_mn = t.b_mn;
    int32_t e = encode_tc_maps(h, p, t, batch, L.bk, L.pair ? 128u : uint32_t(mmr::TC_BN));
    if (e) return cleanup(e);

    mmr::TcParams& q = h->tcp;
    q.m = int(p.m);
    q.n = int(p.n);
    q.k = int(p.k);
    q.batch = int(batch);
    q.tile_m = L.tile_m;
    q.tiles_m = int((p.m + L.tile_m - 1) / L.tile_m);
    q.tiles_n = int((p.n + mmr::TC_BN - 1) / mmr::TC_BN);
    q.tiles_total = int(L.tiles);
    q.k_blocks = L.k_blocks;
    q.chunk_kb = L.chunk_kb;
    q.c = reinterpret_cast<float*>(p.c.base);
    q.c_ld = p.c.s_r;
    q.c_bs = t.c_sb;
    q.a_batched = t.a_batched;
    q.b_batched = t.b_batched;
    q.epilogue = p.epilogue;
    q.bias = reinterpret_cast<const float*>(p.bias);
    q.err = h->d_err;
    q.timeout_ns = h->wait_timeout_ns;
    q.nf = nullptr;
    q.sk_tiles = L.sk_tiles;
    if (h->mode == 1) {
      const size_t words = 2 + 2 * size_t(L.tiles);
      if (cudaMalloc(&h->d_nf, words * sizeof(unsigned int)) != cudaSuccess ||
          cudaMemset(h->d_nf, 0, words * sizeof(unsigned int)) != cudaSuccess)
        return cleanup(fail(MMR_ERR_CUDA, "allocating the non-finite bookkeeping failed"));
      q.nf = h->d_nf;
      fill_simt_params(p, &h->sp);
    }
    if (h->pair) {
      // Stream-K workspace: two partial-sum slots per pair, and an arrival
      // counter per split tile (fewer than two rounds of them) and epilogue
      // warp of each CTA.
      const size_t ws_bytes = size_t(L.npairs) * 2 * mmr::kSkSlotFloats * sizeof(float);
      h->ws_count_bytes = size_t(2 * L.npairs) * 2 * mmr::TC_EPI_WARPS * sizeof(unsigned int);
      if (cudaMalloc(&h->d_ws, ws_bytes) != cudaSuccess ||
          cudaMalloc(&h->d_ws_count, h->ws_count_bytes) != cudaSuccess ||
          cudaMemset(h->d_ws_count, 0, h->ws_count_bytes) != cudaSuccess)
        return cleanup(fail(MMR_ERR_CUDA, "allocating the stream-K workspace failed"));
      q.ws = h->d_ws;
      q.ws_count = h->d_ws_count;
    }
    const cudaError_t ce = mmr::tc_prepare(h->mode, h->pair, t.a_mn, t.b_mn, h->smem);
    if (ce == cudaErrorInvalidConfiguration)
      return cleanup(fail(MMR_ERR_CUDA, "tcgen05 kernel was compiled with too few registers for its warp split"));
    if (ce != cudaSuccess) return cleanup(fail(MMR_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(ce)));
    h->info.cluster = L.cluster_x;
    h->info.stages = L.stages;
    h->info.a_mn_major = t.a_mn;
    h->info.b_mn_major = t.b_mn;
    h->info.tile_m = L.tile_m;
    h->info.tile_n = L.tile_n;
    h->info.tile_k = L.tile_k;
    h->info.tiles = L.tiles;
    h->info.bytes = algorithmic_bytes(p, t.a_batched, t.b_batched);
  } else if (fam == MMR_FAMILY_GEMV && L.gemv_tc) {
    h->gemv_tc = true;
    h->mode = L.mode;
    mmr::GemvTcParams& g = h->gtp;
    g.m = int(p.m);
    g.n = int(p.n);
    g.k = int(p.k);
    g.kslice = L.kslice;
    g.c = reinterpret_cast<float*>(p.c.base);
    g.c_m = p.c.s_r;
    g.bias = reinterpret_cast<const float*>(p.bias);
    g.epilogue = p.epilogue;
    g.err = h->d_err;
    g.timeout_ns = h->wait_timeout_ns;
    // B by 32 x 32 atoms in the 128-byte swizzle with 32-byte atoms (MN-major
    // MMA operand); A by 32-wide K panels of its rows (K-major, 128-byte
    // swizzle); rows of A beyond M arrive as zeros. A one-row A gets any
    // legal row pitch.
    const int64_t a_pitch = p.m > 1 ? p.a.s_r : (p.k + 3) / 4 * 4;
    if (int32_t e = encode_3d(&h->tmB, p.b.base, p.n, p.k, 1, p.b.s_r, 0, 32, mmr::GT_BK, "rhs", true))
      return cleanup(e);
    if (int32_t e = encode_3d(&h->tmA_gv, p.a.base, p.k, p.m, 1, a_pitch, 0, mmr::GT_BK, mmr::GT_MN, "lhs"))
      return cleanup(e);
    g.a = reinterpret_cast<const float*>(p.a.base);
    g.a_m = a_pitch;
    g.b = reinterpret_cast<const float*>(p.b.base);
    g.b_k = p.b.s_r;
    const void* fn = h->mode ? reinterpret_cast<const void*>(mmr::mmr_gemv_tc_kernel<1>)
                             : reinterpret_cast<const void*>(mmr::mmr_gemv_tc_kernel<0>);
    cudaError_t ce = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, h->smem);
    if (ce != cudaSuccess) return cleanup(fail(MMR_ERR_CUDA, "cudaFuncSetAttribute(gemv tc): %s", cudaGetErrorString(ce)));
    h->info.bytes = algorithmic_bytes(p, true, true);
    h->info.cluster = mmr::GT_KSPLIT;
    h->info.tile_m = mmr::GT_MN;
    h->info.tile_n = mmr::GT_COLS;
    h->info.tile_k = mmr::GT_BK;
    h->info.stages = mmr::gt_stages(h->mode);
  } else if (fam == MMR_FAMILY_GEMV) {
    mmr::GemvParams& g = h->gvp;
    g.m = int(p.m);
    g.n = int(p.n);
    g.k = int(p.k);
    g.kslice = L.kslice;
    g.a = reinterpret_cast<const float*>(p.a.base);
    g.a_m = p.a.s_r;
    g.a_k = p.a.s_c;
    g.c = reinterpret_cast<float*>(p.c.base);
    g.c_m = p.c.s_r;
    g.bias = reinterpret_cast<const float*>(p.bias);
    g.epilogue = p.epilogue;
    g.err = h->d_err;
    g.timeout_ns = h->wait_timeout_ns;
    if (int32_t e = encode_3d(&h->tmB, p.b.base, p.n, p.k, 1, p.b.s_r, 0, mmr::GV_COLS, mmr::GV_ROWS, "rhs",
                              false, true))
      return cleanup(e);
    h->gv_mt = L.gv_mt;
    cudaError_t ce = prepare_gemv(h->gv_mt, h->smem);
    if (ce != cudaSuccess) return cleanup(fail(MMR_ERR_CUDA, "cudaFuncSetAttribute(gemv): %s", cudaGetErrorString(ce)));
    h->info.bytes = algorithmic_bytes(p, true, true);
    h->info.cluster = mmr::GV_KSPLIT;
  } else {
    fill_simt_params(p, &h->sp);
    h->info.bytes = algorithmic_bytes(p, true, true);
  }
  h->info.grid = int(h->grid.x * h->grid.y * h->grid.z);
  h->info.block = int(h->block.x);
  h->info.smem_bytes = h->smem;
  *out = h;
  return MMR_OK;
}

namespace {
struct SignalParams {
  unsigned long long* peer_signal[8];  // rank i's signal array (mapped here)
  unsigned long long* local;           // this rank's signal array
  int rank, nranks;
  unsigned long long epoch;
  int* err;
  unsigned long long timeout_ns;
};

// After this rank's GEMM (whose epilogue fenced its peer stores system-wide):
// publish `epoch` into every peer's slot for this rank, then wait, bounded,
// until every peer has published into this rank's array. One warp.
__global__ void mmr_replica_signal_wait_kernel(const SignalParams s) {
  const int t = threadIdx.x;
  const bool peer = t < s.nranks && t != s.rank;
  if (peer) {
    __threadfence_system();
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(s.peer_signal[t] + s.rank), "l"(s.epoch) : "memory");
  }
  __syncwarp();
  if (peer) {
    const uint64_t t0 = mmr::globaltimer_ns();
    for (;;) {
      unsigned long long v;
      asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(s.local + t) : "memory");
      if (v >= s.epoch) break;
      if (mmr::globaltimer_ns() - t0 > s.timeout_ns) {
        atomicCAS(s.err, 0, mmr::kDevTimeoutPeer);
        break;
      }
      __nanosleep(200);
    }
  }
}
}  // namespace

// One run of a host-buffer GEMM: rhs and bias in, then per row panel: lhs
// rows in (copy stream) -> the panel's GEMM (compute stream) -> its output rows
// out (copy-out stream). Copies in and out run in the two PCIe directions at
// once, under the GEMMs of other panels.
static int32_t run_host_pipeline(mmr_gemm_handle* h, cudaStream_t s) {
  using C2 = mmr_gemm_handle::Copy2D;
  auto in = [&](const C2& c, size_t r0, size_t rows) -> cudaError_t {
    if (!rows || !c.width) return cudaSuccess;
    return cudaMemcpy2DAsync(c.dev + r0 * c.dev_pitch, c.dev_pitch, c.host + r0 * c.host_pitch, c.host_pitch, c.width,
                             rows, cudaMemcpyHostToDevice, h->s_in);
  };
  MMR_CUDA_TRY(cudaEventRecord(h->ev_start, s));
  for (cudaStream_t st : {h->s_in, h->s_comp, h->s_out}) {
    MMR_CUDA_TRY(cudaStreamWaitEvent(st, h->ev_start, 0));
    // The staging buffers are the handle's own: a run on another caller
    // stream must not overwrite them while the previous run still uses them.
    if (h->ran) MMR_CUDA_TRY(cudaStreamWaitEvent(st, h->done, 0));
  }
  MMR_CUDA_TRY(in(h->h_rhs, 0, h->h_rhs.rows));
  MMR_CUDA_TRY(in(h->h_bias, 0, h->h_bias.rows));
  MMR_CUDA_TRY(cudaEventRecord(h->ev_rhs, h->s_in));
  const size_t np = h->panel.size();
  for (size_t i = 0; i < np; ++i) {
    MMR_CUDA_TRY(in(h->h_lhs, size_t(h->panel_row[i]), size_t(h->panel_row[i + 1] - h->panel_row[i])));
    MMR_CUDA_TRY(cudaEventRecord(h->ev_lhs[i], h->s_in));
  }
  MMR_CUDA_TRY(cudaStreamWaitEvent(h->s_comp, h->ev_rhs, 0));
  for (size_t i = 0; i < np; ++i) {
    MMR_CUDA_TRY(cudaStreamWaitEvent(h->s_comp, h->ev_lhs[i], 0));
    if (int32_t rc = mmr_gemm_run_on(h->panel[i], h->s_comp)) return rc;
    MMR_CUDA_TRY(cudaEventRecord(h->ev_gemm[i], h->s_comp));
  }
  const C2& c = h->h_out;
  for (size_t i = 0; i < np; ++i) {
    const size_t r0 = size_t(h->panel_row[i]), rows = size_t(h->panel_row[i + 1] - h->panel_row[i]);
    MMR_CUDA_TRY(cudaStreamWaitEvent(h->s_out, h->ev_gemm[i], 0));
    if (rows && c.width)
      MMR_CUDA_TRY(cudaMemcpy2DAsync(c.host + r0 * c.host_pitch, c.host_pitch, c.dev + r0 * c.dev_pitch, c.dev_pitch,
                                     c.width, rows, cudaMemcpyDeviceToHost, h->s_out));
  }
  MMR_CUDA_TRY(cudaEventRecord(h->done, h->s_out));
  MMR_CUDA_TRY(cudaStreamWaitEvent(s, h->done, 0));  // later work on the caller's stream follows
  h->ran = true;
  return MMR_OK;
}

int32_t mmr_gemm_run_on(mmr_gemm_handle* h, void* stream) {
  if (!h) return fail(MMR_ERR_INVALID_ARGUMENT, "null handle");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  DeviceGuard guard(h->device);
  if (!guard.ok) return fail(MMR_ERR_CUDA, "cudaSetDevice(%d) failed", h->device);
  if (h->host) return run_host_pipeline(h, s);
  cudaError_t e = cudaSuccess;
  if (!h->plan.empty) {
    switch (h->family) {
      case MMR_FAMILY_TCGEN05:
        e = mmr::tc_launch(h->mode, h->pair, h->a_mn, h->b_mn, mmr::TcShape{h->grid, h->block, h->smem}, s, h->tmA,
                           h->tmB, h->tmC, h->tcp);
        if (e == cudaSuccess && h->mode == 1)
          e = mmr::launch_kernel(mmr::mmr_tc_nonfinite_fixup_kernel, dim3(h->sms), dim3(256), 0, s, dim3(1, 1, 1), h->sp, h->tcp);
        break;
      case MMR_FAMILY_GEMV:
        e = h->gemv_tc ? launch_gemv_tc(h, s) : launch_gemv(h, s);
        break;
      case MMR_FAMILY_SIMT:
        e = mmr::launch_kernel(mmr::mmr_simt_gemm_exact_kernel, h->grid, h->block, 0, s, dim3(1, 1, 1), h->sp);
        break;
      default: return fail(MMR_ERR_UNSUPPORTED_FAMILY, "no kernel bound");
    }
  }
  if (e == cudaSuccess && h->sharded) {
    SignalParams sp{};
    for (int i = 0; i < 8; ++i) sp.peer_signal[i] = h->peer_signal[i];
    sp.local = h->signal;
    sp.rank = h->rank;
    sp.nranks = h->nranks;
    sp.epoch = ++h->epoch;
    sp.err = h->d_err;
    sp.timeout_ns = h->wait_timeout_ns;
    mmr_replica_signal_wait_kernel<<<1, 32, 0, s>>>(sp);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) return fail(MMR_ERR_CUDA, "kernel launch: %s", cudaGetErrorString(e));
  MMR_CUDA_TRY(cudaEventRecord(h->done, s));
  h->ran = true;
  return MMR_OK;
}

int32_t mmr_gemm_run(mmr_gemm_handle* h) {
  if (!h) return fail(MMR_ERR_INVALID_ARGUMENT, "null handle");
  return mmr_gemm_run_on(h, h->stream);
}

static int32_t poll_event(cudaEvent_t ev, uint64_t timeout_ns) {
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    cudaError_t e = cudaEventQuery(ev);
    if (e == cudaSuccess) return MMR_OK;
    if (e != cudaErrorNotReady) return fail(MMR_ERR_CUDA, "cudaEventQuery: %s", cudaGetErrorString(e));
    const uint64_t el = uint64_t(std::chrono::duration_cast<std::chrono::nanoseconds>(
                                     std::chrono::steady_clock::now() - t0)
                                     .count());
    if (el > timeout_ns) return fail(MMR_ERR_TIMEOUT, "work did not complete within %llu ns", (unsigned long long)timeout_ns);
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

int32_t mmr_gemm_quiesce(mmr_gemm_handle* h, uint64_t timeout_ns) {
  if (!h) return fail(MMR_ERR_INVALID_ARGUMENT, "null handle");
  if (!h->ran) return MMR_OK;
  DeviceGuard guard(h->device);
  int32_t rc = poll_event(h->done, timeout_ns);
  if (rc) return rc;
  if (h->host) {  // every copy has landed; now each panel GEMM's error word
    for (mmr_gemm_handle* sub : h->panel)
      if ((rc = mmr_gemm_quiesce(sub, timeout_ns))) return rc;
    return MMR_OK;
  }
  // Read the device error word (asynchronously, then poll: never block forever).
  MMR_CUDA_TRY(cudaMemcpyAsync(h->h_err, h->d_err, sizeof(int), cudaMemcpyDeviceToHost, h->stream));
  MMR_CUDA_TRY(cudaEventRecord(h->err_ev, h->stream));
  if ((rc = poll_event(h->err_ev, timeout_ns))) return rc;
  const int code = *h->h_err;
  if (code != 0) {
    *h->h_err = 0;
    cudaMemsetAsync(h->d_err, 0, sizeof(int), h->stream);
    // A run that gave up may leave stream-K arrival counts that nothing reset.
    if (h->d_ws_count) cudaMemsetAsync(h->d_ws_count, 0, h->ws_count_bytes, h->stream);
    return fail(code == mmr::kDevTimeoutDrain || code <= mmr::kDevTimeoutXform || code == mmr::kDevTimeoutPeer ||
                        code == mmr::kDevTimeoutReduce
                    ? MMR_ERR_TIMEOUT
                    : MMR_ERR_DEVICE_FAULT_FLAG,
                "kernel reported device error word %d (a bounded wait expired)", code);
  }
  return MMR_OK;
}

int32_t mmr_gemm_destroy(mmr_gemm_handle* h) {
  if (!h) return MMR_OK;
  int32_t rc = MMR_OK;
  {
    DeviceGuard guard(h->device);
    if (h->ran && h->done) rc = poll_event(h->done, 10000000000ull);
    if (h->host) {
      for (mmr_gemm_handle* sub : h->panel) {
        const int32_t r = mmr_gemm_destroy(sub);
        if (rc == MMR_OK) rc = r;
      }
      for (void* b : h->dbuf)
        if (b) cudaFree(b);
      for (cudaStream_t st : {h->s_in, h->s_comp, h->s_out})
        if (st) cudaStreamDestroy(st);
      for (cudaEvent_t ev : h->ev_lhs) cudaEventDestroy(ev);
      for (cudaEvent_t ev : h->ev_gemm) cudaEventDestroy(ev);
      if (h->ev_start) cudaEventDestroy(h->ev_start);
      if (h->ev_rhs) cudaEventDestroy(h->ev_rhs);
    }
    if (h->done) cudaEventDestroy(h->done);
    if (h->err_ev) cudaEventDestroy(h->err_ev);
    if (h->d_err) cudaFree(h->d_err);
    if (h->d_nf) cudaFree(h->d_nf);
    if (h->d_ws) cudaFree(h->d_ws);
    if (h->d_ws_count) cudaFree(h->d_ws_count);
    if (h->d_peer_tm) cudaFree(h->d_peer_tm);
    if (h->h_err) cudaFreeHost(h->h_err);
  }
  delete h;
  return rc;
}

namespace {
__global__ void mmr_bounded_wait_probe_kernel(int* err, unsigned long long limit_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mmr::mbar_init(&bar, 1);
    mmr::fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // Nobody arrives: the wait must expire, record the code and return.
    const mmr::WaitCtl ctl{err, limit_ns};
    mmr::mbar_wait(&bar, 0u, ctl, mmr::kDevTimeoutProbe);
  }
  __syncthreads();
}
}  // namespace

int32_t mmr_selftest_bounded_wait(int32_t device_ordinal, uint64_t limit_ns) {
  DeviceGuard guard(device_ordinal);
  if (!guard.ok) return fail(MMR_ERR_CUDA, "cudaSetDevice(%d) failed", device_ordinal);
  if (limit_ns > 5000000000ull) return fail(MMR_ERR_INVALID_ARGUMENT, "limit above 5 s");
  int* d_err = nullptr;
  MMR_CUDA_TRY(cudaMalloc(&d_err, sizeof(int)));
  int h = -1;
  cudaError_t e = cudaMemset(d_err, 0, sizeof(int));
  if (e == cudaSuccess) {
    mmr_bounded_wait_probe_kernel<<<1, 32>>>(d_err, limit_ns);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpy(&h, d_err, sizeof(int), cudaMemcpyDeviceToHost);
  cudaFree(d_err);
  if (e != cudaSuccess) return fail(MMR_ERR_CUDA, "bounded-wait probe: %s", cudaGetErrorString(e));
  if (h == mmr::kDevTimeoutProbe) return fail(MMR_ERR_TIMEOUT, "probe wait expired as designed");
  return fail(MMR_ERR_DEVICE_FAULT_FLAG, "probe returned error word %d", h);
}

int32_t mmr_shard_columns(int64_t n, int32_t nranks, int32_t rank, int32_t align, int64_t* col0, int64_t* col1) {
  if (!col0 || !col1 || nranks < 1 || rank < 0 || rank >= nranks || n < 0 || align < 1)
    return fail(MMR_ERR_INVALID_ARGUMENT, "bad shard request");
  // Whole `align`-column units are dealt out as evenly as possible; the first
  // (units % nranks) ranks take one extra unit. The last rank absorbs the tail.
  const int64_t units = (n + align - 1) / align;
  const int64_t base = units / nranks, extra = units % nranks;
  const int64_t u0 = rank * base + std::min<int64_t>(rank, extra);
  const int64_t u1 = u0 + base + (rank < extra ? 1 : 0);
  *col0 = std::min<int64_t>(n, u0 * align);
  *col1 = std::min<int64_t>(n, u1 * align);
  return MMR_OK;
}

int32_t mmr_gemm_run_noalloc(const mmr_matmul_desc* desc, int32_t* status_out) {
  Plan p;
  int32_t rc = build_plan(desc, &p);
  if (rc) return rc;
  if (p.math != MMR_MATH_STRICT_FP32)
    return fail(MMR_ERR_UNSUPPORTED_MATH, "the allocation-free entry point runs StrictFp32 (3xTF32) only");
  if (p.family != MMR_FAMILY_AUTO && p.family != MMR_FAMILY_TCGEN05)
    return fail(MMR_ERR_UNSUPPORTED_FAMILY, "the allocation-free entry point runs the tcgen05 family only");
  const TmaLayout t = tma_admission(p);
  if (p.empty) {
    if (status_out) *status_out = 0;
    return MMR_OK;
  }
  if (!t.ok) return fail(MMR_ERR_UNSUPPORTED_FAMILY, "tcgen05 family not admissible: %s", t.why);
  const int64_t batch = p.batch;
  const int64_t tiles_m = (p.m + mmr::TC_BM - 1) / mmr::TC_BM;
  const int64_t tiles_n = (p.n + mmr::TC_BN - 1) / mmr::TC_BN;
  const int64_t tiles = tiles_m * tiles_n * batch;
  if (tiles > MMR_NOALLOC_MAX_TILES)
    return fail(MMR_ERR_INVALID_SHAPE,
                "output needs %lld tiles of 128x256; the allocation-free entry point's static scratch "
                "(%d bytes) holds at most %d",
                (long long)tiles, MMR_NOALLOC_SCRATCH_BYTES, MMR_NOALLOC_MAX_TILES);

  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0)
    return fail(MMR_ERR_UNSUPPORTED_DEVICE, "no CUDA device is visible");
  if (p.device < 0 || p.device >= ndev)
    return fail(MMR_ERR_UNSUPPORTED_DEVICE, "device ordinal %d outside 0..%d", p.device, ndev - 1);
  DeviceGuard guard(p.device);
  if (!guard.ok) return fail(MMR_ERR_CUDA, "cudaSetDevice(%d) failed", p.device);
  int major = 0;
  MMR_CUDA_TRY(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, p.device));
  if (major != 10) return fail(MMR_ERR_UNSUPPORTED_DEVICE, "device %d is not an sm_100 device", p.device);
  const uint64_t addrs[4] = {desc->lhs.address, desc->rhs.address, desc->out.address,
                             mmr::epi_has_bias(desc->epilogue) ? desc->bias.address : 0};
  for (uint64_t a : addrs) {
    if (!a) continue;
    cudaPointerAttributes pa;
    if (cudaPointerGetAttributes(&pa, reinterpret_cast<void*>(a)) != cudaSuccess) {
      cudaGetLastError();
      return fail(MMR_ERR_UNSUPPORTED_DEVICE, "address 0x%llx is not known to CUDA", (unsigned long long)a);
    }
    if ((pa.type != cudaMemoryTypeDevice && pa.type != cudaMemoryTypeManaged) || pa.device != p.device)
      return fail(MMR_ERR_UNSUPPORTED_DEVICE, "address 0x%llx is not device memory of device %d",
                  (unsigned long long)a, p.device);
  }
  NoAllocDevice* dev = nullptr;
  if ((rc = noalloc_setup(p.device, &dev))) return rc;

  // Everything below lives on the stack: descriptors, parameters, launch shape.
  mmr_gemm_handle h;
  h.plan = p;
  h.device = p.device;
  h.mode = 1;
  h.a_mn = t.a_mn;
  h.b_mn = t.b_mn;
  constexpr uint32_t bk = mmr::TcConfig<1>::kBK;
  if (int32_t e = encode_tc_maps(&h, p, t, batch, bk)) return e;

  mmr::TcParams& q = h.tcp;
  q.m = int(p.m);
  q.n = int(p.n);
  q.k = int(p.k);
  q.batch = int(batch);
  q.tile_m = mmr::TC_BM;
  q.tiles_m = int(tiles_m);
  q.tiles_n = int(tiles_n);
  q.tiles_total = int(tiles);
  q.k_blocks = int((p.k + bk - 1) / bk);
  q.chunk_kb = int(256 / bk);
  q.a_batched = t.a_batched;
  q.b_batched = t.b_batched;
  q.epilogue = p.epilogue;
  q.bias = reinterpret_cast<const float*>(p.bias);
  q.c = reinterpret_cast<float*>(p.c.base);
  q.c_ld = p.c.s_r;
  q.c_bs = t.c_sb;
  q.err = reinterpret_cast<int*>(dev->scratch);
  q.timeout_ns = h.wait_timeout_ns;
  q.nf = dev->scratch + 4;
  fill_simt_params(p, &h.sp);
  h.smem = mmr::TcConfig<1>::kSmemBytes;
  h.grid = dim3(unsigned(std::min<int64_t>(tiles, dev->sms)));
  h.block = dim3(mmr::TcConfig<1>::kThreads);

  cudaStream_t s = reinterpret_cast<cudaStream_t>(desc->stream);
  // Clear what the kernels expect at zero: the error word, the flagged-tile
  // count and done counter, and this problem's per-tile flags.
  MMR_CUDA_TRY(cudaMemsetAsync(dev->scratch, 0, (6 + size_t(tiles)) * sizeof(unsigned int), s));
  cudaError_t ce = mmr::tc_launch(1, false, t.a_mn, t.b_mn, mmr::TcShape{h.grid, h.block, h.smem}, s, h.tmA, h.tmB,
                                  h.tmC, h.tcp);
  if (ce == cudaSuccess)
    ce = mmr::launch_kernel(mmr::mmr_tc_nonfinite_fixup_kernel, dim3(dev->sms), dim3(256), 0, s, dim3(1, 1, 1), h.sp, h.tcp);
  if (ce != cudaSuccess) return fail(MMR_ERR_CUDA, "kernel launch: %s", cudaGetErrorString(ce));
  if (status_out)
    MMR_CUDA_TRY(cudaMemcpyAsync(status_out, dev->scratch, sizeof(int32_t), cudaMemcpyDeviceToHost, s));
  return MMR_OK;
}

int32_t mmr_ipc_export(uint64_t address, mmr_ipc_handle* out) {
  if (!address || !out) return fail(MMR_ERR_INVALID_ARGUMENT, "null address or handle");
  cudaPointerAttributes pa;
  if (cudaPointerGetAttributes(&pa, reinterpret_cast<void*>(address)) != cudaSuccess ||
      pa.type != cudaMemoryTypeDevice) {
    cudaGetLastError();
    return fail(MMR_ERR_UNSUPPORTED_DEVICE, "address 0x%llx is not device memory", (unsigned long long)address);
  }
  DeviceGuard guard(pa.device);
  // Driver entry point resolved through the runtime, so the library does not
  // link libcuda directly (it must load on hosts without a driver).
  typedef CUresult (*AddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);
  static AddressRangeFn range_fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &ptr, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      range_fn = reinterpret_cast<AddressRangeFn>(ptr);
  });
  if (!range_fn) return fail(MMR_ERR_CUDA, "cuMemGetAddressRange is unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range_fn(&base, &size, static_cast<CUdeviceptr>(address)) != CUDA_SUCCESS)
    return fail(MMR_ERR_CUDA, "cuMemGetAddressRange failed for 0x%llx", (unsigned long long)address);
  cudaIpcMemHandle_t ih;
  if (cudaError_t e = cudaIpcGetMemHandle(&ih, reinterpret_cast<void*>(base)))
    return fail(MMR_ERR_PEER_ACCESS, "cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
  static_assert(sizeof(ih) == sizeof(out->bytes), "IPC handle size");
  memcpy(out->bytes, &ih, sizeof ih);
  out->offset = address - static_cast<uint64_t>(base);
  return MMR_OK;
}

int32_t mmr_ipc_import(const mmr_ipc_handle* h, int32_t device_ordinal, uint64_t* address_out) {
  if (!h || !address_out) return fail(MMR_ERR_INVALID_ARGUMENT, "null handle or output");
  DeviceGuard guard(device_ordinal);
  if (!guard.ok) return fail(MMR_ERR_CUDA, "cudaSetDevice(%d) failed", device_ordinal);
  cudaIpcMemHandle_t ih;
  memcpy(&ih, h->bytes, sizeof ih);
  void* p = nullptr;
  if (cudaError_t e = cudaIpcOpenMemHandle(&p, ih, cudaIpcMemLazyEnablePeerAccess))
    return fail(MMR_ERR_PEER_ACCESS, "cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
  *address_out = reinterpret_cast<uint64_t>(p) + h->offset;
  return MMR_OK;
}

int32_t mmr_ipc_release(uint64_t address, const mmr_ipc_handle* h) {
  if (!address || !h) return fail(MMR_ERR_INVALID_ARGUMENT, "null address or handle");
  if (cudaError_t e = cudaIpcCloseMemHandle(reinterpret_cast<void*>(address - h->offset)))
    return fail(MMR_ERR_PEER_ACCESS, "cudaIpcCloseMemHandle: %s", cudaGetErrorString(e));
  return MMR_OK;
}

int32_t mmr_shard_local_desc(const mmr_matmul_desc* whole_desc, int32_t rank, int32_t nranks,
                             mmr_matmul_desc* local_out, int64_t* col0, int64_t* col1, uint64_t* out_offset_bytes) {
  if (!whole_desc || !local_out || !col0 || !col1 || !out_offset_bytes)
    return fail(MMR_ERR_INVALID_ARGUMENT, "null descriptor or output");
  if (nranks < 1 || nranks > 8 || rank < 0 || rank >= nranks)
    return fail(MMR_ERR_INVALID_ARGUMENT, "rank %d of %d outside 1..8 ranks", rank, nranks);
  // Validate the whole node first, then narrow to this rank's column block.
  Plan whole;
  int32_t rc = build_plan(whole_desc, &whole);
  if (rc) return rc;
  const mmr_view& O = whole_desc->out;
  if (O.rank < 2 || whole_desc->rhs.rank < 2)
    return fail(MMR_ERR_INVALID_SHAPE, "column sharding needs matrix operands (rank >= 2)");
  int64_t c0 = 0, c1 = 0;
  if ((rc = mmr_shard_columns(whole.n, nranks, rank, mmr::TC_BN, &c0, &c1))) return rc;
  mmr_matmul_desc local = *whole_desc;
  // out[..., c0:c1]
  local.out.base_offset_bytes += uint64_t(c0) * uint64_t(O.strides[O.rank - 1]) * 4u;
  local.out.dims[O.rank - 1] = c1 - c0;
  // rhs[..., :, c0:c1] (columns are the rhs's last axis, or its second to last when transposed)
  const mmr_view& R = whole_desc->rhs;
  const int raxis = whole_desc->transpose_rhs ? R.rank - 2 : R.rank - 1;
  local.rhs.base_offset_bytes += uint64_t(c0) * uint64_t(R.strides[raxis]) * 4u;
  local.rhs.dims[raxis] = c1 - c0;
  if (mmr::epi_has_bias(local.epilogue)) {
    local.bias.base_offset_bytes += uint64_t(c0) * uint64_t(local.bias.strides[0]) * 4u;
    local.bias.dims[0] = c1 - c0;
  }
  *local_out = local;
  *col0 = c0;
  *col1 = c1;
  *out_offset_bytes = local.out.base_offset_bytes;
  return MMR_OK;
}

int32_t mmr_sharded_gemm_bind(const mmr_sharded_desc* d, mmr_gemm_handle** out) {
  if (!d || !out) return fail(MMR_ERR_INVALID_ARGUMENT, "null descriptor or output handle");
  *out = nullptr;
  if (d->nranks < 1 || d->nranks > 8 || d->rank < 0 || d->rank >= d->nranks)
    return fail(MMR_ERR_INVALID_ARGUMENT, "rank %d of %d outside 1..8 ranks", d->rank, d->nranks);
  if (!d->signal) return fail(MMR_ERR_INVALID_ARGUMENT, "null signal array");
  for (int i = 0; i < d->nranks; ++i)
    if (i != d->rank && (!d->peer_out[i] || !d->peer_signal[i]))
      return fail(MMR_ERR_INVALID_ARGUMENT, "rank %d's replica or signal array is not mapped", i);
  mmr_matmul_desc local;
  int64_t c0 = 0, c1 = 0;
  uint64_t out_off = 0;
  int32_t rc = mmr_shard_local_desc(&d->local, d->rank, d->nranks, &local, &c0, &c1, &out_off);
  if (rc) return rc;
  const mmr_view& O = d->local.out;
  local.family = MMR_FAMILY_TCGEN05;
  mmr_gemm_handle* h = nullptr;
  if (c1 > c0) {
    if ((rc = mmr_gemm_bind(&local, &h))) return rc;
  } else {
    // An empty column block still takes part in the completion handshake.
    local.family = MMR_FAMILY_AUTO;
    if ((rc = mmr_gemm_bind(&local, &h))) return rc;
  }
  h->sharded = true;
  h->rank = d->rank;
  h->nranks = d->nranks;
  h->signal = reinterpret_cast<unsigned long long*>(d->signal);
  const uint64_t view_off = local.out.address + local.out.base_offset_bytes - O.address;
  int q = 0;
  for (int i = 0; i < d->nranks; ++i) {
    h->peer_signal[i] = reinterpret_cast<unsigned long long*>(d->peer_signal[i]);
    if (i == d->rank) continue;
    float* pc = reinterpret_cast<float*>(d->peer_out[i] + view_off);
    h->tcp.peer_c[q] = pc;
    h->sp.peer_c[q] = pc;
    ++q;
  }
  h->tcp.npeers = q;
  h->sp.npeers = q;
  // One tensor map per peer replica (the local output's geometry at the
  // peer's address), in device memory: the epilogue stores each finished box
  // to every replica with TMA stores.
  if (h->family == MMR_FAMILY_TCGEN05 && q > 0 && !h->plan.empty) {
    CUtensorMap maps[mmr::kMaxPeers];
    for (int j = 0; j < q; ++j) {
      if ((rc = encode_3d(&maps[j], reinterpret_cast<uint64_t>(h->tcp.peer_c[j]), uint64_t(h->tcp.n),
                          uint64_t(h->tcp.m), uint64_t(h->tcp.batch), h->tcp.c_ld, h->tcp.c_bs, 32, 32,
                          "peer replica"))) {
        mmr_gemm_destroy(h);
        return rc;
      }
    }
    DeviceGuard guard(h->device);
    if (cudaMalloc(&h->d_peer_tm, sizeof(CUtensorMap) * size_t(q)) != cudaSuccess ||
        cudaMemcpy(h->d_peer_tm, maps, sizeof(CUtensorMap) * size_t(q), cudaMemcpyHostToDevice) != cudaSuccess) {
      mmr_gemm_destroy(h);
      return fail(MMR_ERR_CUDA, "storing the peer tensor maps failed");
    }
    h->tcp.peer_tm = h->d_peer_tm;
  }
  // With replicas to feed and under two rounds of tiles, every tile is split
  // stream-K style: the pairs' ranges then end at staggered points inside
  // tiles, so tiles finish (and their stores leave over NVLink) spread across
  // the run instead of a round's worth at once, which would stall every
  // epilogue behind the links together. (With more tiles than that, the
  // round-robin order keeps its L2 reuse.) The counters cover the split: the
  // bind sized them for up to two rounds.
  if (h->pair && q > 0 && h->tcp.tiles_total < int(h->grid.x)) {
    h->tcp.sk_tiles = h->tcp.tiles_total;
    h->launch.sk_tiles = h->tcp.sk_tiles;
  }
  *out = h;
  return MMR_OK;
}

int32_t mmr_gemm_bind_host(const mmr_matmul_desc* d, int32_t panels, mmr_gemm_handle** out) {
  if (!d || !out) return fail(MMR_ERR_INVALID_ARGUMENT, "null descriptor or output handle");
  *out = nullptr;
  if (d->lhs.rank != 2 || d->rhs.rank != 2 || d->out.rank != 2)
    return fail(MMR_ERR_UNSUPPORTED_LAYOUT, "host-buffer GEMM takes rank-2 lhs, rhs and out");
  if (d->transpose_lhs)
    return fail(MMR_ERR_UNSUPPORTED_LAYOUT, "host-buffer GEMM streams lhs by rows: transpose_lhs is not supported");
  if (d->epilogue < MMR_EPI_NONE || d->epilogue > MMR_EPI_BIAS_SILU)
    return fail(MMR_ERR_INVALID_ARGUMENT, "unknown epilogue %d", d->epilogue);
  if (panels < 0 || panels > 64) return fail(MMR_ERR_INVALID_ARGUMENT, "panels %d outside 0..64", panels);
  const bool has_bias = mmr::epi_has_bias(d->epilogue);
  if (has_bias && d->bias.rank != 1) return fail(MMR_ERR_INVALID_SHAPE, "bias must be rank 1");
  // Host views: row-major, unit column stride, inside their buffers, not device memory.
  auto check_host = [&](const mmr_view& v, const char* name) -> int32_t {
    const int64_t rows = v.rank == 2 ? v.dims[0] : 1, cols = v.dims[v.rank - 1];
    const int64_t pitch = v.rank == 2 ? v.strides[0] : cols;
    if (rows < 0 || cols < 0 || v.strides[v.rank - 1] != 1 || (v.rank == 2 && rows > 1 && pitch < cols))
      return fail(MMR_ERR_UNSUPPORTED_LAYOUT, "%s: host buffer must be row-major with unit column stride", name);
    if (v.base_offset_bytes % 4) return fail(MMR_ERR_UNSUPPORTED_LAYOUT, "%s: base offset not f32-aligned", name);
    const uint64_t need = rows && cols ? uint64_t((rows - 1) * pitch + cols) * 4u : 0u;
    if (v.base_offset_bytes + need > v.bytes) return fail(MMR_ERR_INVALID_SHAPE, "%s: view exceeds its host buffer", name);
    if (need && !v.address) return fail(MMR_ERR_INVALID_ARGUMENT, "%s: null host address", name);
    cudaPointerAttributes a{};
    if (need && cudaPointerGetAttributes(&a, reinterpret_cast<void*>(v.address + v.base_offset_bytes)) == cudaSuccess &&
        a.type == cudaMemoryTypeDevice)
      return fail(MMR_ERR_INVALID_ARGUMENT, "%s: device memory given to the host-buffer entry (use mmr_gemm_bind)", name);
    cudaGetLastError();
    return MMR_OK;
  };
  int32_t rc;
  if ((rc = check_host(d->lhs, "lhs")) || (rc = check_host(d->rhs, "rhs")) || (rc = check_host(d->out, "out")) ||
      (has_bias && (rc = check_host(d->bias, "bias"))))
    return rc;
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) return fail(MMR_ERR_UNSUPPORTED_DEVICE, "no CUDA device is visible");
  if (d->device_ordinal < 0 || d->device_ordinal >= ndev)
    return fail(MMR_ERR_UNSUPPORTED_DEVICE, "device ordinal %d outside 0..%d", d->device_ordinal, ndev - 1);
  DeviceGuard guard(d->device_ordinal);
  if (!guard.ok) return fail(MMR_ERR_CUDA, "cudaSetDevice(%d) failed", d->device_ordinal);

  mmr_gemm_handle* h = new mmr_gemm_handle();
  h->host = true;
  h->device = d->device_ordinal;
  h->stream = reinterpret_cast<cudaStream_t>(d->stream);
  auto cleanup = [&](int32_t code) {
    const std::string msg = mmr_last_error();
    mmr_gemm_destroy(h);
    return fail(code, "%s", msg.c_str());
  };
  // Device copies with 16-byte rows (whatever the host pitch).
  mmr_matmul_desc dd = *d;
  auto stage = [&](const mmr_view& v, mmr_gemm_handle::Copy2D& c, mmr_view& dv, int slot) -> int32_t {
    const int64_t rows = v.rank == 2 ? v.dims[0] : 1, cols = v.dims[v.rank - 1];
    const int64_t pitch = v.rank == 2 ? v.strides[0] : cols;
    const int64_t dpitch = std::max<int64_t>((cols + 3) / 4 * 4, 4);
    const size_t bytes = size_t(std::max<int64_t>(rows, 1)) * size_t(dpitch) * 4u;
    if (cudaMalloc(&h->dbuf[slot], bytes) != cudaSuccess)
      return fail(MMR_ERR_CUDA, "cudaMalloc(%zu) for a host-buffer operand failed", bytes);
    c.host = reinterpret_cast<char*>(v.address + v.base_offset_bytes);
    c.host_pitch = size_t(pitch) * 4u;
    c.dev = static_cast<char*>(h->dbuf[slot]);
    c.dev_pitch = size_t(dpitch) * 4u;
    c.width = size_t(cols) * 4u;
    c.rows = size_t(rows);
    dv = v;
    dv.address = reinterpret_cast<uint64_t>(h->dbuf[slot]);
    dv.base_offset_bytes = 0;
    dv.bytes = bytes;
    dv.device_ordinal = d->device_ordinal;
    if (v.rank == 2) dv.strides[0] = dpitch;
    dv.allocation_id = dv.address;
    return MMR_OK;
  };
  if ((rc = stage(d->lhs, h->h_lhs, dd.lhs, 0)) || (rc = stage(d->rhs, h->h_rhs, dd.rhs, 1)) ||
      (rc = stage(d->out, h->h_out, dd.out, 2)) || (has_bias && (rc = stage(d->bias, h->h_bias, dd.bias, 3))))
    return cleanup(rc);
  // The whole node, validated once (shapes, math contract, family).
  if ((rc = mmr_gemm_validate(&dd, &h->info))) return cleanup(rc);
  h->family = h->info.family;
  // Row panels in whole 256-row units, dealt as evenly as possible. By
  // default one panel per two units (512 rows), at most sixteen: the last
  // panel's GEMM and copy-out are what the copies in cannot hide (8192^3:
  // 8 / 12 / 16 panels gave 11.6 / 11.2 / 11.0 ms per run).
  const int64_t m = d->out.dims[0];
  const int64_t units = (m + 255) / 256;
  const int64_t want = panels ? panels : std::min<int64_t>(16, std::max<int64_t>(1, units / 2));
  const int64_t np = std::max<int64_t>(1, std::min<int64_t>(want, std::max<int64_t>(units, 1)));
  for (int64_t i = 0; i <= np; ++i) {
    const int64_t u = i * (units / np) + std::min(i, units % np);
    h->panel_row.push_back(std::min(m, u * 256));
  }
  for (int64_t i = 0; i < np; ++i) {
    const int64_t r0 = h->panel_row[i], r1 = h->panel_row[i + 1];
    mmr_matmul_desc pd = dd;
    pd.lhs.dims[0] = r1 - r0;
    pd.lhs.base_offset_bytes = uint64_t(r0) * uint64_t(dd.lhs.strides[0]) * 4u;
    pd.out.dims[0] = r1 - r0;
    pd.out.base_offset_bytes = uint64_t(r0) * uint64_t(dd.out.strides[0]) * 4u;
    pd.stream = nullptr;
    mmr_gemm_handle* sub = nullptr;
    if ((rc = mmr_gemm_bind(&pd, &sub))) return cleanup(rc);
    h->panel.push_back(sub);
  }
  for (cudaStream_t* st : {&h->s_in, &h->s_comp, &h->s_out})
    if (cudaStreamCreateWithFlags(st, cudaStreamNonBlocking) != cudaSuccess)
      return cleanup(fail(MMR_ERR_CUDA, "cudaStreamCreate failed"));
  auto make_event = [](cudaEvent_t* ev) { return cudaEventCreateWithFlags(ev, cudaEventDisableTiming) == cudaSuccess; };
  bool ok = make_event(&h->ev_start) && make_event(&h->ev_rhs) && make_event(&h->done);
  h->ev_lhs.assign(size_t(np), nullptr);
  h->ev_gemm.assign(size_t(np), nullptr);
  for (int64_t i = 0; ok && i < np; ++i) ok = make_event(&h->ev_lhs[i]) && make_event(&h->ev_gemm[i]);
  if (!ok) return cleanup(fail(MMR_ERR_CUDA, "cudaEventCreate failed"));
  *out = h;
  return MMR_OK;
}

int32_t mmr_gemm_plan_launch(const mmr_matmul_desc* desc, int32_t sm_count, mmr_launch_record* out) {
  if (!out) return fail(MMR_ERR_INVALID_ARGUMENT, "null launch record");
  if (sm_count < 2 || sm_count > 1024) return fail(MMR_ERR_INVALID_ARGUMENT, "SM count %d outside 2..1024", sm_count);
  Plan p;
  int32_t rc = build_plan(desc, &p);
  if (rc) return rc;
  const TmaLayout t = tma_admission(p);
  int32_t fam = MMR_FAMILY_AUTO;
  if ((rc = choose_family(p, t, &fam))) return rc;
  Launch L;
  if ((rc = derive_launch(p, t, fam, sm_count, &L))) return rc;
  to_record(L, p.math, out);
  return MMR_OK;
}

int32_t mmr_gemm_launch_record(const mmr_gemm_handle* h, mmr_launch_record* out) {
  if (!h || !out) return fail(MMR_ERR_INVALID_ARGUMENT, "null handle or launch record");
  if (h->host) return fail(MMR_ERR_INVALID_ARGUMENT, "a host-buffer handle runs one bound GEMM per row panel");
  to_record(h->launch, h->plan.math, out);
  return MMR_OK;
}

int32_t mmr_check_launch_record(const mmr_launch_record* rec) {
  if (!rec) return fail(MMR_ERR_INVALID_ARGUMENT, "null launch record");
  return check_record_rules(*rec);
}

int32_t mmr_gemm_bind_frozen(const mmr_matmul_desc* desc, const mmr_launch_record* frozen, mmr_gemm_handle** out) {
  if (!out || !frozen) return fail(MMR_ERR_INVALID_ARGUMENT, "null launch record or output handle");
  *out = nullptr;
  int32_t rc = check_record_rules(*frozen);
  if (rc) return rc;
  mmr_gemm_handle* h = nullptr;
  if ((rc = mmr_gemm_bind(desc, &h))) return rc;
  mmr_launch_record mine;
  to_record(h->launch, h->plan.math, &mine);
  struct Field {
    const char* name;
    const int32_t *a, *b;
    int n;
  };
  const Field fields[] = {
      {"family", &frozen->family, &mine.family, 1},
      {"math_mode", &frozen->math_mode, &mine.math_mode, 1},
      {"grid", frozen->grid, mine.grid, 3},
      {"block", frozen->block, mine.block, 3},
      {"cluster", frozen->cluster, mine.cluster, 3},
      {"dynamic_shared_bytes", &frozen->dynamic_shared_bytes, &mine.dynamic_shared_bytes, 1},
      {"tmem_columns_per_cta", &frozen->tmem_columns_per_cta, &mine.tmem_columns_per_cta, 1},
      {"tmem_accumulator_stages", &frozen->tmem_accumulator_stages, &mine.tmem_accumulator_stages, 1},
      {"tile_m", &frozen->tile_m, &mine.tile_m, 1},
      {"tile_n", &frozen->tile_n, &mine.tile_n, 1},
      {"tile_k", &frozen->tile_k, &mine.tile_k, 1},
      {"pipeline_stages", &frozen->pipeline_stages, &mine.pipeline_stages, 1},
      {"warps_per_block", &frozen->warps_per_block, &mine.warps_per_block, 1},
      {"producer_warps", &frozen->producer_warps, &mine.producer_warps, 1},
      {"consumer_warps", &frozen->consumer_warps, &mine.consumer_warps, 1},
      {"matrix_acceleration", &frozen->matrix_acceleration, &mine.matrix_acceleration, 1},
      {"async_copy", &frozen->async_copy, &mine.async_copy, 1},
      {"tensor_maps", &frozen->tensor_maps, &mine.tensor_maps, 1},
      {"partition", &frozen->partition, &mine.partition, 1},
      {"split_k", &frozen->split_k, &mine.split_k, 1},
      {"stream_k_slices", &frozen->stream_k_slices, &mine.stream_k_slices, 1},
      {"persistent_ctas_per_sm", &frozen->persistent_ctas_per_sm, &mine.persistent_ctas_per_sm, 1},
      {"cluster_launch", &frozen->cluster_launch, &mine.cluster_launch, 1},
      {"use_distributed_shared_memory", &frozen->use_distributed_shared_memory,
       &mine.use_distributed_shared_memory, 1},
  };
  static_assert(sizeof(mmr_launch_record) == 30 * sizeof(int32_t), "every record field is compared");
  for (const Field& f : fields)
    for (int i = 0; i < f.n; ++i)
      if (f.a[i] != f.b[i]) {
        mmr_gemm_destroy(h);
        return fail(MMR_ERR_PLAN_MISMATCH, "frozen launch record field %s[%d] is %d; this library binds %d", f.name, i,
                    f.a[i], f.b[i]);
      }
  *out = h;
  return MMR_OK;
}

int32_t mmr_gemm_query(const mmr_gemm_handle* h, mmr_gemm_info* info) {
  if (!h || !info) return fail(MMR_ERR_INVALID_ARGUMENT, "null handle or info");
  *info = h->info;
  return MMR_OK;
}

}  // extern "C"
