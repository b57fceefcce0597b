// tc_gemm.cuh -- persistent, warp-specialised tcgen05 f32 GEMM for sm_100a.
//
// Computes, for every batch entry b, C[b] = epilogue(A[b] @ B[b]) where A, B,
// C are f32 views described by TMA tensor maps (zero-copy strided views: A may
// be K- or M-contiguous, B may be K- or N-contiguous). This replaces the
// reference CPU GEMM entries gemm_dot_f32 / gemm_axpy_f32 / gemm_avx2
// (src/momiru/tensor_light/execution/cpu.rs:2989-3098) for a GPU node.
//
// Roles (one CTA per SM, persistent over output tiles of BM x BN):
//   warps 0-7   epilogue (two warpgroups; warp w reads TMEM lane quarter w%4
//               and column half w/4): sums K-chunk partials out of TMEM into
//               f32 registers with round-to-nearest adds, then +bias, ReLU,
//               swizzled shared staging and a TMA store (clipped at the
//               tensor edge; a ragged right edge uses guarded plain stores)
//   warp 8      producer: TMA loads of A/B k-blocks into a 4-stage ring
//   warp 9      MMA issuer: tcgen05.mma kind::tf32 into two TMEM partial
//               accumulators of 256 columns, alternating per K-chunk
//   warps 10-15 (3xTF32 only) split: for each staged f32 operand x, hi is x
//               with the low 13 mantissa bits cleared -- exactly what the
//               tensor core reads from x itself -- and lo = x - hi (exact in
//               f32) is written beside it; the MMA issuer then runs
//               lo*hi + hi*lo + hi*hi per k-step (the error-corrected TF32
//               method of Ootomo & Yokota, 2022).
// K is accumulated in chunks of `chunk_kb` k-blocks (256 wide in 3xTF32): the tensor core's f32
// accumulation is not round-to-nearest, so a single 8192-long chain drifts by
// ~6e-5 relative; short chains summed with RN adds stay near 2e-6.
// Every wait is bounded; on expiry the kernel records an error word, drains
// its in-flight copies and MMAs (bounded), frees TMEM and returns.
// Inputs holding inf or NaN: in 3xTF32 the cross term hi(inf) * lo(b) is
// inf * 0 = NaN whenever b is exactly representable in TF32, which the
// reference order never produces. The split warps flag such tiles (a rare
// path: one atomic per affected stage) and mmr_tc_nonfinite_fixup_kernel
// (fixup.cuh) then recomputes every output of a flagged tile in the
// reference's exact order.
#pragma once
#include "epilogue.cuh"
#include "ptx.cuh"

namespace mmr {

constexpr int TC_BM = 128;
constexpr int TC_BN = 256;
constexpr int TC_CSTAGE_BYTES = 32 * 32 * 4;    // one 32x32 f32 store box
constexpr int TC_EPI_WARPS = 8;
constexpr int TC_PRODUCER_WARP = 8;
constexpr int TC_MMA_WARP = 9;
constexpr int TC_SPLIT_WARP0 = 10;
constexpr int TC_SPLIT_WARPS = 6;
constexpr int TC_GROUP_M = 16;                  // tile raster: M-tiles per group
constexpr int kMaxPeers = 7;                    // replicas on other ranks (8 GPUs)


// Per-mode tile geometry. TF32 stages 32-wide k-blocks (128-byte rows); 3xTF32
// stages 16-wide k-blocks (64-byte rows) so that four stages of raw + split
// operands fit in shared memory and cover the TMA latency.
template <int MODE>
struct TcConfig {
  static constexpr int kBK = MODE ? 16 : 32;
  static constexpr int kABytes = TC_BM * kBK * 4;
  static constexpr int kBBytes = TC_BN * kBK * 4;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = 4;
  static constexpr int kWarps = MODE ? 16 : 12;
  static constexpr int kThreads = 32 * kWarps;
  // Register split by warpgroup (setmaxnreg): the two epilogue warpgroups
  // hold a 128-float running sum per thread; the others need few registers.
  // Launch budget = kThreads * kLaunchRegs; the sum of the split must fit it
  // (checked on the host against the compiled register count before launch).
  static constexpr int kLaunchRegs = MODE ? 128 : 168;
  static constexpr int kEpiRegs = MODE ? 176 : 200;
  static constexpr int kOtherRegs = MODE ? 80 : 96;
  static constexpr int kOperandBytes = kStages * kStageBytes * (MODE ? 2 : 1);
  // Shared-memory descriptor geometry (bytes):
  //  K-major: rows of kBK*4 bytes swizzled with 16-byte atoms (layout 2 for
  //  128-byte rows, 4 for 64-byte rows), 8-row groups kRow*8 apart (SBO),
  //  +32 B per 8-wide k-step.
  //  MN-major tf32 must use the 128-byte swizzle with 32-byte atoms (layout 1,
  //  TMA SWIZZLE_128B_ATOM_32B): 32-element MN atoms kBK*128 apart (LBO),
  //  4-row K groups 512 B apart (SBO), +1024 B per 8-wide k-step.
  static constexpr uint32_t kKmajLayout = kBK == 32 ? 2u : 4u;
  static constexpr uint32_t kKmajSbo = 8u * kBK * 4u;
  static constexpr uint32_t kMnAtomBytes = kBK * 128u;
  static constexpr int kCstageBytes = TC_EPI_WARPS * TC_CSTAGE_BYTES;
  static constexpr int kBarrierBytes = 256;
  // +1024 so the kernel can round its dynamic base up to 1024 bytes.
  static constexpr int kSmemBytes = kOperandBytes + kCstageBytes + kBarrierBytes + 1024;
  static_assert(2 * 128 * kEpiRegs + (kWarps - 8) * 32 * kOtherRegs <= kThreads * kLaunchRegs,
                "register split exceeds the launch budget");
};

struct TcParams {
  int m, n, k;
  int batch;
  int tile_m;                // output tile height: 128 (one CTA) or 256 (CTA pair)
  int tiles_m, tiles_n;
  int tiles_total;
  int k_blocks;
  int chunk_kb;              // k-blocks per TMEM accumulation chunk
  int a_batched, b_batched;  // 0: operand broadcast over the batch
  int epilogue;
  const float* bias;         // [n] when the epilogue adds a bias
  float* c;                  // output base (for the ragged right edge)
  long long c_ld, c_bs;      // output row / batch strides (elements)
  int* err;                  // device error word
  unsigned long long timeout_ns;
  // Non-finite bookkeeping (3xTF32): [0] count, [1] blocks done,
  // [2, 2+tiles) per-tile flags, [2+tiles, 2+2*tiles) flagged tile list.
  unsigned int* nf;
  // Replicated output (column-sharded GEMM): every finished box is also
  // stored into each peer rank's copy of C, at the same element offsets from
  // peer_c[i] as from c (addresses mapped into this process).
  int npeers;
  float* peer_c[kMaxPeers];
  // Tensor maps of the peers' replicas (npeers of them, in device memory),
  // or null: a finished box then leaves for each peer as one TMA store from
  // the staging buffer (asynchronous: the epilogue warp does not issue the
  // NVLink stores itself); the ragged right edge keeps plain stores.
  const CUtensorMap* peer_tm;
  // Stream-K partial sums (CTA-pair kernel): two slots per pair, and arrival
  // counters per split tile and epilogue warp of each CTA (zero between launches).
  float* ws;
  unsigned int* ws_count;
  int sk_tiles;  // trailing tiles split stream-K style (0: whole tiles only)
};

// Copies one finished 32x32 box from the 128B-swizzled staging buffer to each
// peer replica: per instruction the warp writes four 128-byte row segments.
// Called by a whole warp after the staging writes and a __syncwarp.
__device__ __forceinline__ void store_box_to_peers(const TcParams& p, const uint8_t* buf, int row0, int col0,
                                                   int bt, int lane) {
#pragma unroll 1
  for (int it = 0; it < 8; ++it) {
    const int r = it * 4 + (lane >> 3);
    const int ch = lane & 7;
    const float4 v = *reinterpret_cast<const float4*>(buf + r * 128 + ((ch ^ (r & 7)) << 4));
    if (row0 + r < p.m && col0 + ch * 4 < p.n) {
      const long long off = (long long)bt * p.c_bs + (long long)(row0 + r) * p.c_ld + col0 + ch * 4;
      for (int q = 0; q < p.npeers; ++q) *reinterpret_cast<float4*>(p.peer_c[q] + off) = v;
    }
  }
}

// Stores one epilogue warp's 32 x 32 box of C (lane = row; v[i] = column i,
// bias and ReLU already applied in registers): staged in `buf` with the
// 128-byte swizzle, a non-ReLU activation applied there (so the accumulator
// registers are never indexed dynamically), then one TMA store plus the peer
// copies, or, at a ragged right edge (TMA writes whole 16-byte chunks), plain
// stores of the valid columns.
__device__ __forceinline__ void store_box(const TcParams& p, const CUtensorMap* tmC, uint8_t* buf, const float* v,
                                          int row0, int col0, int bt, int lane, int act) {
  if (lane == 0) bulk_wait_group_read<0>();
  __syncwarp();
  // 128B-swizzled row `lane`: 16-byte chunk q lives at q ^ (lane & 7).
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    float4 w4 = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    *reinterpret_cast<float4*>(buf + lane * 128 + ((q ^ (lane & 7)) << 4)) = w4;
  }
  if (act >= ACT_RELU6) {
    __syncwarp();
    float* f = reinterpret_cast<float*>(buf);
    for (int e = lane; e < 32 * 32; e += 32) f[e] = act_other(act, f[e]);
  }
  __syncwarp();
  if ((p.n & 3) && col0 + 32 > p.n) {
    const int row = row0 + lane;
    if (row < p.m) {
      const long long off = (long long)bt * p.c_bs + (long long)row * p.c_ld + col0;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 w = *reinterpret_cast<const float4*>(buf + lane * 128 + ((q ^ (lane & 7)) << 4));
        const float e4[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          if (col0 + 4 * q + i < p.n) {
            p.c[off + 4 * q + i] = e4[i];
            for (int r = 0; r < p.npeers; ++r) p.peer_c[r][off + 4 * q + i] = e4[i];
          }
        }
      }
    }
    return;
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_store_3d(tmC, buf, col0, row0, bt);
    if (p.peer_tm != nullptr)
      for (int q = 0; q < p.npeers; ++q) tma_store_3d(p.peer_tm + q, buf, col0, row0, bt);
    bulk_commit_group();
  }
  if (p.npeers && p.peer_tm == nullptr) store_box_to_peers(p, buf, row0, col0, bt, lane);
}

__device__ __forceinline__ void tc_tile_coords(const TcParams& p, int t, int& mt, int& nt, int& bt) {
  const int per_batch = p.tiles_m * p.tiles_n;
  bt = t / per_batch;
  const int r = t - bt * per_batch;
  const int group_span = TC_GROUP_M * p.tiles_n;
  const int group = r / group_span;
  const int first_m = group * TC_GROUP_M;
  const int gsize = min(p.tiles_m - first_m, TC_GROUP_M);
  const int q = r - group * group_span;
  mt = first_m + q % gsize;
  nt = q / gsize;
}

template <int N>
__device__ __forceinline__ void reg_alloc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;\n" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void reg_dealloc() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;\n" ::"n"(N));
}

template <int MODE, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(TcConfig<MODE>::kThreads, 1)
    mmr_tc_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC, const TcParams p) {
  using Cfg = TcConfig<MODE>;
  constexpr int S = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ops = smem;                                     // [S][A|B]
  uint8_t* lo_ops = smem + S * Cfg::kStageBytes;             // [S][Alo|Blo] (3xTF32)
  uint8_t* cstage = smem + Cfg::kOperandBytes;             // [8 warps][32x32]
  uint64_t* bars = reinterpret_cast<uint64_t*>(cstage + Cfg::kCstageBytes);
  uint64_t* full = bars;             // [S] TMA -> split/MMA
  uint64_t* split_done = bars + S;   // [S] split -> MMA (3xTF32)
  uint64_t* empty = bars + 2 * S;    // [S] MMA -> TMA
  uint64_t* acc_full = bars + 3 * S; // [2] MMA -> epilogue (a K-chunk is done)
  uint64_t* acc_empty = acc_full + 2;// [2] epilogue -> MMA (partial consumed)
  uint64_t* drain = acc_full + 4;    // [1] teardown of the MMA pipe
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const WaitCtl ctl{p.err, p.timeout_ns};

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&split_done[s], TC_SPLIT_WARPS * 32);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], TC_EPI_WARPS * 32);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == TC_PRODUCER_WARP && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmC);
  }
  if (warp == TC_MMA_WARP) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  griddep_wait();
  griddep_release();
  const int n_chunks = (p.k_blocks + p.chunk_kb - 1) / p.chunk_kb;

  if (warp < TC_EPI_WARPS) {
    reg_alloc<Cfg::kEpiRegs>();
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3, half = warp >> 2;
    int acc = 0;
    uint32_t acc_phase = 0;
    uint8_t* buf = cstage + warp * TC_CSTAGE_BYTES;
    const bool add_bias = epi_has_bias(p.epilogue);
    const int act = epi_act(p.epilogue);
    const bool relu = act == ACT_RELU;
    bool ok = true;
    for (int t = blockIdx.x; ok && t < p.tiles_total; t += gridDim.x) {
      int mt, nt, bt;
      tc_tile_coords(p, t, mt, nt, bt);
      const int m0 = mt * TC_BM, n0 = nt * TC_BN;
      float sum[128];
#pragma unroll
      for (int i = 0; i < 128; ++i) sum[i] = 0.0f;
      for (int c = 0; c < n_chunks; ++c) {
        if (!mbar_wait(&acc_full[acc], acc_phase, ctl, kDevTimeoutAcc)) { ok = false; break; }
        tc_fence_after();
        const uint32_t tb = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                            static_cast<uint32_t>(acc * TC_BN + half * 128);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tb + j * 32, r);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) sum[j * 32 + i] = __fadd_rn(sum[j * 32 + i], __uint_as_float(r[i]));
        }
        tc_fence_before();
        mbar_arrive(&acc_empty[acc]);
        if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
      }
      if (!ok) break;
      const int row0 = m0 + quarter * 32;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int col0 = n0 + half * 128 + j * 32;
        float bias_lane = 0.0f;
        if (add_bias && col0 + lane < p.n) bias_lane = __ldg(p.bias + col0 + lane);
        float* v = sum + j * 32;  // epilogue applied in place
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          float x = v[i];
          if (add_bias) x = __fadd_rn(x, __shfl_sync(0xffffffffu, bias_lane, i));
          if (relu) x = act_relu(x);
          v[i] = x;
        }
        if (row0 >= p.m || col0 >= p.n) continue;  // wholly outside C (warp-uniform)
        store_box(p, &tmC, buf, v, row0, col0, bt, lane, act);
      }
    }
    if (lane == 0) bulk_wait_group_all();
    // peer stores (TMA stores complete with the wait above) ordered before
    // the completion signal
    if (p.npeers) {
      fence_proxy_async_global();
      __threadfence_system();
    }
    __syncwarp();
  } else {
    reg_dealloc<Cfg::kOtherRegs>();
    if (warp == TC_PRODUCER_WARP) {
      // ---------------------------------------------------------- producer
      if (lane == 0) {
        int stage = 0;
        uint32_t phase = 0;
        int issued_parity[S];
        for (int s = 0; s < S; ++s) issued_parity[s] = -1;
        bool ok = true;
        for (int t = blockIdx.x; ok && t < p.tiles_total; t += gridDim.x) {
          int mt, nt, bt;
          tc_tile_coords(p, t, mt, nt, bt);
          const int m0 = mt * TC_BM, n0 = nt * TC_BN;
          const int ba = p.a_batched ? bt : 0, bb = p.b_batched ? bt : 0;
          for (int kb = 0; kb < p.k_blocks; ++kb) {
            if (!mbar_wait(&empty[stage], phase ^ 1u, ctl, kDevTimeoutEmpty)) { ok = false; break; }
            uint8_t* sa = ops + stage * Cfg::kStageBytes;
            uint8_t* sb = sa + Cfg::kABytes;
            const int k0 = kb * Cfg::kBK;
            mbar_arrive_expect_tx(&full[stage], Cfg::kStageBytes);
            if (A_MN) {
#pragma unroll
              for (int i = 0; i < TC_BM / 32; ++i)
                tma_load_3d(sa + i * Cfg::kMnAtomBytes, &tmA, &full[stage], m0 + 32 * i, k0, ba);
            } else {
              tma_load_3d(sa, &tmA, &full[stage], k0, m0, ba);
            }
            if (B_MN) {
#pragma unroll
              for (int j = 0; j < TC_BN / 32; ++j)
                tma_load_3d(sb + j * Cfg::kMnAtomBytes, &tmB, &full[stage], n0 + 32 * j, k0, bb);
            } else {
              tma_load_3d(sb, &tmB, &full[stage], k0, n0, bb);
            }
            issued_parity[stage] = static_cast<int>(phase);
            if (++stage == S) { stage = 0; phase ^= 1u; }
          }
        }
        // Drain: every load this thread issued must have landed before the
        // CTA may exit (immediate on the normal path).
        for (int s = 0; s < S; ++s) {
          if (issued_parity[s] >= 0) {
            const uint32_t a = smem_u32(&full[s]);
            const uint64_t t0 = globaltimer_ns();
            while (!mbar_try_wait(a, static_cast<uint32_t>(issued_parity[s]))) {
              if (globaltimer_ns() - t0 > p.timeout_ns) { atomicCAS(p.err, 0, kDevTimeoutDrain); break; }
            }
          }
        }
      }
    } else if (warp == TC_MMA_WARP) {
      // -------------------------------------------------------- MMA issuer
      if (lane == 0) {
        constexpr uint32_t idesc = idesc_tf32(TC_BM, TC_BN, A_MN, B_MN);
        // Descriptor geometry: see TcConfig. Descriptors are fixed offsets from
        // two precomputed ones (the start-address field holds shared-memory
        // addresses >> 4 and never carries), so the issuing thread does little
        // more than issue MMAs.
        constexpr uint32_t a_layout = A_MN ? 1u : Cfg::kKmajLayout, b_layout = B_MN ? 1u : Cfg::kKmajLayout;
        constexpr uint32_t a_lbo = A_MN ? Cfg::kMnAtomBytes : 16u, a_sbo = A_MN ? 512u : Cfg::kKmajSbo;
        constexpr uint32_t b_lbo = B_MN ? Cfg::kMnAtomBytes : 16u, b_sbo = B_MN ? 512u : Cfg::kKmajSbo;
        constexpr uint32_t a_kstep = A_MN ? 1024u : 32u, b_kstep = B_MN ? 1024u : 32u;
        const uint64_t a_desc0 = smem_desc(smem_u32(ops), a_lbo, a_sbo, a_layout);
        const uint64_t b_desc0 = smem_desc(smem_u32(ops) + Cfg::kABytes, b_lbo, b_sbo, b_layout);
        constexpr uint64_t kStageStep = Cfg::kStageBytes >> 4;
        constexpr uint64_t kLoStep = (uint64_t(S) * Cfg::kStageBytes) >> 4;  // raw -> split-off low part
        uint64_t* const ready = MODE ? split_done : full;
        int stage = 0;
        uint32_t phase = 0;
        int acc = 0;
        uint32_t acc_phase = 0;
        bool ok = true;
        bool issued_any = false;
        for (int t = blockIdx.x; ok && t < p.tiles_total; t += gridDim.x) {
          for (int kb = 0; kb < p.k_blocks;) {
            // One TMEM accumulation chunk: k-blocks [kb, chunk_end).
            const int chunk_end = min(kb + p.chunk_kb, p.k_blocks);
            if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1u, ctl, kDevTimeoutAcc)) { ok = false; break; }
            tc_fence_after();
            const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * TC_BN);
            uint32_t accumulate = 0u;
            for (; kb < chunk_end; ++kb) {
              if (!mbar_wait(&ready[stage], phase, ctl, MODE ? kDevTimeoutXform : kDevTimeoutFull)) {
                ok = false;
                break;
              }
              tc_fence_after();
              const uint64_t so = static_cast<uint64_t>(stage) * kStageStep;
#pragma unroll
              for (int kk = 0; kk < Cfg::kBK / 8; ++kk) {
                const uint64_t ad = a_desc0 + so + kk * (a_kstep >> 4);
                const uint64_t bd = b_desc0 + so + kk * (b_kstep >> 4);
                if (MODE) {
                  // Small cross terms first, then hi*hi.
                  umma_tf32(d_tmem, ad + kLoStep, bd, idesc, accumulate);
                  umma_tf32(d_tmem, ad, bd + kLoStep, idesc, 1u);
                  umma_tf32(d_tmem, ad, bd, idesc, 1u);
                } else {
                  umma_tf32(d_tmem, ad, bd, idesc, accumulate);
                }
                accumulate = 1u;
              }
              issued_any = true;
              umma_commit(&empty[stage]);
              if (++stage == S) { stage = 0; phase ^= 1u; }
            }
            if (!ok) break;
            umma_commit(&acc_full[acc]);
            if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
          }
        }
        if (issued_any) {
          // Every MMA must have finished before TMEM is freed.
          umma_commit(drain);
          const uint32_t a = smem_u32(drain);
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(a, 0u)) {
            if (globaltimer_ns() - t0 > p.timeout_ns) { atomicCAS(p.err, 0, kDevTimeoutDrain); break; }
          }
        }
      }
    } else if (MODE && warp >= TC_SPLIT_WARP0 && warp < TC_SPLIT_WARP0 + TC_SPLIT_WARPS) {
      // ------------------------------------------------- 3xTF32 split warps
      const int tid = threadIdx.x - TC_SPLIT_WARP0 * 32;
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < p.tiles_total; t += gridDim.x) {
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, ctl, kDevTimeoutFull)) { ok = false; break; }
          uint4* x = reinterpret_cast<uint4*>(ops + stage * Cfg::kStageBytes);
          uint4* lo = reinterpret_cast<uint4*>(lo_ops + stage * Cfg::kStageBytes);
          bool nonfinite = false;
          // The tensor core reads an f32 operand as TF32 by dropping its low 13
          // mantissa bits, so the staged raw value already is hi; only
          // lo = x - hi is written. Tiles with inf/NaN are flagged and
          // recomputed exactly by the fix-up kernel.
#pragma unroll 4
          for (int i = tid; i < Cfg::kStageBytes / 16; i += TC_SPLIT_WARPS * 32) {
            const uint4 v = x[i];
            uint4 l;
#define MMR_SPLIT1(F)                                                                        \
  {                                                                                          \
    const uint32_t u = v.F;                                                                  \
    const bool nf = (u & 0x7F800000u) == 0x7F800000u;                                        \
    nonfinite |= nf;                                                                         \
    l.F = nf ? 0u : __float_as_uint(__fsub_rn(__uint_as_float(u), __uint_as_float(u & 0xFFFFE000u))); \
  }
            MMR_SPLIT1(x) MMR_SPLIT1(y) MMR_SPLIT1(z) MMR_SPLIT1(w)
#undef MMR_SPLIT1
            lo[i] = l;
          }
          fence_proxy_async_smem();
          mbar_arrive(&split_done[stage]);
          if (__any_sync(0xffffffffu, nonfinite) && lane == 0 && p.nf != nullptr) {
            if (atomicOr(&p.nf[2 + t], 1u) == 0u) p.nf[2 + p.tiles_total + atomicAdd(&p.nf[0], 1u)] = t;
          }
          if (++stage == S) { stage = 0; phase ^= 1u; }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == TC_MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace mmr
