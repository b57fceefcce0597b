// tc_gemm_2sm.cuh -- f32 GEMM on CTA pairs (tcgen05 cta_group::2), in both
// numeric modes: MODE 1 = StrictFp32 (3xTF32), MODE 0 = one TF32 pass.
//
// Same contract and numerics as mmr_tc_gemm_kernel<MODE, ...> (3xTF32 split,
// 256-wide K chunks summed with round-to-nearest adds, exact fix-up of tiles
// with inf/NaN inputs; TF32 keeps one chain per tile segment), but each output
// tile of 256 x 256 is computed by a cluster of two CTAs on two SMs with one
// 256-row MMA per k-step. Each CTA stages only its 128 rows of A and its
// 128-column half of B (plus their lo parts), which halves the per-SM
// shared-memory traffic of the B operand.
//
// Work split: whole tiles round-robin, except the last sk_tiles (the partial
// last round, or the last two rounds when that one is under half full), whose
// k-blocks, in tile-major order, are dealt to the pairs in equal contiguous
// ranges (stream-K), so no pair idles in a last partial round of tiles. A
// range is a list of segments (tile, k-blocks [kb0, kb1)): a whole tile goes
// through the epilogue as usual; a part of a split tile parks its partial sum
// in a workspace slot of its pair and counts itself in on a per-tile counter
// (one per epilogue warp). The warp whose part completes the count adds the
// parts in K order with round-to-nearest adds (so the result is the same
// whichever pair arrives last), stores the tile and resets the counter.
// Nothing waits on another pair, so the pairs need not be co-resident. Odd
// pairs take their segments last-first (PairWork), so a tile shared by an odd
// pair and the next even pair is finished in mid-kernel. When the output is
// replicated to peer GPUs and there are under two rounds of tiles, the binder
// splits every tile this way (sk_tiles = all tiles) to spread tile
// completions, and so the NVLink stores, over the run.
//
// Pair protocol (rank 0 = even CTA issues every MMA of the pair):
//   full[s]        3xTF32: local, TMA -> split warps of the same CTA.
//                  TF32: rank 0's counts the bytes of both CTAs' loads (the
//                  odd CTA's loads name it) and gates the MMA directly.
//   split_done[s]  3xTF32, rank 0 only, 12 arrivals: six split warps of each CTA
//   empty[s]       each CTA, one arrival from rank 0's tcgen05.commit
//   acc_full[a]    each CTA, one arrival from rank 0's tcgen05.commit
//   acc_empty[a]   rank 0 only, 16 arrivals: eight epilogue warps of each CTA
// Commits reach the odd CTA's barriers by their cluster address (no
// multicast). Both CTAs pass a cluster barrier after set-up and before
// freeing TMEM.
#pragma once
#include "tc_gemm.cuh"

namespace mmr {

template <int MODE>
struct Tc2Config {
  // k-block width: 3xTF32 stages raw operands and their split-off low parts
  // (16 wide, six stages); TF32 stages 64-wide k-blocks (two 32-wide K-major
  // panels per operand, three stages), so that each stage carries eight MMAs
  // per barrier wait and commit instead of four (8192^3: 693 -> 748 TFLOP/s).
  static constexpr int kBK = MODE ? 16 : 64;
  static constexpr int kABytes = 128 * kBK * 4;          // this CTA's 128 rows of A
  static constexpr int kBBytes = 128 * kBK * 4;          // this CTA's 128 columns of B
  static constexpr int kStageBytes = kABytes + kBBytes;  // raw operands (+ as much again for lo)
  static constexpr int kStages = MODE ? 6 : 3;
  static constexpr int kWarps = MODE ? 16 : 12;
  static constexpr int kThreads = 32 * kWarps;
  static constexpr int kLaunchRegs = MODE ? 128 : 168;
  static constexpr int kEpiRegs = MODE ? 176 : 200;
  static constexpr int kOtherRegs = MODE ? 80 : 96;
  static constexpr int kOperandBytes = kStages * kStageBytes * (MODE ? 2 : 1);
  static constexpr int kCstageBytes = TC_EPI_WARPS * TC_CSTAGE_BYTES;
  static constexpr int kBarrierBytes = 256;
  static constexpr int kSmemBytes = kOperandBytes + kCstageBytes + kBarrierBytes + 1024;
  static constexpr uint32_t kMnAtomBytes = kBK * 128u;   // 32 MN elements x kBK K rows
  // K-major tiles are stored as panels of at most 32 K (128-byte swizzled
  // rows, one TMA box each); a 64-wide k-block is two panels side by side.
  static constexpr int kPanelK = kBK < 32 ? kBK : 32;
  static constexpr int kPanels = kBK / kPanelK;
  static constexpr uint32_t kPanelBytes = 128u * kPanelK * 4u;  // 128 rows of A or 128 columns of B
  static constexpr uint32_t kKmajLayout = kPanelK == 32 ? 2u : 4u;
  static constexpr uint32_t kKmajSbo = 8u * kPanelK * 4u;
  static_assert(kBK % kPanelK == 0 && kPanels * kPanelBytes == kABytes, "panels tile the k-block");
  static_assert(2 * 128 * kEpiRegs + (kWarps - 8) * 32 * kOtherRegs <= kThreads * kLaunchRegs,
                "register split exceeds the launch budget");
};

// Floats of one partial-sum slot: two CTAs x 128 rows x 256 columns.
constexpr int kSkSlotFloats = 2 * 128 * TC_BN;

// The first tiles_total - sk_tiles tiles are whole tiles dealt round-robin
// (tile = pair + i * npairs), so the pairs running at one time share A and B
// panels in L2; only the last sk_tiles tiles are split stream-K style.
// Equal contiguous ranges of the stream-K (tile, k-block) iteration space:
__device__ __forceinline__ long long sk_unit(const TcParams& p, int pair, int npairs) {
  const long long U = (long long)p.sk_tiles * p.k_blocks;
  return (U / npairs) * pair + (U % npairs) * pair / npairs;
}

// Arrival counter of warp w of CTA `rank` for stream-K tile ts (0-based in
// the split region): each part's warp adds one after parking its partial sum;
// the warp that completes the count finishes the tile and resets it to zero.
__device__ __forceinline__ int sk_counter(int ts, uint32_t rank, int w) {
  return (2 * ts + static_cast<int>(rank)) * TC_EPI_WARPS + w;
}

// The pair whose stream-K range holds unit u.
__device__ __forceinline__ int sk_pair_of(const TcParams& p, long long u, int npairs) {
  const long long U = (long long)p.sk_tiles * p.k_blocks;
  int q = static_cast<int>((u * npairs) / U);
  while (q + 1 < npairs && sk_unit(p, q + 1, npairs) <= u) ++q;
  while (q > 0 && sk_unit(p, q, npairs) > u) --q;
  return q;
}

// One pair's work: its round-robin whole tiles, then its stream-K segments.
// Odd pairs take their segments last-first. Then the tile split between an odd
// pair and the even pair after it has both parts computed first and is
// finished in mid-kernel, instead of at the end where every pair's last tile
// would otherwise land at once (the replicated output leaves over NVLink tile
// by tile, so a burst at the end is time that nothing overlaps).
struct PairWork {
  int pair, npairs, i, dp_rounds, sk_base, kb_per_tile;
  long long u0, u1;
  bool reverse;
  __device__ __forceinline__ PairWork(const TcParams& p, int pair_, int npairs_)
      : pair(pair_), npairs(npairs_), i(0), dp_rounds((p.tiles_total - p.sk_tiles) / npairs_),
        sk_base(p.tiles_total - p.sk_tiles), kb_per_tile(p.k_blocks),
        u0(sk_unit(p, pair_, npairs_)), u1(sk_unit(p, pair_ + 1, npairs_)), reverse(pair_ & 1) {}
  __device__ __forceinline__ bool next(int& t, int& kb0, int& kb1) {
    if (i < dp_rounds) {
      t = pair + i * npairs;
      ++i;
      kb0 = 0;
      kb1 = kb_per_tile;
      return true;
    }
    if (u0 >= u1) return false;
    int ts;
    if (!reverse) {
      ts = static_cast<int>(u0 / kb_per_tile);
      kb0 = static_cast<int>(u0 - (long long)ts * kb_per_tile);
      const long long rem = u1 - u0;
      kb1 = rem < kb_per_tile - kb0 ? kb0 + static_cast<int>(rem) : kb_per_tile;
      u0 += kb1 - kb0;
    } else {
      ts = static_cast<int>((u1 - 1) / kb_per_tile);
      const long long tile_u = (long long)ts * kb_per_tile;
      const long long lo = u0 > tile_u ? u0 : tile_u;
      kb0 = static_cast<int>(lo - tile_u);
      kb1 = static_cast<int>(u1 - tile_u);
      u1 = lo;
    }
    t = sk_base + ts;
    return true;
  }
};

template <int MODE, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(Tc2Config<MODE>::kThreads, 1)
    mmr_tc_gemm_2sm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                       const __grid_constant__ CUtensorMap tmC, const TcParams p) {
  using Cfg = Tc2Config<MODE>;
  constexpr int S = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ops = smem;
  uint8_t* lo_ops = smem + S * Cfg::kStageBytes;
  uint8_t* cstage = smem + Cfg::kOperandBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(cstage + Cfg::kCstageBytes);
  uint64_t* full = bars;
  uint64_t* split_done = bars + S;
  uint64_t* empty = bars + 2 * S;
  uint64_t* acc_full = bars + 3 * S;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_full + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = static_cast<int>(blockIdx.x >> 1);
  const int npairs = static_cast<int>(gridDim.x >> 1);
  const WaitCtl ctl{p.err, p.timeout_ns};

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&split_done[s], 2 * TC_SPLIT_WARPS);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 2 * TC_EPI_WARPS);
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
    tmem_alloc_2sm(tmem_slot, 512);
    tmem_relinquish_2sm();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // barrier inits and both TMEM allocations visible to the pair
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  griddep_wait();
  griddep_release();

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
    const uint32_t acc_empty_leader0 = mapa_shared(smem_u32(&acc_empty[0]), 0);
    // This warp's 32 rows x 128 columns inside a partial-sum slot: 16 KiB of
    // its own, float4 q of lane l at (q * 32 + l), so that each store or load
    // instruction of the warp covers 512 contiguous bytes.
    const int ws_warp = ((static_cast<int>(rank) * 4 + quarter) * 2 + half) * (32 * 128);
    float sum[128];

    // Applies the epilogue (bias, activation) to sum[] and stores this
    // thread's part of tile t.
    // Boxes j in [j0, j1) of this thread's four 32-column boxes.
    auto store_tile = [&](int t, int j0 = 0, int j1 = 4) {
      int mt, nt, bt;
      tc_tile_coords(p, t, mt, nt, bt);
      const int row0 = mt * 256 + static_cast<int>(rank) * 128 + quarter * 32;
      const int nbase = nt * TC_BN + half * 128;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (j < j0 || j >= j1) continue;
        const int col0 = nbase + j * 32;
        float bias_lane = 0.0f;
        if (add_bias && col0 + lane < p.n) bias_lane = __ldg(p.bias + col0 + lane);
        float* v = sum + j * 32;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          float x = v[i];
          if (add_bias) x = __fadd_rn(x, __shfl_sync(0xffffffffu, bias_lane, i));
          if (relu) x = act_relu(x);
          v[i] = x;
        }
        if (row0 >= p.m || col0 >= p.n) continue;
        store_box(p, &tmC, buf, v, row0, col0, bt, lane, act);
      }
    };
    auto save_partial = [&](float* slot) {
      float4* dst = reinterpret_cast<float4*>(slot + ws_warp) + lane;
#pragma unroll
      for (int q = 0; q < 32; ++q)
        dst[q * 32] = make_float4(sum[4 * q], sum[4 * q + 1], sum[4 * q + 2], sum[4 * q + 3]);
    };

    bool ok = true;
    PairWork segs(p, pair, npairs);
    int t, kb0, kb1;
    while (ok && segs.next(t, kb0, kb1)) {
#pragma unroll
      for (int i = 0; i < 128; ++i) sum[i] = 0.0f;
      const int n_chunks = (kb1 - kb0 + p.chunk_kb - 1) / p.chunk_kb;
      for (int c = 0; c < n_chunks; ++c) {
        if (!mbar_wait_cluster(&acc_full[acc], acc_phase, ctl, kDevTimeoutAcc)) { ok = false; break; }
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
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(acc_empty_leader0 + 8u * acc);
        if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
      }
      if (!ok) break;
      if (kb0 == 0 && kb1 == p.k_blocks) {
        store_tile(t);
        continue;
      }
      // One part of a split tile: park it (slot 0 for the part that ends the
      // tile's K range, slot 1 for a head or middle part), then count it in.
      const int ts = t - (p.tiles_total - p.sk_tiles);
      save_partial(p.ws + (2 * pair + (kb1 == p.k_blocks ? 0 : 1)) * kSkSlotFloats);
      __threadfence();
      __syncwarp();
      const int q0 = sk_pair_of(p, (long long)ts * p.k_blocks, npairs);
      const int q1 = sk_pair_of(p, (long long)(ts + 1) * p.k_blocks - 1, npairs);
      unsigned int last = 0;
      if (lane == 0) {
        unsigned int* cnt = p.ws_count + sk_counter(ts, rank, warp);
        unsigned int before;
        asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(before) : "l"(cnt) : "memory");
        last = before == static_cast<unsigned int>(q1 - q0);
        if (last) *cnt = 0u;  // every part has arrived: ready for the next launch
      }
      if (!__shfl_sync(0xffffffffu, last, 0)) continue;
      // Last part in: add the parts in K order (pairs q0 .. q1) with
      // round-to-nearest adds, whichever pair finishes, and store the tile.
      // Done in two 64-column halves so that one part's 16 loads of a half
      // are in flight together beside the 64 live sums (all 32 loads of a
      // part beside all 128 sums would not fit the registers, and the loads
      // would go out a few at a time: several L2 round trips per part).
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
#pragma unroll
        for (int i = 0; i < 64; ++i) sum[hh * 64 + i] = 0.0f;
        for (int q = q0; q <= q1; ++q) {
          const float4* src = reinterpret_cast<const float4*>(p.ws + (2 * q + (q == q1 ? 0 : 1)) * kSkSlotFloats +
                                                              ws_warp) + (hh * 16) * 32 + lane;
          float4 v[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] = __ldcg(src + i * 32);
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            float* d = sum + hh * 64 + 4 * i;
            d[0] = __fadd_rn(d[0], v[i].x);
            d[1] = __fadd_rn(d[1], v[i].y);
            d[2] = __fadd_rn(d[2], v[i].z);
            d[3] = __fadd_rn(d[3], v[i].w);
          }
        }
        store_tile(t, 2 * hh, 2 * hh + 2);
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
        const uint32_t full_leader0 = mapa_shared(smem_u32(&full[0]), 0);
        PairWork segs(p, pair, npairs);
        int t, kb0, kb1;
        while (ok && segs.next(t, kb0, kb1)) {
          int mt, nt, bt;
          tc_tile_coords(p, t, mt, nt, bt);
          const int m0 = mt * 256 + static_cast<int>(rank) * 128;
          const int nb = nt * TC_BN + static_cast<int>(rank) * 128;  // this CTA's half of B
          const int ba = p.a_batched ? bt : 0, bb = p.b_batched ? bt : 0;
          for (int kb = kb0; kb < kb1; ++kb) {
            if (!mbar_wait_cluster(&empty[stage], phase ^ 1u, ctl, kDevTimeoutEmpty)) { ok = false; break; }
            uint8_t* sa = ops + stage * Cfg::kStageBytes;
            uint8_t* sb = sa + Cfg::kABytes;
            const int k0 = kb * Cfg::kBK;
            if (MODE) {
              // 3xTF32: each CTA's loads complete on its own barrier; the
              // split warps gate the MMA.
              mbar_arrive_expect_tx(&full[stage], Cfg::kStageBytes);
              if (A_MN) {
#pragma unroll
                for (int i = 0; i < 4; ++i)
                  tma_load_3d(sa + i * Cfg::kMnAtomBytes, &tmA, &full[stage], m0 + 32 * i, k0, ba);
              } else {
#pragma unroll
                for (int q = 0; q < Cfg::kPanels; ++q)
                  tma_load_3d(sa + q * Cfg::kPanelBytes, &tmA, &full[stage], k0 + q * Cfg::kPanelK, m0, ba);
              }
              if (B_MN) {
#pragma unroll
                for (int j = 0; j < 4; ++j)
                  tma_load_3d(sb + j * Cfg::kMnAtomBytes, &tmB, &full[stage], nb + 32 * j, k0, bb);
              } else {
#pragma unroll
                for (int q = 0; q < Cfg::kPanels; ++q)
                  tma_load_3d(sb + q * Cfg::kPanelBytes, &tmB, &full[stage], k0 + q * Cfg::kPanelK, nb, bb);
              }
            } else {
              // TF32: both CTAs' loads complete on the even CTA's barrier,
              // which expects the bytes of the pair.
              const uint32_t fbar = full_leader0 + 8u * stage;
              if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * Cfg::kStageBytes);
              if (A_MN) {
#pragma unroll
                for (int i = 0; i < 4; ++i)
                  tma_load_3d_pair(sa + i * Cfg::kMnAtomBytes, &tmA, fbar, m0 + 32 * i, k0, ba);
              } else {
#pragma unroll
                for (int q = 0; q < Cfg::kPanels; ++q)
                  tma_load_3d_pair(sa + q * Cfg::kPanelBytes, &tmA, fbar, k0 + q * Cfg::kPanelK, m0, ba);
              }
              if (B_MN) {
#pragma unroll
                for (int j = 0; j < 4; ++j)
                  tma_load_3d_pair(sb + j * Cfg::kMnAtomBytes, &tmB, fbar, nb + 32 * j, k0, bb);
              } else {
#pragma unroll
                for (int q = 0; q < Cfg::kPanels; ++q)
                  tma_load_3d_pair(sb + q * Cfg::kPanelBytes, &tmB, fbar, k0 + q * Cfg::kPanelK, nb, bb);
              }
            }
            issued_parity[stage] = static_cast<int>(phase);
            if (++stage == S) { stage = 0; phase ^= 1u; }
          }
        }
        // Every load this CTA issued must have landed before it may exit. In
        // TF32 mode the odd CTA's loads count on the even CTA's barrier, which
        // the even CTA drains; the closing cluster barrier covers the pair.
        for (int s = 0; (MODE || rank == 0) && s < S; ++s) {
          if (issued_parity[s] >= 0) {
            const uint32_t a = smem_u32(&full[s]);
            const uint64_t t0 = globaltimer_ns();
            while (!mbar_try_wait_cluster(a, static_cast<uint32_t>(issued_parity[s]))) {
              if (globaltimer_ns() - t0 > p.timeout_ns) { atomicCAS(p.err, 0, kDevTimeoutDrain); break; }
            }
          }
        }
      }
    } else if (warp == TC_MMA_WARP) {
      if (lane == 0 && rank == 0) {
        // ----------------------------------------------- MMA issuer (pair)
        // The tensor core only stays busy while this one thread keeps up: a
        // 256x256x8 pair MMA takes 128 cycles, so the per-k-block work of the
        // issuing thread (barrier wait, fence, descriptors, commits) has to
        // stay well below the 768 (3xTF32) or 512 (TF32) cycles of MMAs it
        // issues. Every descriptor is therefore a fixed offset from two
        // precomputed ones, and the chunk bookkeeping is a counter, not a
        // division.
        constexpr uint32_t idesc = idesc_tf32(256, TC_BN, A_MN, B_MN);
        constexpr uint32_t a_layout = A_MN ? 1u : Cfg::kKmajLayout, b_layout = B_MN ? 1u : Cfg::kKmajLayout;
        constexpr uint32_t a_lbo = A_MN ? Cfg::kMnAtomBytes : 16u, a_sbo = A_MN ? 512u : Cfg::kKmajSbo;
        constexpr uint32_t b_lbo = B_MN ? Cfg::kMnAtomBytes : 16u, b_sbo = B_MN ? 512u : Cfg::kKmajSbo;
        constexpr uint32_t a_kstep = A_MN ? 1024u : 32u, b_kstep = B_MN ? 1024u : 32u;
        constexpr int kPerPanel = Cfg::kPanelK / 8;  // 8-wide k-steps per K-major panel
        // Byte offset of k-step kk inside a stage's operand tile.
        constexpr auto kstep_off = [](bool mn, uint32_t step, int kk) -> uint32_t {
          return mn ? step * kk : (kk / kPerPanel) * Cfg::kPanelBytes + (kk % kPerPanel) * step;
        };
        // The start-address field holds shared-memory addresses >> 4 (all below
        // 2^18 bytes, so offsets added to it never carry out of the field).
        const uint64_t a_desc0 = smem_desc(smem_u32(ops), a_lbo, a_sbo, a_layout);
        const uint64_t b_desc0 = smem_desc(smem_u32(ops) + Cfg::kABytes, b_lbo, b_sbo, b_layout);
        constexpr uint64_t kStageStep = Cfg::kStageBytes >> 4;
        constexpr uint64_t kLoStep = (uint64_t(S) * Cfg::kStageBytes) >> 4;  // raw -> split-off low part
        const uint32_t empty_peer0 = mapa_shared(smem_u32(&empty[0]), 1);
        const uint32_t acc_full_peer0 = mapa_shared(smem_u32(&acc_full[0]), 1);
        uint64_t* const ready = MODE ? split_done : full;
        int stage = 0;
        uint32_t phase = 0;
        int acc = 0;
        uint32_t acc_phase = 0;
        bool ok = true;
        bool issued_any = false;
        PairWork segs(p, pair, npairs);
        int t, kb0, kb1;
        while (ok && segs.next(t, kb0, kb1)) {
          for (int kb = kb0; kb < kb1;) {
            // One TMEM accumulation chunk: k-blocks [kb, chunk_end).
            const int chunk_end = min(kb + p.chunk_kb, kb1);
            if (!mbar_wait_cluster(&acc_empty[acc], acc_phase ^ 1u, ctl, kDevTimeoutAcc)) { ok = false; break; }
            tc_fence_after();
            const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * TC_BN);
            uint32_t accumulate = 0u;
            for (; kb < chunk_end; ++kb) {
              if (!mbar_wait_cluster(&ready[stage], phase, ctl, MODE ? kDevTimeoutXform : kDevTimeoutFull)) {
                ok = false;
                break;
              }
              tc_fence_after();
              const uint64_t so = static_cast<uint64_t>(stage) * kStageStep;
#pragma unroll
              for (int kk = 0; kk < Cfg::kBK / 8; ++kk) {
                const uint64_t ad = a_desc0 + so + (kstep_off(A_MN, a_kstep, kk) >> 4);
                const uint64_t bd = b_desc0 + so + (kstep_off(B_MN, b_kstep, kk) >> 4);
                if (MODE) {
                  umma_tf32_2sm(d_tmem, ad + kLoStep, bd, idesc, accumulate);  // lo(A) hi(B)
                  umma_tf32_2sm(d_tmem, ad, bd + kLoStep, idesc, 1u);          // hi(A) lo(B)
                  umma_tf32_2sm(d_tmem, ad, bd, idesc, 1u);                    // hi(A) hi(B)
                } else {
                  umma_tf32_2sm(d_tmem, ad, bd, idesc, accumulate);
                }
                accumulate = 1u;
              }
              issued_any = true;
              umma_commit_2sm(smem_u32(&empty[stage]));
              umma_commit_2sm(empty_peer0 + 8u * stage);
              if (++stage == S) { stage = 0; phase ^= 1u; }
            }
            if (!ok) break;
            umma_commit_2sm(smem_u32(&acc_full[acc]));
            umma_commit_2sm(acc_full_peer0 + 8u * acc);
            if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
          }
        }
        if (issued_any) {
          umma_commit_2sm(smem_u32(drain));
          umma_commit_2sm(mapa_shared(smem_u32(drain), 1));
        }
        if (issued_any) {
          const uint32_t a = smem_u32(drain);
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait_cluster(a, 0u)) {
            if (globaltimer_ns() - t0 > p.timeout_ns) { atomicCAS(p.err, 0, kDevTimeoutDrain); break; }
          }
        }
      }
    } else if (MODE && warp >= TC_SPLIT_WARP0 && warp < TC_SPLIT_WARP0 + TC_SPLIT_WARPS) {
      // ------------------------------------------------------- split warps
      const int tid = threadIdx.x - TC_SPLIT_WARP0 * 32;
      const uint32_t split_done_leader0 = mapa_shared(smem_u32(&split_done[0]), 0);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      PairWork segs(p, pair, npairs);
      int t, kb0, kb1;
      while (ok && segs.next(t, kb0, kb1)) {
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, ctl, kDevTimeoutFull)) { ok = false; break; }
          const uint4* x = reinterpret_cast<const uint4*>(ops + stage * Cfg::kStageBytes);
          uint4* lo = reinterpret_cast<uint4*>(lo_ops + stage * Cfg::kStageBytes);
          bool nonfinite = false;
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
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(split_done_leader0 + 8u * stage);
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
  // On the normal path the epilogue consumed the last chunk's commit, which
  // covers every MMA of the pair. After an error the odd CTA waits (bounded)
  // for the drain commit before its TMEM and shared memory may go.
  if (warp == TC_MMA_WARP && lane == 0 && rank == 1 &&
      *reinterpret_cast<volatile int*>(p.err) != 0) {
    const uint32_t a = smem_u32(drain);
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait_cluster(a, 0u)) {
      if (globaltimer_ns() - t0 > p.timeout_ns) break;
    }
  }
  __syncthreads();
  cluster_sync_all();  // no CTA leaves while its pair may still touch its memory
  if (warp == TC_MMA_WARP) {
    tc_fence_after();
    tmem_dealloc_2sm(tmem_base, 512);
  }
}

}  // namespace mmr
