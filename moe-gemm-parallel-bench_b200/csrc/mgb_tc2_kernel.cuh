// Persistent grouped GEMM on CTA pairs (tcgen05 cta_group::2), fp16 / bf16.
//
// Same contract as tc_grouped_kernel (C_e = A_e @ B_e, fp32 accumulate, cast
// on store) for token-rich problems: a cluster of two CTAs on neighbouring
// SMs owns a 256-token x (256 NH)-weight-column output tile.  CTA r loads
// token rows [128r, 128r + 128) of the tile and, of every 256-column half h,
// weight columns [256h + 128r, 256h + 128r + 128) into its own shared memory;
// the even CTA issues tcgen05.mma.cta_group::2 (M = 256, N = 256) per half,
// which reads both CTAs' halves.  Per SM this halves the weight bytes each MMA
// pulls through shared memory and L2 compared with a one-CTA 128 x 256 tile,
// which is what keeps the tensor pipe fed.
//
// Roles per CTA (192 threads) as in tc_grouped_kernel; only the even CTA's MMA
// lane issues MMAs.  Barriers:
//   full[s]      in CTA 0 only: both CTAs' TMA bytes for stage s land on it
//                (the even CTA's producer posts the expected byte count);
//   empty[s]     in each CTA: the MMA commit multicasts to both;
//   acc_full[b]  in each CTA: the MMA commit multicasts to both epilogues;
//   acc_empty[b] in CTA 0 only: the 8 epilogue warps of the pair arrive.  The
//                256 x 256 tile double-buffers its accumulator (b = buffer);
//                the 256 x 512 tile's single accumulator is freed by halves
//                (b = 256-column half), so the next tile's half-0 MMAs of its
//                first k-blocks run while the epilogue still drains half 1.
// Every wait is bounded; loads carry no multicast.
#pragma once

#include "mgb_tc_kernel.cuh"

namespace mgb {

// NH = number of 256-column MMA halves per cluster tile: 1 gives the 256 x 256
// tile with two TMEM accumulators (the epilogue of one tile overlaps the MMAs
// of the next); 2 gives the 256 x 512 tile, whose single 512-column
// accumulator fills TMEM.  Per k-block a CTA of the wide tile loads 16 KB of
// activations and 32 KB of weights for 128 x 512 x 64 MACs (171 FLOP per
// byte from L2) instead of 16 + 16 KB for 128 x 256 x 64 (128 FLOP per byte).
template <typename T, int NH>
struct Tc2Cfg {
  static constexpr int kElem = static_cast<int>(sizeof(T));
  static_assert(kElem == 2, "the CTA-pair kernel serves fp16 / bf16");
  static_assert(NH == 1 || NH == 2, "one or two 256-column halves");
  static constexpr int kBK = 64;
  static constexpr int kKStep = 16;
  static constexpr int kKSteps = 4;
  static constexpr int kTileM = 256;       // tokens per cluster tile
  static constexpr int kTileN = 256 * NH;  // weight columns per cluster tile
  static constexpr int kHalf = 128;        // per CTA: token rows, and weight columns per MMA half
  static constexpr int kActBytes = kHalf * 128;
  static constexpr int kBoxBytes = kBK * 128;
  static constexpr int kHalfWgtBytes = kHalf * 128;  // one CTA's weight columns of one MMA half
  static constexpr int kWgtBytes = NH * kHalfWgtBytes;
  static constexpr int kStageBytes = kActBytes + kWgtBytes;
  // Two staging blocks per epilogue warp: the shared memory they leave buys
  // a deeper operand ring (4 stages of 48 KB for the wide tile, 6 of 32 KB
  // for 256 x 256), which measured faster on both tiles than four blocks and
  // one stage less; on the wide tile it also lets four k-blocks of half-0
  // MMAs run under the half-1 drain.
  static constexpr int kEpiBlocks = 2;
  static constexpr int kEpiBytes = epi_bytes_row_tile(kEpiBlocks);  // staging blocks of the 4 epilogue warps
  static constexpr int kStagesRaw = (kTcSmemBudget - kEpiBytes) / kStageBytes;
  static constexpr int kStages = kStagesRaw > 12 ? 12 : kStagesRaw;
  static constexpr int kAccCols = kTileN;
  static constexpr int kAccBufs = NH == 1 ? 2 : 1;
  static constexpr int kTmemCols = 512;
  static constexpr uint32_t kFmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
  static constexpr uint32_t kIdesc = instr_desc(kFmt, 0, 1, kTileM, 256);  // one MMA: M = 256, N = 256
  static constexpr int kSmemBytes = kStages * kStageBytes + kEpiBytes + 2048 + 1024;
  static_assert(kAccBufs * kAccCols <= kTmemCols, "accumulators fit in TMEM");
  // The epilogue is exactly four warps (2-5), one per TMEM lane quarter
  // (warp & 3 = 2, 3, 0, 1): the staging blocks are sized for four warps, each
  // warp's blocks start at quarter * kEpiBlocks * kEpiWarpBytes < kEpiBytes,
  // and an accumulator half is released by kEpiArrivals = 2 CTAs x 4 warps
  // arrivals.  A layout with more epilogue warps must resize all three.
  static constexpr int kEpiWarps = (kTcThreads - 64) / 32;
  static constexpr int kEpiArrivals = 2 * kEpiWarps;
  static_assert(kEpiWarps == 4, "one epilogue warp per TMEM lane quarter");
  static_assert(kEpiBytes == kEpiWarps * kEpiBlocks * kEpiWarpBytes, "staging blocks of every epilogue warp");
  // TMEM columns an epilogue warp reads: buf * kAccCols + h * 256 + [0, 256).
  static_assert((kAccBufs - 1) * kAccCols + kTileN <= kTmemCols, "accumulator columns inside the allocation");
  static_assert(kStages >= 3, "operand ring depth");
  // Descriptor offsets are whole 16-byte units, and every shared-memory
  // address fits the descriptor's 14-bit (address >> 4) field.
  static_assert(kStageBytes % 16 == 0 && kActBytes % 16 == 0 && kHalfWgtBytes % 16 == 0, "16-byte offsets");
  static_assert(kSmemBytes < (1 << 18), "addresses fit the descriptor field");
  static_assert(kSmemBytes <= 232448, "shared memory");
};

// This cluster's next work item (items first, first + stride, ...).  Without
// a tail split an item is one tile of the unit walk (half = -1).  With one
// (256 x 512 tile, exact tile count, one tile per unit) item i below
// p.tail_from is global tile i, and from there on consecutive items are the
// two 256-column halves (half = 0, 1) of one tile: a half item accumulates in
// TMEM columns [0, 256) from the weight columns of its half, which the
// producer loads into the first weight slot of the stage.
template <int NH, class Walk>
__device__ __forceinline__ bool next_item(Walk& walk, const GroupedParams& p, int64_t first, int64_t stride,
                                          int64_t& item, int64_t& t, int& half) {
  half = -1;
  if (NH != 2 || !p.tail_split) return walk.next_tile(p, first, stride, t);
  item = item < 0 ? first : item + stride;
  int64_t tile = item;
  if (item >= p.tail_from) {
    tile = p.tail_from + ((item - p.tail_from) >> 1);
    half = static_cast<int>((item - p.tail_from) & 1);
  }
  int64_t t0 = 0, t1 = 0;
  if (!walk.seek_unit(p, tile, 1, t0, t1)) return false;
  const int64_t next = item + stride;
  walk.prefetch_unit(p, next < p.tail_from ? next : p.tail_from + ((next - p.tail_from) >> 1), 1);
  t = t0;
  return true;
}

template <typename T, int NH>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kTcThreads, 1)
    tc2_grouped_kernel(const __grid_constant__ CUtensorMap act_tmpl, const __grid_constant__ CUtensorMap wgt_tmpl,
                       const __grid_constant__ CUtensorMap out_tmpl, const GroupedParams p) {
  using Cfg = Tc2Cfg<T, NH>;
  constexpr int S = Cfg::kStages;
  constexpr int NB = Cfg::kAccBufs;
  constexpr int BK = Cfg::kBK;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;
  uint8_t* epi_stage = smem + S * Cfg::kStageBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(epi_stage + Cfg::kEpiBytes);
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;
  uint64_t* acc_empty = acc_full + 2;  // NB of the two are used
  uint64_t* test_bar = acc_empty + 2;
  uint64_t* drain_bar = test_bar + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* never = abort + 1;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int64_t cluster = blockIdx.x >> 1;
  const int64_t clusters = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], Cfg::kEpiArrivals);
    }
    mbar_init(test_bar, 1);
    mbar_init(drain_bar, 1);
    *abort = 0;
    *never = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the peer's barriers exist before anything lands on them
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const long long budget = p.wait_budget;
  // Programmatic dependent launch behind build_maps_kernel: global memory is
  // read only from here on (see tc_grouped_kernel).
  grid_dependency_wait();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    const CUtensorMap* act_map = &act_tmpl;
    const CUtensorMap* wgt_map = &wgt_tmpl;
    if (p.single && lane == 0) {
      prefetch_tmap(act_map);
      prefetch_tmap(wgt_map);
    }
    // L2 hints: a weight block read by a single token tile is streamed
    // (evict-first); one that several token tiles share keeps normal priority
    // so the sharers hit in L2.  Activation blocks are shared by every weight
    // tile of their expert and are kept (evict-last).
    const uint64_t pol_stream = policy_evict_first();
    const uint64_t pol_shared = policy_evict_normal();
    const uint64_t pol_act = policy_evict_last();
    TileWalk<Cfg::kTileM, Cfg::kTileN> walk;
    uint32_t it = 0;
    int built = -1;
    int ahead_acquired = -1;  // problem whose maps were acquired one unit early
    bool ok = true;
    int64_t item = -1;
    int half = -1;
    for (int64_t t = 0; ok && next_item<NH>(walk, p, cluster, clusters, item, t, half);) {
      const Problem& q = walk.prob;
      if (!tile_legal<T>(p, q)) {
        if (lane == 0 && walk.problem != built) atomicOr(p.error_word, kErrMisaligned);
        continue;
      }
      const int64_t kblocks = (q.k + BK - 1) / BK;
      const uint64_t pol_wgt = walk.m_blocks > 1 ? pol_shared : pol_stream;
      const int32_t m0 = static_cast<int32_t>(walk.m_block(t) * Cfg::kTileM + rank * Cfg::kHalf);
      const int64_t nb = walk.n_block(t);
      for (int64_t kb = 0; kb < kblocks; ++kb) {
        const int s = static_cast<int>(it % S);
        const uint32_t phase = (it / S) & 1u;
        if (!mbar_wait_warp(&empty[s], phase ^ 1u, budget, abort)) {
          if (lane == 0) raise_error(p, kErrWaitEmpty, abort);
          ok = false;
          break;
        }
        if (kb == 0 && !p.single && walk.problem != built) {
          const CUtensorMap* g = problem_maps(p, walk.problem);  // built by build_maps_kernel
          if (lane == 0 && walk.problem != ahead_acquired) {
            tmap_acquire(&g[0]);
            tmap_acquire(&g[1]);
          }
          __syncwarp();
          act_map = &g[0];
          wgt_map = &g[1];
          built = walk.problem;
        }
        if (lane == 0) {
          uint8_t* st_act = ring + s * Cfg::kStageBytes;
          uint8_t* st_wgt = st_act + Cfg::kActBytes;
          const int32_t kx = static_cast<int32_t>(kb * BK);
          const uint32_t bar = mapa_shared(smem_u32(&full[s]), 0);
          // A half item loads one 256-column half of weights (into slot 0).
          const int slots = half < 0 ? NH : 1;
          if (leader) mbar_arrive_expect_tx(&full[s], 2 * (Cfg::kActBytes + slots * Cfg::kHalfWgtBytes));
          tma_load_2d_pair(act_map, bar, st_act, kx, m0, pol_act);
#pragma unroll
          for (int h = 0; h < NH; ++h) {
            if (h >= slots) break;
            const int hc = half < 0 ? h : half;  // weight half loaded into slot h
#pragma unroll
            for (int j = 0; j < Cfg::kHalf / BK; ++j) {
              // Tile-local column 256 hc + 128 rank + 64 j (CTA rank's half of MMA half hc).
              tma_load_2d_pair(wgt_map, bar, st_wgt + h * Cfg::kHalfWgtBytes + j * Cfg::kBoxBytes,
                               weight_col<Cfg::kTileN>(p, q, nb, 256 * hc + Cfg::kHalf * rank + j * BK), kx,
                               pol_wgt);
            }
          }
          if (kb == 0) acquire_ahead_maps(p, walk.ahead_problem, ahead_acquired, 2);
        }
        __syncwarp();
        ++it;
      }
    }
    if (*abort && leader && lane == 0) {
      const uint32_t first = it > static_cast<uint32_t>(S) ? it - S : 0u;
      for (uint32_t j = first; j < it; ++j) {
        if (!mbar_wait(&full[j % S], (j / S) & 1u, budget, never)) {
          atomicOr(p.error_word, kErrWaitTeardown);
          break;
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------- MMA issuer (even CTA only)
    if (lane == 0 && leader) {
      TileWalk<Cfg::kTileM, Cfg::kTileN> walk;
      uint32_t it = 0;
      uint32_t acc_it = 0;
      bool ok = true;
      int64_t item = -1;
      int half = -1;
      // Descriptors of stage 0's operands.  A stage, k-step or weight half is
      // an offset of the 14-bit start-address field (address >> 4); every
      // shared-memory address keeps that field below 2^14, so the 64-bit add
      // never carries out of it, and an MMA costs the issuer one add per
      // operand instead of assembling both descriptors.
      const uint64_t act_desc0 = smem_desc(smem_u32(ring), 16, 1024, kLayoutSw128);
      const uint64_t wgt_desc0 = smem_desc(smem_u32(ring) + Cfg::kActBytes, Cfg::kBoxBytes, 1024, kLayoutSw128);
      for (int64_t t = 0; ok && next_item<NH>(walk, p, cluster, clusters, item, t, half);) {
        const Problem& q = walk.prob;
        if (!tile_legal<T>(p, q) || q.k <= 0) continue;
        const int64_t kblocks = (q.k + BK - 1) / BK;
        const int buf = static_cast<int>(acc_it % NB);
        const uint32_t acc_phase = ((acc_it / NB) & 1u) ^ 1u;
        if (!mbar_wait(&acc_empty[buf], acc_phase, budget, abort)) {
          raise_error(p, kErrWaitAccEmpty, abort);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * Cfg::kAccCols);
        // MMAs of one 256-column half h over the four k-steps of stage s.
        auto issue_half = [&](int s, int h, bool first_kb) {
          const uint64_t stage = static_cast<uint64_t>(s * (Cfg::kStageBytes >> 4));
#pragma unroll
          for (int ks = 0; ks < Cfg::kKSteps; ++ks) {
            const uint64_t act_desc = act_desc0 + stage + ((ks * 32) >> 4);
            const uint64_t wgt_desc = wgt_desc0 + stage + ((h * Cfg::kHalfWgtBytes + ks * Cfg::kKStep * 128) >> 4);
            mma_f16_pair(d_tmem + h * 256, act_desc, wgt_desc, Cfg::kIdesc, (!first_kb || ks > 0) ? 1u : 0u);
          }
        };
        if (NH == 2 && half >= 0) {
          // Half item: every k-block on accumulator half 0 (free above).
          for (int64_t kb = 0; kb < kblocks; ++kb) {
            const int s = static_cast<int>(it % S);
            if (!mbar_wait(&full[s], (it / S) & 1u, budget, abort)) {
              raise_error(p, kErrWaitFull, abort);
              ok = false;
              break;
            }
            tc_fence_after();
            issue_half(s, 0, kb == 0);
            mma_commit_pair(&empty[s], 0x3);
            ++it;
          }
          if (!ok) break;
          // The epilogue arrives on both halves' barriers every item; wait on
          // half 1 as well (before this item's accumulator-full commit, so
          // that barrier is never two phases ahead of this wait).
          if (!mbar_wait(&acc_empty[1], acc_phase, budget, abort)) {
            raise_error(p, kErrWaitAccEmpty, abort);
            ok = false;
            break;
          }
          mma_commit_pair(&acc_full[buf], 0x3);
          ++acc_it;
          continue;
        }
        int64_t held = 0;
        if constexpr (NH == 2) {
          // Half 0 is free (acc_empty[0]): run the half-0 MMAs of the first
          // `held` k-blocks, keeping their stages, then wait for half 1
          // (acc_empty[1]) and finish those k-blocks before the usual order.
          held = kblocks < S ? kblocks : S;
          for (int64_t kb = 0; kb < held; ++kb) {
            const uint32_t j = it + static_cast<uint32_t>(kb);
            if (!mbar_wait(&full[j % S], (j / S) & 1u, budget, abort)) {
              raise_error(p, kErrWaitFull, abort);
              ok = false;
              break;
            }
            tc_fence_after();
            issue_half(static_cast<int>(j % S), 0, kb == 0);
          }
          if (!ok) break;
          if (!mbar_wait(&acc_empty[1], acc_phase, budget, abort)) {
            raise_error(p, kErrWaitAccEmpty, abort);
            ok = false;
            break;
          }
          tc_fence_after();
          for (int64_t kb = 0; kb < held; ++kb) {
            const int s = static_cast<int>((it + static_cast<uint32_t>(kb)) % S);
            issue_half(s, 1, kb == 0);
            mma_commit_pair(&empty[s], 0x3);  // frees stage s in both CTAs
          }
          it += static_cast<uint32_t>(held);
        }
        for (int64_t kb = held; kb < kblocks; ++kb) {
          const int s = static_cast<int>(it % S);
          if (!mbar_wait(&full[s], (it / S) & 1u, budget, abort)) {
            raise_error(p, kErrWaitFull, abort);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t stage = static_cast<uint64_t>(s * (Cfg::kStageBytes >> 4));
#pragma unroll
          for (int ks = 0; ks < Cfg::kKSteps; ++ks) {
            const uint64_t act_desc = act_desc0 + stage + ((ks * 32) >> 4);
#pragma unroll
            for (int h = 0; h < NH; ++h) {
              const uint64_t wgt_desc = wgt_desc0 + stage + ((h * Cfg::kHalfWgtBytes + ks * Cfg::kKStep * 128) >> 4);
              mma_f16_pair(d_tmem + h * 256, act_desc, wgt_desc, Cfg::kIdesc, (kb > 0 || ks > 0) ? 1u : 0u);
            }
          }
          mma_commit_pair(&empty[s], 0x3);  // frees stage s in both CTAs
          ++it;
        }
        if (!ok) break;
        mma_commit_pair(&acc_full[buf], 0x3);  // both epilogues may read their TMEM half
        ++acc_it;
      }
      if (*abort) {
        mma_commit_pair(drain_bar, 0x1);
        if (!mbar_wait(drain_bar, 0, budget, never)) atomicOr(p.error_word, kErrWaitTeardown);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    const int ethread = threadIdx.x - 64;
    if (p.test_flags & 1) {
      if (!mbar_wait_warp(test_bar, 0, budget, never) && lane == 0) atomicOr(p.error_word, kErrTestWait);
    }
    TileWalk<Cfg::kTileM, Cfg::kTileN> walk;
    uint32_t acc_it = 0;
    uint8_t* my_blocks = epi_stage + quarter * Cfg::kEpiBlocks * kEpiWarpBytes;
    int c_built = -1;
    const uint64_t pol_out = policy_evict_first();
    uint32_t chunk_seq = 0;
    bool ok = true;
    int64_t item = -1;
    int half = -1;
    for (int64_t t = 0; ok && next_item<NH>(walk, p, cluster, clusters, item, t, half);) {
      if (!tile_legal<T>(p, walk.prob)) continue;
      Problem q = walk.prob;
      q.n = out_cols(p, q);  // the epilogue addresses C: N/2 columns with SwiGLU
      const int tile_out = p.swiglu ? Cfg::kTileN / 2 : Cfg::kTileN;
      const int64_t m0 = walk.m_block(t) * Cfg::kTileM + rank * Cfg::kHalf;
      const int64_t n0 = walk.n_block(t) * tile_out;
      if (q.k <= 0) {
        for (int idx = ethread; idx < Cfg::kHalf * tile_out; idx += 128) {
          const int64_t row = m0 + idx / tile_out, col = n0 + idx % tile_out;
          if (row < q.m && col < q.n) {
            if (p.scatter_origin != nullptr) {
              char* d = scatter_row(p, q, row);
              if (d != nullptr) store_scalar<T>(d, col, 0.0f);
            } else {
              store_scalar<T>(q.c, row * q.scm + col * q.scn, 0.0f);
            }
          }
        }
        continue;
      }
      const void* cmap = c_tma_legal<T>(q, q.n) ? out_map_for(p, out_tmpl, walk.problem, c_built, lane) : nullptr;
      const int buf = static_cast<int>(acc_it % NB);
      if (!mbar_wait_warp(&acc_full[buf], (acc_it / NB) & 1u, budget, abort)) {
        if (lane == 0) raise_error(p, kErrWaitAccFull, abort);
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                             static_cast<uint32_t>(buf * Cfg::kAccCols);
      if (NH == 2 && half >= 0) {
        // Half item: TMEM half 1 is unused, free it at once; half 0 holds
        // output columns [n0 + 256 half, + 256).
        if (lane == 0) mbar_arrive_cluster_relaxed(mapa_shared(smem_u32(&acc_empty[1]), 0));
        const int64_t row0 = m0 + quarter * 32;
        const int64_t nh = n0 + half * 256;
        if (p.scatter_origin != nullptr) {
          store_rows_scatter<T, 256>(p, q, taddr, row0, nh, my_blocks, lane);
        } else if (cmap != nullptr) {
          store_rows_tma<T, 256, Cfg::kEpiBlocks>(q, cmap, taddr, static_cast<int32_t>(row0), static_cast<int32_t>(nh),
                                                  my_blocks, lane, chunk_seq, pol_out, p.error_word);
        } else {
          store_rows_staged<T, 256>(q, taddr, row0, nh, my_blocks, lane);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster_relaxed(mapa_shared(smem_u32(&acc_empty[0]), 0));
        ++acc_it;
        continue;
      }
      if (p.swiglu) {
        if (cmap != nullptr) {
          store_rows_tma_swiglu<T, Cfg::kTileN / 2, Cfg::kEpiBlocks>(q, cmap, taddr, static_cast<int32_t>(m0 + quarter * 32),
                                                    static_cast<int32_t>(n0), my_blocks, lane, chunk_seq, pol_out,
                                                    p.error_word);
        } else {
          store_rows_scalar_swiglu<T, Cfg::kTileN / 2>(q, taddr, m0 + quarter * 32, n0, lane);
        }
      } else if (NH == 2 && (p.scatter_origin != nullptr || cmap != nullptr)) {
        // By halves: each 256-column half is released as soon as it is drained.
        const int64_t row0 = m0 + quarter * 32;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t th = taddr + static_cast<uint32_t>(h * 256);
          const int64_t nh = n0 + h * 256;
          if (p.scatter_origin != nullptr) {
            store_rows_scatter<T, 256>(p, q, th, row0, nh, my_blocks, lane);
          } else {
            store_rows_tma<T, 256, Cfg::kEpiBlocks>(q, cmap, th, static_cast<int32_t>(row0), static_cast<int32_t>(nh),
                                                    my_blocks, lane, chunk_seq, pol_out, p.error_word);
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster_relaxed(mapa_shared(smem_u32(&acc_empty[h]), 0));
        }
        ++acc_it;
        continue;
      } else if (p.scatter_origin != nullptr) {
        store_rows_scatter<T, Cfg::kTileN>(p, q, taddr, m0 + quarter * 32, n0, my_blocks, lane);
      } else if (cmap != nullptr) {
        store_rows_tma<T, Cfg::kTileN, Cfg::kEpiBlocks>(q, cmap, taddr, static_cast<int32_t>(m0 + quarter * 32),
                                       static_cast<int32_t>(n0), my_blocks, lane, chunk_seq, pol_out, p.error_word);
      } else {
        store_rows_staged<T, Cfg::kTileN>(q, taddr, m0 + quarter * 32, n0, my_blocks, lane);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (NH == 2) {
          // Drained as a whole (SwiGLU pairs columns across the halves): free both.
          mbar_arrive_cluster_relaxed(mapa_shared(smem_u32(&acc_empty[0]), 0));
          mbar_arrive_cluster_relaxed(mapa_shared(smem_u32(&acc_empty[1]), 0));
        } else {
          mbar_arrive_cluster_relaxed(mapa_shared(smem_u32(&acc_empty[buf]), 0));
        }
      }
      ++acc_it;
    }
    if (lane == 0) bulk_wait_group_all();  // tensor stores done before the CTA's shared memory goes away
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // neither CTA leaves while the pair may still touch its memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
  }
}

}  // namespace mgb
