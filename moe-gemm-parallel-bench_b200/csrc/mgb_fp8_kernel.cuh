// Grouped FP8 GEMM with DeepSeek-V3 block scales, sm_100a.
//
//   C_e[M, N] (bf16) = sum over 128-deep K blocks kb of
//       (A_e[:, kb] @ B_e[:, kb]^T) * SA_e[m, kb] * SB_e[n / 128, kb]
//
// A_e: e4m3 [M, K] tokens, K contiguous; SA_e: fp32 [M, ceil(K/128)], one scale
// per token and 128-deep K block (the dynamic 1 x 128 activation blocks).
// B_e: e4m3 [N, K] as checkpoints store a linear weight (output x input
// features, K contiguous); SB_e: fp32 [ceil(N/128), ceil(K/128)], one scale
// per 128 x 128 weight block (quantization_config.weight_block_size of
// model_configs/deepseek-v3.json).  fp32 accumulation, one cast to bf16.
//
// The scales are arbitrary fp32 values, not the power-of-two scales the
// block-scaled MMA kinds take.  So every 128-deep K block is one group of four
// tcgen05.mma.kind::f8f6f4 (K = 32 each, both operands K-major) into a TMEM
// partial that starts from zero, and the epilogue warps "promote" it: read the
// partial, multiply by its token and weight-block scales and add it into fp32
// accumulators held in registers, while the MMA warp fills the other of two
// partial buffers with the next K block.
//
// Roles, as in tc_grouped_kernel:
//   warp 0      TMA producer (per stage: TM token rows and TN weight rows of
//               one 128-deep K block, 128 bytes per row, 128-byte swizzle)
//   warp 1      TMEM allocator; lane 0 issues the MMAs
//   warps 2..   promotion and the output stores (4 warps for swap-AB tiles,
//               8 for row tiles: warp w reads TMEM lanes 32 (w % 4) .. + 31)
// Tiles: SWAP (narrow M): MMA M = 128 weight rows per chunk (TN / 128
// chunks), MMA N = TM tokens; the lane owns a weight row, the registers hold
// its TM token columns.  Row tiles: MMA M = 128 tokens, N = TN = 128 weight
// rows (one scale block); eight promotion warps, two per TMEM lane quarter,
// each own a token row per lane and 64 of the 128 columns.
#pragma once

#include "mgb_tc_kernel.cuh"

namespace mgb {

constexpr int kFp8Block = 128;  // scale block along K (and along N for the weights)
constexpr int kScaleAhead = 4;  // row tiles: K blocks whose scales a promotion lane has in flight

template <bool SWAP, int TM, int TN>
struct Fp8Cfg {
  static constexpr int kBK = kFp8Block;  // K per stage: one 128-byte row, one scale block
  static constexpr int kActBytes = TM * 128;
  static constexpr int kWgtBytes = TN * 128;
  static constexpr int kStageBytes = kActBytes + kWgtBytes;
  // Row tiles promote with 8 warps (two per TMEM lane quarter, 64 columns
  // each): the promotion's FMAs are issued from every sub-partition twice
  // over, which keeps up with the MMA; swap-AB tiles need 4.
  // (10 warps put three on two sub-partitions, whose 16K registers then cap a
  // thread at 168: enough for 64 accumulators, not for the 128 a 128 x 256
  // row tile would need.)
  static constexpr int kEpiWarps = SWAP ? 4 : 8;
  static constexpr int kThreads = 64 + 32 * kEpiWarps;
  static constexpr int kWarpCols = SWAP ? 0 : TN / 2;  // row tiles: columns one promotion warp owns
  // One output staging block per warp: a warp stores a tile once per 128-deep
  // K loop, so double-buffering the stores buys nothing, while the shared
  // memory it frees deepens the operand ring (the FP8 MMA drains a stage in
  // half the time of a bf16 one, so the ring must hide twice as many stages
  // of L2 latency).
  static constexpr int kBlocksPerWarp = 1;
  static constexpr int kEpiBytes = SWAP ? 0 : kEpiWarps * kBlocksPerWarp * kEpiWarpBytes;
  static constexpr int kStagesRaw = (kTcSmemBudget - kEpiBytes) / kStageBytes;
  static constexpr int kStages = kStagesRaw > 12 ? 12 : kStagesRaw;
  static constexpr int kPartCols = SWAP ? (TN / 128) * TM : TN;  // TMEM columns of one partial
  // Partials in flight: the MMA runs up to kPartBufs - 1 K blocks ahead of
  // the promotion, whose per-block latency (barrier wake-up, TMEM load, FMAs)
  // exceeds one block's MMA time; as many as fit in TMEM, at most 4.
  static constexpr int kPartBufs = 512 / kPartCols >= 4 ? 4 : 2;
  static constexpr int kTmemCols = pow2_at_least(kPartBufs * kPartCols);
  // E4M3 x E4M3 (format code 0 for both operands), both K-major, fp32 D.
  static constexpr uint32_t kIdesc = SWAP ? instr_desc(0, 0, 0, 128, TM) : instr_desc(0, 0, 0, TM, TN);
  static constexpr int kSmemBytes = kStages * kStageBytes + kEpiBytes + 2048 + 1024;
  static_assert(TN % 128 == 0 && TN <= 256, "weight tile: whole 128-row scale blocks, one TMA box");
  static_assert(SWAP ? (TM % 16 == 0 && TM >= 16 && TM <= 64) : (TM == 128 && TN == 128), "token tile");
  static_assert(kStages >= 3, "operand ring depth");
  static_assert(kPartBufs * kPartCols <= 512, "the partials fit in TMEM");
  static_assert(kSmemBytes <= 232448, "shared memory");
};

// A problem runs when TMA can address its operands: 16-byte aligned bases,
// K a multiple of 16 (byte rows of A and B), N a multiple of 8 (bf16 C rows).
__device__ __forceinline__ bool fp8_legal(const Problem& q) {
  const uint64_t a = reinterpret_cast<uint64_t>(q.a), b = reinterpret_cast<uint64_t>(q.b),
                 c = reinterpret_cast<uint64_t>(q.c);
  return q.m > 0 && q.n > 0 && q.k >= 0 && a % 16 == 0 && b % 16 == 0 && c % 16 == 0 && q.k % 16 == 0 &&
         q.n % 8 == 0 && q.m < (1ll << 31) && q.n < (1ll << 31) && q.k < (1ll << 31);
}

// Tensor maps of every problem of an FP8 launch (one warp per problem), and
// in the extra block of a heterogeneous launch the walk's unit prefix sums.
// A: u8 [M, K] rows of K bytes; B: u8 [N, K]; C: bf16 [M, N].
__global__ void __launch_bounds__(32)
    build_fp8_maps_kernel(const __grid_constant__ CUtensorMap act_tmpl, const __grid_constant__ CUtensorMap wgt_tmpl,
                          const __grid_constant__ CUtensorMap out_tmpl, const GroupedParams p) {
  __shared__ alignas(128) CUtensorMap staging[kMapsPerProblem];
  const int e = blockIdx.x;
  const int lane = threadIdx.x;
  if (e == p.problem_count && p.unit_start != nullptr) {
    write_unit_prefix(p, lane);
    return;
  }
  if (e >= p.problem_count) return;
  if (lane == 0) {
    const Problem q = load_problem(p, e);
    const CUtensorMap* tmpl[kMapsPerProblem] = {&act_tmpl, &wgt_tmpl, &out_tmpl};
    for (int i = 0; i < kMapsPerProblem; ++i) {
      const uint4* src = reinterpret_cast<const uint4*>(tmpl[i]);
      uint4* dst = reinterpret_cast<uint4*>(&staging[i]);
      for (int j = 0; j < 8; ++j) dst[j] = src[j];
    }
    if (fp8_legal(q)) {
      tmap_replace_address(&staging[0], q.a);
      tmap_replace_address(&staging[1], q.b);
      tmap_replace_address(&staging[2], q.c);
      if (!p.homogeneous) {
        tmap_replace_dim(&staging[0], 0, static_cast<uint32_t>(q.k));
        tmap_replace_dim(&staging[0], 1, static_cast<uint32_t>(q.m));
        tmap_replace_stride1(&staging[0], static_cast<uint64_t>(q.k));
        tmap_replace_dim(&staging[1], 0, static_cast<uint32_t>(q.k));
        tmap_replace_dim(&staging[1], 1, static_cast<uint32_t>(q.n));
        tmap_replace_stride1(&staging[1], static_cast<uint64_t>(q.k));
        tmap_replace_dim(&staging[2], 0, static_cast<uint32_t>(q.n));
        tmap_replace_dim(&staging[2], 1, static_cast<uint32_t>(q.m));
        tmap_replace_stride1(&staging[2], static_cast<uint64_t>(q.n) * 2);
      }
    }
  }
  __syncwarp();
  CUtensorMap* g = reinterpret_cast<CUtensorMap*>(p.desc_slots) + static_cast<int64_t>(kMapsPerProblem) * e;
  for (int i = 0; i < kMapsPerProblem; ++i) tmap_publish(&g[i], &staging[i]);
}

// Row-tile output of one warp: 32 rows (one per lane) x 64 fp32
// accumulators in registers -> bf16, staged like store_rows_tma (in one of the
// warp's kBlocks 4 KB blocks) and written with one tensor store (TMA clips
// rows / columns past C).
template <int kBlocks, int OFF, int W>
__device__ __forceinline__ void store_acc_rows_tma(const Problem& q, const void* cmap, const float (&acc)[W],
                                                   int32_t row0, int32_t x0, uint8_t* blocks, int lane,
                                                   uint32_t& seq, uint64_t policy, uint32_t* error_word) {
  if (row0 >= q.m || x0 >= q.n) return;
  uint8_t* block = blocks + (kBlocks == 2 ? (seq & 1u) * kEpiWarpBytes : 0u);
  if (lane == 0) {
    if constexpr (kBlocks == 2) {
      bulk_wait_group_read<1>();  // the store issued from `block` two chunks ago has read it
    } else {
      bulk_wait_group_read<0>();  // the previous store from the single block has read it
    }
  }
  __syncwarp();
  uint8_t* my_row = block + lane * 128;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int o = OFF + 8 * j;  // compile-time after unrolling: acc stays in registers
    const uint4 packed = make_uint4(pack_pair<__nv_bfloat16>(__float_as_uint(acc[o]), __float_as_uint(acc[o + 1])),
                                    pack_pair<__nv_bfloat16>(__float_as_uint(acc[o + 2]), __float_as_uint(acc[o + 3])),
                                    pack_pair<__nv_bfloat16>(__float_as_uint(acc[o + 4]), __float_as_uint(acc[o + 5])),
                                    pack_pair<__nv_bfloat16>(__float_as_uint(acc[o + 6]), __float_as_uint(acc[o + 7])));
    *reinterpret_cast<uint4*>(my_row + ((j ^ (lane & 7)) << 4)) = packed;
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    if (x0 >= 0 && row0 >= 0) {
      tma_store_2d(cmap, block, x0, row0, policy);
      bulk_commit_group();
    } else {
      atomicOr(error_word, kErrBadStore);
    }
  }
  seq += 1;
}

template <bool SWAP, int TM, int TN>
__global__ void __launch_bounds__(Fp8Cfg<SWAP, TM, TN>::kThreads, 1)
    fp8_grouped_kernel(const __grid_constant__ CUtensorMap act_tmpl, const __grid_constant__ CUtensorMap wgt_tmpl,
                       const __grid_constant__ CUtensorMap out_tmpl, const GroupedParams p) {
  using Cfg = Fp8Cfg<SWAP, TM, TN>;
  constexpr int S = Cfg::kStages;
  constexpr int BK = Cfg::kBK;
  constexpr int kChunks = TN / 128;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;
  uint8_t* epi_stage = smem + S * Cfg::kStageBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(epi_stage + Cfg::kEpiBytes);
  uint64_t* empty = full + S;
  constexpr int NP = Cfg::kPartBufs;
  uint64_t* part_full = empty + S;        // [NP] MMA commit: a partial is ready
  uint64_t* part_empty = part_full + NP;  // [NP] every epilogue warp: a partial was read
  uint64_t* drain_bar = part_empty + NP;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* never = abort + 1;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < NP; ++b) {
      mbar_init(&part_full[b], 1);
      mbar_init(&part_empty[b], Cfg::kEpiWarps);
    }
    mbar_init(drain_bar, 1);
    *abort = 0;
    *never = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const long long budget = p.wait_budget;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    const CUtensorMap* act_map = &act_tmpl;
    const CUtensorMap* wgt_map = &wgt_tmpl;
    const uint64_t pol_stream = policy_evict_first();
    const uint64_t pol_shared = policy_evict_normal();
    const uint64_t pol_act = policy_evict_last();
    TileWalk<TM, TN> walk;
    uint32_t it = 0;
    int built = -1;
    bool ok = true;
    for (int64_t t = 0; ok && walk.next_tile(p, blockIdx.x, gridDim.x, t);) {
      const Problem& q = walk.prob;
      if (!fp8_legal(q)) {
        if (lane == 0 && walk.problem != built) atomicOr(p.error_word, kErrMisaligned);
        continue;
      }
      const int64_t kblocks = (q.k + BK - 1) / BK;
      const uint64_t pol_wgt = walk.m_blocks > 1 ? pol_shared : pol_stream;
      const int32_t m0 = static_cast<int32_t>(walk.m_block(t) * TM);
      const int32_t n0 = static_cast<int32_t>(walk.n_block(t) * TN);
      for (int64_t kb = 0; kb < kblocks; ++kb) {
        const int s = static_cast<int>(it % S);
        if (!mbar_wait_warp(&empty[s], ((it / S) & 1u) ^ 1u, budget, abort)) {
          if (lane == 0) raise_error(p, kErrWaitEmpty, abort);
          ok = false;
          break;
        }
        if (kb == 0 && walk.problem != built) {
          const CUtensorMap* g = problem_maps(p, walk.problem);  // built by build_fp8_maps_kernel
          if (lane == 0) {
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
          mbar_arrive_expect_tx(&full[s], Cfg::kStageBytes);
          tma_load_2d(act_map, &full[s], st_act, kx, m0, pol_act);
          tma_load_2d(wgt_map, &full[s], st_wgt, kx, n0, pol_wgt);
        }
        __syncwarp();
        ++it;
      }
    }
    if (*abort && lane == 0) {
      const uint32_t first = it > static_cast<uint32_t>(S) ? it - S : 0u;
      for (uint32_t j = first; j < it; ++j) {
        if (!mbar_wait(&full[j % S], (j / S) & 1u, budget, never)) {
          atomicOr(p.error_word, kErrWaitTeardown);
          break;
        }
      }
    }
  } else if (warp == 1) {
    // --------------------------------------------------------- MMA issuer
    if (lane == 0) {
      TileWalk<TM, TN> walk;
      uint32_t it = 0;
      uint32_t pit = 0;  // partials issued (all tiles)
      bool ok = true;
      for (int64_t t = 0; ok && walk.next_tile(p, blockIdx.x, gridDim.x, t);) {
        const Problem& q = walk.prob;
        if (!fp8_legal(q)) continue;
        const int64_t kblocks = (q.k + BK - 1) / BK;
        for (int64_t kb = 0; kb < kblocks; ++kb) {
          const int s = static_cast<int>(it % S);
          const int pb = static_cast<int>(pit % NP);
          if (!mbar_wait(&part_empty[pb], ((pit / NP) & 1u) ^ 1u, budget, abort)) {
            raise_error(p, kErrWaitAccEmpty, abort);
            ok = false;
            break;
          }
          if (!mbar_wait(&full[s], (it / S) & 1u, budget, abort)) {
            raise_error(p, kErrWaitFull, abort);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(pb * Cfg::kPartCols);
          const uint32_t a_base = smem_u32(ring + s * Cfg::kStageBytes);
          const uint32_t w_base = a_base + Cfg::kActBytes;
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {
            const uint32_t acc = ks > 0 ? 1u : 0u;  // every partial starts from zero
            const uint64_t act_desc = smem_desc(a_base + ks * 32, 16, 1024, kLayoutSw128);
            if constexpr (SWAP) {
#pragma unroll
              for (int c = 0; c < kChunks; ++c) {
                const uint64_t wgt_desc = smem_desc(w_base + c * 16384 + ks * 32, 16, 1024, kLayoutSw128);
                mma_f8(d_tmem + c * TM, wgt_desc, act_desc, Cfg::kIdesc, acc);
              }
            } else {
              const uint64_t wgt_desc = smem_desc(w_base + ks * 32, 16, 1024, kLayoutSw128);
              mma_f8(d_tmem, act_desc, wgt_desc, Cfg::kIdesc, acc);
            }
          }
          mma_commit(&empty[s]);
          mma_commit(&part_full[pb]);
          ++it;
          ++pit;
        }
      }
      if (*abort) {
        mma_commit(drain_bar);
        if (!mbar_wait(drain_bar, 0, budget, never)) atomicOr(p.error_word, kErrWaitTeardown);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------- promotion and the stores
    const int quarter = warp & 3;
    const int ew = warp - 2;                 // epilogue warp index
    const int half = SWAP ? 0 : ew / 4;      // row tiles: columns [TN/2 half, TN/2 half + TN/2)
    TileWalk<TM, TN> walk;
    uint32_t pit = 0;
    uint8_t* my_blocks = epi_stage + ew * Cfg::kBlocksPerWarp * kEpiWarpBytes;
    int c_built = -1;
    const uint64_t pol_out = policy_evict_first();
    uint32_t chunk_seq = 0;
    bool ok = true;
    for (int64_t t = 0; ok && walk.next_tile(p, blockIdx.x, gridDim.x, t);) {
      const Problem& q = walk.prob;
      if (!fp8_legal(q)) continue;
      const int64_t kblocks = (q.k + BK - 1) / BK;
      const int64_t m0 = walk.m_block(t) * TM;
      const int64_t n0 = walk.n_block(t) * TN;
      const float* sa = reinterpret_cast<const float*>(p.sa_ptrs[walk.problem]);
      const float* sb = reinterpret_cast<const float*>(p.sb_ptrs[walk.problem]);
      const void* cmap = nullptr;
      if constexpr (!SWAP) cmap = out_map_for(p, out_tmpl, walk.problem, c_built, lane);
      if constexpr (SWAP) {
        // Lane l owns weight row n0 + 128 c + 32 quarter + l of each chunk c;
        // acc[c][t] is its output for token m0 + t.
        float acc[kChunks][TM];
#pragma unroll
        for (int c = 0; c < kChunks; ++c) {
#pragma unroll
          for (int i = 0; i < TM; ++i) acc[c][i] = 0.0f;
        }
        const int64_t ta = m0 + lane, tb = m0 + lane + 32;  // tokens whose scales this lane fetches
        auto fetch = [&](int64_t kb, float& s_a0, float& s_a1, float (&s_b)[kChunks]) {
          s_a0 = (lane < TM && ta < q.m) ? sa[ta * kblocks + kb] : 0.0f;
          s_a1 = (lane + 32 < TM && tb < q.m) ? sa[tb * kblocks + kb] : 0.0f;
#pragma unroll
          for (int c = 0; c < kChunks; ++c) {
            const int64_t nblk = (n0 + c * 128) / kFp8Block;
            s_b[c] = n0 + c * 128 < q.n ? sb[nblk * kblocks + kb] : 0.0f;
          }
        };
        float na0 = 0.0f, na1 = 0.0f, nb[kChunks];
        if (kblocks > 0) fetch(0, na0, na1, nb);
        for (int64_t kb = 0; kb < kblocks; ++kb) {
          const float ca0 = na0, ca1 = na1;
          float cb[kChunks];
#pragma unroll
          for (int c = 0; c < kChunks; ++c) cb[c] = nb[c];
          if (kb + 1 < kblocks) fetch(kb + 1, na0, na1, nb);  // next block's scales in flight
          const int pb = static_cast<int>(pit % NP);
          if (!mbar_wait_warp(&part_full[pb], (pit / NP) & 1u, budget, abort)) {
            if (lane == 0) raise_error(p, kErrWaitAccFull, abort);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                                 static_cast<uint32_t>(pb * Cfg::kPartCols);
#pragma unroll
          for (int c = 0; c < kChunks; ++c) {
            uint32_t r[TM / 16][16];
#pragma unroll
            for (int j = 0; j < TM / 16; ++j) tmem_ld16(taddr + c * TM + j * 16, r[j]);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < TM; ++i) {
              const float s_tok = i < 32 ? __shfl_sync(0xffffffffu, ca0, i) : __shfl_sync(0xffffffffu, ca1, i - 32);
              acc[c][i] = fmaf(__uint_as_float(r[i / 16][i % 16]), s_tok * cb[c], acc[c][i]);
            }
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&part_empty[pb]);
          ++pit;
        }
        if (!ok) break;
#pragma unroll
        for (int c = 0; c < kChunks; ++c) {
          const int64_t col = n0 + c * 128 + quarter * 32 + lane;
          if (col < q.n) {
#pragma unroll
            for (int i = 0; i < TM; ++i) {
              const int64_t row = m0 + i;
              if (row < q.m) store_scalar<__nv_bfloat16>(q.c, row * q.n + col, acc[c][i]);
            }
          }
        }
      } else {
        // Lane l owns token row m0 + 32 quarter + l and columns
        // [W half, W half + W) of the tile (W = TN / 2, inside one scale block).
        constexpr int W = Cfg::kWarpCols;
        float acc[W];
#pragma unroll
        for (int i = 0; i < W; ++i) acc[i] = 0.0f;
        const int64_t row = m0 + quarter * 32 + lane;
        const int64_t nblk = (n0 + half * W) / kFp8Block;
        auto fetch = [&](int64_t kb) -> float {
          const float s_a = row < q.m ? sa[row * kblocks + kb] : 0.0f;
          return s_a * sb[nblk * kblocks + kb];
        };
        // The scales of the next kScaleAhead K blocks are in flight: a lane's
        // token scales are kblocks * 4 bytes apart from its neighbours', so
        // each fetch is one sector per lane with L2 latency to hide.
        float ring[kScaleAhead];
#pragma unroll
        for (int j = 0; j < kScaleAhead; ++j) ring[j] = j < kblocks ? fetch(j) : 0.0f;
        for (int64_t kb0 = 0; ok && kb0 < kblocks; kb0 += kScaleAhead) {
#pragma unroll
         for (int j = 0; j < kScaleAhead; ++j) {
          const int64_t kb = kb0 + j;
          if (kb >= kblocks) break;
          const float f = ring[j];
          if (kb + kScaleAhead < kblocks) ring[j] = fetch(kb + kScaleAhead);
          const int pb = static_cast<int>(pit % NP);
          if (!mbar_wait_warp(&part_full[pb], (pit / NP) & 1u, budget, abort)) {
            if (lane == 0) raise_error(p, kErrWaitAccFull, abort);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                                 static_cast<uint32_t>(pb * Cfg::kPartCols + half * W);
          if constexpr (W == 64) {
            uint32_t r0[32], r1[32];
            tmem_ld32(taddr, r0);
            tmem_ld32(taddr + 32, r1);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              acc[i] = fmaf(__uint_as_float(r0[i]), f, acc[i]);
              acc[32 + i] = fmaf(__uint_as_float(r1[i]), f, acc[32 + i]);
            }
          } else {
            // 128 accumulators per lane: one 32-column load in flight at a time.
#pragma unroll
            for (int h = 0; h < W / 32; ++h) {
              uint32_t r[32];
              tmem_ld32(taddr + h * 32, r);
              tmem_ld_wait();
#pragma unroll
              for (int i = 0; i < 32; ++i) acc[h * 32 + i] = fmaf(__uint_as_float(r[i]), f, acc[h * 32 + i]);
            }
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&part_empty[pb]);
          ++pit;
         }
        }
        if (!ok) break;
        if (cmap != nullptr) {
          const int32_t row0 = static_cast<int32_t>(m0 + quarter * 32);
          const int32_t x0 = static_cast<int32_t>(n0 + half * W);
          store_acc_rows_tma<Cfg::kBlocksPerWarp, 0>(q, cmap, acc, row0, x0, my_blocks, lane, chunk_seq, pol_out,
                                                     p.error_word);
          if constexpr (W == 128) {
            store_acc_rows_tma<Cfg::kBlocksPerWarp, 64>(q, cmap, acc, row0, x0 + 64, my_blocks, lane, chunk_seq,
                                                        pol_out, p.error_word);
          }
        }
      }
    }
    if (lane == 0) bulk_wait_group_all();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

// ------------------------------------------------------------------------
// CTA-pair FP8 tiles for token-rich problems: a cluster of two CTAs owns a
// 256-token x TN-weight-row output tile (TN = 128: one weight scale block;
// TN = 256: two).  CTA r loads token rows [128 r, 128 r + 128) and weight rows
// [TN/2 r, TN/2 r + TN/2) of every 128-deep K block into its own shared
// memory; the even CTA issues tcgen05.mma.cta_group::2.kind::f8f6f4
// (M = 256, N = TN), which reads both CTAs' halves and writes rows 0-127 /
// 128-255 of the partial into CTA 0 / 1's TMEM.  Per CTA and K block the
// 256 x 128 tile reads 24 KB from L2 for 128 x 128 x 128 MACs, the 256 x 256
// tile 32 KB for twice the MACs, and each of its MMAs does four times the
// work of a one-CTA 128 x 128 MMA.  Each CTA's eight promotion warps then work
// on their own 128 rows, two per TMEM lane quarter, each on TN / 2 columns
// (one scale block at TN = 256, with 128 fp32 accumulators a lane: see
// Fp8PairCfgT's register split).  Barriers as in tc2_grouped_kernel:
//   full[s]         in CTA 0 only: both CTAs' TMA bytes for stage s land on it
//   empty[s]        in each CTA: the MMA commit multicasts to both
//   part_full[b]    in each CTA: the MMA commit multicasts to both
//   part_empty[b]   in CTA 0 only: the 16 promotion warps of the pair arrive
template <int TN>
struct Fp8PairCfgT {
  static_assert(TN == 128 || TN == 256, "one or two 128-row weight scale blocks per cluster tile");
  static constexpr int kBK = kFp8Block;
  static constexpr int kTileM = 256;      // tokens per cluster tile
  static constexpr int kTileN = TN;       // weight rows per cluster tile
  static constexpr int kHalfM = 128;      // token rows per CTA
  static constexpr int kHalfN = TN / 2;   // weight rows per CTA
  static constexpr int kActBytes = kHalfM * 128;
  static constexpr int kWgtBytes = kHalfN * 128;
  static constexpr int kStageBytes = kActBytes + kWgtBytes;
  static constexpr int kEpiWarps = 8;
  // Warps before the promotion warps.  The 256-row tile keeps whole warpgroups
  // per role (producer, MMA issuer and two idle warps in warpgroup 0, the
  // promotion warps in warpgroups 1 and 2), so each warpgroup runs one
  // setmaxnreg: warpgroup 0 gives registers up, the promotion warpgroups take
  // them for their 128 accumulators per lane.
  static constexpr int kFirstEpiWarp = TN == 256 ? 4 : 2;
  static constexpr int kThreads = 32 * (kFirstEpiWarp + kEpiWarps);
  static constexpr bool kRegSplit = TN == 256;
  static constexpr int kRegsLow = 88;    // warpgroup 0 after setmaxnreg.dec
  static constexpr int kRegsHigh = 208;  // each promotion warpgroup after setmaxnreg.inc
  static constexpr int kWarpCols = kTileN / 2;  // columns one promotion warp owns (one scale block at TN = 256)
  static constexpr int kBlocksPerWarp = 1;  // as in Fp8Cfg: the freed shared memory deepens the ring
  static constexpr int kEpiBytes = kEpiWarps * kBlocksPerWarp * kEpiWarpBytes;
  static constexpr int kStagesRaw = (kTcSmemBudget - kEpiBytes) / kStageBytes;
  static constexpr int kStages = kStagesRaw > 12 ? 12 : kStagesRaw;
  static constexpr int kPartCols = kTileN;             // TMEM columns of one partial (this CTA's 128 rows)
  static constexpr int kPartBufs = TN == 256 ? 2 : 4;  // partials in flight (see Fp8Cfg); 512 TMEM columns
  static constexpr int kTmemCols = kPartBufs * kPartCols;
  static constexpr uint32_t kIdesc = instr_desc(0, 0, 0, kTileM, kTileN);  // E4M3 x E4M3, both K-major
  static constexpr int kSmemBytes = kStages * kStageBytes + kEpiBytes + 2048 + 1024;
  static_assert(kStages >= 3, "operand ring depth");
  static_assert(kSmemBytes <= 232448, "shared memory");
  static_assert(kTmemCols <= 512, "partials fit in TMEM");
  // The split hands out no more than the block was launched with: at most
  // 168 registers a thread for 384 threads (the host also checks the
  // compiled kernel's count before the first launch).
  static_assert(!kRegSplit || (kFirstEpiWarp == 4 && 128 * kRegsLow + 32 * kEpiWarps * kRegsHigh <= kThreads * 168),
                "register split within the launch's registers");
  static_assert(kRegsLow % 8 == 0 && kRegsHigh % 8 == 0 && kRegsLow >= 24 && kRegsHigh <= 256, "setmaxnreg range");
};
using Fp8PairCfg = Fp8PairCfgT<128>;

template <int TN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(Fp8PairCfgT<TN>::kThreads, 1)
    fp8_pair_kernel(const __grid_constant__ CUtensorMap act_tmpl, const __grid_constant__ CUtensorMap wgt_tmpl,
                    const __grid_constant__ CUtensorMap out_tmpl, const GroupedParams p) {
  using Cfg = Fp8PairCfgT<TN>;
  constexpr int S = Cfg::kStages;
  constexpr int BK = Cfg::kBK;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;
  uint8_t* epi_stage = smem + S * Cfg::kStageBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(epi_stage + Cfg::kEpiBytes);
  uint64_t* empty = full + S;
  constexpr int NP = Cfg::kPartBufs;
  uint64_t* part_full = empty + S;
  uint64_t* part_empty = part_full + NP;
  uint64_t* drain_bar = part_empty + NP;
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
    for (int b = 0; b < NP; ++b) {
      mbar_init(&part_full[b], 1);
      mbar_init(&part_empty[b], 2 * Cfg::kEpiWarps);
    }
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

  if (warp < Cfg::kFirstEpiWarp) {
   if constexpr (Cfg::kRegSplit) setmaxnreg_dec<Cfg::kRegsLow>();
   if (warp == 0) {
    // ------------------------------------------------------------ producer
    const CUtensorMap* act_map = &act_tmpl;
    const CUtensorMap* wgt_map = &wgt_tmpl;
    const uint64_t pol_stream = policy_evict_first();
    const uint64_t pol_shared = policy_evict_normal();
    const uint64_t pol_act = policy_evict_last();
    TileWalk<Cfg::kTileM, Cfg::kTileN> walk;
    uint32_t it = 0;
    int built = -1;
    bool ok = true;
    for (int64_t t = 0; ok && walk.next_tile(p, cluster, clusters, t);) {
      const Problem& q = walk.prob;
      if (!fp8_legal(q)) {
        if (lane == 0 && walk.problem != built) atomicOr(p.error_word, kErrMisaligned);
        continue;
      }
      const int64_t kblocks = (q.k + BK - 1) / BK;
      const uint64_t pol_wgt = walk.m_blocks > 1 ? pol_shared : pol_stream;
      const int32_t m0 = static_cast<int32_t>(walk.m_block(t) * Cfg::kTileM + rank * Cfg::kHalfM);
      const int32_t n0 = static_cast<int32_t>(walk.n_block(t) * Cfg::kTileN + rank * Cfg::kHalfN);
      for (int64_t kb = 0; kb < kblocks; ++kb) {
        const int s = static_cast<int>(it % S);
        if (!mbar_wait_warp(&empty[s], ((it / S) & 1u) ^ 1u, budget, abort)) {
          if (lane == 0) raise_error(p, kErrWaitEmpty, abort);
          ok = false;
          break;
        }
        if (kb == 0 && walk.problem != built) {
          const CUtensorMap* g = problem_maps(p, walk.problem);  // built by build_fp8_maps_kernel
          if (lane == 0) {
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
          if (leader) mbar_arrive_expect_tx(&full[s], 2 * Cfg::kStageBytes);
          tma_load_2d_pair(act_map, bar, st_act, kx, m0, pol_act);
          tma_load_2d_pair(wgt_map, bar, st_wgt, kx, n0, pol_wgt);
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
      uint32_t pit = 0;
      bool ok = true;
      for (int64_t t = 0; ok && walk.next_tile(p, cluster, clusters, t);) {
        const Problem& q = walk.prob;
        if (!fp8_legal(q)) continue;
        const int64_t kblocks = (q.k + BK - 1) / BK;
        for (int64_t kb = 0; kb < kblocks; ++kb) {
          const int s = static_cast<int>(it % S);
          const int pb = static_cast<int>(pit % NP);
          if (!mbar_wait(&part_empty[pb], ((pit / NP) & 1u) ^ 1u, budget, abort)) {
            raise_error(p, kErrWaitAccEmpty, abort);
            ok = false;
            break;
          }
          if (!mbar_wait(&full[s], (it / S) & 1u, budget, abort)) {
            raise_error(p, kErrWaitFull, abort);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(pb * Cfg::kPartCols);
          const uint32_t a_base = smem_u32(ring + s * Cfg::kStageBytes);
          const uint32_t w_base = a_base + Cfg::kActBytes;
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {
            const uint64_t act_desc = smem_desc(a_base + ks * 32, 16, 1024, kLayoutSw128);
            const uint64_t wgt_desc = smem_desc(w_base + ks * 32, 16, 1024, kLayoutSw128);
            mma_f8_pair(d_tmem, act_desc, wgt_desc, Cfg::kIdesc, ks > 0 ? 1u : 0u);
          }
          mma_commit_pair(&empty[s], 0x3);      // frees stage s in both CTAs
          mma_commit_pair(&part_full[pb], 0x3);  // both CTAs' promotion warps may read
          ++it;
          ++pit;
        }
      }
      if (*abort) {
        mma_commit_pair(drain_bar, 0x1);
        if (!mbar_wait(drain_bar, 0, budget, never)) atomicOr(p.error_word, kErrWaitTeardown);
      }
    }
    __syncwarp();
   }
  } else {
    // ------------------------------------------- promotion and the stores
    if constexpr (Cfg::kRegSplit) setmaxnreg_inc<Cfg::kRegsHigh>();
    constexpr int W = Cfg::kWarpCols;
    const int quarter = warp & 3;  // TMEM lane quarter this warp may read
    const int ew = warp - Cfg::kFirstEpiWarp;
    const int half = ew / 4;       // columns [W half, W half + W) of the tile
    TileWalk<Cfg::kTileM, Cfg::kTileN> walk;
    uint32_t pit = 0;
    uint8_t* my_blocks = epi_stage + ew * Cfg::kBlocksPerWarp * kEpiWarpBytes;
    int c_built = -1;
    const uint64_t pol_out = policy_evict_first();
    uint32_t chunk_seq = 0;
    bool ok = true;
    for (int64_t t = 0; ok && walk.next_tile(p, cluster, clusters, t);) {
      const Problem& q = walk.prob;
      if (!fp8_legal(q)) continue;
      const int64_t kblocks = (q.k + BK - 1) / BK;
      const int64_t m0 = walk.m_block(t) * Cfg::kTileM + rank * Cfg::kHalfM;
      const int64_t n0 = walk.n_block(t) * Cfg::kTileN;
      const float* sa = reinterpret_cast<const float*>(p.sa_ptrs[walk.problem]);
      const float* sb = reinterpret_cast<const float*>(p.sb_ptrs[walk.problem]);
      const void* cmap = out_map_for(p, out_tmpl, walk.problem, c_built, lane);
      float acc[W];
#pragma unroll
      for (int i = 0; i < W; ++i) acc[i] = 0.0f;
      const int64_t row = m0 + quarter * 32 + lane;
      // This warp's columns lie in one scale block; on the last N tile of the
      // 256-row tile they may all lie past N, where no weight scale exists
      // (those columns are neither computed from real rows nor stored).
      const int64_t nblk = (n0 + half * W) / kFp8Block;
      const bool cols_in = n0 + half * W < q.n;
      auto fetch = [&](int64_t kb) -> float {
        const float s_a = row < q.m ? sa[row * kblocks + kb] : 0.0f;
        return cols_in ? s_a * sb[nblk * kblocks + kb] : 0.0f;
      };
      float ring[kScaleAhead];  // scales of the next K blocks in flight, as in fp8_grouped_kernel
#pragma unroll
      for (int j = 0; j < kScaleAhead; ++j) ring[j] = j < kblocks ? fetch(j) : 0.0f;
      for (int64_t kb0 = 0; ok && kb0 < kblocks; kb0 += kScaleAhead) {
#pragma unroll
       for (int j = 0; j < kScaleAhead; ++j) {
        const int64_t kb = kb0 + j;
        if (kb >= kblocks) break;
        const float f = ring[j];
        if (kb + kScaleAhead < kblocks) ring[j] = fetch(kb + kScaleAhead);
        const int pb = static_cast<int>(pit % NP);
        if (!mbar_wait_warp(&part_full[pb], (pit / NP) & 1u, budget, abort)) {
          if (lane == 0) raise_error(p, kErrWaitAccFull, abort);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                               static_cast<uint32_t>(pb * Cfg::kPartCols + half * W);
#pragma unroll
        for (int g = 0; g < W / 64; ++g) {  // 64 columns (two loads) in flight at a time
          uint32_t r0[32], r1[32];
          tmem_ld32(taddr + g * 64, r0);
          tmem_ld32(taddr + g * 64 + 32, r1);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            acc[g * 64 + i] = fmaf(__uint_as_float(r0[i]), f, acc[g * 64 + i]);
            acc[g * 64 + 32 + i] = fmaf(__uint_as_float(r1[i]), f, acc[g * 64 + 32 + i]);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster_relaxed(mapa_shared(smem_u32(&part_empty[pb]), 0));
        ++pit;
       }
      }
      if (!ok) break;
      if (cmap != nullptr) {
        const int32_t row0 = static_cast<int32_t>(m0 + quarter * 32);
        const int32_t x0 = static_cast<int32_t>(n0 + half * W);
        store_acc_rows_tma<Cfg::kBlocksPerWarp, 0>(q, cmap, acc, row0, x0, my_blocks, lane, chunk_seq, pol_out,
                                                   p.error_word);
        if constexpr (W == 128) {
          store_acc_rows_tma<Cfg::kBlocksPerWarp, 64>(q, cmap, acc, row0, x0 + 64, my_blocks, lane, chunk_seq,
                                                      pol_out, p.error_word);
        }
      }
    }
    if (lane == 0) bulk_wait_group_all();
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
