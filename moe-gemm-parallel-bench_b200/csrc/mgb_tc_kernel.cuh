// Persistent, warp-specialised grouped GEMM for sm_100a: TMA loads into a
// multi-stage 128B-swizzled shared-memory ring, tcgen05.mma accumulating in
// TMEM (two accumulator buffers so the epilogue of one tile overlaps the MMAs
// of the next), and a tcgen05.ld epilogue that converts and stores C.
//
// Computes, for every problem e of a launch, C_e = A_e @ B_e with fp32
// accumulation and a cast on store -- the contract of the reference's
// persistent kernels (kernels/grouped_gemm.py:321-397 homogeneous,
// :399-482 generic) and of its single GEMM (kernels/matmul.py:223-273).
//
// Roles (192 threads):
//   warp 0      TMA producer.  Rebuilds the per-problem tensor maps in a
//               per-CTA global slot when the walk enters a new problem.
//   warp 1      TMEM allocator; lane 0 issues every tcgen05.mma.
//   warps 2..5  epilogue (TMEM lanes 32*(warp%4) .. +31).
//
// Two operand orientations:
//   SWAP = false  MMA M = TM tokens (128), MMA N = TN weight columns.
//   SWAP = true   "swap-AB" for narrow M_e: MMA M = 128 weight columns, MMA N =
//                 TM tokens, so a 16-row expert still drives a 128-wide MMA and
//                 the kernel streams every weight byte exactly once.
// A (activations, [M,K] K contiguous) is always the K-major operand; B (weights,
// [K,N] N contiguous) is always the MN-major operand.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>
#include <type_traits>

#include "mgb_common.cuh"
#include "mgb_ptx.cuh"

namespace mgb {

constexpr int kTcThreads = 192;
constexpr int kTcStageBudget = 220 * 1024;  // shared memory given to the operand ring

constexpr int pow2_at_least(int v) {
  int p = 32;
  while (p < v) p <<= 1;
  return p;
}

template <typename T, bool SWAP, int TM, int TN>
struct TcCfg {
  static constexpr int kElem = static_cast<int>(sizeof(T));
  static constexpr int kBK = 128 / kElem;       // K elements per stage: one 128-byte swizzle row
  static constexpr int kKStep = 32 / kElem;     // K per tcgen05.mma (32 bytes of K)
  static constexpr int kKSteps = kBK / kKStep;  // 4
  static constexpr int kActBytes = TM * 128;
  static constexpr int kBoxBytes = kBK * 128;  // one weight box: kBK columns x kBK K-rows
  static constexpr int kWgtBytes = TN * 128;   // TN / kBK boxes
  static constexpr int kStageBytes = kActBytes + kWgtBytes;
  static constexpr int kStagesRaw = kTcStageBudget / kStageBytes;
  static constexpr int kStages = kStagesRaw > 12 ? 12 : kStagesRaw;
  static constexpr int kSlots = kStages + 1;  // tensor-map slots per CTA (see producer)
  static constexpr int kAccCols = SWAP ? (TN / 128) * TM : TN;
  static constexpr int kTmemCols = pow2_at_least(2 * kAccCols);
  static constexpr uint32_t kFmt = std::is_same<T, float>::value ? 2u
                                   : std::is_same<T, __nv_bfloat16>::value ? 1u
                                                                            : 0u;
  static constexpr uint32_t kIdesc = SWAP ? instr_desc(kFmt, 1, 0, 128, TM) : instr_desc(kFmt, 0, 1, TM, TN);
  static constexpr int kSmemBytes = kStages * kStageBytes + 2048 + 1024;
  // The weight operand is MN-major.  For 16-bit types it uses the plain
  // 128-byte swizzle (8-row K atoms, SBO 1024); MN-major TF32 admits only the
  // 32-byte-granule variant (4-row K atoms, SBO 512), loaded by TMA with the
  // matching 128B_ATOM_32B swizzle.
  static constexpr uint32_t kWgtLayout = kElem == 4 ? kLayoutSw128Base32 : kLayoutSw128;
  static constexpr uint32_t kWgtSbo = kElem == 4 ? 512u : 1024u;

  static_assert(kStages >= 2, "operand ring needs at least two stages");
  static_assert(TM % 16 == 0 && TM >= 16 && TM <= 256, "token tile");
  static_assert(SWAP || TM == 128, "non-swapped tiles use MMA M = 128");
  static_assert(TN % 128 == 0 || (!SWAP && TN == 64), "weight tile");
  static_assert(2 * kAccCols <= 512, "two accumulators must fit in TMEM");
  static_assert(kSmemBytes <= 232448, "shared memory");
};

// A problem is served by the TMA path when its operands satisfy the TMA rules:
// 16-byte aligned bases, unit inner strides, row strides that are multiples of
// 16 bytes, and extents that fit the 32-bit tensor-map fields.
template <typename T>
__device__ __forceinline__ bool tma_legal(const Problem& q) {
  constexpr int E = static_cast<int>(sizeof(T));
  const uint64_t a = reinterpret_cast<uint64_t>(q.a), b = reinterpret_cast<uint64_t>(q.b);
  return (a % 16 == 0) && (b % 16 == 0) && q.sak == 1 && q.sbn == 1 && (q.sam * E) % 16 == 0 &&
         (q.sbk * E) % 16 == 0 && q.sam > 0 && q.sbk > 0 && q.m < (1ll << 31) && q.n < (1ll << 31) &&
         q.k < (1ll << 31);
}

__device__ __forceinline__ void raise_error(const GroupedParams& p, uint32_t bits, volatile int* abort) {
  atomicOr(p.error_word, bits);
  if (abort != nullptr) *abort = 1;
}

// Warp-uniform bounded wait: every lane observes the barrier, lane 0 owns the
// clock, and the verdict is the same for the whole warp (so warp-collective
// instructions that follow never see a split warp).
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity, long long budget, volatile int* abort) {
  const long long start = clock64();
  while (true) {
    const bool done = mbar_try_wait(bar, parity);
    if (__all_sync(0xffffffffu, done)) return true;
    int stop = 0;
    if ((threadIdx.x & 31) == 0) stop = (*abort != 0) || (clock64() - start > budget);
    if (__shfl_sync(0xffffffffu, stop, 0)) return false;
  }
}

template <typename T>
__device__ __forceinline__ void store_scalar(char* base, int64_t elem_offset, float v) {
  T* ptr = reinterpret_cast<T*>(base) + elem_offset;
  if constexpr (std::is_same<T, float>::value) {
    *ptr = v;
  } else if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    *ptr = __float2bfloat16_rn(v);
  } else {
    *ptr = __float2half_rn(v);
  }
}

// 16 consecutive columns of one row: vector stores when the row segment is
// whole, contiguous and 16-byte aligned; element stores otherwise.
template <typename T>
__device__ __forceinline__ void store_row16(const Problem& q, int64_t row, int64_t col0, const uint32_t (&r)[16]) {
  if (row >= q.m) return;
  char* dst = q.c + (row * q.scm + col0 * q.scn) * static_cast<int64_t>(sizeof(T));
  const bool whole = (q.scn == 1) && (col0 + 16 <= q.n) && (reinterpret_cast<uint64_t>(dst) % 16 == 0);
  if (whole) {
    if constexpr (std::is_same<T, float>::value) {
      uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
      for (int i = 0; i < 4; ++i) d[i] = make_uint4(r[4 * i], r[4 * i + 1], r[4 * i + 2], r[4 * i + 3]);
    } else {
      uint32_t packed[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float lo = __uint_as_float(r[2 * i]), hi = __uint_as_float(r[2 * i + 1]);
        if constexpr (std::is_same<T, __nv_bfloat16>::value) {
          __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
          packed[i] = *reinterpret_cast<uint32_t*>(&h);
        } else {
          __half2 h = __floats2half2_rn(lo, hi);
          packed[i] = *reinterpret_cast<uint32_t*>(&h);
        }
      }
      uint4* d = reinterpret_cast<uint4*>(dst);
      d[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
      d[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
    }
    return;
  }
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int64_t col = col0 + i;
    if (col < q.n) store_scalar<T>(q.c, row * q.scm + col * q.scn, __uint_as_float(r[i]));
  }
}

template <typename T, bool SWAP, int TM, int TN>
__global__ void __launch_bounds__(kTcThreads, 1)
    tc_grouped_kernel(const __grid_constant__ CUtensorMap act_tmpl, const __grid_constant__ CUtensorMap wgt_tmpl,
                      const GroupedParams p) {
  using Cfg = TcCfg<T, SWAP, TM, TN>;
  constexpr int S = Cfg::kStages;
  constexpr int BK = Cfg::kBK;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * Cfg::kStageBytes);
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* test_bar = acc_empty + 2;  // never arrived on: the test-only bounded-wait probe
  uint64_t* drain_bar = test_bar + 1;  // teardown: waits for MMAs in flight after an abort
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);  // raised by a role that gave up
  volatile int* never = abort + 1;  // stays 0: for waits no abort may cut short
  CUtensorMap* staging = reinterpret_cast<CUtensorMap*>(
      (reinterpret_cast<uintptr_t>(tmem_slot + 4) + 127) & ~uintptr_t(127));  // [act, wgt]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
    }
    mbar_init(test_bar, 1);
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
    CUtensorMap* slots = reinterpret_cast<CUtensorMap*>(p.desc_slots) +
                         static_cast<int64_t>(blockIdx.x) * Cfg::kSlots * 2;
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
    TileWalk<TM, TN> walk;
    uint32_t it = 0;
    int slot = -1;
    int built = -1;
    bool ok = true;
    for (int64_t t = blockIdx.x; ok && walk.seek(p, t); t += gridDim.x) {
      const Problem& q = walk.prob;
      if (!tma_legal<T>(q)) {
        if (lane == 0 && walk.problem != built) atomicOr(p.error_word, kErrMisaligned);
        continue;
      }
      const int64_t kblocks = (q.k + BK - 1) / BK;
      const uint64_t pol_wgt = walk.m_blocks > 1 ? pol_shared : pol_stream;
      const int32_t m0 = static_cast<int32_t>(walk.m_block(t) * TM);
      const int32_t n0 = static_cast<int32_t>(walk.n_block(t) * TN);
      for (int64_t kb = 0; kb < kblocks; ++kb) {
        const int s = static_cast<int>(it % S);
        const uint32_t phase = (it / S) & 1u;
        if (!mbar_wait_warp(&empty[s], phase ^ 1u, budget, abort)) {
          if (lane == 0) raise_error(p, kErrWaitEmpty, abort);
          ok = false;
          break;
        }
        if (kb == 0 && !p.single && walk.problem != built) {
          // Entering a new problem: rebuild its two tensor maps in the next
          // slot.  A slot is reused only kSlots problems later; each problem
          // issues at least one load, so by then the stage wait just above
          // has proven that every load that read the old maps has landed.
          slot = (slot + 1) % Cfg::kSlots;
          uint64_t* st = reinterpret_cast<uint64_t*>(staging);
          st[lane] = lane < 16 ? reinterpret_cast<const uint64_t*>(&act_tmpl)[lane]
                               : reinterpret_cast<const uint64_t*>(&wgt_tmpl)[lane - 16];
          __syncwarp();
          if (lane == 0) {
            tmap_replace_address(&staging[0], q.a);
            tmap_replace_address(&staging[1], q.b);
            if (!p.homogeneous) {
              tmap_replace_dim(&staging[0], 0, static_cast<uint32_t>(q.k));
              tmap_replace_dim(&staging[0], 1, static_cast<uint32_t>(q.m));
              tmap_replace_stride1(&staging[0], static_cast<uint64_t>(q.sam) * sizeof(T));
              tmap_replace_dim(&staging[1], 0, static_cast<uint32_t>(q.n));
              tmap_replace_dim(&staging[1], 1, static_cast<uint32_t>(q.k));
              tmap_replace_stride1(&staging[1], static_cast<uint64_t>(q.sbk) * sizeof(T));
            }
          }
          __syncwarp();
          CUtensorMap* g = slots + 2 * slot;
          tmap_publish(&g[0], &staging[0]);
          tmap_publish(&g[1], &staging[1]);
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
#pragma unroll
          for (int j = 0; j < TN / BK; ++j) {
            tma_load_2d(wgt_map, &full[s], st_wgt + j * Cfg::kBoxBytes, n0 + j * BK, kx, pol_wgt);
          }
        }
        __syncwarp();
        ++it;
      }
    }
    if (*abort && lane == 0) {
      // Let the loads already issued land before the CTA's shared memory goes away.
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
      uint32_t acc_it = 0;
      bool ok = true;
      for (int64_t t = blockIdx.x; ok && walk.seek(p, t); t += gridDim.x) {
        const Problem& q = walk.prob;
        if (!tma_legal<T>(q) || q.k <= 0) continue;
        const int64_t kblocks = (q.k + BK - 1) / BK;
        const int buf = static_cast<int>(acc_it & 1u);
        if (!mbar_wait(&acc_empty[buf], ((acc_it >> 1) & 1u) ^ 1u, budget, abort)) {
          raise_error(p, kErrWaitAccEmpty, abort);
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * Cfg::kAccCols);
        for (int64_t kb = 0; kb < kblocks; ++kb) {
          const int s = static_cast<int>(it % S);
          if (!mbar_wait(&full[s], (it / S) & 1u, budget, abort)) {
            raise_error(p, kErrWaitFull, abort);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(ring + s * Cfg::kStageBytes);
          const uint32_t w_base = a_base + Cfg::kActBytes;
#pragma unroll
          for (int ks = 0; ks < Cfg::kKSteps; ++ks) {
            const uint32_t acc = (kb > 0 || ks > 0) ? 1u : 0u;
            const uint64_t act_desc = smem_desc(a_base + ks * 32, 16, 1024, kLayoutSw128);
            if constexpr (SWAP) {
#pragma unroll
              for (int c = 0; c < TN / 128; ++c) {
                const uint64_t wgt_desc = smem_desc(w_base + c * 16384 + ks * Cfg::kKStep * 128, Cfg::kBoxBytes,
                                                    Cfg::kWgtSbo, Cfg::kWgtLayout);
                if constexpr (std::is_same<T, float>::value) {
                  mma_tf32(d_tmem + c * TM, wgt_desc, act_desc, Cfg::kIdesc, acc);
                } else {
                  mma_f16(d_tmem + c * TM, wgt_desc, act_desc, Cfg::kIdesc, acc);
                }
              }
            } else {
              const uint64_t wgt_desc =
                  smem_desc(w_base + ks * Cfg::kKStep * 128, Cfg::kBoxBytes, Cfg::kWgtSbo, Cfg::kWgtLayout);
              if constexpr (std::is_same<T, float>::value) {
                mma_tf32(d_tmem, act_desc, wgt_desc, Cfg::kIdesc, acc);
              } else {
                mma_f16(d_tmem, act_desc, wgt_desc, Cfg::kIdesc, acc);
              }
            }
          }
          mma_commit(&empty[s]);  // frees the stage once these MMAs have read it
          ++it;
        }
        if (!ok) break;
        mma_commit(&acc_full[buf]);  // accumulator ready for the epilogue
        ++acc_it;
      }
      if (*abort) {
        mma_commit(drain_bar);
        if (!mbar_wait(drain_bar, 0, budget, never)) {
          atomicOr(p.error_word, kErrWaitTeardown);
        }
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;  // TMEM lanes this warp may read
    const int ethread = threadIdx.x - 64;
    if (p.test_flags & 1) {
      // Test hook: a barrier nothing arrives on must time out, be reported,
      // and leave the launch (and the context) intact.
      if (!mbar_wait_warp(test_bar, 0, budget, never) && lane == 0) {
        atomicOr(p.error_word, kErrTestWait);
      }
    }
    TileWalk<TM, TN> walk;
    uint32_t acc_it = 0;
    for (int64_t t = blockIdx.x; walk.seek(p, t); t += gridDim.x) {
      const Problem& q = walk.prob;
      if (!tma_legal<T>(q)) continue;
      const int64_t m0 = walk.m_block(t) * TM;
      const int64_t n0 = walk.n_block(t) * TN;
      if (q.k <= 0) {
        for (int idx = ethread; idx < TM * TN; idx += 128) {
          const int64_t row = m0 + idx / TN, col = n0 + idx % TN;
          if (row < q.m && col < q.n) store_scalar<T>(q.c, row * q.scm + col * q.scn, 0.0f);
        }
        continue;
      }
      const int buf = static_cast<int>(acc_it & 1u);
      if (!mbar_wait_warp(&acc_full[buf], (acc_it >> 1) & 1u, budget, abort)) {
        if (lane == 0) raise_error(p, kErrWaitAccFull, abort);
        break;
      }
      tc_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                             static_cast<uint32_t>(buf * Cfg::kAccCols);
      if constexpr (SWAP) {
#pragma unroll 1
        for (int c = 0; c < TN / 128; ++c) {
          const int64_t col = n0 + c * 128 + quarter * 32 + lane;
#pragma unroll 1
          for (int j = 0; j < TM / 16; ++j) {
            uint32_t r[16];
            tmem_ld16(taddr + c * TM + j * 16, r);
            tmem_ld_wait();
            if (col < q.n) {
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                const int64_t row = m0 + j * 16 + i;
                if (row < q.m) store_scalar<T>(q.c, row * q.scm + col * q.scn, __uint_as_float(r[i]));
              }
            }
          }
        }
      } else {
        const int64_t row = m0 + quarter * 32 + lane;
#pragma unroll 1
        for (int j = 0; j < TN / 16; ++j) {
          uint32_t r[16];
          tmem_ld16(taddr + j * 16, r);
          tmem_ld_wait();
          store_row16<T>(q, row, n0 + j * 16, r);
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[buf]);
      ++acc_it;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

}  // namespace mgb
