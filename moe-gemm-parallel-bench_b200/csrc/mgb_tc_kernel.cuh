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
//   warp 0      TMA producer.  Grouped launches use the per-problem tensor
//               maps build_maps_kernel wrote just before this kernel.
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
// Dynamic shared memory for the operand ring plus the epilogue staging blocks;
// 3 KB of the 227 KB a CTA may use stay for barriers and the 1024-byte
// alignment of the ring.
constexpr int kTcSmemBudget = 232448 - 3072;
constexpr int kEpiWarpBytes = 32 * 128;  // one staging block: 32 rows x 128 bytes
// Staging blocks per epilogue warp (NB): a block is reused once the tensor
// store issued from it NB chunks earlier has read it, so NB stores of a warp
// can be in flight.  One-CTA row tiles keep 2 (their operand ring needs the
// shared memory: 4 stages of 128 x 256 tiles); CTA-pair tiles take 4, which
// measured faster on the large-M W13 shapes.
constexpr int epi_bytes_row_tile(int blocks) { return 4 * blocks * kEpiWarpBytes; }  // 4 epilogue warps
// Tensor maps of a grouped launch: build_maps_kernel writes A, B and C maps of
// every problem into the scratch buffer before the GEMM kernel runs.
constexpr int kMapsPerProblem = 3;

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
  // Row tiles stage their epilogue through shared memory and store it with
  // TMA (store_rows_tma); swap-AB tiles store column-per-lane, already
  // contiguous across the warp.
  static constexpr int kEpiBlocks = 2;
  static constexpr int kEpiBytes = SWAP ? 0 : epi_bytes_row_tile(kEpiBlocks);
  static constexpr int kStagesRaw = (kTcSmemBudget - kEpiBytes) / kStageBytes;
  static constexpr int kStages = kStagesRaw > 12 ? 12 : kStagesRaw;

  static constexpr int kAccCols = SWAP ? (TN / 128) * TM : TN;
  static constexpr int kTmemCols = pow2_at_least(2 * kAccCols);
  static constexpr uint32_t kFmt = std::is_same<T, float>::value ? 2u
                                   : std::is_same<T, __nv_bfloat16>::value ? 1u
                                                                            : 0u;
  static constexpr uint32_t kIdesc = SWAP ? instr_desc(kFmt, 1, 0, 128, TM) : instr_desc(kFmt, 0, 1, TM, TN);
  static constexpr int kSmemBytes = kStages * kStageBytes + kEpiBytes + 2048 + 1024;
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

// C is stored by TMA when its base is 16-byte aligned, its columns are unit
// stride and its rows are whole multiples of 16 bytes apart (and do not overlap).
template <typename T>
__device__ __forceinline__ bool c_tma_legal(const Problem& q, int64_t cols) {
  constexpr int E = static_cast<int>(sizeof(T));
  return (reinterpret_cast<uint64_t>(q.c) % 16 == 0) && q.scn == 1 && q.scm >= cols && (q.scm * E) % 16 == 0 &&
         q.m < (1ll << 31) && cols < (1ll << 31);
}

// Columns of C: N, or N / 2 with the fused SwiGLU epilogue (B_e packed [gate | up]).
__device__ __forceinline__ int64_t out_cols(const GroupedParams& p, const Problem& q) {
  return p.swiglu ? q.n / 2 : q.n;
}

// A problem runs on the tensor-core path when its operands satisfy the TMA
// rules; with the SwiGLU epilogue its packed weight must also split at a
// 16-byte boundary, so the boxes of the up half start aligned.
template <typename T>
__device__ __forceinline__ bool tile_legal(const GroupedParams& p, const Problem& q) {
  if (!tma_legal<T>(q)) return false;
  if (!p.swiglu) return true;
  return q.n % 2 == 0 && ((q.n / 2) * static_cast<int64_t>(sizeof(T))) % 16 == 0;
}

// Weight column loaded at tile-local column j of a TN-wide tile.  Plain: the
// tile covers weight columns [TN nb, TN nb + TN).  SwiGLU: the tile produces
// output columns [o, o + TN/2), o = nb TN/2, from gate columns o + j (j < TN/2)
// and up columns N/2 + o + j - TN/2, so gate and up of one output column sit
// TN/2 accumulator columns apart.  Columns past the gate half (last tile) read
// up values into accumulator columns whose outputs lie past C and are not stored.
template <int TN>
__device__ __forceinline__ int32_t weight_col(const GroupedParams& p, const Problem& q, int64_t nb, int j) {
  if (!p.swiglu) return static_cast<int32_t>(nb * TN + j);
  const int64_t o = nb * (TN / 2);
  return static_cast<int32_t>(j < TN / 2 ? o + j : q.n / 2 + o + (j - TN / 2));
}

// silu(g) * u = g / (1 + e^-g) * u with the fast exponential and divide
// intrinsics (a few ulp in fp32, far below the bf16 / fp16 output rounding).
// For g -> -inf the denominator overflows to inf and the quotient is 0.
__device__ __forceinline__ float silu_mul(float g, float u) { return __fdividef(g, 1.0f + __expf(-g)) * u; }

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

template <typename T>
__device__ __forceinline__ uint32_t pack_pair(uint32_t lo_bits, uint32_t hi_bits) {
  const float lo = __uint_as_float(lo_bits), hi = __uint_as_float(hi_bits);
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}

// Scatter-mode destination of row `row` of problem q (nullptr: dropped row or
// past the problem's rows); see GroupedParams::scatter_origin.
__device__ __forceinline__ char* scatter_row(const GroupedParams& p, const Problem& q, int64_t row) {
  if (row < 0 || row >= q.m) return nullptr;
  const int64_t origin = p.scatter_origin[q.row0 + row];
  if (origin < 0) return nullptr;
  const int64_t rank = origin >> 40;
  if (rank >= p.scatter_ranks) {
    atomicOr(p.error_word, kErrBadStore);
    return nullptr;
  }
  return reinterpret_cast<char*>(static_cast<uintptr_t>(p.scatter_peers[rank])) + p.scatter_offset +
         (origin & 0xFFFFFFFFFFll) * p.scatter_pitch;
}

// One 128-byte-per-row chunk of a warp's 32 accumulator rows (TMEM lanes):
// loads columns [col0, col0 + 128 / sizeof(T)), converts them and writes row
// `lane` of the 32 x 128-byte block `block` with its 16-byte units rotated by
// lane % 8 -- the 128-byte swizzle TMA uses, which also keeps the
// row-per-lane writes free of bank conflicts.  Returns after the writes;
// the caller synchronises the warp.
template <typename T>
__device__ __forceinline__ void load_chunk_tmem(uint32_t taddr, int col0, uint32_t (&v)[128 / sizeof(T) / 16][16]) {
  constexpr int kLoads = 128 / static_cast<int>(sizeof(T)) / 16;
#pragma unroll
  for (int u = 0; u < kLoads; ++u) tmem_ld16(taddr + col0 + u * 16, v[u]);
}

template <typename T>
__device__ __forceinline__ void write_chunk_smem(const uint32_t (&v)[128 / sizeof(T) / 16][16], uint8_t* block,
                                                 int lane) {
  constexpr int E = static_cast<int>(sizeof(T));
  uint32_t w[32];
  if constexpr (E == 4) {
#pragma unroll
    for (int i = 0; i < 32; ++i) w[i] = v[i / 16][i % 16];
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) w[i] = pack_pair<T>(v[(2 * i) / 16][(2 * i) % 16], v[(2 * i + 1) / 16][(2 * i + 1) % 16]);
  }
  uint8_t* my_row = block + lane * 128;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    *reinterpret_cast<uint4*>(my_row + ((j ^ (lane & 7)) << 4)) =
        make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
  }
}

// Writes 32 accumulator columns (one TMEM load unit) of row `lane` into the
// warp's 32 x 128-byte block at unit position `u` of the row (16-bit: 64
// bytes, units 0 / 1; fp32: the whole 128-byte row), 16-byte pieces rotated by
// lane % 8 as in write_chunk_smem.
template <typename T>
__device__ __forceinline__ void write_unit_smem(const uint32_t (&v)[32], uint8_t* block, int lane, int u) {
  uint8_t* my_row = block + lane * 128;
  if constexpr (sizeof(T) == 4) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      *reinterpret_cast<uint4*>(my_row + ((j ^ (lane & 7)) << 4)) =
          make_uint4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4 packed = make_uint4(pack_pair<T>(v[8 * j], v[8 * j + 1]), pack_pair<T>(v[8 * j + 2], v[8 * j + 3]),
                                      pack_pair<T>(v[8 * j + 4], v[8 * j + 5]),
                                      pack_pair<T>(v[8 * j + 6], v[8 * j + 7]));
      *reinterpret_cast<uint4*>(my_row + (((4 * u + j) ^ (lane & 7)) << 4)) = packed;
    }
  }
}

// Row-tile epilogue of one warp through TMA.  The warp's 32 rows x TN columns
// are read from TMEM in 32-column units, software-pipelined: the load of unit
// g + 1 is in flight while unit g is converted and staged.  Each 128-byte-
// per-row chunk (2 units of 16-bit, 1 of fp32) is staged in one of the warp's
// two 4 KB blocks (double-buffered against the tensor store still reading the
// other) and written by one tensor store of 32 rows x 128 bytes; rows and
// columns past C's extents are clipped by the tensor map.  `seq` counts the
// warp's chunks across tiles and picks the block.
template <typename T, int TN, int NB>
__device__ __forceinline__ void store_rows_tma(const Problem& q, const void* cmap, uint32_t taddr, int32_t row0,
                                               int32_t n0, uint8_t* blocks, int lane, uint32_t& seq,
                                               uint64_t policy, uint32_t* error_word) {
  constexpr int kChunkCols = 128 / static_cast<int>(sizeof(T));
  constexpr int kUnits = kChunkCols / 32;  // TMEM load units per chunk
  constexpr int kTotal = TN / 32;
  static_assert(TN % kChunkCols == 0, "tile width is a whole number of chunks");
  // All 32 rows lie past C (a ragged last M block), or every column does: no
  // TMEM load may be issued then, since only the loop below waits for one (a
  // tcgen05.ld left unwaited writes its registers after they were reused).
  if (row0 >= q.m || n0 >= q.n) return;
  const int64_t cols_left = q.n - n0;
  const int chunks = cols_left >= TN ? TN / kChunkCols : static_cast<int>((cols_left + kChunkCols - 1) / kChunkCols);
  const int units = chunks * kUnits;
  uint32_t v[2][32];
  tmem_ld32(taddr, v[0]);
#pragma unroll
  for (int g = 0; g < kTotal; ++g) {
    if (g >= units) break;
    const int c = g / kUnits;
    const int u = g % kUnits;
    uint8_t* block = blocks + ((seq + static_cast<uint32_t>(c)) % NB) * kEpiWarpBytes;
    if (u == 0) {
      if (lane == 0) bulk_wait_group_read<NB - 1>();  // the store last issued from `block` has read it
      __syncwarp();
    }
    tmem_ld_wait();  // unit g has landed
    if (g + 1 < units) tmem_ld32(taddr + (g + 1) * 32, v[(g + 1) & 1]);
    write_unit_smem<T>(v[g & 1], block, lane, u);
    if (u == kUnits - 1) {
      fence_proxy_async_smem();  // generic-proxy writes -> visible to the TMA store
      __syncwarp();
      if (lane == 0) {
        // Guard: a box must start inside C (stores never start at a negative
        // or past-the-end coordinate); the walk guarantees it.
        const int32_t x = n0 + c * kChunkCols;
        if (x >= 0 && row0 >= 0 && x < q.n && row0 < q.m) {
          tma_store_2d(cmap, block, x, row0, policy);
          bulk_commit_group();
        } else {
          atomicOr(error_word, kErrBadStore);
        }
      }
    }
  }
  seq += static_cast<uint32_t>(chunks);
}

// Row-tile epilogue of one warp in scatter mode: as store_rows_tma, but each
// staged 32 x 128-byte chunk is written by the warp itself, row by row, to the
// row's own destination (scatter_row; peer memory for rows returned to other
// ranks): 8 lanes per 128-byte row segment, 4 rows per store instruction.
// Columns must be a multiple of 8 elements (16 bytes).
template <typename T, int TN>
__device__ __forceinline__ void store_rows_scatter(const GroupedParams& p, const Problem& q, uint32_t taddr,
                                                   int64_t row0, int64_t n0, uint8_t* block, int lane) {
  constexpr int kChunkCols = 128 / static_cast<int>(sizeof(T));
  constexpr int kUnits = kChunkCols / 32;
  constexpr int kTotal = TN / 32;
  if (row0 >= q.m || n0 >= q.n) return;  // as in store_rows_tma: no unwaited TMEM load
  const int64_t cols_left = q.n - n0;
  const int chunks = cols_left >= TN ? TN / kChunkCols : static_cast<int>((cols_left + kChunkCols - 1) / kChunkCols);
  const int units = chunks * kUnits;
  char* my_dst = scatter_row(p, q, row0 + lane);
  uint32_t v[2][32];
  tmem_ld32(taddr, v[0]);
#pragma unroll
  for (int g = 0; g < kTotal; ++g) {
    if (g >= units) break;
    const int c = g / kUnits;
    const int u = g % kUnits;
    tmem_ld_wait();
    if (g + 1 < units) tmem_ld32(taddr + (g + 1) * 32, v[(g + 1) & 1]);
    write_unit_smem<T>(v[g & 1], block, lane, u);
    if (u == kUnits - 1) {
      __syncwarp();
      const int piece = lane & 7;  // 16-byte piece of a 128-byte row segment
      const int64_t col = n0 + c * kChunkCols + piece * (16 / static_cast<int>(sizeof(T)));
#pragma unroll
      for (int it = 0; it < 8; ++it) {
        const int r = it * 4 + (lane >> 3);
        const uint64_t d = __shfl_sync(0xffffffffu, reinterpret_cast<uint64_t>(my_dst), r);
        if (d != 0 && col < q.n) {
          const uint4 val = *reinterpret_cast<const uint4*>(block + r * 128 + ((piece ^ (r & 7)) << 4));
          *reinterpret_cast<uint4*>(reinterpret_cast<char*>(d) + col * static_cast<int64_t>(sizeof(T))) = val;
        }
      }
      __syncwarp();  // every lane has read the block before it is written again
    }
  }
}

// Row-tile SwiGLU epilogue of one warp through TMA: gate accumulators are
// TMEM columns [0, TO), up columns [TO, 2 TO); each 32-column output unit
// loads both, computes silu(gate) * up in fp32 and is staged and stored like
// store_rows_tma.
template <typename T, int TO, int NB>
__device__ __forceinline__ void store_rows_tma_swiglu(const Problem& qo, const void* cmap, uint32_t taddr,
                                                      int32_t row0, int32_t o0, uint8_t* blocks, int lane,
                                                      uint32_t& seq, uint64_t policy, uint32_t* error_word) {
  constexpr int kChunkCols = 128 / static_cast<int>(sizeof(T));
  constexpr int kUnits = kChunkCols / 32;
  static_assert(TO % kChunkCols == 0, "output tile width is a whole number of chunks");
  if (row0 >= qo.m) return;
  const int64_t cols_left = qo.n - o0;
  const int chunks = cols_left >= TO ? TO / kChunkCols : static_cast<int>((cols_left + kChunkCols - 1) / kChunkCols);
  const int units = chunks * kUnits;
#pragma unroll 1
  for (int g = 0; g < units; ++g) {
    const int c = g / kUnits;
    const int u = g % kUnits;
    uint8_t* block = blocks + ((seq + static_cast<uint32_t>(c)) % NB) * kEpiWarpBytes;
    if (u == 0) {
      if (lane == 0) bulk_wait_group_read<NB - 1>();
      __syncwarp();
    }
    uint32_t gate[32], up[32];
    tmem_ld32(taddr + g * 32, gate);
    tmem_ld32(taddr + TO + g * 32, up);
    tmem_ld_wait();
#pragma unroll
    for (int i = 0; i < 32; ++i) gate[i] = __float_as_uint(silu_mul(__uint_as_float(gate[i]), __uint_as_float(up[i])));
    write_unit_smem<T>(gate, block, lane, u);
    if (u == kUnits - 1) {
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        const int32_t x = o0 + c * kChunkCols;
        if (x >= 0 && row0 >= 0 && x < qo.n && row0 < qo.m) {
          tma_store_2d(cmap, block, x, row0, policy);
          bulk_commit_group();
        } else {
          atomicOr(error_word, kErrBadStore);
        }
      }
    }
  }
  seq += static_cast<uint32_t>(chunks);
}

// Row-tile SwiGLU epilogue without TMA (C not addressable by a tensor map):
// element stores with bounds checks.
template <typename T, int TO>
__device__ __forceinline__ void store_rows_scalar_swiglu(const Problem& qo, uint32_t taddr, int64_t row0, int64_t o0,
                                                         int lane) {
  const int64_t row = row0 + lane;
#pragma unroll 1
  for (int g = 0; g < TO / 32; ++g) {
    uint32_t gate[32], up[32];
    tmem_ld32(taddr + g * 32, gate);
    tmem_ld32(taddr + TO + g * 32, up);
    tmem_ld_wait();
    if (row < qo.m) {
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int64_t col = o0 + g * 32 + i;
        if (col < qo.n) {
          store_scalar<T>(qo.c, row * qo.scm + col * qo.scn, silu_mul(__uint_as_float(gate[i]), __uint_as_float(up[i])));
        }
      }
    }
  }
}

// Writes the warp's staged 32 x 128-byte block (rows row0.., columns col0..,
// in the 128-byte swizzle of write_chunk_smem) to C through C's strides:
// every global store instruction writes four whole 128-byte row segments;
// columns past C and rows past M are skipped.
template <typename T>
__device__ __forceinline__ void flush_block_rows(const Problem& q, const uint8_t* block, int64_t row0, int64_t col0,
                                                 int lane) {
  constexpr int E = static_cast<int>(sizeof(T));
  constexpr int kUnitCols = 16 / E;  // columns per 16-byte unit
  const int j = lane & 7;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = 4 * i + (lane >> 3);
    const uint4 val = *reinterpret_cast<const uint4*>(block + r * 128 + ((j ^ (r & 7)) << 4));
    const int64_t row = row0 + r;
    const int64_t col = col0 + j * kUnitCols;
    if (row < q.m) {
      char* dst = q.c + (row * q.scm + col * q.scn) * static_cast<int64_t>(E);
      if (q.scn == 1 && col + kUnitCols <= q.n && (reinterpret_cast<uint64_t>(dst) % 16 == 0)) {
        *reinterpret_cast<uint4*>(dst) = val;
      } else {
        const uint32_t parts[4] = {val.x, val.y, val.z, val.w};
#pragma unroll
        for (int e = 0; e < kUnitCols; ++e) {
          if (col + e >= q.n) break;
          char* d = q.c + (row * q.scm + (col + e) * q.scn) * static_cast<int64_t>(E);
          if constexpr (E == 4) {
            *reinterpret_cast<uint32_t*>(d) = parts[e];
          } else {
            *reinterpret_cast<uint16_t*>(d) = static_cast<uint16_t>(parts[e / 2] >> (16 * (e % 2)));
          }
        }
      }
    }
  }
}

// Row-tile epilogue of one warp without TMA (C not addressable by a tensor
// map): the chunk goes through `block` and is read back so that every global
// store instruction writes four whole 128-byte row segments.
template <typename T, int TN>
__device__ __forceinline__ void store_rows_staged(const Problem& q, uint32_t taddr, int64_t row0, int64_t n0,
                                                  uint8_t* block, int lane) {
  constexpr int E = static_cast<int>(sizeof(T));
  constexpr int kChunkCols = 128 / E;
  static_assert(TN % kChunkCols == 0, "tile width is a whole number of chunks");
  if (lane == 0) bulk_wait_group_read<0>();  // no tensor store of this warp still reads its blocks
  __syncwarp();
#pragma unroll 1
  for (int c = 0; c < TN / kChunkCols; ++c) {
    uint32_t v[kChunkCols / 16][16];
    load_chunk_tmem<T>(taddr, c * kChunkCols, v);
    tmem_ld_wait();
    write_chunk_smem<T>(v, block, lane);
    __syncwarp();
    flush_block_rows<T>(q, block, row0, n0 + c * kChunkCols, lane);
    __syncwarp();  // the block is rewritten by the next chunk
  }
}

// Row-tile epilogue of one warp from fp32 registers (the promoted
// accumulator of an fp32 tile): row `lane` of the warp's 32 rows holds TN
// columns in acc.  Each 32-column chunk is staged in the warp's blocks in the
// 128-byte swizzle and written by a tensor store when C has a map (`cmap`),
// else read back and written as 128-byte row segments (store_rows_staged).
template <int TN, int NB>
__device__ __forceinline__ void store_rows_regs(const Problem& q, const void* cmap, const float (&acc)[TN],
                                                int64_t row0, int64_t n0, uint8_t* blocks, int lane, uint32_t& seq,
                                                uint64_t policy, uint32_t* error_word) {
  static_assert(TN % 32 == 0, "whole 32-column chunks");
  if (row0 >= q.m || n0 >= q.n) return;
  const int64_t cols_left = q.n - n0;
  const int chunks = cols_left >= TN ? TN / 32 : static_cast<int>((cols_left + 31) / 32);
  if (cmap == nullptr) {
    if (lane == 0) bulk_wait_group_read<0>();  // no tensor store of this warp still reads its blocks
    __syncwarp();
  }
#pragma unroll
  for (int c = 0; c < TN / 32; ++c) {
    if (c >= chunks) break;
    uint32_t v[2][16];
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i / 16][i % 16] = __float_as_uint(acc[c * 32 + i]);
    if (cmap != nullptr) {
      uint8_t* block = blocks + ((seq + static_cast<uint32_t>(c)) % NB) * kEpiWarpBytes;
      if (lane == 0) bulk_wait_group_read<NB - 1>();  // the store last issued from `block` has read it
      __syncwarp();
      write_chunk_smem<float>(v, block, lane);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        const int64_t x = n0 + c * 32;
        if (x >= 0 && row0 >= 0 && x < q.n && row0 < q.m) {
          tma_store_2d(cmap, block, static_cast<int32_t>(x), static_cast<int32_t>(row0), policy);
          bulk_commit_group();
        } else {
          atomicOr(error_word, kErrBadStore);
        }
      }
    } else {
      write_chunk_smem<float>(v, blocks, lane);
      __syncwarp();
      flush_block_rows<float>(q, blocks, row0, n0 + c * 32, lane);
      __syncwarp();  // the block is rewritten by the next chunk
    }
  }
  if (cmap != nullptr) seq += static_cast<uint32_t>(chunks);
}

// Tensor maps of problem e in the scratch buffer: [A, B, C].
__device__ __forceinline__ const CUtensorMap* problem_maps(const GroupedParams& p, int e) {
  return reinterpret_cast<const CUtensorMap*>(p.desc_slots) + static_cast<int64_t>(kMapsPerProblem) * e;
}

// Lookahead on the tensormap side (lane 0 of a role): acquires and prefetches
// `count` maps of the problem the walk looked up ahead (`ahead`, -1: none),
// starting at map `first_map`, once, so the switch to that problem neither
// waits on the acquire fence nor on the descriptor fetch.  `acquired` records
// the problem done.
__device__ __forceinline__ void acquire_ahead_maps(const GroupedParams& p, int ahead, int& acquired, int count,
                                                   int first_map = 0) {
  if (p.single || ahead < 0 || ahead == acquired) return;
  const CUtensorMap* g = problem_maps(p, ahead) + first_map;
  for (int i = 0; i < count; ++i) {
    tmap_acquire(&g[i]);
    prefetch_tmap(&g[i]);
  }
  acquired = ahead;
}

// The output map of the epilogue's current problem: the launch's own map for a
// single GEMM, else problem e's C map, acquired when the warp first meets e
// (before the accumulator wait, so the fence overlaps the tile's MMAs).
__device__ __forceinline__ const void* out_map_for(const GroupedParams& p, const CUtensorMap& single_map, int e,
                                                   int& built, int lane) {
  if (p.single) return &single_map;
  const CUtensorMap* g = &problem_maps(p, e)[2];
  if (e != built) {
    if (lane == 0) tmap_acquire(g);
    __syncwarp();
    built = e;
  }
  return g;
}

// The extra block of a heterogeneous launch's map builder (one warp):
// unit_start[e] = units of problems [0, e) for the walk's tile shape and unit
// size (empty or invalid problems have none), lane l summing a contiguous run
// of problems, then a warp-wide exclusive scan.
__device__ __forceinline__ void write_unit_prefix(const GroupedParams& p, int lane) {
  const int per = (p.problem_count + 31) / 32;
  const int lo = lane * per;
  const int hi = lo + per < p.problem_count ? lo + per : p.problem_count;
  const int64_t unit = p.unit_tiles > 0 ? p.unit_tiles : 1;
  auto units_of = [&](int i) -> int64_t {
    const Problem q = load_problem(p, i);
    if (q.m <= 0 || q.n <= 0 || q.k < 0) return 0;
    return ceil_div64(ceil_div64(q.m, p.walk_tm) * ceil_div64(q.n, p.walk_tn), unit);
  };
  int64_t sum = 0;
  for (int i = lo; i < hi; ++i) sum += units_of(i);
  int64_t incl = sum;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int64_t v = __shfl_up_sync(0xffffffffu, incl, d);
    if (lane >= d) incl += v;
  }
  int64_t run = incl - sum;
  for (int i = lo; i < hi; ++i) {
    p.unit_start[i] = run;
    run += units_of(i);
  }
  if (lane == 31) p.unit_start[p.problem_count] = incl;
}

// Builds the tensor maps of every problem of a grouped launch, one warp per
// problem: lane 0 copies the three templates (box shape, swizzle and element
// type final) into shared memory and rewrites the base addresses -- and, for
// heterogeneous groups, the extents and row pitches -- of the problem; the
// warp then publishes the three maps to global memory with a release fence
// for the tensormap proxy.  The GEMM kernel, launched next on the same
// stream, acquires each map before its first TMA operation.  Problems the TMA
// cannot address keep the unmodified template (the GEMM kernel never uses it).
template <typename T>
__global__ void __launch_bounds__(32)
    build_maps_kernel(const __grid_constant__ CUtensorMap act_tmpl, const __grid_constant__ CUtensorMap wgt_tmpl,
                      const __grid_constant__ CUtensorMap out_tmpl, const GroupedParams p) {
  __shared__ alignas(128) CUtensorMap staging[kMapsPerProblem];
  const int e = blockIdx.x;
  const int lane = threadIdx.x;
  // The GEMM kernel that follows may launch now: it only sets up its shared
  // memory and TMEM before waiting for this grid (grid_dependency_wait).
  grid_launch_dependents();
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
    const bool sane = q.m > 0 && q.n > 0 && q.k >= 0;
    if (sane && tile_legal<T>(p, q)) {
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
    if (sane && p.scatter_origin == nullptr && c_tma_legal<T>(q, out_cols(p, q))) {
      tmap_replace_address(&staging[2], q.c);
      if (!p.homogeneous) {
        tmap_replace_dim(&staging[2], 0, static_cast<uint32_t>(out_cols(p, q)));
        tmap_replace_dim(&staging[2], 1, static_cast<uint32_t>(q.m));
        tmap_replace_stride1(&staging[2], static_cast<uint64_t>(q.scm) * sizeof(T));
      }
    }
  }
  __syncwarp();
  CUtensorMap* g = reinterpret_cast<CUtensorMap*>(p.desc_slots) + static_cast<int64_t>(kMapsPerProblem) * e;
  for (int i = 0; i < kMapsPerProblem; ++i) tmap_publish(&g[i], &staging[i]);
}

// K blocks per accumulator chunk of a PROMOTE launch (256 fp32 K).
constexpr int kPromoteBlocks = 8;

// PROMOTE (fp32, 128-token tiles): the tensor core accumulates at most
// kPromoteBlocks k-blocks into a TMEM accumulator, alternating between the two
// accumulators chunk by chunk; the epilogue warps add every chunk into fp32
// registers (round-to-nearest) and store the sum at the end of the tile.
// Long TF32 accumulations inside the tensor core lose accuracy in proportion
// to K (measured: 1.9e-5 relative at K = 8191 for exactly representable
// inputs); chunking bounds that to one 256-deep chunk, which the 3xTF32 split
// of fp32 "ieee" GEMMs needs to reach fp32 accuracy.
template <typename T, bool SWAP, int TM, int TN, bool PROMOTE = false>
__global__ void __launch_bounds__(kTcThreads, 1)
    tc_grouped_kernel(const __grid_constant__ CUtensorMap act_tmpl, const __grid_constant__ CUtensorMap wgt_tmpl,
                      const __grid_constant__ CUtensorMap out_tmpl, const GroupedParams p) {
  using Cfg = TcCfg<T, SWAP, TM, TN>;
  constexpr int S = Cfg::kStages;
  constexpr int BK = Cfg::kBK;
  static_assert(!PROMOTE || (std::is_same<T, float>::value && !SWAP && TM == 128 && TN <= 128),
                "promoted accumulation: fp32 128-token tiles of at most 128 columns");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;
  uint8_t* epi_stage = smem + S * Cfg::kStageBytes;  // kEpiBytes, 1024-byte aligned
  uint64_t* full = reinterpret_cast<uint64_t*>(epi_stage + Cfg::kEpiBytes);
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* test_bar = acc_empty + 2;  // never arrived on: the test-only bounded-wait probe
  uint64_t* drain_bar = test_bar + 1;  // teardown: waits for MMAs in flight after an abort
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);  // raised by a role that gave up
  volatile int* never = abort + 1;  // stays 0: for waits no abort may cut short

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
  // Launched right behind build_maps_kernel with programmatic serialization:
  // nothing above read global memory; everything below may (tables, maps,
  // operands).  Without a programmatic dependency this returns at once.
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
    TileWalk<TM, TN> walk;
    uint32_t it = 0;
    int built = -1;
    int ahead_acquired = -1;  // problem whose maps were acquired one unit early
    bool ok = true;
    for (int64_t t = 0; ok && walk.next_tile(p, blockIdx.x, gridDim.x, t);) {
      const Problem& q = walk.prob;
      if (!tile_legal<T>(p, q)) {
        if (lane == 0 && walk.problem != built) atomicOr(p.error_word, kErrMisaligned);
        continue;
      }
      const int64_t kblocks = (q.k + BK - 1) / BK;
      const uint64_t pol_wgt = walk.m_blocks > 1 ? pol_shared : pol_stream;
      const int32_t m0 = static_cast<int32_t>(walk.m_block(t) * TM);
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
          // Entering a new problem: its maps were built before this kernel
          // started (build_maps_kernel); acquire them for the tensormap proxy
          // (done a unit early when the walk looked this problem up ahead).
          const CUtensorMap* g = problem_maps(p, walk.problem);
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
          mbar_arrive_expect_tx(&full[s], Cfg::kStageBytes);
          tma_load_2d(act_map, &full[s], st_act, kx, m0, pol_act);
#pragma unroll
          for (int j = 0; j < TN / BK; ++j) {
            tma_load_2d(wgt_map, &full[s], st_wgt + j * Cfg::kBoxBytes, weight_col<TN>(p, q, nb, j * BK), kx,
                        pol_wgt);
          }
          if (kb == 0) acquire_ahead_maps(p, walk.ahead_problem, ahead_acquired, 2);
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
      for (int64_t t = 0; ok && walk.next_tile(p, blockIdx.x, gridDim.x, t);) {
        const Problem& q = walk.prob;
        if (!tile_legal<T>(p, q) || q.k <= 0) continue;
        const int64_t kblocks = (q.k + BK - 1) / BK;
        // One accumulator per tile, or per chunk of kPromoteBlocks k-blocks.
        const int64_t chunk_blocks = PROMOTE ? kPromoteBlocks : kblocks;
        for (int64_t kb0 = 0; ok && kb0 < kblocks; kb0 += chunk_blocks) {
        const int64_t kb1 = kb0 + chunk_blocks < kblocks ? kb0 + chunk_blocks : kblocks;
        const int buf = static_cast<int>(acc_it & 1u);
        if (!mbar_wait(&acc_empty[buf], ((acc_it >> 1) & 1u) ^ 1u, budget, abort)) {
          raise_error(p, kErrWaitAccEmpty, abort);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * Cfg::kAccCols);
        for (int64_t kb = kb0; kb < kb1; ++kb) {
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
            const uint32_t acc = (kb > kb0 || ks > 0) ? 1u : 0u;
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
        mma_commit(&acc_full[buf]);  // accumulator (or chunk) ready for the epilogue
        ++acc_it;
        }
        if (!ok) break;
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
    uint8_t* my_blocks = epi_stage + quarter * Cfg::kEpiBlocks * kEpiWarpBytes;
    int c_built = -1;
    const uint64_t pol_out = policy_evict_first();
    uint32_t chunk_seq = 0;
    bool ok = true;
    for (int64_t t = 0; ok && walk.next_tile(p, blockIdx.x, gridDim.x, t);) {
      if (!tile_legal<T>(p, walk.prob)) continue;
      Problem q = walk.prob;
      q.n = out_cols(p, q);  // the epilogue addresses C: N/2 columns with SwiGLU
      const int tile_out = p.swiglu ? TN / 2 : TN;
      const int64_t m0 = walk.m_block(t) * TM;
      const int64_t n0 = walk.n_block(t) * tile_out;
      if (q.k <= 0) {
        for (int idx = ethread; idx < TM * tile_out; idx += 128) {
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
      const void* cmap = nullptr;
      if constexpr (!SWAP) {
        if (c_tma_legal<T>(q, q.n)) cmap = out_map_for(p, out_tmpl, walk.problem, c_built, lane);
      }
      if constexpr (PROMOTE) {
        // Sum the tile's accumulator chunks in fp32 registers (row `lane` of
        // the warp's quarter, TN columns), then store the sum.
        float sum[TN];
#pragma unroll
        for (int i = 0; i < TN; ++i) sum[i] = 0.0f;
        const int64_t kblocks = (q.k + BK - 1) / BK;
        for (int64_t kb0 = 0; kb0 < kblocks; kb0 += kPromoteBlocks) {
          const int cbuf = static_cast<int>(acc_it & 1u);
          if (!mbar_wait_warp(&acc_full[cbuf], (acc_it >> 1) & 1u, budget, abort)) {
            if (lane == 0) raise_error(p, kErrWaitAccFull, abort);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t ctaddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                                  static_cast<uint32_t>(cbuf * Cfg::kAccCols);
          uint32_t v[2][16];  // 16-column units, the next one in flight while one is added
          tmem_ld16(ctaddr, v[0]);
#pragma unroll
          for (int u = 0; u < TN / 16; ++u) {
            tmem_ld_wait();  // unit u has landed
            if (u + 1 < TN / 16) tmem_ld16(ctaddr + (u + 1) * 16, v[(u + 1) & 1]);
#pragma unroll
            for (int i = 0; i < 16; ++i) sum[u * 16 + i] += __uint_as_float(v[u & 1][i]);
          }
          tc_fence_before();
          mbar_arrive_relaxed(&acc_empty[cbuf]);
          ++acc_it;
        }
        if (!ok) break;
        store_rows_regs<TN, Cfg::kEpiBlocks>(q, cmap, sum, m0 + quarter * 32, n0, my_blocks, lane, chunk_seq, pol_out,
                                             p.error_word);
        continue;
      }
      const int buf = static_cast<int>(acc_it & 1u);
      if (!mbar_wait_warp(&acc_full[buf], (acc_it >> 1) & 1u, budget, abort)) {
        if (lane == 0) raise_error(p, kErrWaitAccFull, abort);
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                             static_cast<uint32_t>(buf * Cfg::kAccCols);
      if constexpr (SWAP) {
        if constexpr (TN >= 256) {
          if (p.swiglu) {
            // Chunk 0 holds gate, chunk 1 up, of the same 128 output columns:
            // lane l of quarter w owns output column n0 + 32 w + l.
            const int64_t col = n0 + quarter * 32 + lane;
#pragma unroll 1
            for (int j = 0; j < TM / 16; ++j) {
              uint32_t g[16], u[16];
              tmem_ld16(taddr + j * 16, g);
              tmem_ld16(taddr + TM + j * 16, u);
              tmem_ld_wait();
              if (col < q.n) {
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                  const int64_t row = m0 + j * 16 + i;
                  if (row < q.m) {
                    store_scalar<T>(q.c, row * q.scm + col * q.scn,
                                    silu_mul(__uint_as_float(g[i]), __uint_as_float(u[i])));
                  }
                }
              }
            }
            tc_fence_before();
            mbar_arrive_relaxed(&acc_empty[buf]);
            ++acc_it;
            continue;
          }
        }
#pragma unroll 1
        for (int c = 0; c < TN / 128; ++c) {
          const int64_t col = n0 + c * 128 + quarter * 32 + lane;
#pragma unroll 1
          for (int j = 0; j < TM / 16; ++j) {
            uint32_t r[16];
            tmem_ld16(taddr + c * TM + j * 16, r);
            tmem_ld_wait();
            if (p.scatter_origin != nullptr) {
              // Lane i of the warp resolves row j * 16 + i's destination once.
              char* mine = lane < 16 ? scatter_row(p, q, m0 + j * 16 + lane) : nullptr;
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                const uint64_t d = __shfl_sync(0xffffffffu, reinterpret_cast<uint64_t>(mine), i);
                if (d != 0 && col < q.n) store_scalar<T>(reinterpret_cast<char*>(d), col, __uint_as_float(r[i]));
              }
            } else if (col < q.n) {
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                const int64_t row = m0 + j * 16 + i;
                if (row < q.m) store_scalar<T>(q.c, row * q.scm + col * q.scn, __uint_as_float(r[i]));
              }
            }
          }
        }
      } else {
        bool done = false;
        if constexpr (TN >= 128) {
          if (p.swiglu) {
            if (cmap != nullptr) {
              store_rows_tma_swiglu<T, TN / 2, Cfg::kEpiBlocks>(q, cmap, taddr, static_cast<int32_t>(m0 + quarter * 32),
                                               static_cast<int32_t>(n0), my_blocks, lane, chunk_seq, pol_out,
                                               p.error_word);
            } else {
              store_rows_scalar_swiglu<T, TN / 2>(q, taddr, m0 + quarter * 32, n0, lane);
            }
            done = true;
          }
        }
        if (!done && p.scatter_origin != nullptr) {
          store_rows_scatter<T, TN>(p, q, taddr, m0 + quarter * 32, n0, my_blocks, lane);
          done = true;
        }
        if (!done) {
          if (cmap != nullptr) {
            store_rows_tma<T, TN, Cfg::kEpiBlocks>(q, cmap, taddr, static_cast<int32_t>(m0 + quarter * 32), static_cast<int32_t>(n0),
                                  my_blocks, lane, chunk_seq, pol_out, p.error_word);
          } else {
            store_rows_staged<T, TN>(q, taddr, m0 + quarter * 32, n0, my_blocks, lane);
          }
        }
      }
      tc_fence_before();
      mbar_arrive_relaxed(&acc_empty[buf]);
      ++acc_it;
    }
    if (lane == 0) bulk_wait_group_all();  // tensor stores done before the CTA's shared memory goes away
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

}  // namespace mgb
