// Launch parameters and the device-side problem/tile walk shared by the
// tensor-core kernel and the SIMT kernel.
//
// A launch covers `problem_count` independent GEMMs C_e = A_e @ B_e.  The
// per-problem pointers, dims (M, N, K) and element strides (am, ak, bk, bn,
// cm, cn) are read on the device from the caller's tables, exactly the tables
// the reference builds in kernels/grouped_gemm.py:530-544.  Reading them on the
// device (not on the host) keeps launches graph-capturable and lets callers
// swap a table entry after the workspace was built.
#pragma once

#include <cstdint>

namespace mgb {

// Tile of the generic-stride SIMT kernel (mgb_simt_kernel.cuh).
constexpr int kSimtThreads = 256;
constexpr int kSimtBM = 64;
constexpr int kSimtBN = 64;
constexpr int kSimtBK = 16;

struct GroupedParams {
  // Table mode (grouped launches).
  const int64_t* a_ptrs;
  const int64_t* b_ptrs;
  const int64_t* c_ptrs;
  const int32_t* dims;     // [E, 3]: M, N, K
  const int64_t* strides;  // [E, 6]: am, ak, bk, bn, cm, cn (elements)
  int32_t problem_count;
  int32_t homogeneous;  // every problem has (m, n, k) below and contiguous strides
  int64_t m, n, k;
  // Inline mode (single GEMM): one problem, pointers and strides passed by value.
  int32_t single;
  const void* a;
  const void* b;
  void* c;
  int64_t sam, sak, sbk, sbn, scm, scn;
  // Scratch for the per-CTA tensor-map slots of the TMA path.
  uint8_t* desc_slots;
  // Expert-sorted aggregate mode (offs != nullptr): one A [T, K] (rows of
  // expert e are [offs[e-1], offs[e])), B [E, K, N] with `sbe` elements between
  // experts, C [T, N]; pointers in a / b / c, row strides sam / sbk / scm.
  const int32_t* offs;
  int64_t sbe;
  int32_t b_count;  // > 0: problem e uses B[e % b_count] (segments of several senders share an expert)
  int32_t elem_bytes;
  int32_t unit_tiles;     // tensor-core kernels: consecutive tiles of one problem a CTA takes at a time
  // CTA-pair 256 x 512 launches with an exact tile count and one tile per
  // unit: tail_split = 1 splits every global tile from tail_from on into two
  // 256 x 256 items (one per 256-column half), so a short last wave of wide
  // tiles runs as at most one half-width item per cluster.  0: no split.
  int32_t tail_split;
  int64_t tail_from;
  // Heterogeneous tensor-core launches: unit_start[e] = units of problems
  // [0, e) (E + 1 entries, written by the map builder before the GEMM kernel
  // runs) for the tile shape walk_tm x walk_tn, so the walk finds a unit's
  // problem by binary search instead of scanning the table.
  int64_t* unit_start;
  int32_t walk_tm, walk_tn;
  // FP8 block-scaled launches: per-problem fp32 scale tables, SA_e
  // [M, ceil(K/128)] (per token and 128-deep K block) and SB_e
  // [ceil(N/128), ceil(K/128)] (per 128 x 128 weight block), row-major.
  const int64_t* sa_ptrs;
  const int64_t* sb_ptrs;
  int32_t swiglu;         // 1: fused SwiGLU epilogue, C_e[M, N/2] = silu(A_e B_e[:, :N/2]) * (A_e B_e[:, N/2:])
  // Row-scatter epilogue (aggregate mode, tensor-core kernels, no SwiGLU):
  // row R of the aggregate C is not written to C but to the region of rank
  // scatter_origin[R] >> 40 (base scatter_peers[rank], this process's mapping)
  // at byte scatter_offset + (scatter_origin[R] & 0xFFFFFFFFFF) *
  // scatter_pitch; a negative origin drops the row.  The expert-parallel layer
  // uses it to return W2 rows straight to the ranks that sent the tokens.
  const int64_t* scatter_origin;
  const int64_t* scatter_peers;
  int32_t scatter_ranks;  // entries of scatter_peers; an origin naming another rank drops the row
  int64_t scatter_offset;
  int64_t scatter_pitch;
  long long wait_budget;  // SM clock cycles a barrier wait may take before the launch gives up
  int32_t test_flags;     // bit 0: make the epilogue wait on a barrier nothing arrives on
  uint32_t* error_word;   // where error bits are OR-ed (a __device__ word of this library)
};

struct Problem {
  int64_t m, n, k;
  int64_t row0;  // aggregate mode: row of the launch's A / C where the problem starts
  const char* a;
  const char* b;
  char* c;
  int64_t sam, sak, sbk, sbn, scm, scn;
};

// A problem of a homogeneous table launch from its three pointers: every
// other field is the launch's (contiguous operands; C has N columns, or N/2
// with the SwiGLU epilogue).
__device__ __forceinline__ Problem homogeneous_problem(const GroupedParams& p, const char* a, const char* b, char* c) {
  Problem q;
  q.row0 = 0;
  q.a = a;
  q.b = b;
  q.c = c;
  q.m = p.m; q.n = p.n; q.k = p.k;
  q.sam = p.k; q.sak = 1; q.sbk = p.n; q.sbn = 1; q.scm = p.swiglu ? p.n / 2 : p.n; q.scn = 1;
  return q;
}

__device__ __forceinline__ Problem load_problem(const GroupedParams& p, int e) {
  Problem q;
  q.row0 = 0;
  if (p.single) {
    q.m = p.m; q.n = p.n; q.k = p.k;
    q.a = static_cast<const char*>(p.a);
    q.b = static_cast<const char*>(p.b);
    q.c = static_cast<char*>(p.c);
    q.sam = p.sam; q.sak = p.sak; q.sbk = p.sbk; q.sbn = p.sbn; q.scm = p.scm; q.scn = p.scn;
    return q;
  }
  if (p.offs != nullptr) {
    const int64_t start = e > 0 ? p.offs[e - 1] : 0;
    const int64_t es = p.elem_bytes;
    q.m = static_cast<int64_t>(p.offs[e]) - start;
    q.n = p.n;
    q.k = p.k;
    q.a = static_cast<const char*>(p.a) + start * p.sam * es;
    q.b = static_cast<const char*>(p.b) + (p.b_count > 0 ? e % p.b_count : e) * p.sbe * es;
    q.c = static_cast<char*>(p.c) + start * p.scm * es;
    q.row0 = start;
    q.sam = p.sam; q.sak = 1; q.sbk = p.sbk; q.sbn = 1; q.scm = p.scm; q.scn = 1;
    return q;
  }
  if (p.homogeneous) {
    return homogeneous_problem(p, reinterpret_cast<const char*>(p.a_ptrs[e]),
                               reinterpret_cast<const char*>(p.b_ptrs[e]), reinterpret_cast<char*>(p.c_ptrs[e]));
  }
  q.a = reinterpret_cast<const char*>(p.a_ptrs[e]);
  q.b = reinterpret_cast<const char*>(p.b_ptrs[e]);
  q.c = reinterpret_cast<char*>(p.c_ptrs[e]);
  {
    q.m = p.dims[3 * e + 0];
    q.n = p.dims[3 * e + 1];
    q.k = p.dims[3 * e + 2];
    if (p.strides != nullptr) {
      const int64_t* s = p.strides + 6 * e;
      q.sam = s[0]; q.sak = s[1]; q.sbk = s[2]; q.sbn = s[3]; q.scm = s[4]; q.scn = s[5];
    } else {  // tables without strides (the FP8 path): contiguous A [M, K], B [N, K], C [M, N]
      q.sam = q.k; q.sak = 1; q.sbk = q.k; q.sbn = 1; q.scm = q.n; q.scn = 1;
    }
  }
  return q;
}

__device__ __forceinline__ int64_t ceil_div64(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Walks the flattened tile space problem by problem.  Each CTA visits its
// tiles in increasing order, so the walk only ever moves forward: the whole
// launch costs one pass over the problem table per CTA (the reference scans it
// the same way, kernels/grouped_gemm.py:426-436).  Tiles inside a problem are
// ordered M-block fastest (in bands of 8 M-blocks, see m_block), so CTAs that
// run at the same time share a weight column block in L2.
//
// The tensor-core kernels hand out work in units: U consecutive tiles of one
// problem (the last unit of a problem may be shorter), units strided over the
// CTAs (seek_unit).  With U = 1 this is the plain strided tile schedule; a
// larger U keeps a CTA on one problem for several short-K tiles, so the
// per-problem tensor-map rebuilds are paid once per unit.
template <int TM, int TN>
struct TileWalk {
  int problem = -1;
  int64_t first = 0;   // first global tile of `problem`
  int64_t count = 0;   // tiles of `problem`
  int64_t ufirst = 0;  // first global unit of `problem` (seek_unit)
  int64_t ucount = 0;  // units of `problem` (seek_unit)
  int64_t m_blocks = 1;
  Problem prob;
  // Lookahead of homogeneous table launches: the table pointers of the
  // problem holding this CTA's next unit, loaded while the current unit runs,
  // so a problem switch does not stall a role on a global-memory round trip
  // (the MMA issuer sits on the tensor pipe's critical path there).
  int ahead_problem = -1;
  const char* ahead_a = nullptr;
  const char* ahead_b = nullptr;
  char* ahead_c = nullptr;

  // Issues the loads of the pointers of the problem that holds unit `u`
  // (`unit` tiles each) when it is not the current one; homogeneous table
  // launches only (every problem's shape is known without a load).
  __device__ __forceinline__ void prefetch_unit(const GroupedParams& p, int64_t u, int64_t unit) {
    if (p.single || !p.homogeneous || p.offs != nullptr || count <= 0) return;
    const int64_t e = u / ceil_div64(count, unit);
    if (e >= p.problem_count || e == problem || e == ahead_problem) return;
    ahead_problem = static_cast<int>(e);
    ahead_a = reinterpret_cast<const char*>(p.a_ptrs[e]);
    ahead_b = reinterpret_cast<const char*>(p.b_ptrs[e]);
    ahead_c = reinterpret_cast<char*>(p.c_ptrs[e]);
  }

  // Moves to the problem holding global unit `u` of `unit` tiles each and
  // returns its global tile range [t0, t1); false when `u` is past the end.
  // The walk must only be driven by seek_unit (not mixed with seek).
  __device__ __forceinline__ bool seek_unit(const GroupedParams& p, int64_t u, int64_t unit, int64_t& t0,
                                            int64_t& t1) {
    if (p.single || p.homogeneous) {
      if (problem < 0) {  // every problem is p.m x p.n: no table load needed
        m_blocks = ceil_div64(p.m, TM);
        count = (p.m > 0 && p.n > 0) ? m_blocks * ceil_div64(p.n, TN) : 0;
      }
      const int total_problems = p.single ? 1 : p.problem_count;
      if (count == 0) return false;
      ucount = ceil_div64(count, unit);
      const int64_t e = u / ucount;
      if (e >= total_problems) return false;
      if (e != problem) {
        problem = static_cast<int>(e);
        first = e * count;
        if (problem == ahead_problem) {
          prob = homogeneous_problem(p, ahead_a, ahead_b, ahead_c);
        } else {
          prob = load_problem(p, problem);
        }
      }
      ufirst = e * ucount;
    } else if (p.unit_start != nullptr) {
      // Largest problem whose first unit is <= u (empty problems share their
      // successor's start, so the search lands on the one that owns u).
      const int64_t* us = p.unit_start;
      if (u >= us[p.problem_count]) return false;
      if (problem < 0 || u >= ufirst + ucount) {
        int lo = problem < 0 ? 0 : problem;
        int hi = p.problem_count - 1;
        while (lo < hi) {
          const int mid = (lo + hi + 1) >> 1;
          if (us[mid] <= u) {
            lo = mid;
          } else {
            hi = mid - 1;
          }
        }
        problem = lo;
        prob = load_problem(p, problem);
        m_blocks = ceil_div64(prob.m, TM);
        count = m_blocks * ceil_div64(prob.n, TN);
        first = 0;  // tiles are numbered inside the problem
        ufirst = us[problem];
        ucount = us[problem + 1] - ufirst;
      }
    } else {
      while (problem < 0 || u >= ufirst + ucount) {
        first += count;
        ufirst += ucount;
        ++problem;
        if (problem >= p.problem_count) return false;
        prob = load_problem(p, problem);
        if (prob.m <= 0 || prob.n <= 0 || prob.k < 0) {
          count = 0;
          ucount = 0;
          m_blocks = 1;
          continue;
        }
        m_blocks = ceil_div64(prob.m, TM);
        count = m_blocks * ceil_div64(prob.n, TN);
        ucount = ceil_div64(count, unit);
      }
    }
    t0 = first + (u - ufirst) * unit;
    t1 = t0 + unit < first + count ? t0 + unit : first + count;
    return true;
  }

  // This CTA's next tile under the unit schedule (units first_unit,
  // first_unit + stride, ...; U = p.unit_tiles tiles each): the next tile of
  // the current unit, else the first tile of the next unit.  False at the end.
  int64_t unit_index = -1;
  int64_t unit_next = 0;  // next tile of the current unit
  int64_t unit_end = 0;   // end of the current unit
  __device__ __forceinline__ bool next_tile(const GroupedParams& p, int64_t first_unit, int64_t stride, int64_t& t) {
    if (unit_next < unit_end) {
      t = unit_next++;
      return true;
    }
    unit_index = unit_index < 0 ? first_unit : unit_index + stride;
    int64_t t0 = 0, t1 = 0;
    const int64_t unit = p.unit_tiles > 0 ? p.unit_tiles : 1;
    if (!seek_unit(p, unit_index, unit, t0, t1)) return false;
    prefetch_unit(p, unit_index + stride, unit);
    t = t0;
    unit_next = t0 + 1;
    unit_end = t1;
    return true;
  }

  // Moves to the problem holding global tile `t`; false when `t` is past the end.
  __device__ __forceinline__ bool seek(const GroupedParams& p, int64_t t) {
    if (p.single || p.homogeneous) {
      if (problem < 0) {
        Problem q = load_problem(p, 0);
        m_blocks = ceil_div64(q.m, TM);
        count = (q.m > 0 && q.n > 0) ? m_blocks * ceil_div64(q.n, TN) : 0;
      }
      const int total_problems = p.single ? 1 : p.problem_count;
      if (count == 0) return false;
      const int64_t e = t / count;
      if (e >= total_problems) return false;
      if (e != problem) {
        problem = static_cast<int>(e);
        first = e * count;
        prob = load_problem(p, problem);
      }
      return true;
    }
    while (problem < 0 || t >= first + count) {
      first += count;
      ++problem;
      if (problem >= p.problem_count) return false;
      prob = load_problem(p, problem);
      if (prob.m <= 0 || prob.n <= 0 || prob.k < 0) {
        count = 0;
        m_blocks = 1;
        continue;
      }
      m_blocks = ceil_div64(prob.m, TM);
      count = m_blocks * ceil_div64(prob.n, TN);
    }
    return true;
  }

  // Tiles are rastered in bands of kBand M-blocks: inside a band the M-block
  // runs fastest, then the N-block.  With at most kBand M-blocks (every MoE
  // expert here) that is plain M-fastest order; for one large GEMM it keeps
  // the tiles in flight on a kBand x (grid / kBand) patch whose A rows and B
  // columns both fit in L2, instead of sweeping every A row per B column.
  static constexpr int64_t kBand = 8;

  __device__ __forceinline__ int64_t m_block(int64_t t) const {
    const int64_t local = t - first;
    const int64_t band_tiles = kBand * (count / m_blocks);
    const int64_t band = local / band_tiles;
    const int64_t rows = m_blocks - band * kBand < kBand ? m_blocks - band * kBand : kBand;
    return band * kBand + (local - band * band_tiles) % rows;
  }
  __device__ __forceinline__ int64_t n_block(int64_t t) const {
    const int64_t local = t - first;
    const int64_t band_tiles = kBand * (count / m_blocks);
    const int64_t band = local / band_tiles;
    const int64_t rows = m_blocks - band * kBand < kBand ? m_blocks - band * kBand : kBand;
    return (local - band * band_tiles) / rows;
  }
};

}  // namespace mgb
