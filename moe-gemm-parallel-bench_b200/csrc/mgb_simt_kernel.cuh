// Generic-stride persistent grouped GEMM on the CUDA cores.
//
// Serves what the TMA path cannot: operands whose strides or base addresses
// break the TMA rules (odd row pitches such as a bf16 [17, 13] matrix, the
// `a[:, ::2]` views of the reference's strided test), and fp32 inputs with
// input_precision = "ieee", where the reference's tl.dot performs full-fp32
// FMAs (kernels/matmul.py:268).  Every element is loaded through its own
// (row * stride_r + col * stride_c) address with bounds masks, accumulated in
// fp32 with fused multiply-adds in increasing K order, and cast on store.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>
#include <type_traits>

#include "mgb_common.cuh"

namespace mgb {

template <typename T>
__device__ __forceinline__ float load_as_float(const char* base, int64_t elem_offset) {
  const T v = reinterpret_cast<const T*>(base)[elem_offset];
  if constexpr (std::is_same<T, float>::value) {
    return v;
  } else if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    return __bfloat162float(v);
  } else {
    return __half2float(v);
  }
}

template <typename T>
__device__ __forceinline__ void store_from_float(char* base, int64_t elem_offset, float v) {
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
__global__ void __launch_bounds__(kSimtThreads) simt_grouped_kernel(const GroupedParams p) {
  __shared__ float a_tile[kSimtBK][kSimtBM + 4];  // [k][m]
  __shared__ float b_tile[kSimtBK][kSimtBN + 4];  // [k][n]
  const int tx = threadIdx.x % 16;  // 4 output columns each
  const int ty = threadIdx.x / 16;  // 4 output rows each
  TileWalk<kSimtBM, kSimtBN> walk;
  for (int64_t t = blockIdx.x; walk.seek(p, t); t += gridDim.x) {
    const Problem& q = walk.prob;
    const int64_t m0 = walk.m_block(t) * kSimtBM;
    const int64_t n0 = walk.n_block(t) * kSimtBN;
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
    for (int64_t k0 = 0; k0 < q.k; k0 += kSimtBK) {
      for (int idx = threadIdx.x; idx < kSimtBM * kSimtBK; idx += kSimtThreads) {
        const int mm = idx / kSimtBK, kk = idx % kSimtBK;
        const int64_t gm = m0 + mm, gk = k0 + kk;
        a_tile[kk][mm] = (gm < q.m && gk < q.k) ? load_as_float<T>(q.a, gm * q.sam + gk * q.sak) : 0.0f;
      }
      for (int idx = threadIdx.x; idx < kSimtBK * kSimtBN; idx += kSimtThreads) {
        const int kk = idx / kSimtBN, nn = idx % kSimtBN;
        const int64_t gk = k0 + kk, gn = n0 + nn;
        b_tile[kk][nn] = (gk < q.k && gn < q.n) ? load_as_float<T>(q.b, gk * q.sbk + gn * q.sbn) : 0.0f;
      }
      __syncthreads();
#pragma unroll
      for (int kk = 0; kk < kSimtBK; ++kk) {
        float av[4], bv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) av[i] = a_tile[kk][ty * 4 + i];
#pragma unroll
        for (int j = 0; j < 4; ++j) bv[j] = b_tile[kk][tx * 4 + j];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
      }
      __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t row = m0 + ty * 4 + i;
      if (row >= q.m) continue;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int64_t col = n0 + tx * 4 + j;
        if (col < q.n) store_from_float<T>(q.c, row * q.scm + col * q.scn, acc[i][j]);
      }
    }
  }
}

}  // namespace mgb
