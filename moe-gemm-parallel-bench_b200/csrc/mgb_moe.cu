// MoE routing, permutation and combine: the memory-bound kernels around the
// grouped GEMMs of an expert-parallel layer (C ABI in include/moe_gemm_b200.h).
//
//   moe_route_layout  per-expert slot counts and each slot's position inside
//                     its expert (one atomic per slot)
//   moe_permute       token rows -> expert-sorted rows, one warp per token
//                     (the row is read once for its slots), 16-byte copies
//                     when rows allow it
//   moe_combine       expert-sorted results -> tokens, weighted sum over the
//                     token's top-k slots in fp32, one warp per token
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "../../include/moe_gemm_b200.h"

namespace {

constexpr int kThreads = 256;

int grid_for(int64_t work_items, int per_block) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t blocks = (work_items + per_block - 1) / per_block;
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(blocks, 16ll * sms)));
}

__global__ void __launch_bounds__(kThreads) route_layout_kernel(const int32_t* __restrict__ ids, int64_t slots,
                                                               int32_t experts, int32_t* counts,
                                                               int32_t* __restrict__ position) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < slots;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int32_t e = ids[i];
    position[i] = (e >= 0 && e < experts) ? atomicAdd(&counts[e], 1) : -1;
  }
}

// Slots of one token handled together: their row addresses live in registers.
constexpr int kFan = 8;

// One warp per token: its row is read once per group of kFan slots and
// written to each kept slot's row offsets[e] + position[i] of `sorted`, four
// 16-byte chunks per lane in flight.
__global__ void __launch_bounds__(kThreads)
    permute_kernel(const uint8_t* __restrict__ x, int64_t x_pitch, const int32_t* __restrict__ ids,
                   const int32_t* __restrict__ position, const int32_t* __restrict__ offsets, int64_t tokens,
                   int32_t top_k, int32_t experts, int64_t row_bytes, uint8_t* __restrict__ sorted,
                   int64_t sorted_pitch, int32_t elem_bytes, bool vec16) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x / 32);
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x / 32) + (threadIdx.x >> 5); t < tokens; t += warps) {
    const uint8_t* src = x + t * x_pitch;
    for (int j0 = 0; j0 < top_k; j0 += kFan) {
      uint8_t* dst[kFan];
#pragma unroll
      for (int j = 0; j < kFan; ++j) {
        dst[j] = nullptr;
        if (j0 + j < top_k) {
          const int64_t i = t * top_k + j0 + j;
          const int32_t e = ids[i];
          if (e >= 0 && e < experts && position[i] >= 0) {
            dst[j] = sorted + static_cast<int64_t>(offsets[e] + position[i]) * sorted_pitch;
          }
        }
      }
      if (vec16) {
        constexpr int kBatch = 4;
        for (int64_t b0 = lane * 16; b0 < row_bytes; b0 += kBatch * 32 * 16) {
          uint4 v[kBatch];
#pragma unroll
          for (int u = 0; u < kBatch; ++u) {
            const int64_t b = b0 + u * 32 * 16;
            if (b < row_bytes) v[u] = *reinterpret_cast<const uint4*>(src + b);
          }
#pragma unroll
          for (int j = 0; j < kFan; ++j) {
            if (dst[j] == nullptr) continue;
#pragma unroll
            for (int u = 0; u < kBatch; ++u) {
              const int64_t b = b0 + u * 32 * 16;
              if (b < row_bytes) *reinterpret_cast<uint4*>(dst[j] + b) = v[u];
            }
          }
        }
      } else if (elem_bytes == 4) {
        for (int64_t b = lane * 4; b < row_bytes; b += 32 * 4) {
          const uint32_t v = *reinterpret_cast<const uint32_t*>(src + b);
#pragma unroll
          for (int j = 0; j < kFan; ++j) {
            if (dst[j] != nullptr) *reinterpret_cast<uint32_t*>(dst[j] + b) = v;
          }
        }
      } else {
        for (int64_t b = lane * 2; b < row_bytes; b += 32 * 2) {
          const uint16_t v = *reinterpret_cast<const uint16_t*>(src + b);
#pragma unroll
          for (int j = 0; j < kFan; ++j) {
            if (dst[j] != nullptr) *reinterpret_cast<uint16_t*>(dst[j] + b) = v;
          }
        }
      }
    }
  }
}

// One warp per token: out[t] = sum_j w[t, j] y[offsets[e] + position[t k + j]]
// in fp32, bf16 rows.  A group's row addresses and weights are resolved once
// per token; with 16-byte rows each lane loads its chunk of every slot of the
// group before summing, so kFan loads per lane are in flight.
__global__ void __launch_bounds__(kThreads)
    combine_kernel(const __nv_bfloat16* __restrict__ y, int64_t y_pitch, const int32_t* __restrict__ ids,
                   const float* __restrict__ weights, const int32_t* __restrict__ position,
                   const int32_t* __restrict__ offsets, int64_t tokens, int32_t top_k, int32_t experts,
                   int64_t hidden, __nv_bfloat16* __restrict__ out, int64_t out_pitch, bool vec8) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x / 32);
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x / 32) + (threadIdx.x >> 5); t < tokens; t += warps) {
    __nv_bfloat16* dst = out + t * out_pitch;
    auto resolve = [&](int j0, const __nv_bfloat16* (&src)[kFan], float (&w)[kFan]) {
#pragma unroll
      for (int j = 0; j < kFan; ++j) {
        src[j] = nullptr;
        w[j] = 0.f;
        if (j0 + j < top_k) {
          const int64_t i = t * top_k + j0 + j;
          const int32_t e = ids[i];
          if (e >= 0 && e < experts && position[i] >= 0) {
            src[j] = y + static_cast<int64_t>(offsets[e] + position[i]) * y_pitch;
            w[j] = weights[i];
          }
        }
      }
    };
    const __nv_bfloat16* src[kFan];
    float w[kFan];
    const bool one_group = top_k <= kFan;
    if (one_group) resolve(0, src, w);
    if (vec8) {
      for (int64_t c = lane * 8; c < hidden; c += 32 * 8) {
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int j0 = 0; j0 < top_k; j0 += kFan) {
          if (!one_group) resolve(j0, src, w);
          uint4 raw[kFan];
#pragma unroll
          for (int j = 0; j < kFan; ++j) {
            raw[j] = src[j] != nullptr ? *reinterpret_cast<const uint4*>(src[j] + c) : make_uint4(0, 0, 0, 0);
          }
#pragma unroll
          for (int j = 0; j < kFan; ++j) {
            const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw[j]);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const float2 f = __bfloat1622float2(h[q]);
              acc[2 * q] = fmaf(w[j], f.x, acc[2 * q]);
              acc[2 * q + 1] = fmaf(w[j], f.y, acc[2 * q + 1]);
            }
          }
        }
        uint4 packed;
        __nv_bfloat162* o = reinterpret_cast<__nv_bfloat162*>(&packed);
#pragma unroll
        for (int q = 0; q < 4; ++q) o[q] = __floats2bfloat162_rn(acc[2 * q], acc[2 * q + 1]);
        *reinterpret_cast<uint4*>(dst + c) = packed;
      }
    } else {
      for (int64_t c = lane; c < hidden; c += 32) {
        float acc = 0.f;
        for (int j0 = 0; j0 < top_k; j0 += kFan) {
          if (!one_group) resolve(j0, src, w);
#pragma unroll
          for (int j = 0; j < kFan; ++j) {
            if (src[j] != nullptr) acc = fmaf(w[j], __bfloat162float(src[j][c]), acc);
          }
        }
        dst[c] = __float2bfloat16_rn(acc);
      }
    }
  }
}

bool aligned16(const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

}  // namespace

extern "C" {

int moe_route_layout(const int32_t* topk_ids, int64_t tokens, int32_t top_k, int32_t num_experts, int32_t* counts,
                     int32_t* position, void* stream) {
  if (tokens < 0 || top_k <= 0 || num_experts <= 0 || counts == nullptr ||
      (tokens > 0 && (topk_ids == nullptr || position == nullptr))) {
    return MGB_ERR_INVALID;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(counts, 0, sizeof(int32_t) * num_experts, s) != cudaSuccess) return MGB_ERR_CUDA;
  const int64_t slots = tokens * top_k;
  if (slots == 0) return MGB_OK;
  route_layout_kernel<<<grid_for(slots, kThreads), kThreads, 0, s>>>(topk_ids, slots, num_experts, counts, position);
  return cudaGetLastError() == cudaSuccess ? MGB_OK : MGB_ERR_CUDA;
}

int moe_permute(const void* x, int64_t x_pitch, const int32_t* topk_ids, const int32_t* position,
                const int32_t* offsets, int64_t tokens, int32_t top_k, int32_t num_experts, int64_t hidden,
                void* sorted, int64_t sorted_pitch, int32_t elem_bytes, void* stream) {
  if (tokens < 0 || top_k <= 0 || num_experts <= 0 || hidden < 0 || (elem_bytes != 2 && elem_bytes != 4) ||
      x_pitch < hidden || sorted_pitch < hidden) {
    return MGB_ERR_INVALID;
  }
  const int64_t slots = tokens * top_k;
  if (slots == 0 || hidden == 0) return MGB_OK;
  if (x == nullptr || sorted == nullptr || topk_ids == nullptr || position == nullptr || offsets == nullptr) {
    return MGB_ERR_INVALID;
  }
  const int64_t row_bytes = hidden * elem_bytes;
  const bool vec16 = aligned16(x) && aligned16(sorted) && row_bytes % 16 == 0 && (x_pitch * elem_bytes) % 16 == 0 &&
                     (sorted_pitch * elem_bytes) % 16 == 0;
  permute_kernel<<<grid_for(tokens, kThreads / 32), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(x), x_pitch * elem_bytes, topk_ids, position, offsets, tokens, top_k, num_experts,
      row_bytes, static_cast<uint8_t*>(sorted), sorted_pitch * elem_bytes, elem_bytes, vec16);
  return cudaGetLastError() == cudaSuccess ? MGB_OK : MGB_ERR_CUDA;
}

int moe_combine(const void* y, int64_t y_pitch, const int32_t* topk_ids, const float* weights,
                const int32_t* position, const int32_t* offsets, int64_t tokens, int32_t top_k,
                int32_t num_experts, int64_t hidden, void* out, int64_t out_pitch, void* stream) {
  if (tokens < 0 || top_k <= 0 || num_experts <= 0 || hidden < 0 || out_pitch < hidden || y_pitch < hidden) {
    return MGB_ERR_INVALID;
  }
  if (tokens == 0 || hidden == 0) return MGB_OK;
  if (out == nullptr || topk_ids == nullptr || weights == nullptr || position == nullptr || offsets == nullptr ||
      y == nullptr) {
    return MGB_ERR_INVALID;
  }
  const bool vec8 = aligned16(y) && aligned16(out) && hidden % 8 == 0 && y_pitch % 8 == 0 && out_pitch % 8 == 0;
  combine_kernel<<<grid_for(tokens, kThreads / 32), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(y), y_pitch, topk_ids, weights, position, offsets, tokens, top_k, num_experts,
      hidden, static_cast<__nv_bfloat16*>(out), out_pitch, vec8);
  return cudaGetLastError() == cudaSuccess ? MGB_OK : MGB_ERR_CUDA;
}

}  // extern "C"
