// Instantiates every native variant for one element type (included by the
// per-type translation units with MGB_ELEM defined).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <type_traits>
#include <utility>

#include "mgb_dispatch.cuh"
#include "mgb_simt_kernel.cuh"
#include "mgb_tc2_kernel.cuh"
#include "mgb_tc_kernel.cuh"

namespace mgb {

// The variant list: swap-AB token tiles 16/32/64 (x weight tiles 128/256),
// swap-AB 256 x 128, and MMA-M = 128 token tiles with weight tiles 64/128/256.
#define MGB_FOR_EACH_VARIANT(X) \
  X(true, 16, 128)              \
  X(true, 16, 256)              \
  X(true, 32, 128)              \
  X(true, 32, 256)              \
  X(true, 64, 128)              \
  X(true, 64, 256)              \
  X(true, 256, 128)             \
  X(false, 128, 64)             \
  X(false, 128, 128)            \
  X(false, 128, 256)

// Launches a GEMM kernel on `stream`.  Grouped launches (maps built by
// build_maps_kernel just before) carry programmatic stream serialization, so
// the GEMM grid launches and sets up while the map builder still runs; the
// kernel waits for it (grid_dependency_wait) before reading global memory.
template <typename... Params, typename... Args>
static cudaError_t launch_gemm(void (*kernel)(Params...), int grid, int smem, cudaStream_t stream, bool after_maps,
                               Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
  cfg.blockDim = dim3(kTcThreads, 1, 1);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = after_maps ? attr : nullptr;
  cfg.numAttrs = after_maps ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

template <typename T, bool SWAP, int TM, int TN, bool PROMOTE = false>
static int launch_variant(const CUtensorMap& act, const CUtensorMap& wgt, const CUtensorMap& out,
                          const GroupedParams& p, int grid, cudaStream_t stream) {
  using Cfg = TcCfg<T, SWAP, TM, TN>;
  static bool configured[128] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 128) return static_cast<int>(cudaErrorInvalidDevice);
  if (!configured[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(tc_grouped_kernel<T, SWAP, TM, TN, PROMOTE>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
    if (e != cudaSuccess) return static_cast<int>(e);
    configured[dev] = true;
  }
  const cudaError_t e = launch_gemm(tc_grouped_kernel<T, SWAP, TM, TN, PROMOTE>, grid, Cfg::kSmemBytes, stream,
                                    !p.single, act, wgt, out, p);
  return static_cast<int>(e != cudaSuccess ? e : cudaGetLastError());
}

// The CTA-pair kernel exists for 16-bit types only.
template <typename T>
struct PairKernel {
  static constexpr bool kAvailable = sizeof(T) == 2;
};

// Clusters of two the device keeps resident at once for the pair kernel with
// NH halves (queried once per device; 0 when the query is unavailable).
template <typename T, int NH>
static int pair_max_clusters() {
  if constexpr (!PairKernel<T>::kAvailable) {
    return 0;
  } else {
    static int cached[128] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) return 0;
    if (cached[dev] == 0) {
      using Cfg = Tc2Cfg<T, NH>;
      if (cudaFuncSetAttribute(tc2_grouped_kernel<T, NH>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               Cfg::kSmemBytes) != cudaSuccess) {
        return 0;
      }
      int sms = 0;
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(static_cast<unsigned>(sms & ~1), 1, 1);
      cfg.blockDim = dim3(kTcThreads, 1, 1);
      cfg.dynamicSmemBytes = Cfg::kSmemBytes;
      int clusters = 0;
      if (cudaOccupancyMaxActiveClusters(&clusters, tc2_grouped_kernel<T, NH>, &cfg) != cudaSuccess ||
          clusters <= 0) {
        cudaGetLastError();
        clusters = sms / 2;
      }
      cached[dev] = clusters;
    }
    return cached[dev];
  }
}

template <typename T, int NH>
static int launch_pair(const CUtensorMap& act, const CUtensorMap& wgt, const CUtensorMap& out,
                       const GroupedParams& p, int grid, cudaStream_t stream) {
  if constexpr (!PairKernel<T>::kAvailable) {
    return static_cast<int>(cudaErrorInvalidValue);
  } else {
    using Cfg = Tc2Cfg<T, NH>;
    static bool configured[128] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 128) return static_cast<int>(cudaErrorInvalidDevice);
    if (!configured[dev]) {
      const cudaError_t e = cudaFuncSetAttribute(tc2_grouped_kernel<T, NH>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
      if (e != cudaSuccess) return static_cast<int>(e);
      configured[dev] = true;
    }
    const cudaError_t e = launch_gemm(tc2_grouped_kernel<T, NH>, grid, Cfg::kSmemBytes, stream, !p.single, act, wgt,
                                      out, p);
    return static_cast<int>(e != cudaSuccess ? e : cudaGetLastError());
  }
}

template <typename T, int NH>
static bool pair_variant_info(const TcVariant& v, TcVariantInfo* info) {
  if constexpr (!PairKernel<T>::kAvailable) {
    return false;
  } else {
    using Cfg = Tc2Cfg<T, NH>;
    *info = TcVariantInfo{Cfg::kBK, Cfg::kStages, Cfg::kSmemBytes, pair_max_clusters<T, NH>(), Cfg::kHalf,
                          NH * Cfg::kHalf};
    return v.tm == Cfg::kTileM && v.tn == Cfg::kTileN;
  }
}

template <>
bool tc_variant_info<MGB_ELEM>(const TcVariant& v, TcVariantInfo* info) {
  if (v.promote) {
    if constexpr (std::is_same<MGB_ELEM, float>::value) {
      using Cfg = TcCfg<float, false, 128, 128>;
      *info = TcVariantInfo{Cfg::kBK, Cfg::kStages, Cfg::kSmemBytes, 0, 128, 128};
      return v.tm == 128 && v.tn == 128 && !v.swap && !v.pair;
    }
    return false;
  }
  if (v.pair) return v.tn > 256 ? pair_variant_info<MGB_ELEM, 2>(v, info) : pair_variant_info<MGB_ELEM, 1>(v, info);
#define MGB_INFO(S, M, N)                                                               \
  if (v.swap == S && v.tm == M && v.tn == N) {                                          \
    using Cfg = TcCfg<MGB_ELEM, S, M, N>;                                               \
    *info = TcVariantInfo{Cfg::kBK, Cfg::kStages, Cfg::kSmemBytes, 0, M, N};                \
    return true;                                                                        \
  }
  MGB_FOR_EACH_VARIANT(MGB_INFO)
#undef MGB_INFO
  return false;
}

template <>
int tc_launch<MGB_ELEM>(const TcVariant& v, const CUtensorMap& act, const CUtensorMap& wgt, const CUtensorMap& out,
                        const GroupedParams& p, int grid, cudaStream_t stream) {
  if (v.promote) {
    if constexpr (std::is_same<MGB_ELEM, float>::value) {
      return launch_variant<float, false, 128, 128, true>(act, wgt, out, p, grid, stream);
    }
    return static_cast<int>(cudaErrorInvalidValue);
  }
  if (v.pair) {
    return v.tn > 256 ? launch_pair<MGB_ELEM, 2>(act, wgt, out, p, grid, stream)
                      : launch_pair<MGB_ELEM, 1>(act, wgt, out, p, grid, stream);
  }
#define MGB_LAUNCH(S, M, N) \
  if (v.swap == S && v.tm == M && v.tn == N) return launch_variant<MGB_ELEM, S, M, N>(act, wgt, out, p, grid, stream);
  MGB_FOR_EACH_VARIANT(MGB_LAUNCH)
#undef MGB_LAUNCH
  return static_cast<int>(cudaErrorInvalidValue);
}

template <>
int maps_launch<MGB_ELEM>(const CUtensorMap& act, const CUtensorMap& wgt, const CUtensorMap& out,
                          const GroupedParams& p, cudaStream_t stream) {
  const int blocks = p.problem_count + (p.unit_start != nullptr ? 1 : 0);  // + the unit prefix-sum block
  build_maps_kernel<MGB_ELEM><<<blocks, 32, 0, stream>>>(act, wgt, out, p);
  return static_cast<int>(cudaGetLastError());
}

template <>
int simt_launch<MGB_ELEM>(const GroupedParams& p, int grid, cudaStream_t stream) {
  simt_grouped_kernel<MGB_ELEM><<<grid, kSimtThreads, 0, stream>>>(p);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace mgb
