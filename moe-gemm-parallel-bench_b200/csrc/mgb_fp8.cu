// FP8 block-scaled grouped GEMM: the native variants and their launches.
#include <cuda.h>
#include <cuda_runtime.h>

#include "mgb_dispatch.cuh"
#include "mgb_fp8_kernel.cuh"

namespace mgb {

// swap-AB 16 / 32 / 64 tokens x 256 weight rows, and 128 x 128 row tiles;
// the CTA-pair 256 x 128 and 256 x 256 tiles (fp8_pair_kernel) are handled
// beside them.
#define MGB_FOR_EACH_FP8_VARIANT(X) \
  X(true, 16, 256)                  \
  X(true, 32, 256)                  \
  X(true, 64, 256)                  \
  X(false, 128, 128)

template <bool SWAP, int TM, int TN>
static int launch_fp8_variant(const CUtensorMap& act, const CUtensorMap& wgt, const CUtensorMap& out,
                              const GroupedParams& p, int grid, cudaStream_t stream) {
  using Cfg = Fp8Cfg<SWAP, TM, TN>;
  static bool configured[128] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 128) return static_cast<int>(cudaErrorInvalidDevice);
  if (!configured[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(fp8_grouped_kernel<SWAP, TM, TN>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
    if (e != cudaSuccess) return static_cast<int>(e);
    configured[dev] = true;
  }
  fp8_grouped_kernel<SWAP, TM, TN><<<grid, Cfg::kThreads, Cfg::kSmemBytes, stream>>>(act, wgt, out, p);
  return static_cast<int>(cudaGetLastError());
}

// Clusters of two the device keeps resident at once for a CTA-pair kernel
// (queried once per device; SMs / 2 when the query is unavailable).  For the
// 256-row tile, 0 (not launchable) unless the compiled kernel's registers per
// thread cover its setmaxnreg split: a split above the block's launch
// registers would leave the promotion warps waiting for registers forever.
template <int TN>
static int fp8_pair_max_clusters() {
  using Cfg = Fp8PairCfgT<TN>;
  static int cached[128] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) return 0;
  if (cached[dev] == 0) {
    if (cudaFuncSetAttribute(fp8_pair_kernel<TN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             Cfg::kSmemBytes) != cudaSuccess) {
      return 0;
    }
    if constexpr (Cfg::kRegSplit) {
      cudaFuncAttributes attr = {};
      if (cudaFuncGetAttributes(&attr, fp8_pair_kernel<TN>) != cudaSuccess) return 0;
      const long long launched = static_cast<long long>(attr.numRegs) * Cfg::kThreads;
      const long long split = 128ll * Cfg::kRegsLow + 32ll * Cfg::kEpiWarps * Cfg::kRegsHigh;
      if (launched < split) {
        cached[dev] = -1;
        return 0;
      }
    }
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(sms & ~1), 1, 1);
    cfg.blockDim = dim3(Cfg::kThreads, 1, 1);
    cfg.dynamicSmemBytes = Cfg::kSmemBytes;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, fp8_pair_kernel<TN>, &cfg) != cudaSuccess || clusters <= 0) {
      cudaGetLastError();
      clusters = sms / 2;
    }
    cached[dev] = clusters;
  }
  return cached[dev] > 0 ? cached[dev] : 0;
}

template <int TN>
static bool fp8_pair_info(TcVariantInfo* info) {
  using Cfg = Fp8PairCfgT<TN>;
  const int clusters = fp8_pair_max_clusters<TN>();
  if (clusters <= 0) return false;
  *info = TcVariantInfo{Cfg::kBK, Cfg::kStages, Cfg::kSmemBytes, clusters, Cfg::kHalfM, Cfg::kHalfN};
  return true;
}

template <int TN>
static int fp8_pair_launch(const CUtensorMap& act, const CUtensorMap& wgt, const CUtensorMap& out,
                           const GroupedParams& p, int grid, cudaStream_t stream) {
  using Cfg = Fp8PairCfgT<TN>;
  if (grid % 2 != 0 || fp8_pair_max_clusters<TN>() <= 0) return static_cast<int>(cudaErrorInvalidValue);
  fp8_pair_kernel<TN><<<grid, Cfg::kThreads, Cfg::kSmemBytes, stream>>>(act, wgt, out, p);
  return static_cast<int>(cudaGetLastError());
}

bool fp8_variant_info(const TcVariant& v, TcVariantInfo* info) {
  if (v.pair) {
    if (v.tm != 256) return false;
    if (v.tn == 128) return fp8_pair_info<128>(info);
    if (v.tn == 256) return fp8_pair_info<256>(info);
    return false;
  }
#define MGB_FP8_INFO(S, M, N)                                                         \
  if (v.swap == S && v.tm == M && v.tn == N) {                                        \
    using Cfg = Fp8Cfg<S, M, N>;                                                      \
    *info = TcVariantInfo{Cfg::kBK, Cfg::kStages, Cfg::kSmemBytes, 0, M, N};          \
    return true;                                                                      \
  }
  MGB_FOR_EACH_FP8_VARIANT(MGB_FP8_INFO)
#undef MGB_FP8_INFO
  return false;
}

int fp8_launch(const TcVariant& v, const CUtensorMap& act, const CUtensorMap& wgt, const CUtensorMap& out,
               const GroupedParams& p, int grid, cudaStream_t stream) {
  if (v.pair) {
    if (v.tm == 256 && v.tn == 128) return fp8_pair_launch<128>(act, wgt, out, p, grid, stream);
    if (v.tm == 256 && v.tn == 256) return fp8_pair_launch<256>(act, wgt, out, p, grid, stream);
    return static_cast<int>(cudaErrorInvalidValue);
  }
#define MGB_FP8_LAUNCH(S, M, N) \
  if (v.swap == S && v.tm == M && v.tn == N) return launch_fp8_variant<S, M, N>(act, wgt, out, p, grid, stream);
  MGB_FOR_EACH_FP8_VARIANT(MGB_FP8_LAUNCH)
#undef MGB_FP8_LAUNCH
  return static_cast<int>(cudaErrorInvalidValue);
}

int fp8_maps_launch(const CUtensorMap& act, const CUtensorMap& wgt, const CUtensorMap& out, const GroupedParams& p,
                    cudaStream_t stream) {
  const int blocks = p.problem_count + (p.unit_start != nullptr ? 1 : 0);
  build_fp8_maps_kernel<<<blocks, 32, 0, stream>>>(act, wgt, out, p);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace mgb
