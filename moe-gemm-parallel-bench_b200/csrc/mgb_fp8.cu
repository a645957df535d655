// FP8 block-scaled grouped GEMM: the native variants and their launches.
#include <cuda.h>
#include <cuda_runtime.h>

#include "mgb_dispatch.cuh"
#include "mgb_fp8_kernel.cuh"

namespace mgb {

// swap-AB 16 / 32 / 64 tokens x 256 weight rows, and 128 x 128 row tiles.
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

bool fp8_variant_info(const TcVariant& v, TcVariantInfo* info) {
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
