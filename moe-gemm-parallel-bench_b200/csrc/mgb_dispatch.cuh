// Host-side launch of one native kernel variant.  The variant templates are
// instantiated per element type in mgb_tc_{f16,bf16,f32}.cu so the three
// families compile in parallel.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include "mgb_common.cuh"

namespace mgb {

// A native tensor-core tile: orientation and token / weight tile extents.
// `pair` selects the CTA-pair kernel (tm = tn = 256 per cluster of two CTAs).
struct TcVariant {
  bool swap;
  int tm;
  int tn;
  bool pair = false;
  bool promote = false;  // fp32 only: accumulator chunks summed in registers (tc_grouped_kernel PROMOTE)
};

// Compile-time facts of a variant the host needs (box sizes, ring depth, slots),
// plus, for the CTA-pair kernel, how many clusters the device runs at once.
struct TcVariantInfo {
  int bk;
  int stages;
  int smem_bytes;
  int max_clusters = 0;
  int box_rows = 0;  // token rows one CTA loads per stage (the activation box height)
  int box_cols = 0;  // weight columns one CTA loads per stage
};

// Returns false for a variant that is not instantiated.
template <typename T>
bool tc_variant_info(const TcVariant& v, TcVariantInfo* info);

// Launches tc_grouped_kernel<T, v.swap, v.tm, v.tn> (or the pair kernel);
// returns a cudaError_t value.  `out` is the output map (template for groups).
template <typename T>
int tc_launch(const TcVariant& v, const CUtensorMap& act, const CUtensorMap& wgt, const CUtensorMap& out,
              const GroupedParams& p, int grid, cudaStream_t stream);

// Launches build_maps_kernel<T>: the A / B / C tensor maps of every problem
// of a grouped launch into p.desc_slots; returns a cudaError_t value.
template <typename T>
int maps_launch(const CUtensorMap& act, const CUtensorMap& wgt, const CUtensorMap& out, const GroupedParams& p,
                cudaStream_t stream);

// FP8 block-scaled variants (mgb_fp8.cu): tiles swap-AB {16, 32, 64} x 256
// and 128 x 128; returns false / cudaErrorInvalidValue for others.
bool fp8_variant_info(const TcVariant& v, TcVariantInfo* info);
int fp8_launch(const TcVariant& v, const CUtensorMap& act, const CUtensorMap& wgt, const CUtensorMap& out,
               const GroupedParams& p, int grid, cudaStream_t stream);
int fp8_maps_launch(const CUtensorMap& act, const CUtensorMap& wgt, const CUtensorMap& out, const GroupedParams& p,
                    cudaStream_t stream);

// The current device's error word (device pointer), or nullptr when the CUDA
// runtime cannot resolve it; kernels outside the GEMM families OR their
// kErr* bits into it.
uint32_t* current_error_word();

// Launches simt_grouped_kernel<T>; returns a cudaError_t value.
template <typename T>
int simt_launch(const GroupedParams& p, int grid, cudaStream_t stream);

}  // namespace mgb
