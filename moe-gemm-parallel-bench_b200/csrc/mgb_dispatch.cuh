// Host-side launch of one native kernel variant.  The variant templates are
// instantiated per element type in mgb_tc_{f16,bf16,f32}.cu so the three
// families compile in parallel.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include "mgb_common.cuh"

namespace mgb {

// A native tensor-core tile: orientation and token / weight tile extents.
struct TcVariant {
  bool swap;
  int tm;
  int tn;
};

// Compile-time facts of a variant the host needs (box sizes, ring depth, slots).
struct TcVariantInfo {
  int bk;
  int stages;
  int slots;
  int smem_bytes;
};

// Returns false for a variant that is not instantiated.
template <typename T>
bool tc_variant_info(const TcVariant& v, TcVariantInfo* info);

// Launches tc_grouped_kernel<T, v.swap, v.tm, v.tn>; returns a cudaError_t value.
template <typename T>
int tc_launch(const TcVariant& v, const CUtensorMap& act, const CUtensorMap& wgt, const GroupedParams& p,
              int grid, cudaStream_t stream);

// Launches simt_grouped_kernel<T>; returns a cudaError_t value.
template <typename T>
int simt_launch(const GroupedParams& p, int grid, cudaStream_t stream);

}  // namespace mgb
