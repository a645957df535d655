// grouped_gemm_launch_noalloc: the grouped GEMM launch for callers that cannot
// allocate device memory.
//
// The tensor-core path of a grouped launch needs scratch in global memory: the
// A, B and C tensor maps of every problem (3 x 128 bytes each) and, after them,
// problem_count + 1 int64 tile-walk offsets, all written by the map-builder
// kernel just before the GEMM kernel reads them.  grouped_gemm_launch takes
// that buffer from its caller.  Some callers have no way to obtain one: a
// plugin inside a host process whose framework owns every byte of device
// memory and hands the plugin only its input and output tensors, or a launch
// path that must never enter the driver's allocator (which can block or
// fail).  This entry point takes its scratch from a fixed array compiled into
// the library instead, so it allocates nothing and frees nothing.
//
// The array is a file-scope __device__ object: every GPU that loads this
// library holds kNoAllocScratchBytes of it until the process exits.  In host
// code its name is only a host-side stand-in, never a device address, so the
// device address is looked up once per device (cudaGetSymbolAddress, with that
// device current) and that address is what the kernels receive.  The lookup is
// cached for the life of the process: after cudaDeviceReset() on a device the
// cached address is stale, so a process that resets a device must not call
// this entry point on it again.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "../../include/moe_gemm_b200.h"

namespace {

// Largest scratch one launch may use: 3 tensor maps of 128 bytes and one int64
// walk offset per problem (+ 8 bytes), so 1 MiB covers groups of up to 2674
// problems (DeepSeek-V3 TP ranks hold 256).
constexpr size_t kNoAllocScratchBytes = MGB_NOALLOC_SCRATCH_BYTES;

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 128;
std::mutex g_setup_mutex;
void* g_scratch_address[kMaxDevices] = {};

// Resolves the device address of g_noalloc_scratch for the current device,
// once per device.  Returns nullptr when the lookup fails.
void* scratch_address(int* device_out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  *device_out = dev;
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_scratch_address[dev] == nullptr) {
    void* ptr = nullptr;
    const cudaError_t err = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (err != cudaSuccess || ptr == nullptr) return nullptr;
    g_scratch_address[dev] = ptr;
  }
  return g_scratch_address[dev];
}

}  // namespace

extern "C" {

int grouped_gemm_launch_noalloc(const int64_t* a_ptrs, const int64_t* b_ptrs, const int64_t* c_ptrs,
                                const int32_t* dims, const int64_t* strides, int32_t problem_count,
                                int32_t homogeneous, int64_t m, int64_t n, int64_t k, int32_t dtype,
                                int32_t precision, int32_t operands_tma_aligned, const mgb_tile_config* config,
                                void* stream, mgb_launch_info* info) {
  int sm_count = 0, dev = -1;
  void* scratch = scratch_address(&dev);
  if (scratch == nullptr) return MGB_ERR_CUDA;
  if (cudaDeviceGetAttribute(&sm_count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return MGB_ERR_CUDA;
  // The launch never needs more than grouped_gemm_scratch_bytes(); a group
  // whose maps would not fit the fixed array is refused before any kernel is
  // chosen, so it is refused whichever path (tensor-core or generic) would
  // have run it.
  if (grouped_gemm_scratch_bytes(problem_count, sm_count) > kNoAllocScratchBytes) return MGB_ERR_SCRATCH;
  return grouped_gemm_launch(a_ptrs, b_ptrs, c_ptrs, dims, strides, problem_count, homogeneous, m, n, k, dtype,
                             precision, operands_tma_aligned, config, scratch, kNoAllocScratchBytes, stream, info);
}

}  // extern "C"
