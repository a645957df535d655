// Expert-parallel dispatch and combine over peer memory (NVLink / NVSwitch).
//
// Every rank owns one device region (moe_ep_shared_alloc) that its peers map
// through CUDA IPC; a rank's kernels get the base of every rank's region and
// move data with loads, stores and (dispatch) bulk shared -> global copies to
// peer memory (no NCCL, no multicast).
// Region of one rank (byte offsets from moe_ep_region_layout):
//
//   control    uint32 flags[3][MGB_EP_MAX_WORLD] (phase, source rank), the
//              rank's epoch, a block-completion counter, the receive total
//   counts     int32 [2][world][E]  every rank's per-expert slot counts,
//              written by their owners; double-buffered by epoch parity
//   send_base  int32 [E]   where this rank's slots of expert e start in the
//              owning rank's receive rows (local use)
//   recv_offs  int32 [E_l] cumulative row ends of the local experts in the
//              receive rows: the grouped GEMM's offs
//   recv       rows [capacity][hidden]  token rows sent to this rank, sorted
//              by local expert, then by source rank, then by slot position
//   out        rows [capacity][hidden]  the experts' outputs, same order;
//              the source ranks read their rows back from here
//   origin     int64 [capacity]  per receive row: source rank << 40 | the
//              slot's index on the source (written by the dispatch)
//   ret        rows [max_slots][hidden]  expert outputs returned to this rank
//              by the owners' W2 epilogues, indexed by slot
//
// One forward (all on the caller's stream, no host synchronisation):
//   moe_route_layout         counts[E], position[slot] (local)
//   moe_ep_exchange_counts   epoch += 1; counts row -> every peer; barrier 0;
//                            send_base and recv_offs from the full table
//   moe_ep_dispatch          x rows -> owners' recv rows (peer stores); the
//                            last block signals barrier 1 and waits for it
//   grouped GEMMs            recv -> (W13, SwiGLU) -> (W2) -> out, per expert;
//                            or W2 scattered from its epilogue to the source
//                            ranks' ret rows (grouped_gemm_offsets_scatter_launch)
//   moe_ep_combine           barrier 2; out[t] = sum_j w_tj * owner's out row,
//                            or * this rank's ret row of the slot
//
// Reuse is safe without more barriers: a rank writes into a peer's recv rows
// or counts only after barrier 0 of the next forward, which the peer passes
// only after finishing its previous forward, and overwrites its own out rows
// (or a peer's ret rows) only after barrier 1, which every peer passes only
// after its combine.
// Every wait is bounded by a globaltimer deadline; on expiry the kernel ORs
// kErrPeerWait into the device error word and returns.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstring>

#include "../../include/moe_gemm_b200.h"
#include "mgb_dispatch.cuh"
#include "mgb_ptx.cuh"

namespace {

constexpr int kFlagWords = 3 * MGB_EP_MAX_WORLD;
constexpr int kEpochWord = kFlagWords;       // this rank's forward counter
constexpr int kDoneWord = kFlagWords + 1;    // dispatch blocks finished
constexpr int kRecvTotalWord = kFlagWords + 2;
constexpr int64_t kControlBytes = 256;
constexpr int kThreads = 256;
constexpr int kMaxExperts = 8192;
constexpr long long kDefaultTimeoutNs = 10ll * 1000 * 1000 * 1000;

struct EpArgs {
  const int64_t* peers;  // device [world]: each rank's region base in this process
  int32_t rank;
  int32_t world;
  int32_t experts;
  int32_t local_experts;
  int64_t capacity;
  int64_t max_slots;
  int64_t row_bytes;
  mgb_ep_region layout;
  unsigned long long timeout_ns;
  uint32_t* err;
};

int64_t align_up(int64_t v, int64_t a) { return (v + a - 1) / a * a; }

__device__ __forceinline__ int64_t min64(int64_t x, int64_t y) { return x < y ? x : y; }

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void store_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t load_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ char* region_of(const EpArgs& a, int r) {
  return reinterpret_cast<char*>(static_cast<uintptr_t>(a.peers[r]));
}

__device__ __forceinline__ uint32_t* flag_of(char* region, int phase, int source) {
  return reinterpret_cast<uint32_t*>(region) + phase * MGB_EP_MAX_WORLD + source;
}

// Publishes this rank's arrival at `phase` of forward `epoch` to every rank
// (including itself), then waits until every rank has arrived here.  Called
// by one thread after the writes it covers are ordered before it.
__device__ bool signal_and_wait(const EpArgs& a, int phase, uint32_t epoch) {
  __threadfence_system();
  for (int d = 0; d < a.world; ++d) store_release_sys(flag_of(region_of(a, d), phase, a.rank), epoch);
  const uint32_t* own = flag_of(region_of(a, a.rank), phase, 0);
  const unsigned long long start = global_ns();
  for (int s = 0; s < a.world; ++s) {
    while (static_cast<int32_t>(load_acquire_sys(own + s) - epoch) < 0) {
      if (global_ns() - start > a.timeout_ns) {
        atomicOr(a.err, mgb::kErrPeerWait);
        return false;
      }
      __nanosleep(128);
    }
  }
  __threadfence_system();
  return true;
}

// One block: bump the epoch, publish counts, barrier 0, then the layout.
__global__ void __launch_bounds__(1024) ep_exchange_kernel(const int32_t* __restrict__ counts, EpArgs a) {
  extern __shared__ int32_t s_total[];  // [experts] slots per expert over all ranks
  __shared__ uint32_t s_epoch;
  __shared__ int s_ok;
  char* self = region_of(a, a.rank);
  uint32_t* control = reinterpret_cast<uint32_t*>(self);
  if (threadIdx.x == 0) {
    s_epoch = control[kEpochWord] + 1;
    control[kEpochWord] = s_epoch;
  }
  __syncthreads();
  const uint32_t epoch = s_epoch;
  const int parity = static_cast<int>(epoch & 1u);
  const int E = a.experts;
  for (int i = threadIdx.x; i < a.world * E; i += blockDim.x) {
    const int d = i / E;
    const int e = i - d * E;
    int32_t* table = reinterpret_cast<int32_t*>(region_of(a, d) + a.layout.counts);
    table[(parity * a.world + a.rank) * E + e] = counts[e];
  }
  __syncthreads();
  if (threadIdx.x == 0) s_ok = signal_and_wait(a, 0, epoch) ? 1 : 0;
  __syncthreads();

  const int32_t* table = reinterpret_cast<const int32_t*>(self + a.layout.counts) + parity * a.world * E;
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int32_t total = 0;
    for (int s = 0; s < a.world; ++s) total += __ldcg(table + s * E + e);
    s_total[e] = s_ok ? total : 0;
  }
  __syncthreads();
  int32_t* send_base = reinterpret_cast<int32_t*>(self + a.layout.send_base);
  int32_t* recv_offs = reinterpret_cast<int32_t*>(self + a.layout.recv_offs);
  const int El = a.local_experts;
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int64_t start = 0;
    for (int e2 = (e / El) * El; e2 < e; ++e2) start += s_total[e2];
    int64_t before = 0;
    for (int s = 0; s < a.rank; ++s) before += __ldcg(table + s * E + e);
    // A failed barrier leaves nothing to send: every row lands past capacity.
    send_base[e] = static_cast<int32_t>(s_ok ? min64(start + before, a.capacity) : a.capacity);
  }
  for (int el = threadIdx.x; el < El; el += blockDim.x) {
    int64_t end = 0;
    for (int e2 = a.rank * El; e2 <= a.rank * El + el; ++e2) end += s_total[e2];
    recv_offs[el] = static_cast<int32_t>(min64(end, a.capacity));
    if (el == El - 1) control[kRecvTotalWord] = static_cast<uint32_t>(min64(end, a.capacity));
  }
}

// Slots of one token handled together: their row addresses live in registers.
constexpr int kFan = 8;

// Receive row of slot i on its owner (-1: dropped slot; a slot past capacity
// also reports when `report`).
__device__ __forceinline__ int64_t slot_recv_row(const EpArgs& a, const int32_t* send_base, const int32_t* ids,
                                                 const int32_t* position, int64_t i, bool report) {
  const int32_t e = ids[i];
  const int32_t pos = position[i];
  if (e < 0 || e >= a.experts || pos < 0) return -1;
  const int64_t row = static_cast<int64_t>(send_base[e]) + pos;
  if (row >= a.capacity) {
    if (report) atomicOr(a.err, mgb::kErrCapacity);
    return -1;
  }
  return row;
}

// Address of slot i's row in its owner's region section `section` (recv or
// out), or nullptr for a dropped slot.
__device__ __forceinline__ uint8_t* slot_row(const EpArgs& a, const int32_t* send_base, const int32_t* ids,
                                             const int32_t* position, int64_t i, int64_t section, int lane) {
  const int64_t row = slot_recv_row(a, send_base, ids, position, i, lane == 0 && section == a.layout.recv);
  if (row < 0) return nullptr;
  return reinterpret_cast<uint8_t*>(region_of(a, ids[i] / a.local_experts) + section) + row * a.row_bytes;
}

// Where the expert output of kept slot i is read by the combine: the owner's
// out row, or this rank's ret row i when the owners returned it.
__device__ __forceinline__ const uint8_t* slot_result(const EpArgs& a, const int32_t* send_base, const int32_t* ids,
                                                      const int32_t* position, int64_t i, bool returned) {
  if (!returned) return slot_row(a, send_base, ids, position, i, a.layout.out, 1);
  if (slot_recv_row(a, send_base, ids, position, i, false) < 0) return nullptr;
  return reinterpret_cast<const uint8_t*>(region_of(a, a.rank) + a.layout.ret) + i * a.row_bytes;
}

// One warp per token: its row is read once per group of kFan slots and
// stored to each slot's row in the expert owner's receive rows (peer stores
// for remote owners), four 16-byte chunks per lane in flight.  The block
// that finishes last signals barrier 1 and waits for every rank.
__global__ void __launch_bounds__(kThreads)
    ep_dispatch_kernel(const uint8_t* __restrict__ x, int64_t x_pitch_bytes, const int32_t* __restrict__ ids,
                       const int32_t* __restrict__ position, int64_t tokens, int32_t top_k, bool vec16, EpArgs a) {
  char* self = region_of(a, a.rank);
  uint32_t* control = reinterpret_cast<uint32_t*>(self);
  const int32_t* send_base = reinterpret_cast<const int32_t*>(self + a.layout.send_base);
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x / 32);
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x / 32) + (threadIdx.x >> 5); t < tokens; t += warps) {
    const uint8_t* src = x + t * x_pitch_bytes;
    for (int j0 = 0; j0 < top_k; j0 += kFan) {
      uint8_t* dst[kFan];
#pragma unroll
      for (int j = 0; j < kFan; ++j) {
        const int64_t i = t * top_k + j0 + j;
        const int64_t row = j0 + j < top_k ? slot_recv_row(a, send_base, ids, position, i, lane == 0) : -1;
        dst[j] = nullptr;
        if (row >= 0) {
          char* owner = region_of(a, ids[i] / a.local_experts);
          dst[j] = reinterpret_cast<uint8_t*>(owner + a.layout.recv) + row * a.row_bytes;
          // The owner's W2 epilogue returns this row to (this rank, slot i).
          if (lane == 0) reinterpret_cast<int64_t*>(owner + a.layout.origin)[row] = (static_cast<int64_t>(a.rank) << 40) | i;
        }
      }
      if (vec16) {
        constexpr int kBatch = 4;
        for (int64_t b0 = lane * 16; b0 < a.row_bytes; b0 += kBatch * 32 * 16) {
          uint4 v[kBatch];
#pragma unroll
          for (int u = 0; u < kBatch; ++u) {
            const int64_t b = b0 + u * 32 * 16;
            if (b < a.row_bytes) v[u] = *reinterpret_cast<const uint4*>(src + b);
          }
#pragma unroll
          for (int j = 0; j < kFan; ++j) {
            if (dst[j] == nullptr) continue;
#pragma unroll
            for (int u = 0; u < kBatch; ++u) {
              const int64_t b = b0 + u * 32 * 16;
              if (b < a.row_bytes) *reinterpret_cast<uint4*>(dst[j] + b) = v[u];
            }
          }
        }
      } else {
        for (int64_t b = lane * 2; b < a.row_bytes; b += 32 * 2) {
          const uint16_t v = *reinterpret_cast<const uint16_t*>(src + b);
#pragma unroll
          for (int j = 0; j < kFan; ++j) {
            if (dst[j] != nullptr) *reinterpret_cast<uint16_t*>(dst[j] + b) = v;
          }
        }
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const uint32_t finished = atomicAdd(control + kDoneWord, 1u);
    if (finished == gridDim.x - 1) {
      atomicExch(control + kDoneWord, 0u);
      signal_and_wait(a, 1, __ldcg(control + kEpochWord));
    }
  }
}

// Bulk variant of ep_dispatch_kernel for 16-byte-aligned rows of at most
// kBulkRowBytes: one warp per token stages the row in shared memory (coalesced
// 16-byte loads), then lane j copies it to slot j's receive row with one
// cp.async.bulk shared -> global store (peer memory for remote owners), so each
// row crosses NVLink as one bulk transfer instead of 16-byte stores.  Each warp
// alternates two row buffers; a buffer is refilled only after the copies issued
// from it two tokens earlier have read it.  Before the block's completion
// count, every lane waits for its copies to be performed and fences the async
// proxy against the generic one.
constexpr int kBulkWarps = 4;
constexpr int64_t kBulkRowBytes = 24 * 1024;

__global__ void __launch_bounds__(32 * kBulkWarps)
    ep_dispatch_bulk_kernel(const uint8_t* __restrict__ x, int64_t x_pitch_bytes, const int32_t* __restrict__ ids,
                            const int32_t* __restrict__ position, int64_t tokens, int32_t top_k, EpArgs a) {
  extern __shared__ __align__(128) uint8_t bulk_smem[];
  char* self = region_of(a, a.rank);
  uint32_t* control = reinterpret_cast<uint32_t*>(self);
  const int32_t* send_base = reinterpret_cast<const int32_t*>(self + a.layout.send_base);
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int64_t stride = (a.row_bytes + 127) / 128 * 128;
  uint8_t* buffers = bulk_smem + static_cast<int64_t>(warp) * 2 * stride;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * kBulkWarps;
  uint32_t iter = 0;
  for (int64_t t = blockIdx.x * static_cast<int64_t>(kBulkWarps) + warp; t < tokens; t += warps, ++iter) {
    uint8_t* buf = buffers + (iter & 1u) * stride;
    mgb::bulk_wait_group_read<1>();  // this lane's copies from `buf` (two tokens ago) have read it
    __syncwarp();
    const uint8_t* src = x + t * x_pitch_bytes;
    for (int64_t b = lane * 16; b < a.row_bytes; b += 32 * 16) {
      *reinterpret_cast<uint4*>(buf + b) = *reinterpret_cast<const uint4*>(src + b);
    }
    mgb::fence_proxy_async_smem();  // the row's generic writes -> visible to the bulk copies
    __syncwarp();
    for (int j = lane; j < top_k; j += 32) {
      const int64_t i = t * top_k + j;
      const int64_t row = slot_recv_row(a, send_base, ids, position, i, true);
      if (row < 0) continue;
      char* owner = region_of(a, ids[i] / a.local_experts);
      uint8_t* dst = reinterpret_cast<uint8_t*>(owner + a.layout.recv) + row * a.row_bytes;
      // The owner's W2 epilogue returns this row to (this rank, slot i).
      reinterpret_cast<int64_t*>(owner + a.layout.origin)[row] = (static_cast<int64_t>(a.rank) << 40) | i;
      asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst),
                   "r"(static_cast<uint32_t>(__cvta_generic_to_shared(buf))), "r"(static_cast<uint32_t>(a.row_bytes))
                   : "memory");
    }
    mgb::bulk_commit_group();
  }
  mgb::bulk_wait_group_all();  // this lane's copies are performed
  asm volatile("fence.proxy.async.global;" ::: "memory");
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const uint32_t finished = atomicAdd(control + kDoneWord, 1u);
    if (finished == gridDim.x - 1) {
      atomicExch(control + kDoneWord, 0u);
      signal_and_wait(a, 1, __ldcg(control + kEpochWord));
    }
  }
}

// One thread: barrier 2 (every rank's expert outputs are complete).
__global__ void ep_barrier_kernel(EpArgs a, int phase) {
  if (threadIdx.x == 0) {
    const uint32_t* control = reinterpret_cast<const uint32_t*>(region_of(a, a.rank));
    signal_and_wait(a, phase, __ldcg(control + kEpochWord));
  }
}

// One warp per token: fp32 weighted sum of the token's expert outputs, read
// from the owners' out rows (peer loads for remote owners); bf16 result.
// Each lane loads its 16-byte chunk of all the group's slots before summing,
// so kFan loads per lane are in flight.
__global__ void __launch_bounds__(kThreads)
    ep_combine_kernel(const int32_t* __restrict__ ids, const float* __restrict__ weights,
                      const int32_t* __restrict__ position, int64_t tokens, int32_t top_k,
                      __nv_bfloat16* __restrict__ out, int64_t out_pitch, int64_t hidden, bool vec8, bool returned,
                      EpArgs a) {
  const char* self = region_of(a, a.rank);
  const int32_t* send_base = reinterpret_cast<const int32_t*>(self + a.layout.send_base);
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x / 32);
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x / 32) + (threadIdx.x >> 5); t < tokens; t += warps) {
    __nv_bfloat16* dst = out + t * out_pitch;
    const bool one_group = top_k <= kFan;
    const uint8_t* src[kFan];
    float w[kFan];
    if (one_group) {
#pragma unroll
      for (int j = 0; j < kFan; ++j) {
        src[j] = j < top_k ? slot_result(a, send_base, ids, position, t * top_k + j, returned) : nullptr;
        w[j] = src[j] != nullptr ? weights[t * top_k + j] : 0.f;
      }
    }
    if (vec8) {
      for (int64_t c = lane * 8; c < hidden; c += 32 * 8) {
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int j0 = 0; j0 < top_k; j0 += kFan) {
          if (!one_group) {
#pragma unroll
            for (int j = 0; j < kFan; ++j) {
              src[j] = j0 + j < top_k ? slot_result(a, send_base, ids, position, t * top_k + j0 + j, returned)
                                      : nullptr;
              w[j] = src[j] != nullptr ? weights[t * top_k + j0 + j] : 0.f;
            }
          }
          uint4 raw[kFan];
#pragma unroll
          for (int j = 0; j < kFan; ++j) {
            raw[j] = src[j] != nullptr ? __ldcg(reinterpret_cast<const uint4*>(src[j] + c * 2)) : make_uint4(0, 0, 0, 0);
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
        for (int j = 0; j < top_k; ++j) {
          const uint8_t* y = slot_result(a, send_base, ids, position, t * top_k + j, returned);
          if (y != nullptr) {
            acc = fmaf(weights[t * top_k + j], __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(y)[c]), acc);
          }
        }
        dst[c] = __float2bfloat16_rn(acc);
      }
    }
  }
}

int grid_for(int64_t items, int per_block) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t blocks = (items + per_block - 1) / per_block;
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(blocks, 8ll * sms)));
}

bool aligned16(const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

// Validates a configuration and fills the kernels' argument block.
int make_args(const mgb_ep_config* cfg, const int64_t* peer_regions, EpArgs* a) {
  if (cfg == nullptr || peer_regions == nullptr) return MGB_ERR_INVALID;
  if (cfg->world <= 0 || cfg->world > MGB_EP_MAX_WORLD || cfg->rank < 0 || cfg->rank >= cfg->world ||
      cfg->num_experts <= 0 || cfg->num_experts > kMaxExperts || cfg->num_experts % cfg->world != 0 ||
      cfg->hidden <= 0 || cfg->capacity < 0 || cfg->capacity >= (1ll << 31) || cfg->elem_bytes != 2 ||
      cfg->max_slots < 0 || cfg->max_slots >= (1ll << 40)) {
    return MGB_ERR_INVALID;
  }
  std::memset(a, 0, sizeof(*a));
  if (moe_ep_region_layout(cfg->world, cfg->num_experts, cfg->hidden, cfg->capacity, cfg->max_slots,
                           cfg->elem_bytes, &a->layout) != MGB_OK) {
    return MGB_ERR_INVALID;
  }
  a->err = mgb::current_error_word();
  if (a->err == nullptr) return MGB_ERR_CUDA;
  a->peers = peer_regions;
  a->rank = cfg->rank;
  a->world = cfg->world;
  a->experts = cfg->num_experts;
  a->local_experts = cfg->num_experts / cfg->world;
  a->capacity = cfg->capacity;
  a->max_slots = cfg->max_slots;
  a->row_bytes = cfg->hidden * cfg->elem_bytes;
  a->timeout_ns = static_cast<unsigned long long>(cfg->timeout_ns > 0 ? cfg->timeout_ns : kDefaultTimeoutNs);
  return MGB_OK;
}

}  // namespace

extern "C" {

int moe_ep_region_layout(int32_t world, int32_t num_experts, int64_t hidden, int64_t capacity, int64_t max_slots,
                         int32_t elem_bytes, mgb_ep_region* layout) {
  if (layout == nullptr || world <= 0 || world > MGB_EP_MAX_WORLD || num_experts <= 0 ||
      num_experts % world != 0 || hidden <= 0 || capacity < 0 || max_slots < 0 || elem_bytes <= 0) {
    return MGB_ERR_INVALID;
  }
  mgb_ep_region r;
  r.counts = kControlBytes;
  r.send_base = align_up(r.counts + 2ll * world * num_experts * 4, 256);
  r.recv_offs = align_up(r.send_base + 4ll * num_experts, 256);
  r.recv = align_up(r.recv_offs + 4ll * (num_experts / world), 1024);
  r.out = align_up(r.recv + capacity * hidden * elem_bytes, 1024);
  r.origin = align_up(r.out + capacity * hidden * elem_bytes, 1024);
  r.ret = align_up(r.origin + capacity * 8, 1024);
  r.bytes = align_up(r.ret + max_slots * hidden * elem_bytes, 1024);
  *layout = r;
  return MGB_OK;
}

int moe_ep_shared_alloc(size_t bytes, void** region, void* ipc_handle) {
  if (region == nullptr || bytes == 0) return MGB_ERR_INVALID;
  void* ptr = nullptr;
  if (cudaMalloc(&ptr, bytes) != cudaSuccess) return MGB_ERR_CUDA;
  if (cudaMemset(ptr, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
    cudaFree(ptr);
    return MGB_ERR_CUDA;
  }
  if (ipc_handle != nullptr) {
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, ptr) != cudaSuccess) {
      cudaFree(ptr);
      return MGB_ERR_CUDA;
    }
    static_assert(sizeof(h) == MGB_EP_HANDLE_BYTES, "IPC handle size");
    std::memcpy(ipc_handle, &h, sizeof(h));
  }
  *region = ptr;
  return MGB_OK;
}

int moe_ep_shared_free(void* region) {
  if (region == nullptr) return MGB_OK;
  return cudaFree(region) == cudaSuccess ? MGB_OK : MGB_ERR_CUDA;
}

int moe_ep_peer_open(const void* ipc_handle, void** region) {
  if (ipc_handle == nullptr || region == nullptr) return MGB_ERR_INVALID;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof(h));
  void* ptr = nullptr;
  if (cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return MGB_ERR_CUDA;
  *region = ptr;
  return MGB_OK;
}

int moe_ep_peer_close(void* region) {
  if (region == nullptr) return MGB_OK;
  return cudaIpcCloseMemHandle(region) == cudaSuccess ? MGB_OK : MGB_ERR_CUDA;
}

int moe_ep_exchange_counts(const int32_t* counts, const int64_t* peer_regions, const mgb_ep_config* config,
                           void* stream) {
  EpArgs a;
  if (int st = make_args(config, peer_regions, &a)) return st;
  if (counts == nullptr) return MGB_ERR_INVALID;
  const size_t smem = sizeof(int32_t) * static_cast<size_t>(a.experts);
  ep_exchange_kernel<<<1, 1024, smem, static_cast<cudaStream_t>(stream)>>>(counts, a);
  return cudaGetLastError() == cudaSuccess ? MGB_OK : MGB_ERR_CUDA;
}

int moe_ep_dispatch(const void* x, int64_t x_pitch, const int32_t* topk_ids, const int32_t* position,
                    int64_t tokens, int32_t top_k, const int64_t* peer_regions, const mgb_ep_config* config,
                    void* stream) {
  EpArgs a;
  if (int st = make_args(config, peer_regions, &a)) return st;
  if (tokens < 0 || top_k <= 0 || x_pitch < config->hidden || tokens * top_k > config->max_slots) {
    return MGB_ERR_INVALID;
  }
  if (tokens > 0 && (x == nullptr || topk_ids == nullptr || position == nullptr)) return MGB_ERR_INVALID;
  const int64_t pitch_bytes = x_pitch * config->elem_bytes;
  const bool vec16 = aligned16(x) && a.row_bytes % 16 == 0 && pitch_bytes % 16 == 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // Launched even without slots: every rank takes part in barrier 1.
  if (vec16 && a.row_bytes <= kBulkRowBytes) {
    const size_t smem = static_cast<size_t>(kBulkWarps) * 2 * static_cast<size_t>((a.row_bytes + 127) / 128 * 128);
    static bool configured[128] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) return MGB_ERR_CUDA;
    if (!configured[dev]) {
      if (cudaFuncSetAttribute(ep_dispatch_bulk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(kBulkWarps * 2 * kBulkRowBytes)) != cudaSuccess) {
        return MGB_ERR_CUDA;
      }
      configured[dev] = true;
    }
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t blocks = (tokens + kBulkWarps - 1) / kBulkWarps;
    const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(blocks, sms)));
    ep_dispatch_bulk_kernel<<<grid, 32 * kBulkWarps, smem, s>>>(static_cast<const uint8_t*>(x), pitch_bytes,
                                                                 topk_ids, position, tokens, top_k, a);
  } else {
    ep_dispatch_kernel<<<grid_for(tokens, kThreads / 32), kThreads, 0, s>>>(
        static_cast<const uint8_t*>(x), pitch_bytes, topk_ids, position, tokens, top_k, vec16, a);
  }
  return cudaGetLastError() == cudaSuccess ? MGB_OK : MGB_ERR_CUDA;
}

int moe_ep_combine(const int32_t* topk_ids, const float* topk_weights, const int32_t* position, int64_t tokens,
                   int32_t top_k, const int64_t* peer_regions, const mgb_ep_config* config, int32_t returned,
                   void* out, int64_t out_pitch, void* stream) {
  EpArgs a;
  if (int st = make_args(config, peer_regions, &a)) return st;
  if (tokens < 0 || top_k <= 0 || out_pitch < config->hidden || tokens * top_k > config->max_slots) {
    return MGB_ERR_INVALID;
  }
  if (tokens > 0 && (topk_ids == nullptr || topk_weights == nullptr || position == nullptr || out == nullptr)) {
    return MGB_ERR_INVALID;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  ep_barrier_kernel<<<1, 32, 0, s>>>(a, 2);
  if (cudaGetLastError() != cudaSuccess) return MGB_ERR_CUDA;
  if (tokens == 0) return MGB_OK;
  const bool vec8 = aligned16(out) && config->hidden % 8 == 0 && out_pitch % 8 == 0;
  ep_combine_kernel<<<grid_for(tokens, kThreads / 32), kThreads, 0, s>>>(
      topk_ids, topk_weights, position, tokens, top_k, static_cast<__nv_bfloat16*>(out), out_pitch,
      config->hidden, vec8, returned != 0, a);
  return cudaGetLastError() == cudaSuccess ? MGB_OK : MGB_ERR_CUDA;
}

}  // extern "C"
