/*
 * moe_gemm_b200.h -- C ABI of the B200 (sm_100a) MoE expert-GEMM library.
 *
 * The reference (Steam086/moe-gemm-parallel-bench) is pure Python: its hot path
 * is the Triton persistent grouped GEMM of kernels/grouped_gemm.py and the
 * masked single GEMM of kernels/matmul.py.  This header is the native boundary
 * that replaces those Triton launches.  Every entry point takes plain device
 * pointers, sizes and a CUDA stream handle (cudaStream_t passed as void*); no
 * framework types cross it.  The Python package `kernels` (same module and
 * function names as the reference) binds it through ctypes.
 *
 * Element types, precisions and the tile record follow the reference:
 *   dtype      fp16 | bf16 | fp32           utils/benchmark.py:35-38
 *   precision  "ieee" | "tf32"              kernels/matmul.py:268, grouped_gemm.py:389,475
 *   tile       KernelConfig fields          kernels/matmul.py:19-32
 * All launches are asynchronous on `stream` and synchronise nothing.  Those
 * that take their scratch from the caller allocate nothing and may be
 * recorded into a CUDA graph.
 */
#ifndef MOE_GEMM_B200_H
#define MOE_GEMM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum mgb_dtype { MGB_FP16 = 0, MGB_BF16 = 1, MGB_FP32 = 2 };
/* MGB_TF32_FP32ACC (fp32 only, tensor-core path): TF32 products with the
 * tensor core accumulating at most 256 K at a time, the partial sums added in
 * fp32 registers; for operands that are exact in TF32, such as the halves
 * matrix_split_tf32x3 writes.  No counterpart in the reference. */
enum mgb_precision { MGB_IEEE = 0, MGB_TF32 = 1, MGB_TF32_FP32ACC = 2 };

enum mgb_status {
  MGB_OK = 0,
  MGB_ERR_INVALID = 1,     /* bad argument (shape, dtype, null pointer): the reference's ValueError */
  MGB_ERR_UNSUPPORTED = 2, /* no native kernel for this request: the reference's RuntimeError */
  MGB_ERR_CUDA = 3,        /* a CUDA runtime / driver call failed */
  MGB_ERR_SCRATCH = 4      /* scratch buffer missing or smaller than grouped_gemm_scratch_bytes() */
};

/* The fields of the reference's KernelConfig (kernels/matmul.py:19-32).  The
 * library maps block_m / block_n to one of its native tiles; the other fields
 * are accepted for provenance and do not change the kernel that runs. */
typedef struct mgb_tile_config {
  int32_t block_m, block_n, block_k, group_size_m, num_warps, num_stages, cta_multiplier;
} mgb_tile_config;

/* What a launch actually ran (filled when the pointer is non-null). */
typedef struct mgb_launch_info {
  int32_t path;    /* 0 = TMA + tcgen05 tensor-core kernel, 1 = generic-stride SIMT kernel,
                      2 = TMA + tcgen05 on CTA pairs (cta_group::2, 256 x 256 cluster tiles) */
  int32_t swap_ab; /* 1 when the weight dimension is the MMA M dimension (narrow-M variant) */
  int32_t tile_m, tile_n, tile_k, stages, grid;
} mgb_launch_info;

/* Bytes of scratch a grouped launch of `problem_count` problems needs: the
 * A, B and C tensor maps of every problem (3 x 128 bytes each) plus
 * problem_count + 1 int64 tile-walk offsets, built on the device by a small
 * kernel that runs just before the GEMM kernel.  `sm_count` is not used.  Replaces nothing in the reference: Triton kernels there take
 * raw pointers and need no descriptors. */
size_t grouped_gemm_scratch_bytes(int32_t problem_count, int32_t sm_count);

/* One launch of the persistent grouped GEMM: for e in [0, problem_count)
 *   C_e[M_e, N_e] = A_e[M_e, K_e] @ B_e[K_e, N_e]   (fp32 accumulate, cast on store)
 * Replaces the Triton launches of launch_grouped (kernels/grouped_gemm.py:618-760,
 * kernels _homogeneous_grouped_kernel_impl :321-397 and
 * _generic_grouped_kernel_impl :399-482).  The tables are the reference
 * workspace's device tensors (kernels/grouped_gemm.py:530-544):
 *   a_ptrs, b_ptrs, c_ptrs   int64 [problem_count]   device addresses
 *   dims                     int32 [problem_count, 3] (M, N, K) -- note the M, N, K order
 *   strides                  int64 [problem_count, 6] (am, ak, bk, bn, cm, cn), in elements
 * They are read on the device at run time, so an entry changed after the
 * workspace was built is honoured by the next launch.
 *   homogeneous  1 when every problem is (m, n, k) with contiguous strides
 *                (the reference's `homogeneous` flag, :550-552); then dims and
 *                strides are not read.  Otherwise (m, n, k) are the maxima
 *                (MAX_M / MAX_N / MAX_K, :641-649) and size the grid.
 *   operands_tma_aligned  the caller's promise that every A_e / B_e has a
 *                16-byte aligned base, unit inner stride and 16-byte multiple
 *                row pitch.  Then the tensor-core path runs; a table entry that
 *                breaks the promise is skipped on the device and reported in the
 *                error word (never dereferenced).  0 selects the generic path.
 *   scratch      device buffer of at least grouped_gemm_scratch_bytes() bytes,
 *                owned by the caller; not shared by launches that overlap.
 * A tensor-core launch is two kernels on `stream`: the tensor-map builder
 * (one warp per problem) and the GEMM kernel.
 */
int grouped_gemm_launch(const int64_t* a_ptrs, const int64_t* b_ptrs, const int64_t* c_ptrs,
                        const int32_t* dims, const int64_t* strides, int32_t problem_count,
                        int32_t homogeneous, int64_t m, int64_t n, int64_t k, int32_t dtype,
                        int32_t precision, int32_t operands_tma_aligned, const mgb_tile_config* config,
                        void* scratch, size_t scratch_bytes, void* stream, mgb_launch_info* info);

/* Grouped GEMM with the fused SwiGLU epilogue: for e in [0, problem_count)
 *   C_e[M_e, N_e/2] = silu(A_e @ B_e[:, :N_e/2]) * (A_e @ B_e[:, N_e/2:])
 * (silu(x) = x / (1 + exp(-x)), fp32 accumulate, epilogue math in fp32, one
 * cast on store).  B_e is the packed W13 weight [gate | up] of
 * build_fused_gate_up_workspace (kernels/grouped_gemm.py:575-594); the tables
 * and arguments are those of grouped_gemm_launch, with (m, n, k) and `dims`
 * giving the packed N and `strides` C's [M, N/2] strides.  Runs on the
 * tensor-core path only: fp16 / bf16, or fp32 with MGB_TF32, TMA-aligned A / B
 * (operands_tma_aligned = 1) and N/2 a multiple of 16 bytes of elements;
 * otherwise MGB_ERR_UNSUPPORTED (MGB_ERR_INVALID for odd N).  No counterpart
 * in the reference, which leaves SiLU(gate) * up outside its timed GEMM
 * (README.md:55-60): this writes [M, F] instead of [M, 2F] and never reads
 * the [gate | up] intermediate back. */
int grouped_gemm_swiglu_launch(const int64_t* a_ptrs, const int64_t* b_ptrs, const int64_t* c_ptrs,
                               const int32_t* dims, const int64_t* strides, int32_t problem_count,
                               int32_t homogeneous, int64_t m, int64_t n, int64_t k, int32_t dtype,
                               int32_t precision, int32_t operands_tma_aligned, const mgb_tile_config* config,
                               void* scratch, size_t scratch_bytes, void* stream, mgb_launch_info* info);

/* Grouped GEMM over the expert-sorted aggregate layout: for e in [0, problem_count)
 *   C[r0:r1, :] = A[r0:r1, :] @ B[e]      with r0 = offs[e-1] (0 for e = 0), r1 = offs[e]
 * A is one [total_rows, k] matrix of tokens sorted by expert, B one [E, k, n]
 * tensor, C one [total_rows, n] matrix (n / 2 columns with swiglu = 1, which
 * applies the fused SwiGLU epilogue to a packed [gate | up] B).  Row strides
 * are in elements; columns are contiguous; stride_be is the element distance
 * between consecutive experts' B.  `offs` is int32 [problem_count] of
 * cumulative row ends, read on the device (no host synchronisation; empty
 * experts are fine), the format of torch.nn.functional.grouped_mm that the
 * reference's torch provider builds (kernels/torch_grouped_gemm.py:142-158).
 * No counterpart in the reference's own kernels, which take per-expert
 * pointer tables; this removes the tables for callers whose tokens are
 * already permuted by expert.  Tensor-core path when A / B are 16-byte
 * aligned with 16-byte multiple row strides (fp16 / bf16, or fp32 with
 * MGB_TF32); the generic kernel otherwise (swiglu requires the former).
 * Scratch: grouped_gemm_scratch_bytes(problem_count, *). */
int grouped_gemm_offsets_launch(const void* a, const void* b, void* c, const int32_t* offs, int32_t problem_count,
                                int64_t total_rows, int64_t n, int64_t k, int64_t stride_am, int64_t stride_be,
                                int64_t stride_bk, int64_t stride_cm, int32_t dtype, int32_t precision,
                                int32_t swiglu, const mgb_tile_config* config, void* scratch, size_t scratch_bytes,
                                void* stream, mgb_launch_info* info);

/* FP8 block-scaled grouped GEMM (DeepSeek-V3 quantization): for e in [0, problem_count)
 *   C_e[M, N] = sum_kb (A_e[:, kb] @ B_e[:, kb]^T) * SA_e[:, kb] * SB_e[n / 128, kb]
 * over 128-deep K blocks kb, fp32 accumulation, bf16 output.
 *   a_ptrs   e4m3 A_e [M, K], contiguous (tokens)
 *   b_ptrs   e4m3 B_e [N, K], contiguous (a linear weight as checkpoints store it)
 *   c_ptrs   bf16 C_e [M, N], contiguous
 *   sa_ptrs  fp32 SA_e [M, ceil(K/128)]: one scale per token and K block
 *   sb_ptrs  fp32 SB_e [ceil(N/128), ceil(K/128)]: one scale per 128 x 128 weight block
 *   dims     int32 [problem_count, 3] (M, N, K) unless homogeneous (then m, n, k)
 * The tensor-core path needs 16-byte aligned bases, K a multiple of 16 and N a
 * multiple of 8; a homogeneous group that breaks it is refused with
 * MGB_ERR_UNSUPPORTED, a heterogeneous entry is skipped and reported in the
 * error word.  config->block_m picks the tile (<= 16 / 32 / 64: swap-AB with
 * that many tokens x 256 weight rows; up to 255: 128 x 128; from 256: a CTA
 * pair of 256 tokens x 128 weight rows, or x 256 when config->block_n >= 256,
 * refused with MGB_ERR_UNSUPPORTED where the device cannot run that tile).  Scratch:
 * grouped_gemm_scratch_bytes(problem_count, *).  No counterpart in the
 * reference, which runs every expert in fp16 / bf16 / fp32 and notes that the
 * model's FP8 quantization is not emulated (README.md:298). */
int grouped_gemm_fp8_launch(const int64_t* a_ptrs, const int64_t* b_ptrs, const int64_t* c_ptrs,
                            const int64_t* sa_ptrs, const int64_t* sb_ptrs, const int32_t* dims,
                            int32_t problem_count, int32_t homogeneous, int64_t m, int64_t n, int64_t k,
                            const mgb_tile_config* config, void* scratch, size_t scratch_bytes, void* stream,
                            mgb_launch_info* info);

/* grouped_gemm_offsets_launch where several row segments share one B: with
 * b_count > 0, segment e multiplies B[e % b_count] (b_count = 0 is the plain
 * call).  An expert-parallel rank that received P senders' tokens, each sender's
 * block sorted by the rank's b_count local experts, runs its experts over the
 * received buffer as P * b_count segments without re-sorting it. */
int grouped_gemm_offsets_launch_ex(const void* a, const void* b, void* c, const int32_t* offs,
                                   int32_t problem_count, int32_t b_count, int64_t total_rows, int64_t n, int64_t k,
                                   int64_t stride_am, int64_t stride_be, int64_t stride_bk, int64_t stride_cm,
                                   int32_t dtype, int32_t precision, int32_t swiglu, const mgb_tile_config* config,
                                   void* scratch, size_t scratch_bytes, void* stream, mgb_launch_info* info);

/* MoE routing, permutation and combine (an expert-parallel layer around the
 * grouped GEMMs; the reference excludes routing and all-to-all, README.md:14,
 * README.md:35).  topk_ids: int32 [tokens, top_k] global expert ids in
 * [0, num_experts) (others are dropped).  All device pointers, `stream` the
 * caller's.
 *
 * moe_route_layout: counts [num_experts] (int32, zeroed by the call) = slots
 * per expert; position [tokens * top_k] = the slot's index inside its expert
 * (-1 for a dropped slot).  Slots of one expert keep no particular order. */
int moe_route_layout(const int32_t* topk_ids, int64_t tokens, int32_t top_k, int32_t num_experts, int32_t* counts,
                     int32_t* position, void* stream);

/* moe_permute: sorted[offsets[e] + position[i], :] = x[i / top_k, :] for every
 * kept slot i (offsets = exclusive prefix sum of counts, int32
 * [num_experts]); rows of `hidden` elements of elem_bytes (2 or 4), row
 * pitches in elements. */
int moe_permute(const void* x, int64_t x_pitch, const int32_t* topk_ids, const int32_t* position,
                const int32_t* offsets, int64_t tokens, int32_t top_k, int32_t num_experts, int64_t hidden,
                void* sorted, int64_t sorted_pitch, int32_t elem_bytes, void* stream);

/* moe_combine: out[t, :] = sum_j weights[t, j] * y[offsets[e_tj] + position[t*top_k + j], :]
 * over the kept slots of token t (fp32 accumulate, bf16 in and out; a token
 * with no kept slot gets zeros). */
int moe_combine(const void* y, int64_t y_pitch, const int32_t* topk_ids, const float* weights,
                const int32_t* position, const int32_t* offsets, int64_t tokens, int32_t top_k,
                int32_t num_experts, int64_t hidden, void* out, int64_t out_pitch, void* stream);

/* Expert-parallel dispatch and combine over peer memory.  No reference
 * counterpart: the reference stops at the expert GEMMs and leaves routing and
 * the all-to-all out (README.md:14, README.md:35).  Rank r of `world` owns
 * experts [r * E / world, (r + 1) * E / world).  Each rank allocates one
 * region (moe_ep_shared_alloc), sends its IPC handle to the others (any host
 * channel), maps theirs (moe_ep_peer_open) and keeps a device int64 [world]
 * table of every rank's region base as mapped in its own process.  A forward
 * is, on one stream and without host synchronisation:
 *   moe_route_layout -> moe_ep_exchange_counts -> moe_ep_dispatch ->
 *   grouped GEMMs on the region's recv rows (offs = recv_offs, one segment per
 *   local expert) writing its out rows -> moe_ep_combine.
 * Every rank must run every step of every forward (with zero tokens too);
 * barrier waits are bounded by `timeout_ns` (<= 0: 10 s) and report
 * expiry as error bit 9, rows beyond `capacity` as bit 10 (dropped). */
#define MGB_EP_MAX_WORLD 16
#define MGB_EP_HANDLE_BYTES 64

typedef struct mgb_ep_config {
  int32_t rank;
  int32_t world;       /* 1 .. MGB_EP_MAX_WORLD */
  int32_t num_experts; /* global experts E, a multiple of world */
  int32_t elem_bytes;  /* 2: bf16 token rows */
  int64_t hidden;      /* row width H in elements */
  int64_t capacity;    /* receive rows per rank (world * tokens * top_k never drops) */
  int64_t timeout_ns;
  int64_t max_slots;   /* tokens * top_k bound of one forward: rows of the return buffer */
} mgb_ep_config;

/* Byte offsets inside one rank's region (all ranks share the layout):
 * counts int32 [2][world][E], send_base int32 [E], recv_offs int32 [E / world]
 * (cumulative row ends of the local experts: the grouped GEMM's offs), recv and
 * out rows [capacity][hidden], origin int64 [capacity] (receive row -> source
 * rank << 40 | source slot, written by the dispatch), ret rows
 * [max_slots][hidden] (expert outputs returned to this rank, by slot). */
typedef struct mgb_ep_region {
  int64_t counts;
  int64_t send_base;
  int64_t recv_offs;
  int64_t recv;
  int64_t out;
  int64_t origin;
  int64_t ret;
  int64_t bytes;
} mgb_ep_region;

int moe_ep_region_layout(int32_t world, int32_t num_experts, int64_t hidden, int64_t capacity, int64_t max_slots,
                         int32_t elem_bytes, mgb_ep_region* layout);
/* Zero-filled device allocation of `bytes` on the current device; writes its
 * MGB_EP_HANDLE_BYTES-byte CUDA IPC handle when `ipc_handle` is non-null. */
int moe_ep_shared_alloc(size_t bytes, void** region, void* ipc_handle);
int moe_ep_shared_free(void* region);
/* Maps a peer's region (peer access enabled on demand). */
int moe_ep_peer_open(const void* ipc_handle, void** region);
int moe_ep_peer_close(void* region);
/* counts: this rank's moe_route_layout counts [E].  Publishes them to every
 * rank, waits for all ranks, then writes send_base and recv_offs. */
int moe_ep_exchange_counts(const int32_t* counts, const int64_t* peer_regions, const mgb_ep_config* config,
                           void* stream);
/* Copies row i / top_k of x (pitch in elements) to the owner of expert
 * topk_ids[i], at send_base[e] + position[i] of its recv rows; returns after
 * every rank's rows have arrived. */
int moe_ep_dispatch(const void* x, int64_t x_pitch, const int32_t* topk_ids, const int32_t* position,
                    int64_t tokens, int32_t top_k, const int64_t* peer_regions, const mgb_ep_config* config,
                    void* stream);
/* Waits until every rank's out rows are complete, then
 * out[t, :] = sum_j topk_weights[t, j] * (owner's out row of slot t * top_k + j)
 * (fp32 accumulate, bf16 out; dropped slots add nothing).  With `returned`
 * nonzero the rows are read from this rank's own ret rows instead (row
 * t * top_k + j), where the owners' W2 launches stored them
 * (grouped_gemm_offsets_scatter_launch over the origin table). */
int moe_ep_combine(const int32_t* topk_ids, const float* topk_weights, const int32_t* position, int64_t tokens,
                   int32_t top_k, const int64_t* peer_regions, const mgb_ep_config* config, int32_t returned,
                   void* out, int64_t out_pitch, void* stream);

/* Aggregate-layout grouped GEMM whose output rows are scattered: row R of the
 * product (rows of segment e = [offs[e-1], offs[e]), weights B[e % b_count]
 * or B[e]) is stored at byte dst_offset + (row_origin[R] & 0xFFFFFFFFFF) *
 * dst_pitch_bytes of rank (row_origin[R] >> 40)'s region, whose base in this
 * process is peer_regions[rank] (device int64 table of peer_count entries; a
 * negative origin drops the row, a rank >= peer_count drops it and sets error
 * bit 8).  The expert-parallel layer's W2 uses it to return each output row
 * straight to the rank that sent the token, from the GEMM epilogue.
 * Tensor-core path only (16-byte aligned operands; N * element size a multiple
 * of 16 bytes); no SwiGLU. */
int grouped_gemm_offsets_scatter_launch(const void* a, const void* b, const int32_t* offs, int32_t problem_count,
                                        int32_t b_count, int64_t total_rows, int64_t n, int64_t k, int64_t stride_am,
                                        int64_t stride_be, int64_t stride_bk, const int64_t* row_origin,
                                        const int64_t* peer_regions, int32_t peer_count, int64_t dst_offset,
                                        int64_t dst_pitch_bytes, int32_t dtype, int32_t precision,
                                        const mgb_tile_config* config, void* scratch, size_t scratch_bytes,
                                        void* stream, mgb_launch_info* info);

/* Masked single GEMM C[m, n] = A[m, k] @ B[k, n] with arbitrary element strides.
 * Replaces the Triton launch of launch_matmul (kernels/matmul.py:332-392,
 * kernel _matmul_kernel_impl :223-273).  Operands that satisfy the TMA rules
 * run on the tensor cores; others on the generic-stride kernel. */
int matmul_launch(const void* a, const void* b, void* c, int64_t m, int64_t n, int64_t k, int64_t stride_am,
                  int64_t stride_ak, int64_t stride_bk, int64_t stride_bn, int64_t stride_cm, int64_t stride_cn,
                  int32_t dtype, int32_t precision, const mgb_tile_config* config, void* stream,
                  mgb_launch_info* info);

/* Copies a rows x cols matrix with arbitrary element strides into `dst`, a
 * row-major buffer with a row pitch of `dst_pitch` elements (elements past
 * `cols` in each row are left untouched).  The masked single GEMM uses it to
 * give the tensor-core path operands whose row pitch the TMA cannot address
 * (e.g. fp32 rows of 127 or 8191 elements).  No counterpart in the reference:
 * its Triton kernel reads every element through masked loads. */
int matrix_repack(const void* src, int64_t rows, int64_t cols, int64_t stride_r, int64_t stride_c, void* dst,
                  int64_t dst_pitch, int32_t elem_bytes, void* stream);

/* The 3xTF32 operand split behind input_precision="ieee" fp32 GEMMs on the
 * tensor cores (kernels/matmul.py:268 in the reference asks for full fp32
 * products; its Triton kernel runs them as fp32 FMAs).  Each fp32 element x
 * becomes hi = tf32(x) and lo = tf32(x - hi) (round to nearest even, kept in
 * fp32 words with the low 13 bits zero), laid out along K so that one TF32
 * GEMM of depth 3K computes hi(A) hi(B) + lo(A) hi(B) + hi(A) lo(B):
 *   side 0, A [rows = M, cols = K]: dst [M, 3K] = [hi | lo | hi]
 *   side 1, B [rows = K, cols = N]: dst [3K, N] = [hi ; hi ; lo]
 * src has arbitrary element strides; dst is row-major with a row pitch of
 * dst_pitch elements (>= 3 cols for side 0, >= cols for side 1).  No
 * counterpart in the reference. */
int matrix_split_tf32x3(const float* src, int64_t rows, int64_t cols, int64_t stride_r, int64_t stride_c, float* dst,
                        int64_t dst_pitch, int32_t side, void* stream);

/* The reduction of a single GEMM whose K was split over several problems of
 * one grouped launch (kernels/matmul.py does this for fp32 GEMMs with too
 * few output tiles to fill the GPU and a long K): C = sum over s of
 * partials[s], partials fp32 [splits][rows][cols] contiguous, summed in the
 * order s = 0, 1, ... in fp32 and rounded once to dtype, C written through
 * its element strides.  No counterpart in the reference, whose Triton matmul
 * runs each output tile's whole K in one program (kernels/matmul.py:256-268). */
int matrix_sum_partials(const float* partials, int32_t splits, int64_t rows, int64_t cols, void* c, int64_t stride_cm,
                        int64_t stride_cn, int32_t dtype, void* stream);

/* Size of the scratch array compiled into the library for
 * grouped_gemm_launch_noalloc (bytes, per GPU that loads the library). */
#define MGB_NOALLOC_SCRATCH_BYTES (1u << 20)

/* grouped_gemm_launch for callers that cannot allocate device memory.  No
 * counterpart in the reference (its Triton launches need no scratch).
 *
 * Same arguments and result as grouped_gemm_launch, minus the scratch buffer:
 * the per-problem tensor maps and tile-walk offsets live in a fixed
 * MGB_NOALLOC_SCRATCH_BYTES array inside this library, so the call allocates
 * and frees nothing.  It serves callers with no device allocator of their
 * own: a plugin in a process whose framework owns all device memory and hands
 * it only the input and output tensors, or a launch path that must never
 * enter the driver's allocator.
 *   - The first call on a device looks up the array's device address (once per
 *     device, with that device current, cached for the process); make that
 *     first call before any stream capture, and do not call this again on a
 *     device after cudaDeviceReset() in the same process.
 *   - A group of more than 2674 problems (whose maps would exceed
 *     MGB_NOALLOC_SCRATCH_BYTES) is refused with MGB_ERR_SCRATCH, whichever
 *     kernel would have run it.
 *   - Every call shares the one array and leaves its last contents behind;
 *     nothing in it has to start at zero (each launch writes every map and
 *     offset before reading it), but calls that overlap on the GPU -- other
 *     streams, other threads -- race on it and must be serialised by the
 *     caller. */
int grouped_gemm_launch_noalloc(const int64_t* a_ptrs, const int64_t* b_ptrs, const int64_t* c_ptrs,
                                const int32_t* dims, const int64_t* strides, int32_t problem_count,
                                int32_t homogeneous, int64_t m, int64_t n, int64_t k, int32_t dtype,
                                int32_t precision, int32_t operands_tma_aligned, const mgb_tile_config* config,
                                void* stream, mgb_launch_info* info);

/* Reads and clears the device's error word: OR of the bits the kernels raised
 * since the last call (bounded waits that gave up, table entries that broke
 * the TMA promise).  Synchronous.  The reference has no counterpart: Triton
 * kernels there cannot report device-side failures. */
int read_and_clear_error_word(int32_t device, uint32_t* word);

/* Test hook: the wait budget (SM clock cycles) of every bounded barrier wait
 * and test flags for later launches in this process (bit 0: make the epilogue
 * wait on a barrier nothing arrives on, which must time out and be reported).
 * budget <= 0 restores the default. */
int mgb_set_debug(int64_t wait_budget_cycles, int32_t test_flags);

/* Human-readable text for an mgb_status value. */
const char* mgb_status_string(int32_t status);

/* ABI version of this header (bumped on any signature change). */
int32_t mgb_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* MOE_GEMM_B200_H */
