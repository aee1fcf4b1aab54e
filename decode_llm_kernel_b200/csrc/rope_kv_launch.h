// Host-visible launch interface between the C ABI layer (abi.cpp) and the kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace drk {

// Threads per block the kernels are compiled for (__launch_bounds__).
constexpr int kMaxThreadsPerBlock = 256;
constexpr int kStagedThreadsPerBlock = 128;

// Head rows a thread holds in registers at once (its loads are all issued before any store),
// and the blocks of kMaxThreadsPerBlock threads per SM the register budget is set for.
#ifndef DRK_ROWS_PER_THREAD
#define DRK_ROWS_PER_THREAD 3
#endif
#ifndef DRK_MIN_BLOCKS_PER_SM
#define DRK_MIN_BLOCKS_PER_SM 1
#endif
constexpr int kRowsPerThread = DRK_ROWS_PER_THREAD;

struct KernelParams {
  const char* q;              // Q (fused/rope)
  const char* k;              // K (fused/rope) or k_rot (append)
  const char* v;              // V (fused/append)
  char* q_out;                // contiguous [T, Hq, D]
  char* k_dst;                // k cache, or contiguous k_out [T, Hkv, D] in rope mode
  char* v_dst;                // v cache
  const float* cos_t;
  const float* sin_t;
  const float* inv_freq;      // in-register trig only
  const void* positions;
  const void* request_indices;
  const void* block_table;    // paged only
  uint32_t* status;           // may be null
  int64_t T;
  int64_t q_ts, q_hs, k_ts, k_hs, v_ts, v_hs;  // element strides of the sources
  int64_t c_bs, c_ss, c_hs;   // cache element strides: batch (paged: block), position, head
  int64_t B, S;               // cache rows and positions (paged: requests, max positions)
  int64_t num_blocks, block_size, bt_stride;
  int64_t table_rows, table_stride;
  int32_t Hq, Hkv, D, R;
  int32_t nslots, nrot, G;
  int32_t inreg_trig;
  int32_t table_vec4;         // table base and row stride allow 16-byte loads
  int32_t pdl;                // launched with programmatic dependent launch
  int32_t rows_per_thread;    // register kernel: 1 (small batches) or kRowsPerThread
  // Bulk-copy kernel, for testing its timeout path only (drk_testing_staged_timeout): the
  // token whose Q/K/V loads are not issued (-1: none) and the wait limit in ns (0: the
  // compiled default).
  int64_t test_skip_token = -1;
  int64_t wait_limit_ns = 0;
};

enum { kElemF32 = 0, kElemF16 = 1, kElemBF16 = 2, kElemF64 = 3 };
enum { kModeFused = 0, kModeRope = 1, kModeAppend = 2 };
enum { kCacheStrided = 0, kCachePaged = 1 };

struct LaunchShape {
  int grid;      // CTAs along x; each walks tokens blockIdx.x, blockIdx.x + grid, ...
  int splits;    // gridDim.y: CTAs sharing one token's head rows (register kernel)
  int lanes;     // blockDim.x: lanes per head row (nslots)
  int groups;    // blockDim.y: row groups (G)
  bool pdl;
  bool allow_lean = false;  // register kernel, one row per thread, fused into a strided cache:
                            // the launcher may take the 56-register form when that puts the
                            // grid in one wave where the 64-register form needs more
};

cudaError_t launch_rope_kv(const KernelParams& p, int elem_code, int index_bits, int vb,
                           int mode, int cache, const LaunchShape& shape, cudaStream_t stream);

// Shared memory one CTA of the bulk-copy kernel may use for its stages.
#ifndef DRK_STAGED_SMEM_BUDGET
#define DRK_STAGED_SMEM_BUDGET (192 * 1024)
#endif

// Stage geometry of the bulk-copy kernel (rope_kv_staged.cuh), in bytes.
struct StagedParams {
  uint32_t q_bytes;      // Hq * D * es: one token's Q rows
  uint32_t kv_bytes;     // Hkv * D * es: one token's K (or V) rows
  uint32_t stage_bytes;  // q_bytes + 2 * kv_bytes, rounded up to 128
  int32_t stages;        // pipeline depth
  int32_t deepen;        // the launcher may add a stage when CTAs walk many tokens each
  int32_t early_issue;   // set by the launcher for launches without programmatic dependent
                         // launch: the first copies go out during the metadata round trip
};
// Token metadata a CTA of the bulk-copy kernel keeps in shared memory: two blocks of 32 tokens
// of 24 bytes (position, cache slot, status bits, flags), after the stages and their barriers.
constexpr int kStagedMetaBlock = 32;
constexpr size_t kStagedMetaBytes = 2 * kStagedMetaBlock * 24;

// Fused mode only. shape.grid is ignored: the launcher sizes a persistent grid of
// min(T, SMs x resident CTAs per SM).
cudaError_t launch_rope_kv_staged(const KernelParams& p, const StagedParams& sp, int elem_code,
                                  int index_bits, int vb, int cache, const LaunchShape& shape,
                                  cudaStream_t stream);

// Streaming multiprocessors of a device (cached per device).
int device_sm_count(int device);

// rope_kv_attention.cu: the fused RoPE + append + decode attention kernel.
struct AttentionParams {
  float* workspace;      // [T, Hq, max_chunks, D + 2] fp32: acc[D], m, l of each chunk
  int* counters;         // [T, Hkv, nhb], zero on entry, zero again on exit
  void* attn_out;        // contiguous [T, Hq, D] of the storage type
  char* q_out;           // contiguous [T, Hq, D] or null
  float scale_log2;      // softmax scale * log2(e)
  int32_t chunk;         // positions per CTA
  int32_t max_chunks;    // ceil(S / chunk)
  int32_t group;         // Hq / Hkv
  int32_t nhb;           // head blocks per KV head
  int32_t q_vec;         // tensor-core kernel: full rotary with 16-byte q rows and table rows
  int32_t box_rows;      // tensor-core kernel: positions per TMA box (128, or the page size of
                         // a paged cache when it is smaller)
};

struct AttentionShape {
  int grid_x;   // max_chunks * nhb
  int grid_y;   // Hkv
  int grid_z;   // T
  int lpr;      // lanes per K/V row: 8, 16 or 32
  int hpb;      // query heads per CTA: 1, 2, 4 or 8
  bool pdl;
};
cudaError_t launch_rope_kv_attention(const KernelParams& p, const AttentionParams& a,
                                     int elem_code, int index_bits, const AttentionShape& s,
                                     cudaStream_t stream);

// rope_kv_attention_tc.cu: the tcgen05 form (16-bit, head_dim 64 or 128), a persistent grid over
// `units` = T * Hkv * nhb * max_chunks work units of up to 16 query heads.
cudaError_t launch_rope_kv_attention_tc(const KernelParams& p, const AttentionParams& a,
                                        int elem_code, int index_bits, int64_t units, bool pdl,
                                        cudaStream_t stream);

// positions.cu
cudaError_t launch_advance_positions(void* data, int index_bits, int64_t n, int64_t delta,
                                     bool pdl, cudaStream_t stream);

// smoke.cu
cudaError_t launch_smoke_fill(void* data, int elem_code, int64_t numel, double value,
                              cudaStream_t stream);
cudaError_t run_arch_probe(int* arch_out, cudaStream_t stream);
cudaError_t launch_empty(int count, bool pdl, cudaStream_t stream);
// `count` chained copies of `vectors` 16-byte vectors (an even number), launch i from
// src + i * stride_vectors to dst + i * stride_vectors, `threads` per CTA, two vectors a
// thread (see copy_probe_kernel).
cudaError_t launch_copy_probe(const void* src, void* dst, int64_t vectors, int64_t stride_vectors,
                              int count, int threads, bool pdl, bool prefetch,
                              cudaStream_t stream);

}  // namespace drk
