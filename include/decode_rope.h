/*
 * decode_rope.h -- C ABI of the B200 (sm_100a) decode-step RoPE + KV-cache append library,
 * libdecode_rope.so.
 *
 * Every entry point takes plain tensor descriptors (a data pointer, a dtype code, sizes and
 * element strides), an optional device status word and a CUDA stream. No entry point
 * allocates device memory, synchronises the stream or reads device memory on the host, except
 * drk_build_info, which is a diagnostic. Return value: DRK_OK, or a negative DRK_ERR_* code
 * with a message available from drk_last_error() on the same thread.
 *
 * The argument checks and their messages follow the reference's host checks
 * (csrc/kernel_common.cuh:56-125 and csrc/fused_rope_kv_append.cu:93-115 of the reference
 * project), so a binding that raises the message reproduces the reference's errors.
 *
 * Out-of-range positions or request indices do not trap (the reference uses a device assert,
 * csrc/kernel_common.cuh:38-51, which ends the CUDA context): the kernel skips that token's
 * cache writes and ORs a DRK_STATUS_* bit into *status when status is not NULL. The caller
 * reads the word when it chooses to (outside any timed region).
 */
#ifndef DECODE_ROPE_H_
#define DECODE_ROPE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define DRK_API __attribute__((visibility("default")))
#else
#define DRK_API
#endif

/* Same object as cudaStream_t; NULL is the legacy default stream. */
typedef struct CUstream_st* drk_stream_t;

/* Element type codes. */
enum {
  DRK_F32 = 0,
  DRK_F16 = 1,
  DRK_BF16 = 2,
  DRK_F64 = 3,
  DRK_I32 = 4,
  DRK_I64 = 5
};

/* Return codes. */
enum {
  DRK_OK = 0,
  DRK_ERR_INVALID = -1,     /* an argument check failed; see drk_last_error() */
  DRK_ERR_CUDA = -2,        /* a CUDA runtime call failed; see drk_last_error() */
  DRK_ERR_UNSUPPORTED = -3  /* a dtype or layout this build has no kernel for */
};

/* Bits a kernel ORs into the optional status word. */
enum {
  DRK_STATUS_POSITION_OUT_OF_CACHE = 1u << 0, /* position < 0 or >= cache_alloc_len */
  DRK_STATUS_REQUEST_OUT_OF_RANGE = 1u << 1,  /* request index < 0 or >= batch */
  DRK_STATUS_POSITION_OUT_OF_TABLE = 1u << 2, /* position >= rows of the cos/sin table */
  DRK_STATUS_BLOCK_OUT_OF_RANGE = 1u << 3,    /* paged cache: block id outside the pool */
  DRK_STATUS_TIMEOUT = 1u << 4                /* a bounded in-kernel wait ran out; the CTA
                                                 stopped early (no valid input causes this) */
};

/* Launch options (drk_options.flags). */
enum {
  /* Launch with programmatic dependent launch: the kernel reads positions, request indices,
   * the block table of a paged cache and the cos/sin rows before waiting on the preceding
   * kernel in the stream, then waits (griddepcontrol.wait) before it reads q/k/v or writes
   * anything. The caller guarantees the immediately preceding kernel writes none of those
   * (positions, request indices, block table, tables). */
  DRK_FLAG_PDL = 1u << 0,
  /* Accept caches with any element strides whose last dim is contiguous (e.g. head-major
   * [B, Hkv, S, D] passed as its [B, S, Hkv, D] transposed view). Without it the cache must be
   * contiguous token-major, as the reference requires. */
  DRK_FLAG_STRIDED_CACHE = 1u << 1,
  /* Take cos/sin from sincosf of position * inv_freq in registers instead of the table
   * (needs drk_options.inv_freq). Not bit-exact: sincosf and the table's cos/sin differ by an
   * fp32 ulp at times, which cancellation in x1*c - x2*s can magnify for near-zero outputs;
   * results stay within the reference's tolerance (bf16 8e-3, fp16 1e-3). */
  DRK_FLAG_INREG_TRIG = 1u << 2,
  /* Kernel choice for the fused op. By default calls with many tokens whose Q/K/V row blocks
   * and cache slots are contiguous and 16-byte aligned use the bulk-copy (TMA) kernel that
   * stages tokens through shared memory; other calls use the register kernel. These force
   * one (forcing the bulk-copy kernel on an ineligible layout returns DRK_ERR_UNSUPPORTED). */
  DRK_FLAG_FORCE_REGISTER_PATH = 1u << 3,
  DRK_FLAG_FORCE_STAGED_PATH = 1u << 4
};

/* A strided view of device (or host) memory. Sizes and strides are in elements; unused
 * trailing dims are ignored. device is the CUDA ordinal, or -1 for host memory. */
typedef struct drk_tensor {
  void* data;
  int32_t dtype;
  int32_t ndim;
  int32_t device;
  int32_t reserved;
  int64_t sizes[4];
  int64_t strides[4];
} drk_tensor;

/* Extensions beyond the reference contract; zero-initialised means reference behaviour. */
typedef struct drk_options {
  uint32_t flags;         /* DRK_FLAG_* */
  int32_t rotary_dim;     /* 0: the table width must equal head_dim (reference). Otherwise the
                             table width, even and <= head_dim; dims past it are copied raw. */
  const float* inv_freq;  /* [rotary_dim/2] fp32 device array, only for DRK_FLAG_INREG_TRIG */
  int32_t row_splits;     /* register kernel: CTAs sharing one token's head rows (0 = chosen
                             by the library from the token count and the SM count) */
  int32_t rows_per_thread; /* register kernel: head rows a thread holds, 1 or 3 (0 = chosen by
                              the library: 1 up to 256 tokens, 3 above) */
  int64_t k_position_limit; /* drk_kv_append only: when > 0, the K row of a token whose
                               position is >= this is not written (its V row still is). A
                               separate RoPE-then-append passes the cos/sin table's row count,
                               because drk_rope_forward leaves k_rot rows of such tokens
                               unwritten, so they hold no defined value. 0: every K row is
                               written (the reference's kv_append). */
  int32_t staged_stages;  /* bulk-copy kernel: tokens staged per CTA at once, 2..8 (0 = the
                             library's choice, bounded by shared memory) */
  int32_t reserved1;
  int64_t reserved;
} drk_options;

/*
 * Fused RoPE + KV append, one launch.
 * Replaces fused_rope_kv_append (csrc/fused_rope_kv_append.cu:89-141, bound at
 * csrc/bindings.cpp:30-33 of the reference). q [T, Hq, D], k and v [T, Hkv, D] with a
 * contiguous last dim and any token/head strides; positions and request_indices [T], both
 * int32 or both int64; cos and sin fp32 contiguous [P, D]; k_cache and v_cache contiguous
 * [B, S, Hkv, D] of q's dtype; q_out contiguous [T, Hq, D] of q's dtype, allocated by the
 * caller (the reference returns a fresh tensor). Writes q_out = RoPE(q),
 * k_cache[ri[t], pos[t]] = RoPE(k[t]), v_cache[ri[t], pos[t]] = v[t] (byte copy).
 * Q and K are bit-exact to the reference's PyTorch oracle.
 */
DRK_API int drk_fused_rope_kv_append(const drk_tensor* q, const drk_tensor* k, const drk_tensor* v,
                             const drk_tensor* positions, const drk_tensor* cos,
                             const drk_tensor* sin, const drk_tensor* k_cache,
                             const drk_tensor* v_cache, const drk_tensor* request_indices,
                             const drk_tensor* q_out, uint32_t* status, drk_stream_t stream);

/* drk_fused_rope_kv_append with the extensions in *opts (NULL = none). */
DRK_API int drk_fused_rope_kv_append_ex(const drk_tensor* q, const drk_tensor* k, const drk_tensor* v,
                                const drk_tensor* positions, const drk_tensor* cos,
                                const drk_tensor* sin, const drk_tensor* k_cache,
                                const drk_tensor* v_cache, const drk_tensor* request_indices,
                                const drk_tensor* q_out, const drk_options* opts,
                                uint32_t* status, drk_stream_t stream);

/*
 * RoPE only: q_out = RoPE(q), k_out = RoPE(k), both contiguous and caller-allocated.
 * Replaces rope_forward (csrc/rope.cu:64-105, bound at csrc/bindings.cpp:22-24).
 */
DRK_API int drk_rope_forward(const drk_tensor* q, const drk_tensor* k, const drk_tensor* positions,
                     const drk_tensor* cos, const drk_tensor* sin, const drk_tensor* q_out,
                     const drk_tensor* k_out, const drk_options* opts, uint32_t* status,
                     drk_stream_t stream);

/*
 * Append only: byte copies of k_rot and v into k_cache/v_cache at [ri[t], pos[t]].
 * Replaces kv_append (csrc/kv_append.cu:45-86, bound at csrc/bindings.cpp:25-27).
 */
DRK_API int drk_kv_append(const drk_tensor* k_rot, const drk_tensor* v, const drk_tensor* positions,
                  const drk_tensor* request_indices, const drk_tensor* k_cache,
                  const drk_tensor* v_cache, const drk_options* opts, uint32_t* status,
                  drk_stream_t stream);

/*
 * Fused RoPE + append into a paged KV cache (no counterpart in the reference, whose cache is
 * one contiguous row per request; this is the block-table layout its notes name as the next
 * step). k_pages and v_pages are [num_blocks, block_size, Hkv, D] contiguous; block_table is
 * [num_requests, max_blocks_per_request] contiguous, of the index dtype; token t lands in
 * block block_table[ri[t], pos[t] / block_size], row pos[t] % block_size.
 */
DRK_API int drk_paged_rope_kv_append(const drk_tensor* q, const drk_tensor* k, const drk_tensor* v,
                             const drk_tensor* positions, const drk_tensor* cos,
                             const drk_tensor* sin, const drk_tensor* k_pages,
                             const drk_tensor* v_pages, const drk_tensor* block_table,
                             const drk_tensor* request_indices, const drk_tensor* q_out,
                             const drk_options* opts, uint32_t* status, drk_stream_t stream);

/*
 * The separate op (drk_rope_forward, then drk_kv_append) for callers that cannot allocate
 * device memory when they launch it. It has no counterpart in the reference: it is this
 * library's allocation-free form of the separate RoPE-then-append op, whose k_rot intermediate
 * is otherwise allocated per call.
 *
 * Callers it is for: code recorded under a global-mode stream capture (where cudaMalloc is not
 * allowed), serving runtimes that have given all free HBM to their KV-cache pool, and hosts
 * reaching the library through this C ABI without an allocator of their own. The caller still
 * provides every input and output (q_out included); the k_rot intermediate lives in an 8 MiB
 * static device array inside the library, which every GPU that loads the library holds until
 * the process exits. Arguments go through the checks of drk_rope_forward and drk_kv_append
 * first; then calls whose k_rot ([T, Hkv, D] of k's dtype) exceeds 8 MiB are rejected with
 * DRK_ERR_INVALID, before any launch. The first call on a device looks up the array's address
 * with that device current and keeps it for the life of the process: make it before any stream
 * capture, and do not use this entry point after cudaDeviceReset in the same process. All calls
 * share the array, so calls that overlap on the GPU race. Nothing in the array needs to start
 * zeroed: a K slot is written only from a k_rot row the same call wrote (a token past the
 * cos/sin table sets DRK_STATUS_POSITION_OUT_OF_TABLE and keeps its K slot, as in the fused
 * op). Results are bit-identical to drk_rope_forward + drk_kv_append with a caller-allocated
 * k_rot and k_position_limit set to the table's row count.
 */
DRK_API int drk_separate_rope_kv_append_noalloc(
    const drk_tensor* q, const drk_tensor* k, const drk_tensor* v, const drk_tensor* positions,
    const drk_tensor* cos, const drk_tensor* sin, const drk_tensor* k_cache,
    const drk_tensor* v_cache, const drk_tensor* request_indices, const drk_tensor* q_out,
    uint32_t* status, drk_stream_t stream);

/* Tuning and semantics of drk_fused_rope_kv_append_attention; zero-initialised = defaults. */
typedef struct drk_attention_options {
  double scale;           /* softmax scale; 0 means 1 / sqrt(head_dim) */
  int32_t chunk;          /* cache positions per work unit; 0 = chosen from the shape and SM
                             count (the tensor-core kernel rounds it up to a multiple of 128) */
  int32_t heads_per_cta;  /* CUDA-core kernel: query heads per CTA, 0 (chosen), 1, 2, 4 or 8 */
  int32_t path;           /* DRK_ATTN_PATH_* */
  int32_t flags;          /* DRK_ATTN_WORKSPACE_ZEROED */
  int64_t reserved;
} drk_attention_options;

/* drk_attention_options.flags. The workspace's counters are already zero, so the call skips
 * zeroing them (one memset node less per call, which a graph-captured decode loop notices).
 * Every call leaves a workspace's counters at zero again, so a workspace zeroed once (e.g.
 * cudaMemset to 0 at allocation) may be passed with this flag call after call -- except after
 * a call that set DRK_STATUS_TIMEOUT: zero it again before the next. */
enum { DRK_ATTN_WORKSPACE_ZEROED = 1u << 0 };

/* Kernel choice of drk_fused_rope_kv_append_attention (drk_attention_options.path). AUTO takes
 * the tensor-core (tcgen05 + TMA) kernel for fp16/bf16 with head_dim 64 or 128 and the
 * CUDA-core kernel otherwise; forcing the tensor-core kernel on another shape returns
 * DRK_ERR_UNSUPPORTED. */
enum {
  DRK_ATTN_PATH_AUTO = 0,
  DRK_ATTN_PATH_CUDA_CORES = 1,
  DRK_ATTN_PATH_TENSOR_CORES = 2
};

/*
 * Bytes of device workspace drk_fused_rope_kv_append_attention needs for this shape, with the
 * same options and device; negative (a DRK_ERR_* code) if the shape is rejected. dtype is the
 * element type code of q/k/v. The workspace holds per-chunk partial results (fp32) and the
 * arrival counters of the cross-chunk merge.
 */
DRK_API int64_t drk_attention_workspace_bytes(int64_t num_tokens, int32_t num_q_heads,
                                              int32_t num_kv_heads, int32_t head_dim,
                                              int64_t cache_alloc_len, int32_t dtype,
                                              const drk_attention_options* attn,
                                              int32_t device);

/*
 * The fused append followed by the decode attention that consumes the cache, in one launch:
 * the write side of drk_fused_rope_kv_append and the read side the reference prices separately
 * (SDPA over the token-major cache viewed head-major, benchmarks/probe_cache_read.py:26-172 and
 * results/LIMITATIONS.md:153-157 of the reference). No counterpart kernel in the reference.
 *
 * For each token t it performs the fused op's append exactly (K slot = RoPE(k[t]), V slot =
 * v[t], bit-identical to drk_fused_rope_kv_append), optionally writes q_out = RoPE(q) (NULL to
 * skip), and writes attn_out[t, h] = softmax(scale * q_rot[t, h] . K[ri, p, g]) V[ri, p, g]
 * over cache positions p = 0..pos[t] of request ri[t] and KV head g = h / (Hq / Hkv), with the
 * new token's own K/V at p = pos[t]. Softmax and accumulation run in fp32; attn_out
 * ([T, Hq, D] contiguous, q's dtype) is rounded once.
 *
 * Each request appears at most once per call (one new token per sequence, the decode
 * contract). fp32, fp16 and bf16; head_dim * element size a multiple of 16 bytes and head_dim
 * <= 256 (16-bit) or 128 (fp32); cache base and strides 16-byte aligned; T <= 65535. opts
 * accepts DRK_FLAG_PDL, DRK_FLAG_STRIDED_CACHE and rotary_dim. workspace is device memory of
 * at least drk_attention_workspace_bytes for the same arguments; calls that overlap on the
 * GPU need separate workspaces. Other shapes return DRK_ERR_UNSUPPORTED.
 */
DRK_API int drk_fused_rope_kv_append_attention(
    const drk_tensor* q, const drk_tensor* k, const drk_tensor* v, const drk_tensor* positions,
    const drk_tensor* cos, const drk_tensor* sin, const drk_tensor* k_cache,
    const drk_tensor* v_cache, const drk_tensor* request_indices, const drk_tensor* q_out,
    const drk_tensor* attn_out, const drk_attention_options* attn, void* workspace,
    size_t workspace_bytes, const drk_options* opts, uint32_t* status, drk_stream_t stream);

/*
 * drk_fused_rope_kv_append_attention over a paged KV cache: k_pages and v_pages are
 * [num_blocks, block_size, Hkv, D] contiguous, block_table [num_requests, max_blocks_per_request]
 * contiguous of the index dtype; position p of request r lives in block block_table[r, p /
 * block_size], row p % block_size (the layout of drk_paged_rope_kv_append). No counterpart in
 * the reference, whose cache is one contiguous row per request and whose notes name the
 * block-table layout as the next step. fp16/bf16 with head_dim 64 or 128; block_size a
 * multiple of 8 that divides 128, or a multiple of 128. Size the workspace with
 * drk_attention_workspace_bytes for cache_alloc_len = max_blocks_per_request * block_size.
 * Block-table entries outside the pool are read as zeros, skip the append, and set
 * DRK_STATUS_BLOCK_OUT_OF_RANGE.
 */
DRK_API int drk_paged_rope_kv_append_attention(
    const drk_tensor* q, const drk_tensor* k, const drk_tensor* v, const drk_tensor* positions,
    const drk_tensor* cos, const drk_tensor* sin, const drk_tensor* k_pages,
    const drk_tensor* v_pages, const drk_tensor* block_table,
    const drk_tensor* request_indices, const drk_tensor* q_out, const drk_tensor* attn_out,
    const drk_attention_options* attn, void* workspace, size_t workspace_bytes,
    const drk_options* opts, uint32_t* status, drk_stream_t stream);

/*
 * positions[t] += delta for every token: the device-side step of a decode loop, so a captured
 * step ending with this call replays without a host-side position copy. No counterpart in the
 * reference, whose graph runner copies new positions in before every replay
 * (benchmarks/impls.py:144-150). positions is a contiguous int32 or int64 [T] device tensor.
 * With DRK_FLAG_PDL in flags it launches as a programmatic dependent and still writes only after
 * the preceding kernel has finished (every layer of the step has read the positions).
 */
DRK_API int drk_advance_positions(const drk_tensor* positions, int64_t delta, uint32_t flags,
                                  drk_stream_t stream);

/*
 * Fills a contiguous fp64/fp32/fp16/bf16 tensor with value (converted once on the host, so
 * fp64 keeps full precision). Replaces smoke_fill (csrc/smoke.cu:42-60, bound at
 * csrc/bindings.cpp:19-20).
 */
DRK_API int drk_smoke_fill(const drk_tensor* tensor, double value, drk_stream_t stream);

/*
 * Writes "key=value" lines (gencode_arch, cuda_version_compiled, cuda_version_runtime,
 * cuda_version_driver, nvcc_version, fast_math) into buf. gencode_arch comes from a kernel
 * run on the current device, so this call synchronises the stream. Replaces build_info
 * (csrc/smoke.cu:62-87, bound at csrc/bindings.cpp:21).
 */
DRK_API int drk_build_info(char* buf, size_t len, drk_stream_t stream);

/* Launch-floor probe: `count` back-to-back launches of an empty one-warp kernel on stream,
 * with programmatic dependent launch when pdl != 0. */
DRK_API int drk_launch_empty(int count, int pdl, drk_stream_t stream);

/* Dependent-copy floor probe: `count` launches chained like the layers of a decode step; launch
 * i copies `bytes` (a multiple of 32) from src + i * stride_bytes to dst + i * stride_bytes,
 * two 16-byte vectors per thread, threads_per_cta threads per CTA, with programmatic dependent
 * launch when pdl != 0. Each launch loads only after griddepcontrol.wait; with prefetch != 0
 * its threads first pull their source lines toward L2 while they wait. It is one layer of the
 * fused op without its arithmetic and index work, so a layer's time against it shows what the
 * op adds to the cost of a chained dependent read and write. The caller guarantees src and dst
 * hold (count - 1) * stride_bytes + bytes bytes. No counterpart in the reference, whose floor
 * probe (benchmarks/probe_graph_floor.py:36-112) launches empty kernels only. */
DRK_API int drk_launch_copy_probe(const void* src, void* dst, int64_t bytes, int64_t stride_bytes,
                                  int count, int threads_per_cta, int pdl, int prefetch,
                                  drk_stream_t stream);

/* Message of the last failed call on this thread ("" if none). */
DRK_API const char* drk_last_error(void);

/* Human-readable description of a status word's bits. */
DRK_API const char* drk_status_string(uint32_t status);

/* Library version, e.g. "0.1.0". */
DRK_API const char* drk_version(void);

#ifdef __cplusplus
}
#endif

#endif /* DECODE_ROPE_H_ */
