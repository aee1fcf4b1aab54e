// C ABI of libdecode_rope.so (include/decode_rope.h): argument checks, launch shape, dispatch.
//
// The checks, their order and their messages follow the reference's host launchers
// (csrc/fused_rope_kv_append.cu:93-115, csrc/rope.cu:67-79, csrc/kv_append.cu:53-71) and
// helpers (csrc/kernel_common.cuh:56-125), so a binding that raises the message reproduces the
// reference's RuntimeErrors. Nothing here allocates, synchronises or reads device memory
// (drk_build_info excepted, a diagnostic).
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <sstream>
#include <stdexcept>
#include <string>

#include "decode_rope.h"
#include "rope_kv_launch.h"

namespace {

thread_local std::string g_last_error;
thread_local std::string g_status_text;

struct InvalidArgument : std::runtime_error {
  using std::runtime_error::runtime_error;
};
struct Unsupported : std::runtime_error {
  using std::runtime_error::runtime_error;
};
struct CudaFailure : std::runtime_error {
  using std::runtime_error::runtime_error;
};

template <typename... A>
std::string cat(const A&... a) {
  std::ostringstream os;
  (os << ... << a);
  return os.str();
}

template <typename... A>
[[noreturn]] void invalid(const A&... a) {
  throw InvalidArgument(cat(a...));
}

const char* dtype_name(int32_t dt) {
  switch (dt) {
    case DRK_F32: return "Float";
    case DRK_F16: return "Half";
    case DRK_BF16: return "BFloat16";
    case DRK_F64: return "Double";
    case DRK_I32: return "Int";
    case DRK_I64: return "Long";
    default: return "Unknown";
  }
}

std::string device_name(int32_t d) { return d < 0 ? std::string("cpu") : cat("cuda:", d); }

std::string sizes_str(const drk_tensor* t) {
  std::ostringstream os;
  os << "[";
  for (int i = 0; i < t->ndim; ++i) os << (i ? ", " : "") << t->sizes[i];
  os << "]";
  return os.str();
}

int64_t elem_size(int32_t dt) {
  switch (dt) {
    case DRK_F32: case DRK_I32: return 4;
    case DRK_F16: case DRK_BF16: return 2;
    case DRK_F64: case DRK_I64: return 8;
    default: return 0;
  }
}

bool is_float(int32_t dt) {
  return dt == DRK_F32 || dt == DRK_F16 || dt == DRK_BF16 || dt == DRK_F64;
}

int64_t numel(const drk_tensor* t) {
  int64_t n = 1;
  for (int i = 0; i < t->ndim; ++i) n *= t->sizes[i];
  return n;
}

// Row-major contiguity with PyTorch's rule: strides of size-1 dims do not matter.
bool is_contiguous(const drk_tensor* t) {
  if (numel(t) == 0) return true;
  int64_t expected = 1;
  for (int i = t->ndim - 1; i >= 0; --i) {
    if (t->sizes[i] != 1 && t->strides[i] != expected) return false;
    expected *= t->sizes[i];
  }
  return true;
}

void require(const drk_tensor* t, const char* name) {
  if (t == nullptr) invalid(name, " is NULL");
  if (t->ndim < 0 || t->ndim > 4) invalid(name, " has an unsupported number of dims ", t->ndim);
  for (int i = 0; i < t->ndim; ++i)
    if (t->sizes[i] < 0) invalid(name, " has a negative size ", t->sizes[i], " in dim ", i);
}

void check_device(const drk_tensor* t, const char* name, int32_t device) {
  if (t->device < 0) invalid(name, " must be a CUDA tensor, got ", device_name(t->device));
  if (t->device != device)
    invalid(name, " is on ", device_name(t->device), " but the operation runs on ",
            device_name(device), "; every tensor must be on one device");
}

// csrc/kernel_common.cuh:62-74, plus the partial-rotary extension.
void check_rope_tables(const drk_tensor* cos, const drk_tensor* sin, int64_t head_dim,
                       int32_t rotary_dim, int32_t device) {
  require(cos, "cos");
  require(sin, "sin");
  check_device(cos, "cos", device);
  check_device(sin, "sin", device);
  if (cos->dtype != DRK_F32 || sin->dtype != DRK_F32)
    invalid("cos/sin must be FP32 per the locked RoPE semantics, got ", dtype_name(cos->dtype),
            "/", dtype_name(sin->dtype));
  if (!is_contiguous(cos) || !is_contiguous(sin)) invalid("cos/sin must be contiguous");
  if (cos->ndim != 2 || sin->ndim != 2) invalid("cos/sin must be [max_position, head_dim]");
  if (rotary_dim == 0) {
    if (cos->sizes[1] != head_dim || sin->sizes[1] != head_dim)
      invalid("cos/sin head_dim ", cos->sizes[1], " does not match q/k head_dim ", head_dim);
  } else if (cos->sizes[1] != rotary_dim || sin->sizes[1] != rotary_dim) {
    invalid("cos/sin width ", cos->sizes[1], " does not match rotary_dim ", rotary_dim);
  }
  if (cos->sizes[0] != sin->sizes[0] || cos->sizes[1] != sin->sizes[1])
    invalid("cos and sin must have the same shape");
}

// csrc/kernel_common.cuh:78-88
void check_qkv(const drk_tensor* t, const char* name, int64_t num_tokens, int64_t head_dim,
               int32_t device) {
  require(t, name);
  check_device(t, name, device);
  if (t->ndim != 3)
    invalid(name, " must be [num_tokens, num_heads, head_dim], got ", t->ndim, " dims");
  if (t->sizes[0] != num_tokens)
    invalid(name, " has ", t->sizes[0], " tokens, expected ", num_tokens);
  if (t->sizes[2] != head_dim) invalid(name, " head_dim ", t->sizes[2], " expected ", head_dim);
  if (t->strides[2] != 1)
    invalid(name, " needs a contiguous head_dim (last-dim stride ", t->strides[2], ")");
}

// csrc/kernel_common.cuh:90-98
void check_index_tensor(const drk_tensor* t, const char* name, int64_t num_tokens,
                        int32_t device) {
  require(t, name);
  check_device(t, name, device);
  if (t->dtype != DRK_I32 && t->dtype != DRK_I64)
    invalid(name, " must be int32 or int64, got ", dtype_name(t->dtype));
  if (t->ndim != 1 || t->sizes[0] != num_tokens)
    invalid(name, " must be [num_tokens]; got ", sizes_str(t));
  if (!is_contiguous(t)) invalid(name, " must be contiguous");
}

// csrc/kernel_common.cuh:100-114; DRK_FLAG_STRIDED_CACHE relaxes contiguity to a contiguous
// last dim.
void check_cache(const drk_tensor* cache, const char* name, int32_t like_dtype,
                 int64_t num_kv_heads, int64_t head_dim, int32_t device, bool strided_ok) {
  require(cache, name);
  check_device(cache, name, device);
  if (!strided_ok && !is_contiguous(cache)) invalid(name, " must be contiguous, token-major");
  if (cache->ndim != 4)
    invalid(name, " must be [batch, cache_alloc_len, num_kv_heads, head_dim], got ",
            cache->ndim, " dims");
  if (cache->sizes[2] != num_kv_heads || cache->sizes[3] != head_dim)
    invalid(name, " kv-head/head_dim ", cache->sizes[2], "/", cache->sizes[3], " expected ",
            num_kv_heads, "/", head_dim);
  if (cache->dtype != like_dtype)
    invalid(name, " dtype ", dtype_name(cache->dtype), " must match its source dtype ",
            dtype_name(like_dtype));
  if (strided_ok && numel(cache) != 0 && cache->strides[3] != 1)
    invalid(name, " needs a contiguous head_dim (last-dim stride ", cache->strides[3], ")");
}

// csrc/kernel_common.cuh:116-125
void check_caches_are_distinct(const drk_tensor* k_cache, const drk_tensor* v_cache) {
  bool same_shape = k_cache->ndim == v_cache->ndim;
  for (int i = 0; same_shape && i < k_cache->ndim; ++i)
    same_shape = k_cache->sizes[i] == v_cache->sizes[i];
  if (!same_shape) invalid("k_cache and v_cache must have the same shape");
  if (numel(k_cache) != 0 && k_cache->data == v_cache->data)
    invalid("k_cache and v_cache must be distinct buffers; sharing one makes the K and V "
            "writes race for the same slot");
  for (int i = 0; numel(k_cache) != 0 && i < k_cache->ndim; ++i)
    if (k_cache->sizes[i] != 1 && k_cache->strides[i] != v_cache->strides[i])
      invalid("k_cache and v_cache must have the same strides");
}

void check_output(const drk_tensor* t, const char* name, int32_t dtype, int64_t d0, int64_t d1,
                  int64_t d2, int32_t device) {
  require(t, name);
  check_device(t, name, device);
  if (t->dtype != dtype)
    invalid(name, " dtype ", dtype_name(t->dtype), " must match its source dtype ",
            dtype_name(dtype));
  if (t->ndim != 3 || t->sizes[0] != d0 || t->sizes[1] != d1 || t->sizes[2] != d2 ||
      !is_contiguous(t))
    invalid(name, " must be a contiguous [", d0, ", ", d1, ", ", d2, "] tensor, got ",
            sizes_str(t));
}

void check_float_dtype(int32_t dt, const char* op) {
  if (!is_float(dt)) invalid("\"", op, "\" not implemented for '", dtype_name(dt), "'");
}

int32_t elem_code(int32_t dt) {
  switch (dt) {
    case DRK_F32: return drk::kElemF32;
    case DRK_F16: return drk::kElemF16;
    case DRK_BF16: return drk::kElemBF16;
    default: return drk::kElemF64;
  }
}

// Widest vector (bytes) such that every row segment a lane moves starts on a VB boundary.
struct Aligner {
  int64_t es;
  int64_t R, D;
  uintptr_t ptr_or = 0;    // OR of every base address
  int64_t stride_or = 0;   // OR of every relevant element stride
  void ptr(const void* p) { ptr_or |= reinterpret_cast<uintptr_t>(p); }
  void stride(int64_t size, int64_t s) {
    if (size > 1) stride_or |= s;
  }
  int pick() const {
    for (int vb : {16, 8, 4, 2}) {
      if (vb < es || vb % es) continue;
      const int64_t vec = vb / es;
      if ((R / 2) % vec || ((D - R) / 2) % vec || (D / 2) % vec) continue;
      if (ptr_or % vb) continue;
      if ((stride_or * es) % vb) continue;
      return vb;
    }
    return 0;
  }
};

struct Shape {
  int vb;
  int nslots, nrot, G, threads;
  int rows;    // head rows per thread in flight
  int splits;  // CTAs sharing one token's rows
};

// Small batches run one head row per thread (more threads per token, shorter per-thread
// chains: the latency regime); larger ones kRowsPerThread rows per thread.
#ifndef DRK_SMALL_BATCH_TOKENS
#define DRK_SMALL_BATCH_TOKENS 256
#endif
constexpr int kRowsPerSplitCta = 20;

Shape plan(const Aligner& al, int nrows, bool rotates, int64_t tokens, int32_t splits_hint,
           int32_t rows_hint = 0) {
  Shape s{};
  s.vb = al.pick();
  if (s.vb == 0) throw Unsupported("tensors are not aligned to their element size");
  const int64_t vec = s.vb / al.es;
  const int64_t nslots = al.D / (2 * vec);
  if (nslots > drk::kMaxThreadsPerBlock)
    throw Unsupported(cat("head_dim ", al.D, " needs ", nslots,
                          " lanes per row at this alignment; at most ",
                          drk::kMaxThreadsPerBlock, " are supported"));
  s.nslots = static_cast<int>(nslots);
  s.nrot = rotates ? static_cast<int>(al.R / (2 * vec)) : 0;
  if (rows_hint != 0 && rows_hint != 1 && rows_hint != drk::kRowsPerThread)
    invalid("rows_per_thread must be 0 (chosen by the library), 1 or ", drk::kRowsPerThread,
            ", got ", rows_hint);
  s.rows = rows_hint ? rows_hint : (tokens <= DRK_SMALL_BATCH_TOKENS ? 1 : drk::kRowsPerThread);
  const int max_threads = s.rows == 1 ? 1024 : drk::kMaxThreadsPerBlock;
  // `rows` rows per thread; a block holds whole row groups.
  const int want_groups = std::max(1, (nrows + s.rows - 1) / s.rows);
  s.G = std::max(1, std::min(want_groups, max_threads / s.nslots));
  // With one row per thread, a token's rows are shared by several CTAs of about
  // kRowsPerSplitCta rows each: smaller CTAs spread over more SMs finish a small launch sooner
  // (measured on B200: 70B-shaped 80-row tokens 4.56 -> 3.41 us at 256 tokens).
  int splits = 1;
  if (splits_hint > 0) {
    splits = splits_hint;
  } else if (s.rows == 1 && tokens > 0) {
    splits = std::max(1, nrows / kRowsPerSplitCta);
  }
  const int groups_needed = (nrows + s.rows - 1) / s.rows;
  splits = std::max(1, std::min(splits, groups_needed));
  if (splits > 1)
    s.G = std::max(1, std::min((groups_needed + splits - 1) / splits, max_threads / s.nslots));
  s.splits = splits;
  s.threads = s.G * s.nslots;
  return s;
}

// The bulk-copy kernel's plan: eligible only if every row block it copies is one contiguous,
// 16-byte-aligned run. It takes calls of DRK_STAGED_MIN_TOKENS tokens and up; measured on B200
// (Mistral-shaped rows, fp16, graph-replayed launches with programmatic dependent launch), the
// register kernel is faster at 512 tokens (2.96 against 3.84 us at the best depth) and the
// bulk-copy kernel from 768 (4.70-4.80 against 4.96 us; 2048: 10.0 against 11.1; 4096: 17.7
// against 21.1 us).
#ifndef DRK_STAGED_MIN_TOKENS
#define DRK_STAGED_MIN_TOKENS 768
#endif
// Pipeline depth of the bulk-copy kernel and the shared memory one CTA may use for its stages.
#ifndef DRK_STAGED_STAGES
#define DRK_STAGED_STAGES 3
#endif

struct StagedPlan {
  bool ok = false;
  std::string why;
  int vb = 0, nrot = 0, groups = 0;
  drk::StagedParams sp{};
};

StagedPlan plan_staged(const drk_tensor* q, const drk_tensor* k, const drk_tensor* v,
                       const drk_tensor* q_out, const drk_tensor* k_cache,
                       const drk_tensor* v_cache, int64_t T, int64_t Hq, int64_t Hkv,
                       int64_t D, int64_t R, int64_t es, int32_t stages_hint = 0) {
  StagedPlan pl;
  auto fail = [&](const char* why) {
    pl.why = why;
    return pl;
  };
  auto rows_contig = [&](const drk_tensor* t, int64_t heads) {
    return heads == 1 || t->strides[1] == D;
  };
  if (!rows_contig(q, Hq) || !rows_contig(k, Hkv) || !rows_contig(v, Hkv))
    return fail("a token's q/k/v heads are not one contiguous run (head stride != head_dim)");
  if (Hkv > 1 && k_cache->strides[2] != D)
    return fail("a cache slot is not contiguous (head stride != head_dim)");
  const int64_t q_bytes = Hq * D * es, kv_bytes = Hkv * D * es;
  if (q_bytes % 16 || kv_bytes % 16) return fail("row blocks are not multiples of 16 bytes");
  uintptr_t addr = 0;
  for (const drk_tensor* t : {q, k, v, q_out, k_cache, v_cache})
    addr |= reinterpret_cast<uintptr_t>(t->data);
  if (addr % 16) return fail("a base address is not 16-byte aligned");
  int64_t strides = 0;
  if (T > 1) strides |= q->strides[0] | k->strides[0] | v->strides[0];
  for (int i = 0; i < 2; ++i)
    if (k_cache->sizes[i] > 1) strides |= k_cache->strides[i];
  if ((strides * es) % 16) return fail("a token or cache stride is not a multiple of 16 bytes");
  for (int vb : {16, 8, 4, 2}) {
    if (vb < es || vb % es) continue;
    const int64_t vec = vb / es;
    if ((R / 2) % vec || (D * es) % vb) continue;
    pl.vb = vb;
    pl.nrot = static_cast<int>(R / (2 * vec));
    break;
  }
  if (pl.vb == 0 || pl.nrot > drk::kStagedThreadsPerBlock)
    return fail("no vector width fits the rotary dims");
  const int64_t rot_rows = Hq + Hkv;
  pl.groups = static_cast<int>(std::max<int64_t>(
      1, std::min<int64_t>(rot_rows, drk::kStagedThreadsPerBlock / pl.nrot)));
  const int64_t stage = (q_bytes + 2 * kv_bytes + 127) / 128 * 128;
  if (stages_hint < 0 || stages_hint == 1 || stages_hint > 8)
    invalid("staged_stages must be 0 (chosen by the library) or in [2, 8], got ", stages_hint);
  int stages = static_cast<int>(std::min<int64_t>(stages_hint ? stages_hint : DRK_STAGED_STAGES,
                                                  DRK_STAGED_SMEM_BUDGET / stage));
  if (stages < 2) {
    if (2 * stage > 200 * 1024) return fail("one token's rows do not fit two shared-memory stages");
    stages = 2;
  }
  pl.sp.q_bytes = static_cast<uint32_t>(q_bytes);
  pl.sp.kv_bytes = static_cast<uint32_t>(kv_bytes);
  pl.sp.stage_bytes = static_cast<uint32_t>(stage);
  pl.sp.stages = stages;
  pl.sp.deepen = stages_hint == 0 ? 1 : 0;
  pl.ok = true;
  return pl;
}

int grid_for(int64_t tokens) {
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(tokens, 1 << 20)));
}

class DeviceGuard {
 public:
  explicit DeviceGuard(int device) {
    int cur = -1;
    if (cudaGetDevice(&cur) != cudaSuccess) throw CudaFailure("cudaGetDevice failed");
    if (cur != device) {
      if (cudaSetDevice(device) != cudaSuccess)
        throw CudaFailure(cat("cudaSetDevice(", device, ") failed"));
      prev_ = cur;
    }
  }
  ~DeviceGuard() {
    if (prev_ >= 0) cudaSetDevice(prev_);
  }

 private:
  int prev_ = -1;
};

void check_launch(cudaError_t err) {
  if (err != cudaSuccess) throw CudaFailure(cat("kernel launch failed: ", cudaGetErrorString(err)));
}

template <typename F>
int guarded(F&& body) {
  try {
    body();
    g_last_error.clear();
    return DRK_OK;
  } catch (const InvalidArgument& e) {
    g_last_error = e.what();
    return DRK_ERR_INVALID;
  } catch (const Unsupported& e) {
    g_last_error = e.what();
    return DRK_ERR_UNSUPPORTED;
  } catch (const CudaFailure& e) {
    g_last_error = e.what();
    return DRK_ERR_CUDA;
  } catch (const std::exception& e) {
    g_last_error = e.what();
    return DRK_ERR_INVALID;
  }
}

drk_options options_or_default(const drk_options* opts) {
  drk_options o{};
  if (opts) o = *opts;
  return o;
}

int32_t resolve_rotary(const drk_options& o, int64_t head_dim) {
  if (o.rotary_dim == 0) return 0;
  if (o.rotary_dim < 0 || o.rotary_dim % 2 || o.rotary_dim > head_dim)
    invalid("rotary_dim must be even and in (0, head_dim]; got ", o.rotary_dim, " for head_dim ",
            head_dim);
  return o.rotary_dim == head_dim ? 0 : o.rotary_dim;
}

void fill_table(drk::KernelParams& p, const drk_tensor* cos, const drk_tensor* sin,
                const drk_options& o, int64_t R) {
  p.cos_t = static_cast<const float*>(cos->data);
  p.sin_t = static_cast<const float*>(sin->data);
  p.table_rows = cos->sizes[0];
  p.table_stride = cos->sizes[1];
  p.table_vec4 = (reinterpret_cast<uintptr_t>(cos->data) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(sin->data) % 16 == 0 &&
                  (p.table_stride * 4) % 16 == 0) ? 1 : 0;
  if (o.flags & DRK_FLAG_INREG_TRIG) {
    if (o.inv_freq == nullptr) invalid("DRK_FLAG_INREG_TRIG needs opts->inv_freq");
    p.inv_freq = o.inv_freq;
    p.inreg_trig = 1;
  }
  (void)R;
}

// The common body of the fused entry points (strided and paged caches).
void fused_impl(const drk_tensor* q, const drk_tensor* k, const drk_tensor* v,
                const drk_tensor* positions, const drk_tensor* cos, const drk_tensor* sin,
                const drk_tensor* k_cache, const drk_tensor* v_cache,
                const drk_tensor* block_table, const drk_tensor* request_indices,
                const drk_tensor* q_out, const drk_options* opts, uint32_t* status,
                drk_stream_t stream, int64_t test_skip_token = -1, int64_t wait_limit_ns = 0) {
  const drk_options o = options_or_default(opts);
  const bool paged = block_table != nullptr;
  require(q, "q");
  if (q->ndim != 3) invalid("q must be [num_tokens, num_q_heads, head_dim]");
  const int64_t T = q->sizes[0], Hq = q->sizes[1], D = q->sizes[2];
  if (D % 2) invalid("head_dim must be even for split-half RoPE, got ", D);
  const int32_t device = q->device;
  check_qkv(q, "q", T, D, device);
  check_qkv(k, "k", T, D, device);
  check_qkv(v, "v", T, D, device);
  const int64_t Hkv = k->sizes[1];
  if (v->sizes[1] != Hkv) invalid("v has ", v->sizes[1], " kv heads, expected ", Hkv);
  if (q->dtype != k->dtype || q->dtype != v->dtype) invalid("q, k and v must share a dtype");
  check_index_tensor(positions, "positions", T, device);
  check_index_tensor(request_indices, "request_indices", T, device);
  if (positions->dtype != request_indices->dtype)
    invalid("positions and request_indices must share a dtype, got ",
            dtype_name(positions->dtype), "/", dtype_name(request_indices->dtype));
  const int32_t rot = resolve_rotary(o, D);
  check_rope_tables(cos, sin, D, rot, device);
  const bool strided_ok = (o.flags & DRK_FLAG_STRIDED_CACHE) != 0;
  check_cache(k_cache, paged ? "k_pages" : "k_cache", k->dtype, Hkv, D, device,
              strided_ok && !paged);
  check_cache(v_cache, paged ? "v_pages" : "v_cache", v->dtype, Hkv, D, device,
              strided_ok && !paged);
  check_caches_are_distinct(k_cache, v_cache);
  if (paged) {
    require(block_table, "block_table");
    check_device(block_table, "block_table", device);
    if (block_table->dtype != positions->dtype)
      invalid("block_table must share the index dtype of positions, got ",
              dtype_name(block_table->dtype), "/", dtype_name(positions->dtype));
    if (block_table->ndim != 2 || !is_contiguous(block_table))
      invalid("block_table must be a contiguous [num_requests, max_blocks_per_request] tensor");
    if (k_cache->sizes[1] <= 0 && numel(k_cache) != 0) invalid("block_size must be positive");
  }
  check_output(q_out, "q_out", q->dtype, T, Hq, D, device);
  check_float_dtype(q->dtype, "fused_rope_kv_append");
  if (T == 0) return;

  const int64_t R = rot ? rot : D;
  const int64_t es = elem_size(q->dtype);
  drk::KernelParams p{};
  p.q = static_cast<const char*>(q->data);
  p.k = static_cast<const char*>(k->data);
  p.v = static_cast<const char*>(v->data);
  p.q_out = static_cast<char*>(q_out->data);
  p.k_dst = static_cast<char*>(k_cache->data);
  p.v_dst = static_cast<char*>(v_cache->data);
  p.positions = positions->data;
  p.request_indices = request_indices->data;
  p.status = status;
  p.T = T;
  p.q_ts = q->strides[0]; p.q_hs = q->strides[1];
  p.k_ts = k->strides[0]; p.k_hs = k->strides[1];
  p.v_ts = v->strides[0]; p.v_hs = v->strides[1];
  p.c_bs = k_cache->strides[0]; p.c_ss = k_cache->strides[1]; p.c_hs = k_cache->strides[2];
  if (paged) {
    p.block_table = block_table->data;
    p.num_blocks = k_cache->sizes[0];
    p.block_size = k_cache->sizes[1];
    p.bt_stride = block_table->sizes[1];
    p.B = block_table->sizes[0];
    p.S = block_table->sizes[1] * k_cache->sizes[1];
  } else {
    p.B = k_cache->sizes[0];
    p.S = k_cache->sizes[1];
  }
  p.Hq = static_cast<int32_t>(Hq);
  p.Hkv = static_cast<int32_t>(Hkv);
  p.D = static_cast<int32_t>(D);
  p.R = static_cast<int32_t>(R);
  fill_table(p, cos, sin, o, R);

  p.test_skip_token = test_skip_token;
  p.wait_limit_ns = wait_limit_ns;

  const int index_bits = positions->dtype == DRK_I32 ? 32 : 64;
  const bool pdl = (o.flags & DRK_FLAG_PDL) != 0;
  const bool force_staged = (o.flags & DRK_FLAG_FORCE_STAGED_PATH) != 0;
  const bool force_register = (o.flags & DRK_FLAG_FORCE_REGISTER_PATH) != 0;
  if (force_staged && force_register)
    invalid("DRK_FLAG_FORCE_STAGED_PATH and DRK_FLAG_FORCE_REGISTER_PATH are exclusive");
  if (!force_register && (force_staged || T >= DRK_STAGED_MIN_TOKENS)) {
    const StagedPlan pl = plan_staged(q, k, v, q_out, k_cache, v_cache, T, Hq, Hkv, D, R, es,
                                      o.staged_stages);
    if (pl.ok) {
      p.nrot = pl.nrot;
      p.G = pl.groups;
      p.nslots = pl.nrot;
      DeviceGuard guard(device);
      const drk::LaunchShape shape{0, 1, pl.nrot, pl.groups, pdl};
      check_launch(drk::launch_rope_kv_staged(p, pl.sp, elem_code(q->dtype), index_bits, pl.vb,
                                              paged ? drk::kCachePaged : drk::kCacheStrided,
                                              shape, reinterpret_cast<cudaStream_t>(stream)));
      return;
    }
    if (force_staged) throw Unsupported("the bulk-copy kernel cannot take this call: " + pl.why);
  }

  Aligner al{es, R, D};
  for (const drk_tensor* t : {q, k, v, q_out, k_cache, v_cache}) al.ptr(t->data);
  al.stride(T, q->strides[0]); al.stride(Hq, q->strides[1]);
  al.stride(T, k->strides[0]); al.stride(Hkv, k->strides[1]);
  al.stride(T, v->strides[0]); al.stride(Hkv, v->strides[1]);
  for (int i = 0; i < 3; ++i) al.stride(k_cache->sizes[i], k_cache->strides[i]);
  const int nrows = static_cast<int>(Hq + 2 * Hkv);
  const Shape s = plan(al, nrows, true, T, o.row_splits, o.rows_per_thread);
  p.nslots = s.nslots; p.nrot = s.nrot; p.G = s.G; p.rows_per_thread = s.rows;
  p.pdl = pdl ? 1 : 0;

  DeviceGuard guard(device);
  drk::LaunchShape shape{grid_for(T), s.splits, s.nslots, s.G, pdl};
  shape.allow_lean = s.rows == 1;
  check_launch(drk::launch_rope_kv(p, elem_code(q->dtype), index_bits, s.vb, drk::kModeFused,
                                   paged ? drk::kCachePaged : drk::kCacheStrided, shape,
                                   reinterpret_cast<cudaStream_t>(stream)));
}

// ---- fused append + decode attention: the plan both the workspace query and the launch use ----

struct AttentionPlan {
  bool tc = false;              // the tensor-core kernel (16 heads per unit)
  int64_t chunk = 0, max_chunks = 0;
  int hpb = 0, nhb = 0, lpr = 0;
  int64_t counter_bytes = 0;    // arrival counters, rounded up to 256 bytes
  int64_t partial_bytes = 0;    // fp32 [T, Hq, max_chunks, D + 2]
};

// CTAs of one attention instantiation resident per SM, from its register use (128 threads).
int attention_ctas_per_sm(int hpb, int64_t es) {
  if (es == 4) return hpb >= 8 ? 4 : 8;
  return hpb >= 8 ? 2 : (hpb == 4 ? 4 : 8);
}

AttentionPlan plan_attention(int64_t T, int64_t Hq, int64_t Hkv, int64_t D, int64_t S,
                             int32_t dtype, const drk_attention_options& ao, int device) {
  if (dtype != DRK_F32 && dtype != DRK_F16 && dtype != DRK_BF16)
    throw Unsupported(cat("fused attention supports fp32, fp16 and bf16, got ", dtype_name(dtype)));
  if (T < 0 || Hq <= 0 || Hkv <= 0 || D <= 0 || S < 0)
    invalid("fused attention: sizes must be positive");
  if (Hq % Hkv) invalid("num_q_heads (", Hq, ") must be a multiple of num_kv_heads (", Hkv, ")");
  const int64_t es = elem_size(dtype);
  const int64_t vl = 16 / es;
  if (D % vl) throw Unsupported(cat("fused attention needs head_dim * element size to be a ",
                                    "multiple of 16 bytes, got head_dim ", D));
  if (D > 32 * vl)
    throw Unsupported(cat("fused attention supports head_dim <= ", 32 * vl, " for ",
                          dtype_name(dtype), ", got ", D));
  if (T > 65535 || Hkv > 65535) throw Unsupported("fused attention: at most 65535 tokens and kv heads");
  AttentionPlan pl;
  if (ao.path < DRK_ATTN_PATH_AUTO || ao.path > DRK_ATTN_PATH_TENSOR_CORES)
    invalid("path must be DRK_ATTN_PATH_AUTO, _CUDA_CORES or _TENSOR_CORES, got ", ao.path);
  const bool tc_shape = es == 2 && (D == 128 || D == 64);
  if (ao.path == DRK_ATTN_PATH_TENSOR_CORES && !tc_shape)
    throw Unsupported(
        "the tensor-core attention kernel takes fp16/bf16 with head_dim 64 or 128");
  if (tc_shape && ao.path != DRK_ATTN_PATH_CUDA_CORES) {
    pl.tc = true;
    pl.hpb = 16;
    pl.nhb = static_cast<int>((Hq / Hkv + 15) / 16);
    int64_t chunk = ao.chunk;
    if (chunk < 0) invalid("chunk must be >= 0, got ", chunk);
    if (chunk == 0) {
      // Cost model of the persistent grid, fitted to B200 sweeps (batch 1..64, 2048..32768
      // positions, GQA and MQA): units of one chunk run in rounds of one per SM; a full round
      // streams at the HBM rate, a partial round of r units at min(HBM, r x one SM's rate:
      // ~90 GB/s with 128 dims, ~45 GB/s with 64, where a 64 KB tile takes 24 tensor-core
      // products instead of 16); every round adds ~3 us of unit start and epilogue, and ~3 us
      // more when chunks are merged. Positions live on the device, so every sequence is taken
      // as S long. Candidates: 512 doubling up to S, then S itself (no merge).
      constexpr double kHbm = 6.6e12, kRound = 3e-6, kMerge = 3e-6;
      const double kPerSm = D == 64 ? 45e9 : 90e9;
      const int64_t heads = std::max<int64_t>(1, T * Hkv * pl.nhb);
      const int64_t sms = std::max(1, drk::device_sm_count(device));
      const double row_bytes = 2.0 * D * es;
      const int64_t whole = (std::max<int64_t>(S, 1) + 127) / 128 * 128;
      double best = 0;
      for (int64_t c = 512;; c <<= 1) {
        const int64_t cand = std::min(c, whole);
        const int64_t nch = (S + cand - 1) / cand;
        const int64_t units = heads * std::max<int64_t>(nch, 1);
        const int64_t rounds = units / sms, rem = units % sms;
        const double unit_bytes = row_bytes * cand;
        double t = rounds * (sms * unit_bytes / kHbm);
        if (rem) t += rem * unit_bytes / std::min(kHbm, rem * kPerSm);
        t += (rounds + (rem ? 1 : 0)) * (kRound + (nch > 1 ? kMerge : 0.0));
        if (chunk == 0 || t < best) { best = t; chunk = cand; }
        if (cand >= whole) break;
      }
    }
    // Whole tiles: 128 positions of 128 dims, or 256 of 64 dims (64 KB of K and V either way).
    const int64_t tile = D == 64 ? 256 : 128;
    pl.chunk = (chunk + tile - 1) / tile * tile;
    pl.max_chunks = std::max<int64_t>(1, (S + pl.chunk - 1) / pl.chunk);
    // Arrival counters of the units, then the persistent grid's unit counter (reset by the
    // grid's last take).
    pl.counter_bytes = ((T * Hkv * pl.nhb + 1) * 4 + 255) / 256 * 256;
    pl.partial_bytes = T * Hq * pl.max_chunks * (D + 2) * 4;
    return pl;
  }
  int lanes = 8;
  while (lanes * vl < D) lanes <<= 1;
  pl.lpr = lanes;
  const int64_t group = Hq / Hkv;
  int hpb = ao.heads_per_cta;
  if (hpb == 0) {
    hpb = 1;
    while (hpb < group && hpb < 8) hpb <<= 1;
    // Eight 16-bit heads per CTA need ~250 registers a thread; two blocks of four re-read each
    // chunk (from L2) but keep twice the CTAs resident.
    if (hpb == 8 && es == 2) hpb = 4;
  }
  if (hpb != 1 && hpb != 2 && hpb != 4 && hpb != 8)
    invalid("heads_per_cta must be 0, 1, 2, 4 or 8, got ", hpb);
  pl.hpb = hpb;
  pl.nhb = static_cast<int>((group + hpb - 1) / hpb);
  int64_t chunk = ao.chunk;
  if (chunk < 0) invalid("chunk must be >= 0, got ", chunk);
  if (chunk == 0) {
    // About one wave of resident CTAs: a CTA streams its chunk at a latency-bound rate, so
    // more, shorter chunks finish sooner until the grid fills the SMs, while each extra chunk
    // costs a partial and a share of the merge. The power of two nearest to
    // units * S / (SMs x resident CTAs per SM), within [128, 1024] (B200 sweeps of batch
    // 1..32, 2048..8192 positions, GQA and MQA: the fastest chunk or within 11% of it).
    const int64_t units = std::max<int64_t>(1, T * Hkv * pl.nhb);
    const int64_t slots = static_cast<int64_t>(drk::device_sm_count(device)) *
                          attention_ctas_per_sm(hpb, es);
    const double want = static_cast<double>(units) * std::max<int64_t>(S, 1) / slots;
    chunk = 128;
    while (chunk < 1024 && want >= chunk * 1.41421356) chunk <<= 1;
  }
  pl.chunk = chunk;
  pl.max_chunks = std::max<int64_t>(1, (S + chunk - 1) / chunk);
  if (pl.max_chunks * pl.nhb > 0x7fffffffLL) throw Unsupported("fused attention: grid too large");
  pl.counter_bytes = (T * Hkv * pl.nhb * 4 + 255) / 256 * 256;
  pl.partial_bytes = T * Hq * pl.max_chunks * (D + 2) * 4;
  return pl;
}

drk_attention_options attention_or_default(const drk_attention_options* a) {
  drk_attention_options o{};
  if (a) o = *a;
  return o;
}

// The body of both fused attention entry points; block_table is NULL for a contiguous (or
// strided) cache and the page table of a paged one.
void attention_impl(const drk_tensor* q, const drk_tensor* k, const drk_tensor* v,
                    const drk_tensor* positions, const drk_tensor* cos, const drk_tensor* sin,
                    const drk_tensor* k_cache, const drk_tensor* v_cache,
                    const drk_tensor* block_table,
                    const drk_tensor* request_indices, const drk_tensor* q_out,
                    const drk_tensor* attn_out, const drk_attention_options* attn,
                    void* workspace, size_t workspace_bytes, const drk_options* opts,
                    uint32_t* status, drk_stream_t stream) {
  const drk_options o = options_or_default(opts);
  const drk_attention_options ao = attention_or_default(attn);
  if (o.flags & ~static_cast<uint32_t>(DRK_FLAG_PDL | DRK_FLAG_STRIDED_CACHE))
    throw Unsupported("fused attention accepts only DRK_FLAG_PDL and DRK_FLAG_STRIDED_CACHE");
  require(q, "q");
  if (q->ndim != 3) invalid("q must be [num_tokens, num_q_heads, head_dim]");
  const int64_t T = q->sizes[0], Hq = q->sizes[1], D = q->sizes[2];
  if (D % 2) invalid("head_dim must be even for split-half RoPE, got ", D);
  const int32_t device = q->device;
  check_qkv(q, "q", T, D, device);
  check_qkv(k, "k", T, D, device);
  check_qkv(v, "v", T, D, device);
  const int64_t Hkv = k->sizes[1];
  if (v->sizes[1] != Hkv) invalid("v has ", v->sizes[1], " kv heads, expected ", Hkv);
  if (q->dtype != k->dtype || q->dtype != v->dtype) invalid("q, k and v must share a dtype");
  check_index_tensor(positions, "positions", T, device);
  check_index_tensor(request_indices, "request_indices", T, device);
  if (positions->dtype != request_indices->dtype)
    invalid("positions and request_indices must share a dtype, got ",
            dtype_name(positions->dtype), "/", dtype_name(request_indices->dtype));
  const int32_t rot = resolve_rotary(o, D);
  check_rope_tables(cos, sin, D, rot, device);
  const bool paged = block_table != nullptr;
  const bool strided_ok = (o.flags & DRK_FLAG_STRIDED_CACHE) != 0 && !paged;
  check_cache(k_cache, paged ? "k_pages" : "k_cache", k->dtype, Hkv, D, device, strided_ok);
  check_cache(v_cache, paged ? "v_pages" : "v_cache", v->dtype, Hkv, D, device, strided_ok);
  check_caches_are_distinct(k_cache, v_cache);
  int64_t block_size = 0;
  if (paged) {
    check_device(block_table, "block_table", device);
    if (block_table->dtype != positions->dtype)
      invalid("block_table must share the index dtype of positions, got ",
              dtype_name(block_table->dtype), "/", dtype_name(positions->dtype));
    if (block_table->ndim != 2 || !is_contiguous(block_table))
      invalid("block_table must be a contiguous [num_requests, max_blocks_per_request] tensor");
    block_size = k_cache->sizes[1];
    if (block_size <= 0 || block_size % 8 || (128 % block_size && block_size % 128))
      throw Unsupported(cat("paged fused attention takes block sizes that are multiples of 8 ",
                            "dividing 128, or multiples of 128; got ", block_size));
  }
  if (q_out != nullptr) check_output(q_out, "q_out", q->dtype, T, Hq, D, device);
  check_output(attn_out, "attn_out", q->dtype, T, Hq, D, device);
  check_float_dtype(q->dtype, "fused_rope_kv_append_attention");
  const int64_t S = paged ? block_table->sizes[1] * block_size : k_cache->sizes[1];
  const AttentionPlan pl = plan_attention(T, Hq, Hkv, D, S, q->dtype, ao, device);
  if (paged && !pl.tc)
    throw Unsupported("paged fused attention takes fp16/bf16 with head_dim 64 or 128 (the "
                      "tensor-core kernel)");
  if (T == 0) return;
  const int64_t es = elem_size(q->dtype);
  uintptr_t addr = reinterpret_cast<uintptr_t>(k_cache->data) |
                   reinterpret_cast<uintptr_t>(v_cache->data);
  int64_t strides = 0;
  for (int i = 0; i < 3; ++i)
    if (k_cache->sizes[i] > 1) strides |= k_cache->strides[i];
  if (addr % 16 || (strides * es) % 16)
    throw Unsupported("fused attention needs 16-byte aligned cache rows (base and strides)");
  if (workspace == nullptr ||
      workspace_bytes < static_cast<size_t>(pl.counter_bytes + pl.partial_bytes))
    invalid("workspace needs ", pl.counter_bytes + pl.partial_bytes, " bytes, got ",
            workspace == nullptr ? 0 : workspace_bytes);
  if (reinterpret_cast<uintptr_t>(workspace) % 16) invalid("workspace must be 16-byte aligned");
  if (ao.scale < 0) invalid("scale must be >= 0 (0 = 1/sqrt(head_dim))");

  const int64_t R = rot ? rot : D;
  drk::KernelParams p{};
  p.q = static_cast<const char*>(q->data);
  p.k = static_cast<const char*>(k->data);
  p.v = static_cast<const char*>(v->data);
  p.k_dst = static_cast<char*>(k_cache->data);
  p.v_dst = static_cast<char*>(v_cache->data);
  p.positions = positions->data;
  p.request_indices = request_indices->data;
  p.status = status;
  p.T = T;
  p.q_ts = q->strides[0]; p.q_hs = q->strides[1];
  p.k_ts = k->strides[0]; p.k_hs = k->strides[1];
  p.v_ts = v->strides[0]; p.v_hs = v->strides[1];
  p.c_bs = k_cache->strides[0]; p.c_ss = k_cache->strides[1]; p.c_hs = k_cache->strides[2];
  p.B = paged ? block_table->sizes[0] : k_cache->sizes[0];
  p.S = S;
  if (paged) {
    p.block_table = block_table->data;
    p.num_blocks = k_cache->sizes[0];
    p.block_size = block_size;
    p.bt_stride = block_table->sizes[1];
  }
  p.Hq = static_cast<int32_t>(Hq);
  p.Hkv = static_cast<int32_t>(Hkv);
  p.D = static_cast<int32_t>(D);
  p.R = static_cast<int32_t>(R);
  fill_table(p, cos, sin, o, R);

  drk::AttentionParams a{};
  a.box_rows = paged ? static_cast<int32_t>(std::min<int64_t>(block_size, 128)) : 128;
  char* ws = static_cast<char*>(workspace);
  a.counters = reinterpret_cast<int*>(ws);
  a.workspace = reinterpret_cast<float*>(ws + pl.counter_bytes);
  a.attn_out = attn_out->data;
  a.q_out = q_out ? static_cast<char*>(q_out->data) : nullptr;
  const double scale = ao.scale > 0 ? ao.scale : 1.0 / std::sqrt(static_cast<double>(D));
  a.scale_log2 = static_cast<float>(scale * 1.4426950408889634);
  a.chunk = static_cast<int32_t>(pl.chunk);
  a.max_chunks = static_cast<int32_t>(pl.max_chunks);
  a.group = static_cast<int32_t>(Hq / Hkv);
  a.nhb = pl.nhb;

  DeviceGuard guard(device);
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // Every call returns the counters to zero (unless a bounded wait ran out), so a caller that
  // keeps its workspace and says it is zeroed saves this memset node.
  if (!(ao.flags & DRK_ATTN_WORKSPACE_ZEROED) &&
      cudaMemsetAsync(workspace, 0, static_cast<size_t>(pl.counter_bytes), s) != cudaSuccess)
    throw CudaFailure("cudaMemsetAsync of the attention counters failed");
  const int index_bits_tc = positions->dtype == DRK_I32 ? 32 : 64;
  if (pl.tc) {
    const int64_t units = T * Hkv * pl.nhb * pl.max_chunks;
    if (units > 0x7fffffffLL) throw Unsupported("fused attention: more than 2^31 work units");
    // One round of 16-byte loads for the query rotation: full rotary, aligned q rows, q_out and
    // table rows.
    const uintptr_t qa = reinterpret_cast<uintptr_t>(q->data) |
                         (q_out ? reinterpret_cast<uintptr_t>(q_out->data) : 0);
    const int64_t qs = (T > 1 ? q->strides[0] : 0) | (Hq > 1 ? q->strides[1] : 0);
    a.q_vec = (R == D && qa % 16 == 0 && (qs * es) % 16 == 0 && p.table_vec4) ? 1 : 0;
    check_launch(drk::launch_rope_kv_attention_tc(p, a, elem_code(q->dtype), index_bits_tc, units,
                                                  (o.flags & DRK_FLAG_PDL) != 0, s));
    return;
  }
  const drk::AttentionShape shape{static_cast<int>(pl.max_chunks * pl.nhb),
                                  static_cast<int>(Hkv), static_cast<int>(T), pl.lpr, pl.hpb,
                                  (o.flags & DRK_FLAG_PDL) != 0};
  const int index_bits = positions->dtype == DRK_I32 ? 32 : 64;
  check_launch(drk::launch_rope_kv_attention(p, a, elem_code(q->dtype), index_bits, shape, s));
}

void rope_forward_impl(const drk_tensor* q, const drk_tensor* k, const drk_tensor* positions,
                       const drk_tensor* cos, const drk_tensor* sin, const drk_tensor* q_out,
                       const drk_tensor* k_out, const drk_options* opts, uint32_t* status,
                       drk_stream_t stream, bool launch) {
  const drk_options o = options_or_default(opts);
  require(q, "q");
  if (q->ndim != 3) invalid("q must be [num_tokens, num_q_heads, head_dim]");
  const int64_t T = q->sizes[0], Hq = q->sizes[1], D = q->sizes[2];
  if (D % 2) invalid("head_dim must be even for split-half RoPE, got ", D);
  const int32_t device = q->device;
  check_qkv(q, "q", T, D, device);
  check_qkv(k, "k", T, D, device);
  if (q->dtype != k->dtype)
    invalid("q and k must share a dtype, got ", dtype_name(q->dtype), "/",
            dtype_name(k->dtype));
  check_index_tensor(positions, "positions", T, device);
  const int32_t rot = resolve_rotary(o, D);
  check_rope_tables(cos, sin, D, rot, device);
  const int64_t Hkv = k->sizes[1];
  check_output(q_out, "q_out", q->dtype, T, Hq, D, device);
  check_output(k_out, "k_out", k->dtype, T, Hkv, D, device);
  check_float_dtype(q->dtype, "rope_forward");
  if (T == 0 || !launch) return;

  const int64_t R = rot ? rot : D;
  drk::KernelParams p{};
  p.q = static_cast<const char*>(q->data);
  p.k = static_cast<const char*>(k->data);
  p.q_out = static_cast<char*>(q_out->data);
  p.k_dst = static_cast<char*>(k_out->data);
  p.positions = positions->data;
  p.status = status;
  p.T = T;
  p.q_ts = q->strides[0]; p.q_hs = q->strides[1];
  p.k_ts = k->strides[0]; p.k_hs = k->strides[1];
  p.Hq = static_cast<int32_t>(Hq);
  p.Hkv = static_cast<int32_t>(Hkv);
  p.D = static_cast<int32_t>(D);
  p.R = static_cast<int32_t>(R);
  fill_table(p, cos, sin, o, R);
  Aligner al{elem_size(q->dtype), R, D};
  for (const drk_tensor* t : {q, k, q_out, k_out}) al.ptr(t->data);
  al.stride(T, q->strides[0]); al.stride(Hq, q->strides[1]);
  al.stride(T, k->strides[0]); al.stride(Hkv, k->strides[1]);
  const Shape s = plan(al, static_cast<int>(Hq + Hkv), true, T, o.row_splits);
  p.nslots = s.nslots; p.nrot = s.nrot; p.G = s.G; p.rows_per_thread = s.rows;
  p.pdl = (o.flags & DRK_FLAG_PDL) ? 1 : 0;
  DeviceGuard guard(device);
  const drk::LaunchShape shape{grid_for(T), s.splits, s.nslots, s.G, (o.flags & DRK_FLAG_PDL) != 0};
  const int index_bits = positions->dtype == DRK_I32 ? 32 : 64;
  check_launch(drk::launch_rope_kv(p, elem_code(q->dtype), index_bits, s.vb, drk::kModeRope,
                                   drk::kCacheStrided, shape,
                                   reinterpret_cast<cudaStream_t>(stream)));
}

void kv_append_impl(const drk_tensor* k_rot, const drk_tensor* v, const drk_tensor* positions,
                    const drk_tensor* request_indices, const drk_tensor* k_cache,
                    const drk_tensor* v_cache, const drk_options* opts, uint32_t* status,
                    drk_stream_t stream, bool launch) {
  const drk_options o = options_or_default(opts);
  require(k_rot, "k_rot");
  if (k_rot->ndim != 3) invalid("k_rot must be [num_tokens, num_kv_heads, head_dim]");
  const int64_t T = k_rot->sizes[0], Hkv = k_rot->sizes[1], D = k_rot->sizes[2];
  const int32_t device = k_rot->device;
  check_qkv(k_rot, "k_rot", T, D, device);
  check_qkv(v, "v", T, D, device);
  if (v->sizes[1] != Hkv) invalid("v has ", v->sizes[1], " kv heads, expected ", Hkv);
  if (k_rot->dtype != v->dtype)
    invalid("k_rot and v must share a dtype, got ", dtype_name(k_rot->dtype), "/",
            dtype_name(v->dtype));
  check_index_tensor(positions, "positions", T, device);
  check_index_tensor(request_indices, "request_indices", T, device);
  if (positions->dtype != request_indices->dtype)
    invalid("positions and request_indices must share a dtype, got ",
            dtype_name(positions->dtype), "/", dtype_name(request_indices->dtype));
  const bool strided_ok = (o.flags & DRK_FLAG_STRIDED_CACHE) != 0;
  check_cache(k_cache, "k_cache", k_rot->dtype, Hkv, D, device, strided_ok);
  check_cache(v_cache, "v_cache", v->dtype, Hkv, D, device, strided_ok);
  check_caches_are_distinct(k_cache, v_cache);
  check_float_dtype(k_rot->dtype, "kv_append");
  if (o.k_position_limit < 0)
    invalid("k_position_limit must be >= 0, got ", o.k_position_limit);
  if (T == 0 || !launch) return;
  if (D % 2)
    throw Unsupported(cat("kv_append needs an even head_dim, got ", D));

  drk::KernelParams p{};
  p.k = static_cast<const char*>(k_rot->data);
  p.v = static_cast<const char*>(v->data);
  p.k_dst = static_cast<char*>(k_cache->data);
  p.v_dst = static_cast<char*>(v_cache->data);
  p.positions = positions->data;
  p.request_indices = request_indices->data;
  p.status = status;
  p.T = T;
  p.k_ts = k_rot->strides[0]; p.k_hs = k_rot->strides[1];
  p.v_ts = v->strides[0]; p.v_hs = v->strides[1];
  p.c_bs = k_cache->strides[0]; p.c_ss = k_cache->strides[1]; p.c_hs = k_cache->strides[2];
  p.B = k_cache->sizes[0];
  p.S = k_cache->sizes[1];
  p.Hkv = static_cast<int32_t>(Hkv);
  p.D = static_cast<int32_t>(D);
  p.R = 0;
  p.table_rows = o.k_position_limit > 0 ? o.k_position_limit : INT64_MAX;
  Aligner al{elem_size(k_rot->dtype), 0, D};
  for (const drk_tensor* t : {k_rot, v, k_cache, v_cache}) al.ptr(t->data);
  al.stride(T, k_rot->strides[0]); al.stride(Hkv, k_rot->strides[1]);
  al.stride(T, v->strides[0]); al.stride(Hkv, v->strides[1]);
  for (int i = 0; i < 3; ++i) al.stride(k_cache->sizes[i], k_cache->strides[i]);
  const Shape s = plan(al, static_cast<int>(2 * Hkv), false, T, o.row_splits);
  p.nslots = s.nslots; p.nrot = 0; p.G = s.G; p.rows_per_thread = s.rows;
  p.pdl = (o.flags & DRK_FLAG_PDL) ? 1 : 0;
  DeviceGuard guard(device);
  const drk::LaunchShape shape{grid_for(T), s.splits, s.nslots, s.G, (o.flags & DRK_FLAG_PDL) != 0};
  const int index_bits = positions->dtype == DRK_I32 ? 32 : 64;
  check_launch(drk::launch_rope_kv(p, elem_code(k_rot->dtype), index_bits, s.vb,
                                   drk::kModeAppend, drk::kCacheStrided, shape,
                                   reinterpret_cast<cudaStream_t>(stream)));
}

}  // namespace

namespace drk {
// The host checks of drk_rope_forward and drk_kv_append without the launch: DRK_OK, or the
// error code with the message drk_last_error() returns. (noalloc.cu validates a call before it
// touches its scratch array.)
int validate_rope_forward(const drk_tensor* q, const drk_tensor* k, const drk_tensor* positions,
                          const drk_tensor* cos, const drk_tensor* sin, const drk_tensor* q_out,
                          const drk_tensor* k_out) {
  return guarded([&] {
    rope_forward_impl(q, k, positions, cos, sin, q_out, k_out, nullptr, nullptr, nullptr, false);
  });
}
int validate_kv_append(const drk_tensor* k_rot, const drk_tensor* v, const drk_tensor* positions,
                       const drk_tensor* request_indices, const drk_tensor* k_cache,
                       const drk_tensor* v_cache, const drk_options* opts) {
  return guarded([&] {
    kv_append_impl(k_rot, v, positions, request_indices, k_cache, v_cache, opts, nullptr,
                   nullptr, false);
  });
}
// For entry points defined in other files of this library (noalloc.cu).
void set_last_error(const std::string& message) { g_last_error = message; }
}  // namespace drk

extern "C" {

int drk_fused_rope_kv_append(const drk_tensor* q, const drk_tensor* k, const drk_tensor* v,
                             const drk_tensor* positions, const drk_tensor* cos,
                             const drk_tensor* sin, const drk_tensor* k_cache,
                             const drk_tensor* v_cache, const drk_tensor* request_indices,
                             const drk_tensor* q_out, uint32_t* status, drk_stream_t stream) {
  return guarded([&] {
    fused_impl(q, k, v, positions, cos, sin, k_cache, v_cache, nullptr, request_indices, q_out,
               nullptr, status, stream);
  });
}

int drk_fused_rope_kv_append_ex(const drk_tensor* q, const drk_tensor* k, const drk_tensor* v,
                                const drk_tensor* positions, const drk_tensor* cos,
                                const drk_tensor* sin, const drk_tensor* k_cache,
                                const drk_tensor* v_cache, const drk_tensor* request_indices,
                                const drk_tensor* q_out, const drk_options* opts,
                                uint32_t* status, drk_stream_t stream) {
  return guarded([&] {
    fused_impl(q, k, v, positions, cos, sin, k_cache, v_cache, nullptr, request_indices, q_out,
               opts, status, stream);
  });
}

int drk_paged_rope_kv_append(const drk_tensor* q, const drk_tensor* k, const drk_tensor* v,
                             const drk_tensor* positions, const drk_tensor* cos,
                             const drk_tensor* sin, const drk_tensor* k_pages,
                             const drk_tensor* v_pages, const drk_tensor* block_table,
                             const drk_tensor* request_indices, const drk_tensor* q_out,
                             const drk_options* opts, uint32_t* status, drk_stream_t stream) {
  return guarded([&] {
    if (block_table == nullptr) invalid("block_table is NULL");
    fused_impl(q, k, v, positions, cos, sin, k_pages, v_pages, block_table, request_indices,
               q_out, opts, status, stream);
  });
}

int drk_rope_forward(const drk_tensor* q, const drk_tensor* k, const drk_tensor* positions,
                     const drk_tensor* cos, const drk_tensor* sin, const drk_tensor* q_out,
                     const drk_tensor* k_out, const drk_options* opts, uint32_t* status,
                     drk_stream_t stream) {
  return guarded([&] {
    rope_forward_impl(q, k, positions, cos, sin, q_out, k_out, opts, status, stream, true);
  });
}

int drk_kv_append(const drk_tensor* k_rot, const drk_tensor* v, const drk_tensor* positions,
                  const drk_tensor* request_indices, const drk_tensor* k_cache,
                  const drk_tensor* v_cache, const drk_options* opts, uint32_t* status,
                  drk_stream_t stream) {
  return guarded([&] {
    kv_append_impl(k_rot, v, positions, request_indices, k_cache, v_cache, opts, status, stream,
                   true);
  });
}

int drk_advance_positions(const drk_tensor* positions, int64_t delta, uint32_t flags,
                          drk_stream_t stream) {
  return guarded([&] {
    require(positions, "positions");
    if (positions->device < 0)
      invalid("positions must be a CUDA tensor, got ", device_name(positions->device));
    if (positions->dtype != DRK_I32 && positions->dtype != DRK_I64)
      invalid("positions must be int32 or int64, got ", dtype_name(positions->dtype));
    if (positions->ndim != 1 || !is_contiguous(positions))
      invalid("positions must be a contiguous [num_tokens] tensor");
    const int64_t n = positions->sizes[0];
    if (n == 0) return;
    DeviceGuard guard(positions->device);
    check_launch(drk::launch_advance_positions(positions->data,
                                               positions->dtype == DRK_I32 ? 32 : 64, n, delta,
                                               (flags & DRK_FLAG_PDL) != 0,
                                               reinterpret_cast<cudaStream_t>(stream)));
  });
}

int drk_smoke_fill(const drk_tensor* tensor, double value, drk_stream_t stream) {
  return guarded([&] {
    require(tensor, "tensor");
    if (tensor->device < 0)
      invalid("smoke_fill expects a CUDA tensor, got ", device_name(tensor->device));
    if (!is_contiguous(tensor)) invalid("smoke_fill expects a contiguous tensor");
    check_float_dtype(tensor->dtype, "smoke_fill");
    const int64_t n = numel(tensor);
    if (n == 0) return;
    DeviceGuard guard(tensor->device);
    check_launch(drk::launch_smoke_fill(tensor->data, elem_code(tensor->dtype), n, value,
                                        reinterpret_cast<cudaStream_t>(stream)));
  });
}

int drk_build_info(char* buf, size_t len, drk_stream_t stream) {
  return guarded([&] {
    if (buf == nullptr || len == 0) invalid("buf is NULL or empty");
    int arch = 0, runtime = 0, driver = 0;
    cudaError_t err = drk::run_arch_probe(&arch, reinterpret_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) throw CudaFailure(cat("arch probe failed: ", cudaGetErrorString(err)));
    cudaRuntimeGetVersion(&runtime);
    cudaDriverGetVersion(&driver);
    auto ver = [](int packed) {
      return packed <= 0 ? std::string() : cat(packed / 1000, ".", (packed % 1000) / 10);
    };
#if defined(__FAST_MATH__) || defined(__USE_FAST_MATH__)
    const char* fast_math = "1";
#else
    const char* fast_math = "0";
#endif
    const std::string text =
        cat("gencode_arch=", arch, "\ncuda_version_compiled=", ver(CUDART_VERSION),
            "\ncuda_version_runtime=", ver(runtime), "\ncuda_version_driver=", ver(driver),
            "\nnvcc_version=", __CUDACC_VER_MAJOR__, ".", __CUDACC_VER_MINOR__, ".",
            __CUDACC_VER_BUILD__, "\nfast_math=", fast_math, "\n");
    if (text.size() + 1 > len) invalid("buf too small: need ", text.size() + 1, " bytes");
    std::memcpy(buf, text.c_str(), text.size() + 1);
  });
}

int64_t drk_attention_workspace_bytes(int64_t num_tokens, int32_t num_q_heads,
                                      int32_t num_kv_heads, int32_t head_dim,
                                      int64_t cache_alloc_len, int32_t dtype,
                                      const drk_attention_options* attn, int32_t device) {
  int64_t bytes = 0;
  const int rc = guarded([&] {
    const AttentionPlan pl = plan_attention(num_tokens, num_q_heads, num_kv_heads, head_dim,
                                            cache_alloc_len, dtype, attention_or_default(attn),
                                            device);
    bytes = pl.counter_bytes + pl.partial_bytes;
  });
  return rc == DRK_OK ? bytes : rc;
}

int drk_fused_rope_kv_append_attention(
    const drk_tensor* q, const drk_tensor* k, const drk_tensor* v, const drk_tensor* positions,
    const drk_tensor* cos, const drk_tensor* sin, const drk_tensor* k_cache,
    const drk_tensor* v_cache, const drk_tensor* request_indices, const drk_tensor* q_out,
    const drk_tensor* attn_out, const drk_attention_options* attn, void* workspace,
    size_t workspace_bytes, const drk_options* opts, uint32_t* status, drk_stream_t stream) {
  return guarded([&] {
    attention_impl(q, k, v, positions, cos, sin, k_cache, v_cache, nullptr, request_indices,
                   q_out, attn_out, attn, workspace, workspace_bytes, opts, status, stream);
  });
}

int drk_paged_rope_kv_append_attention(
    const drk_tensor* q, const drk_tensor* k, const drk_tensor* v, const drk_tensor* positions,
    const drk_tensor* cos, const drk_tensor* sin, const drk_tensor* k_pages,
    const drk_tensor* v_pages, const drk_tensor* block_table,
    const drk_tensor* request_indices, const drk_tensor* q_out, const drk_tensor* attn_out,
    const drk_attention_options* attn, void* workspace, size_t workspace_bytes,
    const drk_options* opts, uint32_t* status, drk_stream_t stream) {
  return guarded([&] {
    require(block_table, "block_table");
    attention_impl(q, k, v, positions, cos, sin, k_pages, v_pages, block_table, request_indices,
                   q_out, attn_out, attn, workspace, workspace_bytes, opts, status, stream);
  });
}

int drk_launch_empty(int count, int pdl, drk_stream_t stream) {
  return guarded([&] {
    if (count < 0) invalid("count must be >= 0");
    check_launch(drk::launch_empty(count, pdl != 0, reinterpret_cast<cudaStream_t>(stream)));
  });
}

// Testing the bounded-wait timeout path of the bulk-copy kernel, without a GPU fault: the
// fused op forced onto that kernel, with the loads of token `skip_token` not issued and every
// wait limited to `wait_limit_ns`. The CTA that owns the token waits for copies that were never
// issued; when the limit passes it sets DRK_STATUS_TIMEOUT, waits for its other copies in
// flight and returns, and the other CTAs finish normally. Not declared in the public header.
DRK_API int drk_testing_staged_timeout(
    const drk_tensor* q, const drk_tensor* k, const drk_tensor* v, const drk_tensor* positions,
    const drk_tensor* cos, const drk_tensor* sin, const drk_tensor* k_cache,
    const drk_tensor* v_cache, const drk_tensor* request_indices, const drk_tensor* q_out,
    int64_t skip_token, int64_t wait_limit_ns, uint32_t* status, drk_stream_t stream) {
  return guarded([&] {
    if (wait_limit_ns <= 0 || wait_limit_ns > 2000000000ll)
      invalid("wait_limit_ns must be in (0, 2e9], got ", wait_limit_ns);
    drk_options o{};
    o.flags = DRK_FLAG_FORCE_STAGED_PATH;
    fused_impl(q, k, v, positions, cos, sin, k_cache, v_cache, nullptr, request_indices, q_out,
               &o, status, stream, skip_token, wait_limit_ns);
  });
}

int drk_launch_copy_probe(const void* src, void* dst, int64_t bytes, int64_t stride_bytes,
                          int count, int threads_per_cta, int pdl, int prefetch,
                          drk_stream_t stream) {
  return guarded([&] {
    if (count < 0) invalid("count must be >= 0");
    if (bytes <= 0 || bytes % 32) invalid("bytes must be a positive multiple of 32, got ", bytes);
    if (stride_bytes < bytes || stride_bytes % 16)
      invalid("stride_bytes must be >= bytes and a multiple of 16, got ", stride_bytes);
    if (threads_per_cta < 32 || threads_per_cta > 1024 || threads_per_cta % 32)
      invalid("threads_per_cta must be a multiple of 32 in [32, 1024], got ", threads_per_cta);
    if (src == nullptr || dst == nullptr || reinterpret_cast<uintptr_t>(src) % 16 ||
        reinterpret_cast<uintptr_t>(dst) % 16)
      invalid("src and dst must be non-null and 16-byte aligned");
    check_launch(drk::launch_copy_probe(src, dst, bytes / 16, stride_bytes / 16, count,
                                        threads_per_cta, pdl != 0, prefetch != 0,
                                        reinterpret_cast<cudaStream_t>(stream)));
  });
}

const char* drk_last_error(void) { return g_last_error.c_str(); }

const char* drk_status_string(uint32_t status) {
  if (status == 0) {
    g_status_text = "ok";
    return g_status_text.c_str();
  }
  std::string s;
  auto add = [&](uint32_t bit, const char* text) {
    if (status & bit) s += (s.empty() ? "" : "; ") + std::string(text);
  };
  add(DRK_STATUS_POSITION_OUT_OF_CACHE, "a position was outside [0, cache_alloc_len)");
  add(DRK_STATUS_REQUEST_OUT_OF_RANGE, "a request index was outside [0, batch)");
  add(DRK_STATUS_POSITION_OUT_OF_TABLE, "a position was outside the cos/sin table");
  add(DRK_STATUS_BLOCK_OUT_OF_RANGE, "a block-table entry was outside the page pool");
  add(DRK_STATUS_TIMEOUT, "a bounded in-kernel wait ran out and a CTA stopped early");
  if (status & ~0x1Fu) s += (s.empty() ? "" : "; ") + cat("unknown bits 0x", std::hex, status);
  g_status_text = s;
  return g_status_text.c_str();
}

const char* drk_version(void) { return "0.1.0"; }

}  // extern "C"
