// PyTorch binding over the C ABI (include/decode_rope.h): the drop-in for the reference's
// decode_kernels.cuda._ext module (csrc/bindings.cpp:18-34 of the reference), with the same
// function names, keyword names, return types and error messages.
//
// The binding owns what the C ABI leaves to its caller: it allocates outputs through PyTorch's
// caching allocator (so calls stay graph-capturable), launches on the current stream of the
// inputs' device, and keeps one status word per device for the kernels' bounds reports.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

#include <atomic>
#include <map>
#include <mutex>
#include <string>
#include <tuple>
#include <vector>

#include "decode_rope.h"

namespace {

int32_t dtype_code(at::ScalarType t) {
  switch (t) {
    case at::kFloat: return DRK_F32;
    case at::kHalf: return DRK_F16;
    case at::kBFloat16: return DRK_BF16;
    case at::kDouble: return DRK_F64;
    case at::kInt: return DRK_I32;
    case at::kLong: return DRK_I64;
    default: return -1;
  }
}

drk_tensor describe(const at::Tensor& t) {
  drk_tensor d{};
  d.data = t.data_ptr();
  d.dtype = dtype_code(t.scalar_type());
  d.ndim = static_cast<int32_t>(std::min<int64_t>(t.dim(), 4));
  d.device = t.is_cuda() ? t.get_device() : -1;
  for (int i = 0; i < d.ndim; ++i) {
    d.sizes[i] = t.size(i);
    d.strides[i] = t.stride(i);
  }
  if (t.dim() > 4) d.ndim = static_cast<int32_t>(t.dim());  // rejected by the ABI's checks
  return d;
}

void raise_on_error(int rc) {
  if (rc == DRK_OK) return;
  TORCH_CHECK(false, drk_last_error());
}

cudaStream_t stream_for(const at::Tensor& t) {
  if (!t.is_cuda()) return nullptr;
  return at::cuda::getCurrentCUDAStream(t.get_device()).stream();
}

// One zero-initialised uint32 per device, allocated outside any stream capture's view (relaxed
// capture mode) so the first call may happen while a graph is being captured. The fast path
// is one atomic load; the mutex only guards the first allocation on a device.
constexpr int kMaxStatusDevices = 64;
std::mutex g_status_mutex;
std::atomic<uint32_t*> g_status[kMaxStatusDevices];

uint32_t* status_word(int device) {
  TORCH_CHECK(device >= 0 && device < kMaxStatusDevices, "device ordinal ", device,
              " is beyond the ", kMaxStatusDevices, " devices this binding tracks");
  uint32_t* fast = g_status[device].load(std::memory_order_acquire);
  if (fast != nullptr) return fast;
  std::lock_guard<std::mutex> lock(g_status_mutex);
  if (uint32_t* again = g_status[device].load(std::memory_order_acquire)) return again;
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;
  cudaThreadExchangeStreamCaptureMode(&mode);
  uint32_t* ptr = nullptr;
  cudaError_t err = cudaMalloc(&ptr, sizeof(uint32_t));
  cudaStream_t side = nullptr;
  if (err == cudaSuccess) err = cudaStreamCreateWithFlags(&side, cudaStreamNonBlocking);
  if (err == cudaSuccess) err = cudaMemsetAsync(ptr, 0, sizeof(uint32_t), side);
  if (err == cudaSuccess) err = cudaStreamSynchronize(side);
  if (side) cudaStreamDestroy(side);
  cudaThreadExchangeStreamCaptureMode(&mode);
  TORCH_CHECK(err == cudaSuccess, "could not allocate the status word: ",
              cudaGetErrorString(err));
  g_status[device].store(ptr, std::memory_order_release);
  return ptr;
}

uint32_t* status_for(const at::Tensor& t) {
  return t.is_cuda() ? status_word(t.get_device()) : nullptr;
}

drk_options make_options(uint32_t flags, int64_t rotary_dim,
                         const c10::optional<at::Tensor>& inv_freq, int64_t head_dim = 0) {
  drk_options o{};
  o.flags = flags;
  o.rotary_dim = static_cast<int32_t>(rotary_dim);
  if (inv_freq.has_value() && inv_freq->defined()) {
    TORCH_CHECK(inv_freq->is_cuda() && inv_freq->scalar_type() == at::kFloat &&
                    inv_freq->is_contiguous(),
                "inv_freq must be a contiguous fp32 CUDA tensor");
    const int64_t width = rotary_dim ? rotary_dim : head_dim;
    TORCH_CHECK(inv_freq->numel() == width / 2, "inv_freq must hold rotary_dim/2 = ", width / 2,
                " frequencies, got ", inv_freq->numel());
    o.inv_freq = inv_freq->data_ptr<float>();
    o.flags |= DRK_FLAG_INREG_TRIG;
  }
  return o;
}

uint32_t path_flags(const std::string& path) {
  if (path == "auto") return 0u;
  if (path == "register") return DRK_FLAG_FORCE_REGISTER_PATH;
  if (path == "staged") return DRK_FLAG_FORCE_STAGED_PATH;
  TORCH_CHECK(false, "path must be 'auto', 'register' or 'staged', got '", path, "'");
}

int32_t attention_path(const std::string& path) {
  if (path == "auto") return DRK_ATTN_PATH_AUTO;
  if (path == "cuda_cores") return DRK_ATTN_PATH_CUDA_CORES;
  if (path == "tensor_cores") return DRK_ATTN_PATH_TENSOR_CORES;
  TORCH_CHECK(false, "path must be 'auto', 'cuda_cores' or 'tensor_cores', got '", path, "'");
}

at::Tensor empty_like_rows(const at::Tensor& src, int64_t heads) {
  return at::empty({src.size(0), heads, src.size(2)}, src.options());
}

// ---- the reference's five functions ----

at::Tensor fused_rope_kv_append(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor positions,
                                at::Tensor cos, at::Tensor sin, at::Tensor k_cache,
                                at::Tensor v_cache, at::Tensor request_indices) {
  at::Tensor q_out;
  if (q.dim() == 3) q_out = empty_like_rows(q, q.size(1));
  const drk_tensor dq = describe(q), dk = describe(k), dv = describe(v),
                   dp = describe(positions), dc = describe(cos), ds = describe(sin),
                   dkc = describe(k_cache), dvc = describe(v_cache),
                   dri = describe(request_indices);
  drk_tensor dqo{};
  if (q_out.defined()) dqo = describe(q_out);
  raise_on_error(drk_fused_rope_kv_append(&dq, &dk, &dv, &dp, &dc, &ds, &dkc, &dvc, &dri,
                                          q_out.defined() ? &dqo : nullptr, status_for(q),
                                          stream_for(q)));
  return q_out;
}

std::tuple<at::Tensor, at::Tensor> rope_forward(at::Tensor q, at::Tensor k, at::Tensor positions,
                                                at::Tensor cos, at::Tensor sin) {
  at::Tensor q_out, k_out;
  if (q.dim() == 3) q_out = empty_like_rows(q, q.size(1));
  if (k.dim() == 3) k_out = empty_like_rows(k, k.size(1));
  const drk_tensor dq = describe(q), dk = describe(k), dp = describe(positions),
                   dc = describe(cos), ds = describe(sin);
  drk_tensor dqo{}, dko{};
  if (q_out.defined()) dqo = describe(q_out);
  if (k_out.defined()) dko = describe(k_out);
  raise_on_error(drk_rope_forward(&dq, &dk, &dp, &dc, &ds, q_out.defined() ? &dqo : nullptr,
                                  k_out.defined() ? &dko : nullptr, nullptr, status_for(q),
                                  stream_for(q)));
  return {q_out, k_out};
}

void kv_append(at::Tensor k_rot, at::Tensor v, at::Tensor positions, at::Tensor request_indices,
               at::Tensor k_cache, at::Tensor v_cache) {
  const drk_tensor dk = describe(k_rot), dv = describe(v), dp = describe(positions),
                   dri = describe(request_indices), dkc = describe(k_cache),
                   dvc = describe(v_cache);
  raise_on_error(drk_kv_append(&dk, &dv, &dp, &dri, &dkc, &dvc, nullptr, status_for(k_rot),
                               stream_for(k_rot)));
}

// rope_forward then the append, in one call from Python: k_rot is materialised (the separate
// op's defining intermediate) and the append is told the cos/sin row count, so a token past the
// table keeps its K slot as in the fused op.
at::Tensor separate_rope_kv_append(at::Tensor q, at::Tensor k, at::Tensor v,
                                   at::Tensor positions, at::Tensor cos, at::Tensor sin,
                                   at::Tensor k_cache, at::Tensor v_cache,
                                   at::Tensor request_indices) {
  auto rotated = rope_forward(q, k, positions, cos, sin);
  const at::Tensor& k_rot = std::get<1>(rotated);
  drk_options o{};
  o.k_position_limit = cos.dim() == 2 ? cos.size(0) : 0;
  const drk_tensor dk = describe(k_rot), dv = describe(v), dp = describe(positions),
                   dri = describe(request_indices), dkc = describe(k_cache),
                   dvc = describe(v_cache);
  raise_on_error(drk_kv_append(&dk, &dv, &dp, &dri, &dkc, &dvc, &o, status_for(k_rot),
                               stream_for(k_rot)));
  return std::get<0>(rotated);
}

void smoke_fill(at::Tensor tensor, double value) {
  const drk_tensor d = describe(tensor);
  raise_on_error(drk_smoke_fill(&d, value, stream_for(tensor)));
}

std::map<std::string, std::string> build_info() {
  const int device = c10::cuda::current_device();
  char buf[1024];
  raise_on_error(drk_build_info(buf, sizeof(buf), at::cuda::getCurrentCUDAStream(device).stream()));
  std::map<std::string, std::string> info;
  std::string text(buf);
  size_t start = 0;
  while (start < text.size()) {
    size_t end = text.find('\n', start);
    if (end == std::string::npos) end = text.size();
    const std::string line = text.substr(start, end - start);
    const size_t eq = line.find('=');
    if (eq != std::string::npos) info[line.substr(0, eq)] = line.substr(eq + 1);
    start = end + 1;
  }
  return info;
}

// ---- extensions (no counterpart in the reference's binding) ----

at::Tensor fused_rope_kv_append_ex(at::Tensor q, at::Tensor k, at::Tensor v,
                                   at::Tensor positions, at::Tensor cos, at::Tensor sin,
                                   at::Tensor k_cache, at::Tensor v_cache,
                                   at::Tensor request_indices, int64_t rotary_dim, bool pdl,
                                   bool strided_cache, c10::optional<at::Tensor> inv_freq,
                                   c10::optional<at::Tensor> q_out_opt, const std::string& path,
                                   int64_t row_splits, int64_t rows_per_thread,
                                   int64_t staged_stages) {
  at::Tensor q_out;
  if (q_out_opt.has_value() && q_out_opt->defined()) q_out = *q_out_opt;
  else if (q.dim() == 3) q_out = empty_like_rows(q, q.size(1));
  drk_options o = make_options((pdl ? DRK_FLAG_PDL : 0u) |
                                   (strided_cache ? DRK_FLAG_STRIDED_CACHE : 0u) |
                                   path_flags(path),
                               rotary_dim, inv_freq, q.dim() == 3 ? q.size(2) : 0);
  TORCH_CHECK(row_splits >= 0 && row_splits <= 64, "row_splits must be in [0, 64], got ",
              row_splits);
  o.row_splits = static_cast<int32_t>(row_splits);
  o.rows_per_thread = static_cast<int32_t>(rows_per_thread);
  o.staged_stages = static_cast<int32_t>(staged_stages);
  const drk_tensor dq = describe(q), dk = describe(k), dv = describe(v),
                   dp = describe(positions), dc = describe(cos), ds = describe(sin),
                   dkc = describe(k_cache), dvc = describe(v_cache),
                   dri = describe(request_indices);
  drk_tensor dqo{};
  if (q_out.defined()) dqo = describe(q_out);
  raise_on_error(drk_fused_rope_kv_append_ex(&dq, &dk, &dv, &dp, &dc, &ds, &dkc, &dvc, &dri,
                                             q_out.defined() ? &dqo : nullptr, &o,
                                             status_for(q), stream_for(q)));
  return q_out;
}

at::Tensor paged_rope_kv_append(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor positions,
                                at::Tensor cos, at::Tensor sin, at::Tensor k_pages,
                                at::Tensor v_pages, at::Tensor block_table,
                                at::Tensor request_indices, int64_t rotary_dim, bool pdl,
                                const std::string& path) {
  at::Tensor q_out;
  if (q.dim() == 3) q_out = empty_like_rows(q, q.size(1));
  const drk_options o =
      make_options((pdl ? DRK_FLAG_PDL : 0u) | path_flags(path), rotary_dim, c10::nullopt);
  const drk_tensor dq = describe(q), dk = describe(k), dv = describe(v),
                   dp = describe(positions), dc = describe(cos), ds = describe(sin),
                   dkp = describe(k_pages), dvp = describe(v_pages), dbt = describe(block_table),
                   dri = describe(request_indices);
  drk_tensor dqo{};
  if (q_out.defined()) dqo = describe(q_out);
  raise_on_error(drk_paged_rope_kv_append(&dq, &dk, &dv, &dp, &dc, &ds, &dkp, &dvp, &dbt, &dri,
                                          q_out.defined() ? &dqo : nullptr, &o, status_for(q),
                                          stream_for(q)));
  return q_out;
}

std::tuple<at::Tensor, at::Tensor> rope_forward_ex(at::Tensor q, at::Tensor k,
                                                   at::Tensor positions, at::Tensor cos,
                                                   at::Tensor sin, int64_t rotary_dim,
                                                   bool pdl) {
  at::Tensor q_out, k_out;
  if (q.dim() == 3) q_out = empty_like_rows(q, q.size(1));
  if (k.dim() == 3) k_out = empty_like_rows(k, k.size(1));
  const drk_options o = make_options(pdl ? DRK_FLAG_PDL : 0u, rotary_dim, c10::nullopt);
  const drk_tensor dq = describe(q), dk = describe(k), dp = describe(positions),
                   dc = describe(cos), ds = describe(sin);
  drk_tensor dqo{}, dko{};
  if (q_out.defined()) dqo = describe(q_out);
  if (k_out.defined()) dko = describe(k_out);
  raise_on_error(drk_rope_forward(&dq, &dk, &dp, &dc, &ds, q_out.defined() ? &dqo : nullptr,
                                  k_out.defined() ? &dko : nullptr, &o, status_for(q),
                                  stream_for(q)));
  return {q_out, k_out};
}

void kv_append_ex(at::Tensor k_rot, at::Tensor v, at::Tensor positions,
                  at::Tensor request_indices, at::Tensor k_cache, at::Tensor v_cache, bool pdl,
                  bool strided_cache, int64_t k_position_limit) {
  drk_options o = make_options((pdl ? DRK_FLAG_PDL : 0u) |
                                   (strided_cache ? DRK_FLAG_STRIDED_CACHE : 0u),
                               0, c10::nullopt);
  o.k_position_limit = k_position_limit;
  const drk_tensor dk = describe(k_rot), dv = describe(v), dp = describe(positions),
                   dri = describe(request_indices), dkc = describe(k_cache),
                   dvc = describe(v_cache);
  raise_on_error(drk_kv_append(&dk, &dv, &dp, &dri, &dkc, &dvc, &o, status_for(k_rot),
                               stream_for(k_rot)));
}

// Fused append + decode attention. attn_out (and the workspace) come from the caching
// allocator unless given; q_out is written only when given.
at::Tensor fused_rope_kv_append_attention(
    at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor positions, at::Tensor cos,
    at::Tensor sin, at::Tensor k_cache, at::Tensor v_cache, at::Tensor request_indices,
    double scale, c10::optional<at::Tensor> q_out_opt, c10::optional<at::Tensor> attn_out_opt,
    int64_t chunk, int64_t heads_per_cta, int64_t rotary_dim, bool pdl, bool strided_cache,
    c10::optional<at::Tensor> workspace_opt, const std::string& path, bool workspace_zeroed) {
  TORCH_CHECK(q.dim() == 3 && k.dim() == 3 && k_cache.dim() == 4,
              "q must be [num_tokens, num_q_heads, head_dim], k [num_tokens, num_kv_heads, "
              "head_dim] and k_cache [batch, cache_alloc_len, num_kv_heads, head_dim]");
  at::Tensor attn_out;
  if (attn_out_opt.has_value() && attn_out_opt->defined()) attn_out = *attn_out_opt;
  else attn_out = empty_like_rows(q, q.size(1));
  drk_attention_options ao{};
  ao.scale = scale;
  ao.chunk = static_cast<int32_t>(chunk);
  ao.heads_per_cta = static_cast<int32_t>(heads_per_cta);
  ao.path = attention_path(path);
  const bool given = workspace_opt.has_value() && workspace_opt->defined();
  TORCH_CHECK(!workspace_zeroed || given, "workspace_zeroed=True needs a workspace");
  ao.flags = workspace_zeroed ? DRK_ATTN_WORKSPACE_ZEROED : 0;
  const int32_t device = q.is_cuda() ? q.get_device() : -1;
  const int64_t need = drk_attention_workspace_bytes(
      q.size(0), static_cast<int32_t>(q.size(1)), static_cast<int32_t>(k.size(1)),
      static_cast<int32_t>(q.size(2)), k_cache.size(1), dtype_code(q.scalar_type()), &ao,
      device < 0 ? 0 : device);
  if (need < 0) raise_on_error(static_cast<int>(need));
  at::Tensor workspace;
  if (workspace_opt.has_value() && workspace_opt->defined()) workspace = *workspace_opt;
  else workspace = at::empty({std::max<int64_t>(need, 16)}, q.options().dtype(at::kByte));
  TORCH_CHECK(workspace.is_contiguous(), "workspace must be contiguous");
  const drk_options o = make_options((pdl ? DRK_FLAG_PDL : 0u) |
                                         (strided_cache ? DRK_FLAG_STRIDED_CACHE : 0u),
                                     rotary_dim, c10::nullopt);
  const drk_tensor dq = describe(q), dk = describe(k), dv = describe(v),
                   dp = describe(positions), dc = describe(cos), ds = describe(sin),
                   dkc = describe(k_cache), dvc = describe(v_cache),
                   dri = describe(request_indices), dao = describe(attn_out);
  drk_tensor dqo{};
  const bool has_q_out = q_out_opt.has_value() && q_out_opt->defined();
  if (has_q_out) dqo = describe(*q_out_opt);
  raise_on_error(drk_fused_rope_kv_append_attention(
      &dq, &dk, &dv, &dp, &dc, &ds, &dkc, &dvc, &dri, has_q_out ? &dqo : nullptr, &dao, &ao,
      workspace.data_ptr(), static_cast<size_t>(workspace.numel() * workspace.element_size()),
      &o, status_for(q), stream_for(q)));
  return attn_out;
}

// Fused append + decode attention over a paged cache ([num_blocks, block_size, Hkv, D] pages
// and a block table); attn_out and the workspace come from the caching allocator unless given.
at::Tensor paged_rope_kv_append_attention(
    at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor positions, at::Tensor cos,
    at::Tensor sin, at::Tensor k_pages, at::Tensor v_pages, at::Tensor block_table,
    at::Tensor request_indices, double scale, c10::optional<at::Tensor> q_out_opt,
    c10::optional<at::Tensor> attn_out_opt, int64_t chunk, int64_t rotary_dim, bool pdl,
    c10::optional<at::Tensor> workspace_opt, bool workspace_zeroed) {
  TORCH_CHECK(q.dim() == 3 && k.dim() == 3 && k_pages.dim() == 4 && block_table.dim() == 2,
              "q must be [num_tokens, num_q_heads, head_dim], k [num_tokens, num_kv_heads, "
              "head_dim], k_pages [num_blocks, block_size, num_kv_heads, head_dim] and "
              "block_table [num_requests, max_blocks_per_request]");
  at::Tensor attn_out;
  if (attn_out_opt.has_value() && attn_out_opt->defined()) attn_out = *attn_out_opt;
  else attn_out = empty_like_rows(q, q.size(1));
  drk_attention_options ao{};
  ao.scale = scale;
  ao.chunk = static_cast<int32_t>(chunk);
  ao.path = DRK_ATTN_PATH_TENSOR_CORES;
  const bool given = workspace_opt.has_value() && workspace_opt->defined();
  TORCH_CHECK(!workspace_zeroed || given, "workspace_zeroed=True needs a workspace");
  ao.flags = workspace_zeroed ? DRK_ATTN_WORKSPACE_ZEROED : 0;
  const int32_t device = q.is_cuda() ? q.get_device() : -1;
  const int64_t need = drk_attention_workspace_bytes(
      q.size(0), static_cast<int32_t>(q.size(1)), static_cast<int32_t>(k.size(1)),
      static_cast<int32_t>(q.size(2)), block_table.size(1) * k_pages.size(1),
      dtype_code(q.scalar_type()), &ao, device < 0 ? 0 : device);
  if (need < 0) raise_on_error(static_cast<int>(need));
  at::Tensor workspace;
  if (workspace_opt.has_value() && workspace_opt->defined()) workspace = *workspace_opt;
  else workspace = at::empty({std::max<int64_t>(need, 16)}, q.options().dtype(at::kByte));
  TORCH_CHECK(workspace.is_contiguous(), "workspace must be contiguous");
  const drk_options o = make_options(pdl ? DRK_FLAG_PDL : 0u, rotary_dim, c10::nullopt);
  const drk_tensor dq = describe(q), dk = describe(k), dv = describe(v),
                   dp = describe(positions), dc = describe(cos), ds = describe(sin),
                   dkp = describe(k_pages), dvp = describe(v_pages), dbt = describe(block_table),
                   dri = describe(request_indices), dao = describe(attn_out);
  drk_tensor dqo{};
  const bool has_q_out = q_out_opt.has_value() && q_out_opt->defined();
  if (has_q_out) dqo = describe(*q_out_opt);
  raise_on_error(drk_paged_rope_kv_append_attention(
      &dq, &dk, &dv, &dp, &dc, &ds, &dkp, &dvp, &dbt, &dri, has_q_out ? &dqo : nullptr, &dao,
      &ao, workspace.data_ptr(),
      static_cast<size_t>(workspace.numel() * workspace.element_size()), &o, status_for(q),
      stream_for(q)));
  return attn_out;
}

int64_t attention_workspace_bytes(int64_t num_tokens, int64_t num_q_heads, int64_t num_kv_heads,
                                  int64_t head_dim, int64_t cache_alloc_len,
                                  at::ScalarType dtype, int64_t chunk, int64_t heads_per_cta,
                                  int64_t device, const std::string& path) {
  drk_attention_options ao{};
  ao.chunk = static_cast<int32_t>(chunk);
  ao.heads_per_cta = static_cast<int32_t>(heads_per_cta);
  ao.path = attention_path(path);
  const int64_t need = drk_attention_workspace_bytes(
      num_tokens, static_cast<int32_t>(num_q_heads), static_cast<int32_t>(num_kv_heads),
      static_cast<int32_t>(head_dim), cache_alloc_len, dtype_code(dtype), &ao,
      static_cast<int32_t>(device));
  if (need < 0) raise_on_error(static_cast<int>(need));
  return need;
}

// Reads (and by default clears) the device's status word. Synchronises the current stream:
// call it outside timed regions.
int64_t read_status(int64_t device, bool clear) {
  uint32_t* word = status_word(static_cast<int>(device));
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(static_cast<c10::DeviceIndex>(device));
  uint32_t host = 0;
  cudaError_t err = cudaMemcpyAsync(&host, word, sizeof(uint32_t), cudaMemcpyDeviceToHost, stream);
  if (err == cudaSuccess) err = cudaStreamSynchronize(stream);
  if (err == cudaSuccess && clear) {
    err = cudaMemsetAsync(word, 0, sizeof(uint32_t), stream);
    if (err == cudaSuccess) err = cudaStreamSynchronize(stream);
  }
  TORCH_CHECK(err == cudaSuccess, "reading the status word failed: ", cudaGetErrorString(err));
  return static_cast<int64_t>(host);
}

int64_t status_address(int64_t device) {
  return static_cast<int64_t>(reinterpret_cast<uintptr_t>(status_word(static_cast<int>(device))));
}

std::string status_string(int64_t status) {
  return drk_status_string(static_cast<uint32_t>(status));
}

void advance_positions(at::Tensor positions, int64_t delta, bool pdl) {
  const drk_tensor d = describe(positions);
  raise_on_error(drk_advance_positions(&d, delta, pdl ? DRK_FLAG_PDL : 0u, stream_for(positions)));
}

void launch_empty(int64_t count, bool pdl) {
  const int device = c10::cuda::current_device();
  raise_on_error(drk_launch_empty(static_cast<int>(count), pdl ? 1 : 0,
                                  at::cuda::getCurrentCUDAStream(device).stream()));
}

// The dependent-copy floor probe over two device tensors, whose sizes bound every launch.
void launch_copy_probe(at::Tensor src, at::Tensor dst, int64_t bytes, int64_t stride_bytes,
                       int64_t count, int64_t threads, bool pdl, bool prefetch) {
  TORCH_CHECK(src.is_cuda() && dst.is_cuda() && src.get_device() == dst.get_device(),
              "src and dst must be CUDA tensors on one device");
  TORCH_CHECK(src.is_contiguous() && dst.is_contiguous(), "src and dst must be contiguous");
  const int64_t need = count > 0 ? (count - 1) * stride_bytes + bytes : 0;
  TORCH_CHECK(src.numel() * src.element_size() >= need &&
                  dst.numel() * dst.element_size() >= need,
              "src and dst must hold (count - 1) * stride_bytes + bytes = ", need, " bytes");
  c10::cuda::CUDAGuard guard(src.device());
  raise_on_error(drk_launch_copy_probe(src.data_ptr(), dst.data_ptr(), bytes, stride_bytes,
                                       static_cast<int>(count), static_cast<int>(threads),
                                       pdl ? 1 : 0, prefetch ? 1 : 0, stream_for(src)));
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("smoke_fill", &smoke_fill, py::arg("tensor"), py::arg("value"),
        "Fill a contiguous CUDA tensor in place; exercises launch + dtype dispatch.");
  m.def("build_info", &build_info, "Compile-time and runtime facts about this binary.");
  m.def("rope_forward", &rope_forward, py::arg("q"), py::arg("k"), py::arg("positions"),
        py::arg("cos"), py::arg("sin"),
        "Split-half RoPE over strided Q and K in one launch; returns (q_rot, k_rot).");
  m.def("kv_append", &kv_append, py::arg("k_rot"), py::arg("v"), py::arg("positions"),
        py::arg("request_indices"), py::arg("k_cache"), py::arg("v_cache"),
        "Scatter rotated K and raw V into a contiguous token-major cache, in place.");
  m.def("separate_rope_kv_append", &separate_rope_kv_append, py::arg("q"), py::arg("k"),
        py::arg("v"), py::arg("positions"), py::arg("cos"), py::arg("sin"), py::arg("k_cache"),
        py::arg("v_cache"), py::arg("request_indices"),
        "rope_forward then kv_append (k_rot materialised); returns q_rot.");
  m.def("fused_rope_kv_append", &fused_rope_kv_append, py::arg("q"), py::arg("k"),
        py::arg("v"), py::arg("positions"), py::arg("cos"), py::arg("sin"), py::arg("k_cache"),
        py::arg("v_cache"), py::arg("request_indices"),
        "Rotate Q and K and append K/V to the cache in one launch; returns q_rot.");

  m.def("fused_rope_kv_append_ex", &fused_rope_kv_append_ex, py::arg("q"), py::arg("k"),
        py::arg("v"), py::arg("positions"), py::arg("cos"), py::arg("sin"), py::arg("k_cache"),
        py::arg("v_cache"), py::arg("request_indices"), py::arg("rotary_dim") = 0,
        py::arg("pdl") = false, py::arg("strided_cache") = false,
        py::arg("inv_freq") = py::none(), py::arg("q_out") = py::none(),
        py::arg("path") = "auto", py::arg("row_splits") = 0, py::arg("rows_per_thread") = 0,
        py::arg("staged_stages") = 0,
        "fused_rope_kv_append with partial rotary, PDL, strided caches, in-register trig.");
  m.def("paged_rope_kv_append", &paged_rope_kv_append, py::arg("q"), py::arg("k"),
        py::arg("v"), py::arg("positions"), py::arg("cos"), py::arg("sin"), py::arg("k_pages"),
        py::arg("v_pages"), py::arg("block_table"), py::arg("request_indices"),
        py::arg("rotary_dim") = 0, py::arg("pdl") = false, py::arg("path") = "auto",
        "Fused RoPE + append into a paged (block-table) KV cache; returns q_rot.");
  m.def("rope_forward_ex", &rope_forward_ex, py::arg("q"), py::arg("k"), py::arg("positions"),
        py::arg("cos"), py::arg("sin"), py::arg("rotary_dim") = 0, py::arg("pdl") = false);
  m.def("kv_append_ex", &kv_append_ex, py::arg("k_rot"), py::arg("v"), py::arg("positions"),
        py::arg("request_indices"), py::arg("k_cache"), py::arg("v_cache"),
        py::arg("pdl") = false, py::arg("strided_cache") = false,
        py::arg("k_position_limit") = 0);
  m.def("fused_rope_kv_append_attention", &fused_rope_kv_append_attention, py::arg("q"),
        py::arg("k"), py::arg("v"), py::arg("positions"), py::arg("cos"), py::arg("sin"),
        py::arg("k_cache"), py::arg("v_cache"), py::arg("request_indices"),
        py::arg("scale") = 0.0, py::arg("q_out") = py::none(), py::arg("attn_out") = py::none(),
        py::arg("chunk") = 0, py::arg("heads_per_cta") = 0, py::arg("rotary_dim") = 0,
        py::arg("pdl") = false, py::arg("strided_cache") = false,
        py::arg("workspace") = py::none(), py::arg("path") = "auto",
        py::arg("workspace_zeroed") = false,
        "Fused RoPE + KV append + decode attention over positions [0, pos]; returns attn_out.");
  m.def("paged_rope_kv_append_attention", &paged_rope_kv_append_attention, py::arg("q"),
        py::arg("k"), py::arg("v"), py::arg("positions"), py::arg("cos"), py::arg("sin"),
        py::arg("k_pages"), py::arg("v_pages"), py::arg("block_table"),
        py::arg("request_indices"), py::arg("scale") = 0.0, py::arg("q_out") = py::none(),
        py::arg("attn_out") = py::none(), py::arg("chunk") = 0, py::arg("rotary_dim") = 0,
        py::arg("pdl") = false, py::arg("workspace") = py::none(),
        py::arg("workspace_zeroed") = false,
        "Fused RoPE + append + decode attention over a paged (block-table) KV cache.");
  m.def("attention_workspace_bytes", &attention_workspace_bytes, py::arg("num_tokens"),
        py::arg("num_q_heads"), py::arg("num_kv_heads"), py::arg("head_dim"),
        py::arg("cache_alloc_len"), py::arg("dtype"), py::arg("chunk") = 0,
        py::arg("heads_per_cta") = 0, py::arg("device") = 0, py::arg("path") = "auto");
  m.def("read_status", &read_status, py::arg("device"), py::arg("clear") = true);
  m.def("status_address", &status_address, py::arg("device"));
  m.def("status_string", &status_string, py::arg("status"));
  m.def("launch_empty", &launch_empty, py::arg("count"), py::arg("pdl") = false);
  m.def("launch_copy_probe", &launch_copy_probe, py::arg("src"), py::arg("dst"),
        py::arg("bytes"), py::arg("stride_bytes"), py::arg("count"), py::arg("threads"),
        py::arg("pdl") = true, py::arg("prefetch") = true,
        "Chained dependent copies with one decode layer's memory pattern (launch floor).");
  m.def("advance_positions", &advance_positions, py::arg("positions"), py::arg("delta") = 1,
        py::arg("pdl") = false, "positions += delta on the device (a decode loop's step).");
}
