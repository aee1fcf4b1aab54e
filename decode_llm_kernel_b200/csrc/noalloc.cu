// drk_separate_rope_kv_append_noalloc: the separate RoPE-then-append op with its k_rot
// intermediate in a fixed device array instead of caller- or allocator-provided memory.
//
// Who needs it: callers that cannot call cudaMalloc (or any allocating routine) at the point
// where they launch this op -- for example code recorded under a global-mode stream capture,
// where allocation calls are prohibited; serving runtimes that have handed every free byte of
// HBM to their KV-cache pool and allocate nothing afterwards; and foreign-language hosts that
// reach this library through the C ABI without owning an allocator for the device. They still
// pass every input and output; only the intermediate lives here.
//
// Limits and behaviour:
//  * Every argument goes through the same host checks as drk_rope_forward and drk_kv_append
//    first (same messages). Only then is the intermediate k_rot ([T, Hkv, D] of k's dtype)
//    measured against kScratchBytes (8 MiB); larger calls are rejected with DRK_ERR_INVALID
//    before anything is launched.
//  * The array is a file-scope static __device__ object: every GPU that loads this library
//    holds its 8 MiB until the process exits.
//  * The first call on a device looks up the array's device address (cudaGetSymbolAddress,
//    with that device current) and caches it for the life of the process; make that first
//    call before any stream capture. The cached address belongs to the device's primary
//    context: do not use this entry point after cudaDeviceReset (or any teardown of that
//    context) in the same process.
//  * All calls share the one array, and it keeps the last call's contents. Nothing in it needs
//    to start at zero: the append step writes a K slot only from a k_rot row this call's rope
//    step wrote (rows of tokens past the cos/sin table are skipped in both steps, as in the
//    fused op). Calls that overlap on the GPU -- on different streams, or from different host
//    threads -- race on the array.
//  * No cudaMalloc, cudaFree or other allocating routine is called.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "decode_rope.h"

namespace {

constexpr size_t kScratchBytes = size_t(8) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

std::mutex g_scratch_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

int64_t elem_bytes(int32_t dt) {
  switch (dt) {
    case DRK_F32: return 4;
    case DRK_F16: case DRK_BF16: return 2;
    case DRK_F64: return 8;
    default: return 0;
  }
}

// Device address of the scratch array on `device`, looked up once per device with that
// device current (the previous device is restored).
cudaError_t scratch_on(int device, void** out) {
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_ptr[device] == nullptr) {
    int prev = -1;
    cudaError_t err = cudaGetDevice(&prev);
    if (err != cudaSuccess) return err;
    if (prev != device && (err = cudaSetDevice(device)) != cudaSuccess) return err;
    void* ptr = nullptr;
    err = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (prev != device) cudaSetDevice(prev);
    if (err != cudaSuccess) return err;
    g_scratch_ptr[device] = ptr;
  }
  *out = g_scratch_ptr[device];
  return cudaSuccess;
}

// The [T, Hkv, D] contiguous k_rot descriptor over `data` for k's shape and dtype.
drk_tensor k_rot_like(const drk_tensor* k, void* data) {
  drk_tensor t{};
  t.data = data;
  t.dtype = k->dtype;
  t.ndim = 3;
  t.device = k->device;
  t.sizes[0] = k->sizes[0];
  t.sizes[1] = k->sizes[1];
  t.sizes[2] = k->sizes[2];
  t.strides[2] = 1;
  t.strides[1] = k->sizes[2];
  t.strides[0] = k->sizes[1] * k->sizes[2];
  return t;
}

}  // namespace

namespace drk {
void set_last_error(const std::string& message);  // abi.cu: the text drk_last_error() returns
int validate_rope_forward(const drk_tensor* q, const drk_tensor* k, const drk_tensor* positions,
                          const drk_tensor* cos, const drk_tensor* sin, const drk_tensor* q_out,
                          const drk_tensor* k_out);
int validate_kv_append(const drk_tensor* k_rot, const drk_tensor* v, const drk_tensor* positions,
                       const drk_tensor* request_indices, const drk_tensor* k_cache,
                       const drk_tensor* v_cache, const drk_options* opts);
}  // namespace drk

extern "C" {

int drk_separate_rope_kv_append_noalloc(const drk_tensor* q, const drk_tensor* k,
                                        const drk_tensor* v, const drk_tensor* positions,
                                        const drk_tensor* cos, const drk_tensor* sin,
                                        const drk_tensor* k_cache, const drk_tensor* v_cache,
                                        const drk_tensor* request_indices,
                                        const drk_tensor* q_out, uint32_t* status,
                                        drk_stream_t stream) {
  // 1. The regular checks, in the order the two steps make them, with k_rot described over a
  //    placeholder (no check reads its address).
  if (k == nullptr || k->ndim != 3) {
    return drk::validate_rope_forward(q, k, positions, cos, sin, q_out, nullptr);
  }
  const drk_tensor probe = k_rot_like(k, nullptr);
  int rc = drk::validate_rope_forward(q, k, positions, cos, sin, q_out, &probe);
  if (rc != DRK_OK) return rc;
  drk_options opts{};
  opts.k_position_limit = cos->sizes[0];   // validated: cos is [P, D] with P >= 0
  rc = drk::validate_kv_append(&probe, v, positions, request_indices, k_cache, v_cache, &opts);
  if (rc != DRK_OK) return rc;

  // 2. The intermediate must fit the array. The sizes are validated non-negative; the product
  //    is formed with overflow checks all the same.
  int64_t need = elem_bytes(k->dtype);
  for (int i = 0; i < 3; ++i) {
    if (__builtin_mul_overflow(need, k->sizes[i], &need)) {
      need = -1;
      break;
    }
  }
  if (need < 0 || need > static_cast<int64_t>(kScratchBytes)) {
    drk::set_last_error(
        "k_rot needs " + (need < 0 ? std::string("more than 2^63") : std::to_string(need)) +
        " bytes but the no-alloc scratch holds at most " + std::to_string(kScratchBytes) +
        " bytes (8 MiB); use drk_rope_forward + drk_kv_append with a caller-allocated k_rot");
    return DRK_ERR_INVALID;
  }
  if (q->device >= kMaxDevices) {
    drk::set_last_error("the no-alloc entry point supports device ordinals below " +
                        std::to_string(kMaxDevices));
    return DRK_ERR_INVALID;
  }

  // 3. The array's address on this device, then the two launches.
  void* scratch = nullptr;
  const cudaError_t err = scratch_on(q->device, &scratch);
  if (err != cudaSuccess) {
    drk::set_last_error(std::string("cudaGetSymbolAddress of the no-alloc scratch failed: ") +
                        cudaGetErrorString(err));
    return DRK_ERR_CUDA;
  }
  const drk_tensor k_rot = k_rot_like(k, scratch);
  rc = drk_rope_forward(q, k, positions, cos, sin, q_out, &k_rot, nullptr, status, stream);
  if (rc != DRK_OK) return rc;
  return drk_kv_append(&k_rot, v, positions, request_indices, k_cache, v_cache, &opts, status,
                       stream);
}

}  // extern "C"
