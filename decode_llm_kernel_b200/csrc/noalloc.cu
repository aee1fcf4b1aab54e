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
//  * The intermediate k_rot ([T, Hkv, D] of k's dtype) must fit kScratchBytes (8 MiB); larger
//    calls are rejected with DRK_ERR_INVALID before anything is launched.
//  * The array is a file-scope static __device__ object: every GPU that loads this library
//    holds its 8 MiB until the process exits.
//  * The first call on a device looks up the array's device address (cudaGetSymbolAddress,
//    with that device current) and caches it; make that first call before any stream capture.
//  * All calls share the one array, and it keeps the last call's contents. Nothing in it needs
//    to start at zero (each call fully writes the k_rot rows it later reads). Calls that
//    overlap on the GPU -- on different streams, or from different host threads -- race on it.
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

// Device address of the scratch array on `device`, looked up once per device.
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

}  // namespace

namespace drk {
void set_last_error(const std::string& message);  // abi.cu: the text drk_last_error() returns
}

extern "C" {

int drk_separate_rope_kv_append_noalloc(const drk_tensor* q, const drk_tensor* k,
                                        const drk_tensor* v, const drk_tensor* positions,
                                        const drk_tensor* cos, const drk_tensor* sin,
                                        const drk_tensor* k_cache, const drk_tensor* v_cache,
                                        const drk_tensor* request_indices,
                                        const drk_tensor* q_out, uint32_t* status,
                                        drk_stream_t stream) {
  if (q == nullptr || k == nullptr || q->device < 0 || k->ndim != 3) {
    // Not a device q or not a [T, Hkv, D] k: the regular checks reject these with the
    // reference's messages before anything is launched.
    return drk_rope_forward(q, k, positions, cos, sin, q_out, nullptr, nullptr, status, stream);
  }
  if (q->device >= kMaxDevices) {
    drk::set_last_error("the no-alloc entry point supports device ordinals below " +
                        std::to_string(kMaxDevices));
    return DRK_ERR_INVALID;
  }
  const int64_t es = elem_bytes(k->dtype);
  const int64_t need = k->sizes[0] * k->sizes[1] * k->sizes[2] * (es ? es : 1);
  if (need > static_cast<int64_t>(kScratchBytes)) {
    drk::set_last_error("k_rot needs " + std::to_string(need) +
                        " bytes but the no-alloc scratch holds at most " +
                        std::to_string(kScratchBytes) + " bytes (8 MiB); use "
                        "drk_rope_forward + drk_kv_append with a caller-allocated k_rot");
    return DRK_ERR_INVALID;
  }
  void* scratch = nullptr;
  const cudaError_t err = scratch_on(q->device, &scratch);
  if (err != cudaSuccess) {
    drk::set_last_error(std::string("cudaGetSymbolAddress of the no-alloc scratch failed: ") +
                        cudaGetErrorString(err));
    return DRK_ERR_CUDA;
  }
  drk_tensor k_rot{};
  k_rot.data = scratch;
  k_rot.dtype = k->dtype;
  k_rot.ndim = 3;
  k_rot.device = q->device;
  k_rot.sizes[0] = k->sizes[0];
  k_rot.sizes[1] = k->sizes[1];
  k_rot.sizes[2] = k->sizes[2];
  k_rot.strides[2] = 1;
  k_rot.strides[1] = k->sizes[2];
  k_rot.strides[0] = k->sizes[1] * k->sizes[2];
  int rc = drk_rope_forward(q, k, positions, cos, sin, q_out, &k_rot, nullptr, status, stream);
  if (rc != DRK_OK) return rc;
  return drk_kv_append(&k_rot, v, positions, request_indices, k_cache, v_cache, nullptr, status,
                       stream);
}

}  // extern "C"
