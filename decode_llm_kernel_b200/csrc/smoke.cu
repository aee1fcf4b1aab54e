// Smoke fill, build-info probe and the empty kernel used to measure the launch floor.
//
// smoke_fill keeps the reference's contract (csrc/smoke.cu:17-24,42-60): fill a contiguous
// tensor with one value converted once on the host, so an fp64 tensor keeps full precision.
// The arch probe reports the __CUDA_ARCH__ of the code that actually ran (csrc/smoke.cu:27-33).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "rope_kv_launch.h"

namespace drk {
namespace {

template <typename T>
__global__ void smoke_fill_kernel(T* __restrict__ out, int64_t numel, T value) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < numel;
       i += stride) {
    out[i] = value;
  }
}

__device__ int g_arch_probe;

__global__ void arch_probe_kernel() {
#ifdef __CUDA_ARCH__
  g_arch_probe = __CUDA_ARCH__;
#endif
}

__global__ void empty_kernel() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

constexpr int kFillThreads = 256;

template <typename T>
cudaError_t fill(void* data, int64_t numel, T value, cudaStream_t stream) {
  int device = 0, sms = 148;
  cudaGetDevice(&device);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  const int64_t want = (numel + kFillThreads - 1) / kFillThreads;
  const int blocks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, sms * 16)));
  smoke_fill_kernel<T><<<blocks, kFillThreads, 0, stream>>>(static_cast<T*>(data), numel, value);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_smoke_fill(void* data, int elem_code, int64_t numel, double value,
                              cudaStream_t stream) {
  switch (elem_code) {
    case kElemF64: return fill<double>(data, numel, value, stream);
    case kElemF32: return fill<float>(data, numel, static_cast<float>(value), stream);
    case kElemF16: {
      const __half h = __float2half_rn(static_cast<float>(value));
      return fill<unsigned short>(data, numel, __half_as_ushort(h), stream);
    }
    case kElemBF16: {
      const __nv_bfloat16 b = __float2bfloat16_rn(static_cast<float>(value));
      return fill<unsigned short>(data, numel, __bfloat16_as_ushort(b), stream);
    }
    default:
      return cudaErrorInvalidValue;
  }
}

cudaError_t run_arch_probe(int* arch_out, cudaStream_t stream) {
  arch_probe_kernel<<<1, 1, 0, stream>>>();
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return err;
  err = cudaMemcpyFromSymbolAsync(arch_out, g_arch_probe, sizeof(int), 0,
                                  cudaMemcpyDeviceToHost, stream);
  if (err != cudaSuccess) return err;
  return cudaStreamSynchronize(stream);
}

cudaError_t launch_empty(int count, bool pdl, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1, 1, 1);
  cfg.blockDim = dim3(32, 1, 1);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  if (pdl) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  for (int i = 0; i < count; ++i) {
    cudaError_t err = cudaLaunchKernelEx(&cfg, empty_kernel);
    if (err != cudaSuccess) return err;
  }
  return cudaSuccess;
}

}  // namespace drk
