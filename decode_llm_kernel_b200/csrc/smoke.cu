// Smoke fill, build-info probe, and the two kernels that measure launch floors: an empty kernel
// and a dependent copy with the memory pattern of one decode-step layer.
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

// The dependent-copy floor: thread i copies the 16-byte vectors i and i + half from src to
// dst with a streaming load and a streaming store, after griddepcontrol.wait. With `prefetch`
// each thread first pulls both source lines toward L2 while it waits, as the fused kernel
// does with its q/k/v rows. It is one layer of the fused op with the arithmetic, the index
// and table loads and the slot computation taken out: the cost of a chained launch that must
// read after the previous launch and write before the next.
__global__ void copy_probe_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst,
                                  int64_t half, int prefetch) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (prefetch && i < half) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(src + i));
    asm volatile("prefetch.global.L2 [%0];" ::"l"(src + i + half));
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (i < half) {
    const uint4 a = __ldcs(src + i);
    const uint4 b = __ldcs(src + i + half);
    __stcs(dst + i, a);
    __stcs(dst + i + half, b);
  }
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

cudaError_t launch_copy_probe(const void* src, void* dst, int64_t vectors, int64_t stride_vectors,
                              int count, int threads, bool pdl, bool prefetch,
                              cudaStream_t stream) {
  const int64_t half = vectors / 2;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>((half + threads - 1) / threads), 1, 1);
  cfg.blockDim = dim3(threads, 1, 1);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  if (pdl) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  for (int i = 0; i < count; ++i) {
    const uint4* s = static_cast<const uint4*>(src) + i * stride_vectors;
    uint4* d = static_cast<uint4*>(dst) + i * stride_vectors;
    cudaError_t err = cudaLaunchKernelEx(&cfg, copy_probe_kernel, s, d, half,
                                         prefetch ? 1 : 0);
    if (err != cudaSuccess) return err;
  }
  return cudaSuccess;
}

}  // namespace drk
