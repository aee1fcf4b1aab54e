// Advances a decode loop's positions on the device: positions[t] += delta for every token.
//
// A captured decode step that ends with this kernel can be replayed step after step with no
// host-side position copy between replays (the reference's graph runner copies new positions
// into the graph's static buffer before every replay, benchmarks/impls.py:144-150). Launched
// as a programmatic dependent of the step's last layer it still writes only after
// griddepcontrol.wait, i.e. after every layer of the step has read the positions.
#include <cuda_runtime.h>

#include <algorithm>

#include "rope_kv_launch.h"

namespace drk {
namespace {

template <typename Idx>
__global__ void advance_positions_kernel(Idx* __restrict__ positions, int64_t n, int64_t delta) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += stride) {
    positions[i] = static_cast<Idx>(positions[i] + delta);
  }
}

template <typename Idx>
cudaError_t launch(void* data, int64_t n, int64_t delta, bool pdl, cudaStream_t stream) {
  constexpr int kThreads = 256;
  const int blocks = static_cast<int>(std::max<int64_t>(
      1, std::min<int64_t>((n + kThreads - 1) / kThreads, 1024)));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(blocks, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  if (pdl) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, advance_positions_kernel<Idx>, static_cast<Idx*>(data), n,
                            delta);
}

}  // namespace

cudaError_t launch_advance_positions(void* data, int index_bits, int64_t n, int64_t delta,
                                     bool pdl, cudaStream_t stream) {
  if (index_bits == 32) return launch<int>(data, n, delta, pdl, stream);
  return launch<long long>(data, n, delta, pdl, stream);
}

}  // namespace drk
