// Instantiation and launch of the RoPE + KV-append kernels (rope_kv_kernels.cuh).
//
// The host layer (abi.cpp) has already validated the arguments and picked the widest vector
// width VB the alignment allows; this file maps (dtype, index type, VB, mode, cache kind) to a
// kernel instantiation and launches it with cudaLaunchKernelEx, adding the programmatic
// stream serialization attribute when the caller asked for PDL.
#include "rope_kv_kernels.cuh"
#include "rope_kv_launch.h"

namespace drk {
namespace {

template <typename E, typename Idx, int VB, Mode M, Cache C>
cudaError_t launch_one(const KernelParams& p, const LaunchShape& shape, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(shape.grid, 1, 1);
  cfg.blockDim = dim3(shape.threads, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  if (shape.pdl) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, rope_kv_kernel<E, Idx, VB, M, C>, p);
}

template <typename E, typename Idx, int VB>
cudaError_t launch_mode(const KernelParams& p, int mode, int cache, const LaunchShape& shape,
                        cudaStream_t stream) {
  switch (mode) {
    case kModeFused:
      if (cache == kCachePaged)
        return launch_one<E, Idx, VB, Mode::kFused, Cache::kPaged>(p, shape, stream);
      return launch_one<E, Idx, VB, Mode::kFused, Cache::kStrided>(p, shape, stream);
    case kModeRope:
      return launch_one<E, Idx, VB, Mode::kRope, Cache::kStrided>(p, shape, stream);
    case kModeAppend:
      return launch_one<E, Idx, VB, Mode::kAppend, Cache::kStrided>(p, shape, stream);
    default:
      return cudaErrorInvalidValue;
  }
}

template <typename E, typename Idx>
cudaError_t launch_vb(const KernelParams& p, int vb, int mode, int cache,
                      const LaunchShape& shape, cudaStream_t stream) {
  constexpr int es = static_cast<int>(sizeof(typename E::raw));
  switch (vb) {
    case 16: return launch_mode<E, Idx, 16>(p, mode, cache, shape, stream);
    case 8: return launch_mode<E, Idx, 8>(p, mode, cache, shape, stream);
    case 4:
      if constexpr (es <= 4) return launch_mode<E, Idx, 4>(p, mode, cache, shape, stream);
      break;
    case 2:
      if constexpr (es <= 2) return launch_mode<E, Idx, 2>(p, mode, cache, shape, stream);
      break;
    default:
      break;
  }
  return cudaErrorInvalidValue;
}

template <typename E>
cudaError_t launch_idx(const KernelParams& p, int index_bits, int vb, int mode, int cache,
                       const LaunchShape& shape, cudaStream_t stream) {
  if (index_bits == 32) return launch_vb<E, int>(p, vb, mode, cache, shape, stream);
  return launch_vb<E, long long>(p, vb, mode, cache, shape, stream);
}

}  // namespace

cudaError_t launch_rope_kv(const KernelParams& p, int elem_code, int index_bits, int vb,
                           int mode, int cache, const LaunchShape& shape, cudaStream_t stream) {
  switch (elem_code) {
    case kElemF32: return launch_idx<F32>(p, index_bits, vb, mode, cache, shape, stream);
    case kElemF16: return launch_idx<F16>(p, index_bits, vb, mode, cache, shape, stream);
    case kElemBF16: return launch_idx<BF16>(p, index_bits, vb, mode, cache, shape, stream);
    case kElemF64: return launch_idx<F64>(p, index_bits, vb, mode, cache, shape, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace drk
