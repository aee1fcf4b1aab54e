// Instantiation and launch of the fused RoPE + KV append + decode attention kernel
// (rope_kv_attention.cuh). The host layer (abi.cu) has validated the call and picked the lanes
// per row (LPR) and query heads per CTA (HPB); this file maps them to an instantiation.
#include "rope_kv_attention.cuh"
#include "rope_kv_launch.h"

namespace drk {
namespace {

template <typename E, typename Idx, int LPR, int HPB>
cudaError_t attention_one(const KernelParams& p, const AttentionParams& a,
                          const AttentionShape& s, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(s.grid_x, s.grid_y, s.grid_z);
  cfg.blockDim = dim3(kAttnThreads, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  if (s.pdl) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, rope_kv_attention_kernel<E, Idx, LPR, HPB>, p, a);
}

template <typename E, typename Idx, int LPR>
cudaError_t attention_hpb(const KernelParams& p, const AttentionParams& a,
                          const AttentionShape& s, cudaStream_t stream) {
  switch (s.hpb) {
    case 1: return attention_one<E, Idx, LPR, 1>(p, a, s, stream);
    case 2: return attention_one<E, Idx, LPR, 2>(p, a, s, stream);
    case 4: return attention_one<E, Idx, LPR, 4>(p, a, s, stream);
    case 8: return attention_one<E, Idx, LPR, 8>(p, a, s, stream);
    default: return cudaErrorInvalidValue;
  }
}

template <typename E, typename Idx>
cudaError_t attention_lpr(const KernelParams& p, const AttentionParams& a,
                          const AttentionShape& s, cudaStream_t stream) {
  switch (s.lpr) {
    case 8: return attention_hpb<E, Idx, 8>(p, a, s, stream);
    case 16: return attention_hpb<E, Idx, 16>(p, a, s, stream);
    case 32: return attention_hpb<E, Idx, 32>(p, a, s, stream);
    default: return cudaErrorInvalidValue;
  }
}

template <typename E>
cudaError_t attention_idx(const KernelParams& p, const AttentionParams& a, int index_bits,
                          const AttentionShape& s, cudaStream_t stream) {
  if (index_bits == 32) return attention_lpr<E, int>(p, a, s, stream);
  return attention_lpr<E, long long>(p, a, s, stream);
}

}  // namespace

cudaError_t launch_rope_kv_attention(const KernelParams& p, const AttentionParams& a,
                                     int elem_code, int index_bits, const AttentionShape& s,
                                     cudaStream_t stream) {
  switch (elem_code) {
    case kElemF32: return attention_idx<F32>(p, a, index_bits, s, stream);
    case kElemF16: return attention_idx<F16>(p, a, index_bits, s, stream);
    case kElemBF16: return attention_idx<BF16>(p, a, index_bits, s, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace drk
