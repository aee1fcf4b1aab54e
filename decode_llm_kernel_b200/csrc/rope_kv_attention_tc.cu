// Host side of the tensor-core attention kernel (rope_kv_attention_tc.cuh): the TMA tensor
// maps of the two caches and the persistent launch.
//
// The caches are described to TMA as 4-D tensors (dims, kv heads, positions, batch rows) with
// their own element strides, so token-major and head-major caches take the same kernel; a box
// is [1 row][128 positions][1 head][64 dims] with the 128-byte swizzle the tcgen05 shared-memory
// descriptors expect. cuTensorMapEncodeTiled is reached through the runtime's driver entry
// point, so the library does not link the driver API.
#include <cudaTypedefs.h>

#include <map>
#include <mutex>

#include "rope_kv_attention_tc.cuh"
#include "rope_kv_launch.h"

namespace drk {
namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// The cache as a 4-D tensor (dims, kv heads, positions, rows): rows are requests for a
// contiguous cache and pages for a paged one (positions then run within a page).
cudaError_t encode_cache_map(CUtensorMap* map, const void* base, bool bf16,
                             const KernelParams& p, int box_rows) {
  auto fn = encode_fn();
  if (fn == nullptr) return cudaErrorNotSupported;
  const CUtensorMapDataType type =
      bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const cuuint32_t estride[5] = {1, 1, 1, 1, 1};
  CUresult r;
  if (p.block_table != nullptr && p.D == 64) {
    // Page pool [num_blocks, block_size, Hkv, 64] over its own strides as {64 dims, Hkv,
    // block_size, pages}: a box holds a page slice's 128-byte rows of one head, which land as
    // the tile's 1024-byte swizzle atoms [row group][8 rows][128 bytes].
    const cuuint64_t dims[4] = {64, static_cast<cuuint64_t>(p.Hkv),
                                static_cast<cuuint64_t>(p.block_size),
                                static_cast<cuuint64_t>(p.num_blocks)};
    const cuuint64_t strides[3] = {static_cast<cuuint64_t>(p.c_hs) * 2,
                                   static_cast<cuuint64_t>(p.c_ss) * 2,
                                   static_cast<cuuint64_t>(p.c_bs) * 2};
    const cuuint32_t box[4] = {64, 1, static_cast<cuuint32_t>(box_rows), 1};
    r = fn(map, type, 4, const_cast<void*>(base), dims, strides, box, estride,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else if (p.block_table != nullptr) {
    // Page pool [num_blocks, block_size, Hkv, 128], contiguous, as
    // {64 dims, 8 rows, 2 * Hkv half rows, block_size / 8 row groups, pages}: one box holds
    // a page slice's whole rows of one head (half rows 2g and 2g + 1) as 1024-byte swizzle
    // atoms [row group][half][8 rows][128 bytes].
    const cuuint64_t dims[5] = {64, 8, static_cast<cuuint64_t>(2 * p.Hkv),
                                static_cast<cuuint64_t>(p.block_size / 8),
                                static_cast<cuuint64_t>(p.num_blocks)};
    const cuuint64_t strides[4] = {static_cast<cuuint64_t>(p.c_ss) * 2, 128,
                                   static_cast<cuuint64_t>(p.c_ss) * 16,
                                   static_cast<cuuint64_t>(p.c_bs) * 2};
    const cuuint32_t box[5] = {64, 8, 2, static_cast<cuuint32_t>(box_rows / 8), 1};
    r = fn(map, type, 5, const_cast<void*>(base), dims, strides, box, estride,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else {
    // Cache [B, S, Hkv, D] over its own strides as {D, Hkv, S, B}; boxes of 64 dims x 128 rows.
    const cuuint64_t dims[4] = {static_cast<cuuint64_t>(p.D), static_cast<cuuint64_t>(p.Hkv),
                                static_cast<cuuint64_t>(p.S), static_cast<cuuint64_t>(p.B)};
    const cuuint64_t strides[3] = {static_cast<cuuint64_t>(p.c_hs) * 2,
                                   static_cast<cuuint64_t>(p.c_ss) * 2,
                                   static_cast<cuuint64_t>(p.c_bs) * 2};
    const cuuint32_t box[4] = {64, 1, static_cast<cuuint32_t>(box_rows), 1};
    r = fn(map, type, 4, const_cast<void*>(base), dims, strides, box, estride,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  }
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

template <typename E, typename Idx, int HR, int DIM>
cudaError_t launch_tc(const KernelParams& p, const AttentionParams& a, int64_t units, bool pdl,
                      cudaStream_t stream) {
  auto kernel = rope_kv_attention_tc_kernel<E, Idx, HR, DIM>;
  constexpr size_t smem = tc_smem_bytes<DIM>();
  static_assert(smem <= 232448, "the kernel's shared memory exceeds a B200 CTA's 227 KB");
  int device = 0;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) return err;
  {
    static std::mutex mu;
    static std::map<int, bool> opted_in;
    std::lock_guard<std::mutex> lock(mu);
    if (!opted_in[device]) {
      err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(smem));
      if (err != cudaSuccess) return err;
      opted_in[device] = true;
    }
  }
  CUtensorMap kmap, vmap;
  constexpr bool bf16 = std::is_same<E, BF16>::value;
  err = encode_cache_map(&kmap, p.k_dst, bf16, p, a.box_rows);
  if (err != cudaSuccess) return err;
  err = encode_cache_map(&vmap, p.v_dst, bf16, p, a.box_rows);
  if (err != cudaSuccess) return err;
  const int64_t sms = device_sm_count(device);
  const int grid = static_cast<int>(units < sms ? units : sms);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(kTcBlock, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  if (pdl) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, kernel, p, a, kmap, vmap, units);
}

template <typename E, typename Idx, int DIM>
cudaError_t launch_tc_hr(const KernelParams& p, const AttentionParams& a, int64_t units, bool pdl,
                         cudaStream_t stream) {
  // Real query heads per unit: the group size rounded up to a power of two, at most 16.
  const int g = a.group < kTcHeads ? a.group : kTcHeads;
  if (g <= 1) return launch_tc<E, Idx, 1, DIM>(p, a, units, pdl, stream);
  if (g <= 2) return launch_tc<E, Idx, 2, DIM>(p, a, units, pdl, stream);
  if (g <= 4) return launch_tc<E, Idx, 4, DIM>(p, a, units, pdl, stream);
  if (g <= 8) return launch_tc<E, Idx, 8, DIM>(p, a, units, pdl, stream);
  return launch_tc<E, Idx, 16, DIM>(p, a, units, pdl, stream);
}

}  // namespace

cudaError_t launch_rope_kv_attention_tc(const KernelParams& p, const AttentionParams& a,
                                        int elem_code, int index_bits, int64_t units, bool pdl,
                                        cudaStream_t stream) {
  if (units <= 0) return cudaSuccess;
  if (p.D != 64 && p.D != 128) return cudaErrorInvalidValue;
  const bool d64 = p.D == 64;
  switch (elem_code) {
    case kElemF16:
      if (index_bits == 32)
        return d64 ? launch_tc_hr<F16, int, 64>(p, a, units, pdl, stream)
                   : launch_tc_hr<F16, int, 128>(p, a, units, pdl, stream);
      return d64 ? launch_tc_hr<F16, long long, 64>(p, a, units, pdl, stream)
                 : launch_tc_hr<F16, long long, 128>(p, a, units, pdl, stream);
    case kElemBF16:
      if (index_bits == 32)
        return d64 ? launch_tc_hr<BF16, int, 64>(p, a, units, pdl, stream)
                   : launch_tc_hr<BF16, int, 128>(p, a, units, pdl, stream);
      return d64 ? launch_tc_hr<BF16, long long, 64>(p, a, units, pdl, stream)
                 : launch_tc_hr<BF16, long long, 128>(p, a, units, pdl, stream);
    default:
      return cudaErrorInvalidValue;
  }
}

}  // namespace drk
