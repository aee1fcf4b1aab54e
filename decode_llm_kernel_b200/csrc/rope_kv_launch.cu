// Instantiation and launch of the RoPE + KV-append kernels (rope_kv_kernels.cuh).
//
// The host layer (abi.cpp) has already validated the arguments and picked the widest vector
// width VB the alignment allows; this file maps (dtype, index type, VB, mode, cache kind) to a
// kernel instantiation and launches it with cudaLaunchKernelEx, adding the programmatic
// stream serialization attribute when the caller asked for PDL.
#include <map>
#include <mutex>
#include <utility>

#include "rope_kv_kernels.cuh"
#include "rope_kv_launch.h"
#include "rope_kv_staged.cuh"

namespace drk {
namespace {

int sm_count(int device);

// CTAs of `kernel` with `threads` threads one SM holds (cached per kernel, block size, device).
template <typename K>
int resident_ctas(K kernel, int threads) {
  static std::mutex mu;
  static std::map<std::pair<const void*, std::pair<int, int>>, int> cache;
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return 0;
  std::lock_guard<std::mutex> lock(mu);
  const auto key = std::make_pair(reinterpret_cast<const void*>(kernel),
                                  std::make_pair(device, threads));
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, threads, 0) != cudaSuccess) n = 0;
  cache[key] = n;
  return n;
}

template <typename E, typename Idx, int VB, Mode M, Cache C, int NR, bool Lean = false>
cudaError_t launch_one(const KernelParams& p, const LaunchShape& shape, cudaStream_t stream) {
  if constexpr (NR == 1 && !Lean && M == Mode::kFused && C == Cache::kStrided) {
    // Waves of the 64-register form against the 56-register (Lean) form: take Lean when it
    // fits the grid in fewer waves (both resident counts come from the occupancy calculator).
    const int64_t ctas = static_cast<int64_t>(shape.grid) * shape.splits;
    int device = 0;
    if (shape.allow_lean && cudaGetDevice(&device) == cudaSuccess) {
      const int64_t sms = sm_count(device);
      const int threads = shape.lanes * shape.groups;
      if (ctas > sms) {
        const int64_t full =
            sms * resident_ctas(rope_kv_kernel<E, Idx, VB, M, C, 1, false>, threads);
        const int64_t lean =
            sms * resident_ctas(rope_kv_kernel<E, Idx, VB, M, C, 1, true>, threads);
        if (full > 0 && lean > 0 && (ctas + lean - 1) / lean < (ctas + full - 1) / full)
          return launch_one<E, Idx, VB, M, C, 1, true>(p, shape, stream);
      }
    }
  }
  if (!shape.pdl) {
    // The plain launch path: no attributes to process on the host.
    rope_kv_kernel<E, Idx, VB, M, C, NR, Lean>
        <<<dim3(shape.grid, shape.splits, 1), dim3(shape.lanes, shape.groups, 1), 0, stream>>>(p);
    return cudaGetLastError();
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(shape.grid, shape.splits, 1);
  cfg.blockDim = dim3(shape.lanes, shape.groups, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  if (shape.pdl) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, rope_kv_kernel<E, Idx, VB, M, C, NR, Lean>, p);
}

template <typename E, typename Idx, int VB, int NR>
cudaError_t launch_mode_nr(const KernelParams& p, int mode, int cache, const LaunchShape& shape,
                           cudaStream_t stream) {
  switch (mode) {
    case kModeFused:
      if (cache == kCachePaged)
        return launch_one<E, Idx, VB, Mode::kFused, Cache::kPaged, NR>(p, shape, stream);
      return launch_one<E, Idx, VB, Mode::kFused, Cache::kStrided, NR>(p, shape, stream);
    case kModeRope:
      return launch_one<E, Idx, VB, Mode::kRope, Cache::kStrided, NR>(p, shape, stream);
    case kModeAppend:
      return launch_one<E, Idx, VB, Mode::kAppend, Cache::kStrided, NR>(p, shape, stream);
    default:
      return cudaErrorInvalidValue;
  }
}

template <typename E, typename Idx, int VB>
cudaError_t launch_mode(const KernelParams& p, int mode, int cache, const LaunchShape& shape,
                        cudaStream_t stream) {
  if (p.rows_per_thread == 1) return launch_mode_nr<E, Idx, VB, 1>(p, mode, cache, shape, stream);
  return launch_mode_nr<E, Idx, VB, kRowsPerThread>(p, mode, cache, shape, stream);
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

// ---- the staged (TMA bulk copy) kernel ----

int sm_count(int device) {
  static std::mutex mu;
  static std::map<int, int> cache;
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(device);
  if (it != cache.end()) return it->second;
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n <= 0)
    n = 1;
  cache[device] = n;
  return n;
}

template <typename E, typename Idx, int VB, Cache C>
cudaError_t launch_staged_one(const KernelParams& p, const StagedParams& sp_in,
                              const LaunchShape& shape, cudaStream_t stream) {
  auto kernel = rope_kv_staged_kernel<E, Idx, VB, C>;
  StagedParams sp = sp_in;
  const int threads = shape.lanes * shape.groups;
  int device = 0;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) return err;
  // Per instantiation and device: the dynamic shared-memory opt-in (raised once to the
  // device's limit, so any stage size a later call needs is allowed) and the occupancy per
  // (smem, threads).
  static std::mutex mu;
  static std::map<int, bool> opted_in;
  static std::map<std::pair<int, std::pair<size_t, int>>, int> occupancy;
  int per_sm = 0;
  size_t smem =
      static_cast<size_t>(sp.stages) * (sp.stage_bytes + sizeof(uint64_t)) + kStagedMetaBytes;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!opted_in[device]) {
      int limit = 0;
      err = cudaDeviceGetAttribute(&limit, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
      if (err != cudaSuccess) return err;
      err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 limit - 1024);
      if (err != cudaSuccess) return err;
      opted_in[device] = true;
    }
    auto resident = [&](size_t bytes, int* out) -> cudaError_t {
      const auto key = std::make_pair(device, std::make_pair(bytes, threads));
      auto it = occupancy.find(key);
      if (it != occupancy.end()) {
        *out = it->second;
        return cudaSuccess;
      }
      cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(out, kernel, threads, bytes);
      if (e != cudaSuccess) return e;
      occupancy[key] = *out;
      return cudaSuccess;
    };
    err = resident(smem, &per_sm);
    if (err != cudaSuccess) return err;
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    // A deeper pipeline when every CTA walks many tokens: measured on B200 with Mistral-shaped
    // fp16 rows (12 KB a token, PDL chain), one more stage -- one CTA fewer per SM -- gains
    // 2-3% from about 4.8 tokens a CTA up (4096 tokens: 19.4 -> 18.9 us), while below that
    // the CTA it costs shows as a longer tail (2048 tokens: 10.4 -> 11.2 us).
    if (sp.deepen) {
      const double per_cta =
          static_cast<double>(p.T) / (static_cast<double>(sm_count(device)) * per_sm);
      const size_t deeper =
          static_cast<size_t>(sp.stages + 1) * (sp.stage_bytes + sizeof(uint64_t)) +
          kStagedMetaBytes;
      int per_sm_deeper = 0;
      if (per_cta >= 4.8 && deeper <= static_cast<size_t>(DRK_STAGED_SMEM_BUDGET) &&
          resident(deeper, &per_sm_deeper) == cudaSuccess && per_sm_deeper >= 1) {
        sp.stages += 1;
        smem = deeper;
        per_sm = per_sm_deeper;
      }
    }
  }
  const int64_t slots = static_cast<int64_t>(sm_count(device)) * per_sm;
  const int grid = static_cast<int>(p.T < slots ? p.T : slots);
  sp.early_issue = shape.pdl ? 0 : 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(shape.lanes, shape.groups, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  if (shape.pdl) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, kernel, p, sp);
}

template <typename E, typename Idx, int VB>
cudaError_t launch_staged_cache(const KernelParams& p, const StagedParams& sp, int cache,
                                const LaunchShape& shape, cudaStream_t stream) {
  if (cache == kCachePaged)
    return launch_staged_one<E, Idx, VB, Cache::kPaged>(p, sp, shape, stream);
  return launch_staged_one<E, Idx, VB, Cache::kStrided>(p, sp, shape, stream);
}

template <typename E, typename Idx>
cudaError_t launch_staged_vb(const KernelParams& p, const StagedParams& sp, int vb, int cache,
                             const LaunchShape& shape, cudaStream_t stream) {
  constexpr int es = static_cast<int>(sizeof(typename E::raw));
  switch (vb) {
    case 16: return launch_staged_cache<E, Idx, 16>(p, sp, cache, shape, stream);
    case 8: return launch_staged_cache<E, Idx, 8>(p, sp, cache, shape, stream);
    case 4:
      if constexpr (es <= 4) return launch_staged_cache<E, Idx, 4>(p, sp, cache, shape, stream);
      break;
    case 2:
      if constexpr (es <= 2) return launch_staged_cache<E, Idx, 2>(p, sp, cache, shape, stream);
      break;
    default:
      break;
  }
  return cudaErrorInvalidValue;
}

template <typename E>
cudaError_t launch_staged_idx(const KernelParams& p, const StagedParams& sp, int index_bits,
                              int vb, int cache, const LaunchShape& shape, cudaStream_t stream) {
  if (index_bits == 32) return launch_staged_vb<E, int>(p, sp, vb, cache, shape, stream);
  return launch_staged_vb<E, long long>(p, sp, vb, cache, shape, stream);
}

}  // namespace

int device_sm_count(int device) { return sm_count(device); }

cudaError_t launch_rope_kv_staged(const KernelParams& p, const StagedParams& sp, int elem_code,
                                  int index_bits, int vb, int cache, const LaunchShape& shape,
                                  cudaStream_t stream) {
  switch (elem_code) {
    case kElemF32: return launch_staged_idx<F32>(p, sp, index_bits, vb, cache, shape, stream);
    case kElemF16: return launch_staged_idx<F16>(p, sp, index_bits, vb, cache, shape, stream);
    case kElemBF16: return launch_staged_idx<BF16>(p, sp, index_bits, vb, cache, shape, stream);
    case kElemF64: return launch_staged_idx<F64>(p, sp, index_bits, vb, cache, shape, stream);
    default: return cudaErrorInvalidValue;
  }
}

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
