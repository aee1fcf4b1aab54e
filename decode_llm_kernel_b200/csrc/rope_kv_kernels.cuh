// Device side of the decode-step RoPE + KV-cache append path, written for sm_100a.
//
// What one launch does (fused mode), per token t of the step:
//   q_out[t, h]                = RoPE(q[t, h], pos[t])        for the Hq query heads
//   k_cache[ri[t], pos[t], h]  = RoPE(k[t, h], pos[t])        for the Hkv key heads
//   v_cache[ri[t], pos[t], h]  = v[t, h]  (byte copy)         for the Hkv value heads
// which is the reference's fused_rope_kv_append (csrc/fused_rope_kv_append.cu:14-84) with its
// oracle's arithmetic (decode_kernels/reference/rope_cache.py:20-36). The rope-only and
// append-only modes are the reference's two separate kernels (csrc/rope.cu:14-59,
// csrc/kv_append.cu:11-40) on the same code.
//
// Work layout. A CTA owns one token at a time (grid-stride over tokens). Its threads form
// `G` row groups of `nslots` lanes: lane j of a group moves two vectors of VB bytes of one head
// row -- for a rotated row, x1 = x[j*VEC ..) and x2 = x[R/2 + j*VEC ..), which is exactly the
// rotate_half pairing, so the rotation needs no data exchange between lanes. Rows are the
// token's Q heads, then its K heads, then its V heads; group g takes rows g, g+G, g+2G, ...
// Each lane loads the position, request index and its slice of the cos/sin row once per token
// and reuses them for every row it owns, and issues the loads of up to kMaxRowsInFlight rows
// before any store so several 32-byte requests per thread are in flight.
//
// Arithmetic. Each output is fl(fl(x1*c) - fl(x2*s)) or fl(fl(x2*c) + fl(x1*s)) in fp32 with
// explicitly rounded multiplies and adds (__fmul_rn/__fadd_rn/__fsub_rn, never contracted to
// an FMA), then one round-to-nearest-even conversion to the storage type. That is what the
// reference's PyTorch oracle computes, so Q and K are bit-exact to it. The table is built as
// concat(f, f), so cos[i + R/2] == cos[i] and only the first R/2 columns are read (the same
// observation csrc/kernel_common.cuh:21-30 of the reference makes). V and the pass-through
// dims of a partial-rotary row are moved as raw bits.
//
// Bounds. An out-of-range position or request index is not a trap (the reference's
// CUDA_KERNEL_ASSERT, csrc/kernel_common.cuh:38-51, kills the context): the token's writes
// that would need the bad index are skipped and a bit is ORed into the status word.
//
// Programmatic dependent launch. The indices and the table slice are read before
// griddepcontrol.wait; q/k/v are read and every store is issued after it. Launched without the
// PDL attribute the wait returns at once.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "rope_kv_launch.h"

namespace drk {

enum class Mode : int { kFused = 0, kRope = 1, kAppend = 2 };
enum class Cache : int { kStrided = 0, kPaged = 1 };

constexpr int kMaxRowsInFlight = 4;

enum : uint32_t {
  kStatusPosCache = 1u << 0,
  kStatusRequest = 1u << 1,
  kStatusPosTable = 1u << 2,
  kStatusBlock = 1u << 3,
};

// KernelParams lives in rope_kv_launch.h so the host layer can fill it.

// ---- element traits: storage bits <-> fp32 ----
struct F32 {
  using raw = float;
  static __device__ __forceinline__ float to_f(raw x) { return x; }
  static __device__ __forceinline__ raw from_f(float f) { return f; }
};
struct F16 {
  using raw = unsigned short;
  static __device__ __forceinline__ float to_f(raw x) { return __half2float(__ushort_as_half(x)); }
  static __device__ __forceinline__ raw from_f(float f) {
    return __half_as_ushort(__float2half_rn(f));
  }
};
struct BF16 {
  using raw = unsigned short;
  static __device__ __forceinline__ float to_f(raw x) {
    return __uint_as_float(static_cast<unsigned int>(x) << 16);
  }
  static __device__ __forceinline__ raw from_f(float f) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(f));
  }
};
struct F64 {
  using raw = double;
  static __device__ __forceinline__ float to_f(raw x) { return __double2float_rn(x); }
  static __device__ __forceinline__ raw from_f(float f) { return static_cast<double>(f); }
};

template <int VB> struct VecBits;
template <> struct VecBits<16> { using type = uint4; };
template <> struct VecBits<8> { using type = uint2; };
template <> struct VecBits<4> { using type = unsigned int; };
template <> struct VecBits<2> { using type = unsigned short; };

template <typename E, int VB>
union Pack {
  typename VecBits<VB>::type bits;
  typename E::raw e[VB / sizeof(typename E::raw)];
};

// Sources are read once: evict-first in L1 and L2.
template <int VB>
__device__ __forceinline__ typename VecBits<VB>::type load_stream(const char* p) {
  return __ldcs(reinterpret_cast<const typename VecBits<VB>::type*>(p));
}
// Cache slots are written once per step and not re-read by this kernel: evict-first.
template <int VB>
__device__ __forceinline__ void store_stream(char* p, typename VecBits<VB>::type x) {
  __stcs(reinterpret_cast<typename VecBits<VB>::type*>(p), x);
}
// q_out is read next by the attention kernel: a normal write-back store keeps it in L2.
template <int VB>
__device__ __forceinline__ void store_keep(char* p, typename VecBits<VB>::type x) {
  *reinterpret_cast<typename VecBits<VB>::type*>(p) = x;
}

template <typename Idx>
__device__ __forceinline__ int64_t load_index(const void* base, int64_t i) {
  return static_cast<int64_t>(__ldg(static_cast<const Idx*>(base) + i));
}

__device__ __forceinline__ void pdl_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Row kinds of one token: which source, destination and whether it rotates.
enum RowKind : int { kRowQ = 0, kRowK = 1, kRowV = 2 };

template <Mode M>
__device__ __forceinline__ int num_rows(const KernelParams& p) {
  if constexpr (M == Mode::kFused) return p.Hq + 2 * p.Hkv;
  else if constexpr (M == Mode::kRope) return p.Hq + p.Hkv;
  else return 2 * p.Hkv;
}

template <Mode M>
__device__ __forceinline__ void row_kind(const KernelParams& p, int r, int& kind, int& head) {
  if constexpr (M == Mode::kAppend) {
    kind = r < p.Hkv ? kRowK : kRowV;
    head = r < p.Hkv ? r : r - p.Hkv;
  } else {
    if (r < p.Hq) { kind = kRowQ; head = r; }
    else if (r < p.Hq + p.Hkv) { kind = kRowK; head = r - p.Hq; }
    else { kind = kRowV; head = r - p.Hq - p.Hkv; }
  }
}

template <typename E, typename Idx, int VB, Mode M, Cache C>
__global__ void __launch_bounds__(kMaxThreadsPerBlock)
rope_kv_kernel(const __grid_constant__ KernelParams p) {
  using raw = typename E::raw;
  using Bits = typename VecBits<VB>::type;
  constexpr int VEC = VB / static_cast<int>(sizeof(raw));
  constexpr int64_t ES = static_cast<int64_t>(sizeof(raw));

  // Let the next kernel in the stream start its own prologue while this one runs.
  pdl_launch_dependents();

  const int lane = static_cast<int>(threadIdx.x) % p.nslots;
  const int grp = static_cast<int>(threadIdx.x) / p.nslots;
  if (grp >= p.G) return;
  const int nrows = num_rows<M>(p);
  const int half_r = p.R >> 1;
  const bool lane_rotates = (M != Mode::kAppend) && lane < p.nrot;
  bool waited = false;

  for (int64_t t = blockIdx.x; t < p.T; t += gridDim.x) {
    // ---- prologue: indices, bounds, table slice (independent of the preceding kernel) ----
    const int64_t pos = load_index<Idx>(p.positions, t);
    uint32_t bad = 0;
    const bool table_ok = pos >= 0 && pos < p.table_rows;
    if (!table_ok && M != Mode::kAppend) bad |= kStatusPosTable;
    int64_t slot = 0;
    bool cache_ok = true;
    if constexpr (M != Mode::kRope) {
      const int64_t ri = load_index<Idx>(p.request_indices, t);
      const bool pos_ok = pos >= 0 && pos < p.S;
      const bool ri_ok = ri >= 0 && ri < p.B;
      if (!pos_ok) bad |= kStatusPosCache;
      if (!ri_ok) bad |= kStatusRequest;
      cache_ok = pos_ok && ri_ok;
      if constexpr (C == Cache::kStrided) {
        slot = ri * p.c_bs + pos * p.c_ss;
      } else {
        if (cache_ok) {
          const int64_t blk_i = pos / p.block_size;
          const int64_t blk = load_index<Idx>(p.block_table, ri * p.bt_stride + blk_i);
          if (blk < 0 || blk >= p.num_blocks) {
            bad |= kStatusBlock;
            cache_ok = false;
          }
          slot = blk * p.c_bs + (pos - blk_i * p.block_size) * p.c_ss;
        }
      }
    }
    if (bad && threadIdx.x == 0 && p.status != nullptr) atomicOr(p.status, bad);

    float c[VEC], s[VEC];
    if (lane_rotates && table_ok) {
      if (p.inreg_trig) {
        const float pf = static_cast<float>(pos);
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
          const float ang = __fmul_rn(pf, __ldg(p.inv_freq + lane * VEC + j));
          sincosf(ang, &s[j], &c[j]);
        }
      } else {
        const float* crow = p.cos_t + pos * p.table_stride + lane * VEC;
        const float* srow = p.sin_t + pos * p.table_stride + lane * VEC;
        if constexpr (VEC % 4 == 0) {
          if (p.table_vec4) {
#pragma unroll
            for (int j = 0; j < VEC; j += 4) {
              const float4 cv = __ldg(reinterpret_cast<const float4*>(crow + j));
              const float4 sv = __ldg(reinterpret_cast<const float4*>(srow + j));
              c[j] = cv.x; c[j + 1] = cv.y; c[j + 2] = cv.z; c[j + 3] = cv.w;
              s[j] = sv.x; s[j + 1] = sv.y; s[j + 2] = sv.z; s[j + 3] = sv.w;
            }
          } else {
#pragma unroll
            for (int j = 0; j < VEC; ++j) { c[j] = __ldg(crow + j); s[j] = __ldg(srow + j); }
          }
        } else {
#pragma unroll
          for (int j = 0; j < VEC; ++j) { c[j] = __ldg(crow + j); s[j] = __ldg(srow + j); }
        }
      }
    }

    // ---- everything below may depend on the preceding kernel ----
    if (!waited) {
      pdl_wait();
      waited = true;
    }

    for (int r0 = grp; r0 < nrows; r0 += p.G * kMaxRowsInFlight) {
      Pack<E, VB> x1[kMaxRowsInFlight], x2[kMaxRowsInFlight];
      // Issue every load of this batch of rows first.
#pragma unroll
      for (int i = 0; i < kMaxRowsInFlight; ++i) {
        const int r = r0 + i * p.G;
        if (r < nrows) {
          int kind, head;
          row_kind<M>(p, r, kind, head);
          const char* src;
          if (kind == kRowQ) src = p.q + (t * p.q_ts + head * p.q_hs) * ES;
          else if (kind == kRowK) src = p.k + (t * p.k_ts + head * p.k_hs) * ES;
          else src = p.v + (t * p.v_ts + head * p.v_hs) * ES;
          const bool rot = lane_rotates && kind != kRowV;
          const int rb = (kind == kRowV || M == Mode::kAppend) ? 0 : p.R;
          const int off1 = rot ? lane * VEC : rb + (lane - (rb ? p.nrot : 0)) * VEC;
          const int off2 = rot ? half_r + lane * VEC : off1 + ((p.D - rb) >> 1);
          x1[i].bits = load_stream<VB>(src + off1 * ES);
          x2[i].bits = load_stream<VB>(src + off2 * ES);
        }
      }
#pragma unroll
      for (int i = 0; i < kMaxRowsInFlight; ++i) {
        const int r = r0 + i * p.G;
        if (r < nrows) {
          int kind, head;
          row_kind<M>(p, r, kind, head);
          const bool rot = lane_rotates && kind != kRowV;
          const int rb = (kind == kRowV || M == Mode::kAppend) ? 0 : p.R;
          const int off1 = rot ? lane * VEC : rb + (lane - (rb ? p.nrot : 0)) * VEC;
          const int off2 = rot ? half_r + lane * VEC : off1 + ((p.D - rb) >> 1);
          if (rot) {
#pragma unroll
            for (int j = 0; j < VEC; ++j) {
              const float a = E::to_f(x1[i].e[j]);
              const float b = E::to_f(x2[i].e[j]);
              const float y1 = __fsub_rn(__fmul_rn(a, c[j]), __fmul_rn(b, s[j]));
              const float y2 = __fadd_rn(__fmul_rn(b, c[j]), __fmul_rn(a, s[j]));
              x1[i].e[j] = E::from_f(y1);
              x2[i].e[j] = E::from_f(y2);
            }
          }
          if (kind == kRowQ) {
            if (table_ok) {
              char* dst = p.q_out + ((t * p.Hq + head) * static_cast<int64_t>(p.D)) * ES;
              store_keep<VB>(dst + off1 * ES, x1[i].bits);
              store_keep<VB>(dst + off2 * ES, x2[i].bits);
            }
          } else if (M == Mode::kRope) {
            if (table_ok) {
              char* dst = p.k_dst + ((t * p.Hkv + head) * static_cast<int64_t>(p.D)) * ES;
              store_keep<VB>(dst + off1 * ES, x1[i].bits);
              store_keep<VB>(dst + off2 * ES, x2[i].bits);
            }
          } else {
            const bool ok = cache_ok && (kind == kRowV || M == Mode::kAppend || table_ok);
            if (ok) {
              char* base = kind == kRowK ? p.k_dst : p.v_dst;
              char* dst = base + (slot + head * p.c_hs) * ES;
              store_stream<VB>(dst + off1 * ES, x1[i].bits);
              store_stream<VB>(dst + off2 * ES, x2[i].bits);
            }
          }
        }
      }
    }
  }
  if (!waited) pdl_wait();
}

}  // namespace drk
