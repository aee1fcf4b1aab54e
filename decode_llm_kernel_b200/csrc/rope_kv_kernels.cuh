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
// Work layout. A CTA walks tokens (grid-stride). Its threads form `G` row groups (threadIdx.y)
// of `nslots` lanes (threadIdx.x): lane j of a group moves two vectors of VB bytes of one head
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
// Order of a token's memory traffic. The position and request-index loads are issued first
// (before griddepcontrol.wait: they never come from the preceding kernel); then every q/k/v
// row load of the thread, which do not depend on the position; only then is the position
// consumed for the bounds, the cache slot and the table slice. So a CTA's HBM reads are in
// flight while its index and table loads resolve, instead of after them. Launched without the
// programmatic-dependent-launch attribute, griddepcontrol.wait returns at once.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "rope_kv_launch.h"

namespace drk {

enum class Mode : int { kFused = 0, kRope = 1, kAppend = 2 };
enum class Cache : int { kStrided = 0, kPaged = 1 };

constexpr int kMinBlocksPerSM = DRK_MIN_BLOCKS_PER_SM;
#ifndef DRK_ONE_ROW_LEAN_REGS
#define DRK_ONE_ROW_LEAN_REGS 56
#endif

enum : uint32_t {
  kStatusPosCache = 1u << 0,
  kStatusRequest = 1u << 1,
  kStatusPosTable = 1u << 2,
  kStatusBlock = 1u << 3,
};

// KernelParams lives in rope_kv_launch.h so the host layer can fill it.

// ---- element traits: storage bits <-> fp32, one element or a packed pair ----
// A pair is two adjacent elements in one 32-bit word, element j in the low half.
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
  static __device__ __forceinline__ float2 pair_to_f(unsigned int w) {
    __half2 h;
    memcpy(&h, &w, 4);
    return __half22float2(h);
  }
  static __device__ __forceinline__ unsigned int pair_from_f(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    unsigned int w;
    memcpy(&w, &h, 4);
    return w;
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
  static __device__ __forceinline__ float2 pair_to_f(unsigned int w) {
    return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
  }
  static __device__ __forceinline__ unsigned int pair_from_f(float lo, float hi) {
    const __nv_bfloat162 b = __floats2bfloat162_rn(lo, hi);
    unsigned int w;
    memcpy(&w, &b, 4);
    return w;
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
  unsigned int w[VB >= 4 ? VB / 4 : 1];
};

// x1 <- fl(fl(x1*c) - fl(x2*s)), x2 <- fl(fl(x2*c) + fl(x1*s)), element by element, rounded to
// the storage type once. 16-bit types unpack and repack two elements per 32-bit word; the
// arithmetic is the scalar __fmul_rn / __fsub_rn / __fadd_rn chain, which the compiler may not
// contract into a fused multiply-add.
template <typename E, int VB>
__device__ __forceinline__ void rotate_pack(Pack<E, VB>& x1, Pack<E, VB>& x2, const float* c,
                                            const float* s) {
  using raw = typename E::raw;
  constexpr int VEC = VB / static_cast<int>(sizeof(raw));
  if constexpr (sizeof(raw) == 2 && VB >= 4) {
#pragma unroll
    for (int w = 0; w < VB / 4; ++w) {
      const float2 a = E::pair_to_f(x1.w[w]);
      const float2 b = E::pair_to_f(x2.w[w]);
      const float c0 = c[2 * w], c1 = c[2 * w + 1], s0 = s[2 * w], s1 = s[2 * w + 1];
      const float y1lo = __fsub_rn(__fmul_rn(a.x, c0), __fmul_rn(b.x, s0));
      const float y1hi = __fsub_rn(__fmul_rn(a.y, c1), __fmul_rn(b.y, s1));
      const float y2lo = __fadd_rn(__fmul_rn(b.x, c0), __fmul_rn(a.x, s0));
      const float y2hi = __fadd_rn(__fmul_rn(b.y, c1), __fmul_rn(a.y, s1));
      x1.w[w] = E::pair_from_f(y1lo, y1hi);
      x2.w[w] = E::pair_from_f(y2lo, y2hi);
    }
  } else {
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      const float a = E::to_f(x1.e[j]);
      const float b = E::to_f(x2.e[j]);
      const float y1 = __fsub_rn(__fmul_rn(a, c[j]), __fmul_rn(b, s[j]));
      const float y2 = __fadd_rn(__fmul_rn(b, c[j]), __fmul_rn(a, s[j]));
      x1.e[j] = E::from_f(y1);
      x2.e[j] = E::from_f(y2);
    }
  }
}

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

__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

// Threads per block the kernel is compiled for: NR == 1 (one head row per thread, the small-batch
// shape) runs up to 1024 threads, otherwise kMaxThreadsPerBlock. Registers per thread: one row
// per thread takes 64, or 56 in the Lean form (an 8-byte spill), which lets an SM hold 36 warps
// instead of 32. The host takes the Lean form only when that turns a launch of more than one
// wave into one (a 70B-shaped call: 256 tokens x 80 rows x 8 lanes = 164k threads fits 148 SMs
// at 36 warps, not at 32); for launches that fit either way the spill costs latency.
template <int NR, bool Lean>
struct RegisterKernelBounds {
  static constexpr int kThreads = NR == 1 ? 1024 : kMaxThreadsPerBlock;
  static constexpr int kMinBlocks = NR == 1 ? 1 : kMinBlocksPerSM;
  static constexpr int kMaxRegs = NR == 1 ? (Lean ? DRK_ONE_ROW_LEAN_REGS : 64) : 128;
};

template <typename E, typename Idx, int VB, Mode M, Cache C, int NR, bool Lean = false>
__global__ void __launch_bounds__(RegisterKernelBounds<NR, Lean>::kThreads,
                                  RegisterKernelBounds<NR, Lean>::kMinBlocks)
__maxnreg__((RegisterKernelBounds<NR, Lean>::kMaxRegs))
rope_kv_kernel(const __grid_constant__ KernelParams p) {
  using raw = typename E::raw;
  constexpr int VEC = VB / static_cast<int>(sizeof(raw));
  constexpr int64_t ES = static_cast<int64_t>(sizeof(raw));

  // Let the next kernel in the stream start its own prologue while this one runs.
  pdl_launch_dependents();

  // blockDim = (nslots, G): threadIdx.x is the lane within a row, threadIdx.y the row group.
  const int lane = static_cast<int>(threadIdx.x);
  const int grp = static_cast<int>(threadIdx.y);
  const int nrows = num_rows<M>(p);
  const bool lane_rotates = (M != Mode::kAppend) && lane < p.nrot;
  // Element offsets of the lane's two vectors: in a Q/K row (the rotate_half pair, or two
  // pass-through vectors past the rotary dims) and in a V row (a plain copy).
  const int qk_base = (M == Mode::kAppend) ? 0 : p.R;
  const int qk_off1 = lane_rotates ? lane * VEC : qk_base + (lane - (qk_base ? p.nrot : 0)) * VEC;
  const int qk_off2 = lane_rotates ? (p.R >> 1) + lane * VEC : qk_off1 + ((p.D - qk_base) >> 1);
  const int v_off1 = lane * VEC;
  const int v_off2 = v_off1 + (p.D >> 1);
  const bool lead = threadIdx.x == 0 && threadIdx.y == 0 && blockIdx.y == 0;
  bool waited = false;

  // gridDim.y CTAs share a token's rows: CTA y takes row groups y*G .. y*G + G-1.
  const int groups_total = p.G * static_cast<int>(gridDim.y);
  for (int r0 = static_cast<int>(blockIdx.y) * p.G + grp; r0 < nrows; r0 += groups_total * NR) {
    // Per-row constants of this batch of rows: which tensor, the byte offset of the lane's
    // first vector inside a token's source row and inside its destination row, the distance
    // to the second vector.
    int kind[NR];
    int64_t src_off[NR], dst_off[NR];
    int gap[NR];
#pragma unroll
    for (int i = 0; i < NR; ++i) {
      const int r = r0 + i * groups_total;
      int k = kRowV, head = 0;
      if (r < nrows) row_kind<M>(p, r, k, head);
      kind[i] = r < nrows ? k : -1;
      const int o1 = k == kRowV ? v_off1 : qk_off1;
      const int o2 = k == kRowV ? v_off2 : qk_off2;
      gap[i] = (o2 - o1) * static_cast<int>(ES);
      const int64_t hs = k == kRowQ ? p.q_hs : (k == kRowK ? p.k_hs : p.v_hs);
      src_off[i] = (head * hs + o1) * ES;
      if (k == kRowQ || M == Mode::kRope) dst_off[i] = (static_cast<int64_t>(head) * p.D + o1) * ES;
      else dst_off[i] = (head * p.c_hs + o1) * ES;
    }

    for (int64_t t = blockIdx.x; t < p.T; t += gridDim.x) {
      const char* src[NR];
#pragma unroll
      for (int i = 0; i < NR; ++i) {
        const char* base = kind[i] == kRowQ ? p.q + t * p.q_ts * ES
                         : kind[i] == kRowK ? p.k + t * p.k_ts * ES
                                            : p.v + t * p.v_ts * ES;
        src[i] = base + src_off[i];
      }
      // Indices first: they never come from the preceding kernel.
      const int64_t pos = load_index<Idx>(p.positions, t);
      int64_t ri = 0;
      if constexpr (M != Mode::kRope) ri = load_index<Idx>(p.request_indices, t);

      uint32_t bad = 0;
      bool table_ok = false, cache_ok = true;
      int64_t slot = 0;
      float c[VEC], s[VEC];
      // Bounds, destination slot and the table slice: everything that needs the position.
      auto resolve = [&]() {
        table_ok = pos >= 0 && pos < p.table_rows;
        if (!table_ok && M != Mode::kAppend) bad |= kStatusPosTable;
        if constexpr (M != Mode::kRope) {
          const bool pos_ok = pos >= 0 && pos < p.S;
          const bool ri_ok = ri >= 0 && ri < p.B;
          if (!pos_ok) bad |= kStatusPosCache;
          if (!ri_ok) bad |= kStatusRequest;
          cache_ok = pos_ok && ri_ok;
          if constexpr (C == Cache::kStrided) {
            slot = ri * p.c_bs + pos * p.c_ss;
          } else if (cache_ok) {
            const int64_t blk_i = pos / p.block_size;
            const int64_t blk = load_index<Idx>(p.block_table, ri * p.bt_stride + blk_i);
            if (blk < 0 || blk >= p.num_blocks) {
              bad |= kStatusBlock;
              cache_ok = false;
            }
            slot = blk * p.c_bs + (pos - blk_i * p.block_size) * p.c_ss;
          }
          // Warm the address translation of this token's cache slots before the stores.
          if (cache_ok && lead) {
            prefetch_l2(p.k_dst + slot * ES);
            prefetch_l2(p.v_dst + slot * ES);
          }
        }
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
            bool vec4 = false;
            if constexpr (VEC % 4 == 0) vec4 = p.table_vec4 != 0;
            if (vec4) {
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
          }
        }
      };

      Pack<E, VB> x1[NR], x2[NR];
      auto load_rows = [&]() {
#pragma unroll
        for (int i = 0; i < NR; ++i) {
          if (kind[i] >= 0) {
            x1[i].bits = load_stream<VB>(src[i]);
            x2[i].bits = load_stream<VB>(src[i] + gap[i]);
          }
        }
      };

      if (!waited && p.pdl) {
        // Launched as a dependent: the preceding kernel may still be writing q/k/v, so they are
        // only loaded after griddepcontrol.wait. Until then, pull their lines toward L2 (L2 is
        // the coherence point, so a line written later is still read fresh) and resolve
        // everything that needs the position.
#pragma unroll
        for (int i = 0; i < NR; ++i) {
          if (kind[i] >= 0) {
            prefetch_l2(src[i]);
            prefetch_l2(src[i] + gap[i]);
          }
        }
        resolve();
        pdl_wait();
        waited = true;
        load_rows();
      } else {
        if (!waited) {
          pdl_wait();   // returns at once when not launched as a dependent
          waited = true;
        }
        // Row loads first: they do not depend on the position, so they are in flight while the
        // position-dependent work resolves.
        load_rows();
        resolve();
      }
      if (bad && lead && p.status != nullptr) atomicOr(p.status, bad);

#pragma unroll
      for (int i = 0; i < NR; ++i) {
        if (kind[i] < 0) continue;
        if (lane_rotates && kind[i] != kRowV) rotate_pack<E, VB>(x1[i], x2[i], c, s);
        if (kind[i] == kRowQ) {
          if (table_ok) {
            char* dst = p.q_out + t * (static_cast<int64_t>(p.Hq) * p.D * ES) + dst_off[i];
            store_keep<VB>(dst, x1[i].bits);
            store_keep<VB>(dst + gap[i], x2[i].bits);
          }
        } else if (M == Mode::kRope) {
          if (table_ok) {
            char* dst = p.k_dst + t * (static_cast<int64_t>(p.Hkv) * p.D * ES) + dst_off[i];
            store_keep<VB>(dst, x1[i].bits);
            store_keep<VB>(dst + gap[i], x2[i].bits);
          }
        } else if (cache_ok && (kind[i] == kRowV || table_ok)) {
          // K rows need table_ok: in fused mode the row was rotated with this token's table
          // row; in append mode table_rows is the caller's k_position_limit (INT64_MAX unless
          // set), past which the rope step left the k_rot row unwritten.
          char* dst = (kind[i] == kRowK ? p.k_dst : p.v_dst) + slot * ES + dst_off[i];
          store_stream<VB>(dst, x1[i].bits);
          store_stream<VB>(dst + gap[i], x2[i].bits);
        }
      }
    }
  }
  if (!waited) pdl_wait();
}

}  // namespace drk
