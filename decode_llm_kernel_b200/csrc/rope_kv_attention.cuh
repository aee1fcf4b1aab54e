// Fused RoPE + KV append + grouped-query decode attention over the cache, in one launch.
//
// For token t (request ri, position pos) and query head h of KV head g (h / group == g):
//   q_rot          = RoPE(q[t, h]), rounded to the storage type (exactly the fused op's q_out)
//   cache slot     = RoPE(k[t, g]), v[t, g] at [ri, pos, g]       (exactly the fused op's append)
//   attn_out[t, h] = sum_{p <= pos} softmax_p(scale * q_rot . K[ri, p, g]) * V[ri, p, g]
//
// Grid: x = chunk * nhb + hb, y = KV head g, z = token t. A CTA covers positions
// [chunk * C, min((chunk + 1) * C, pos + 1)) of one KV head for up to HPB of its query heads
// (head block hb of nhb); CTAs whose chunk starts past pos exit at once.
//
// Inside a CTA each lane owns VL = 16 / sizeof(element) consecutive dims of a K/V row and a
// warp covers 32 / LPR positions per step (LPR lanes per row), so a row is one coalesced
// 16-byte-per-lane read. Each lane keeps the head block's scaled queries for its dims in
// registers, forms partial dot products, reduces them over its LPR lanes with xor-shuffles and
// updates an online softmax (running max m, sum l, accumulator acc) per head, in base 2.
// Warps then merge into one (m, l, acc) per head for the chunk.
//
// The new token's K and V rows are formed in shared memory first. Head block 0 of the CTA whose
// chunk holds pos writes them to the cache slot; every CTA that covers pos reads that position
// from shared memory, so no CTA depends on another's global write.
//
// Chunks of one (token, KV head, head block) combine without waiting on each other: each writes
// (acc, m, l) per head to the workspace, fences, and increments that unit's counter. The CTA
// that sees the last arrival merges every chunk, writes attn_out and returns the counter to zero.
#pragma once

#include "rope_kv_kernels.cuh"

namespace drk {

constexpr int kAttnThreads = 128;
constexpr int kAttnWarps = kAttnThreads / 32;

// AttentionParams lives in rope_kv_launch.h so the host layer can fill it.

// Eight (16-bit types) or four (fp32) consecutive elements of a 16-byte vector as fp32.
template <typename E>
__device__ __forceinline__ void unpack16(const uint4& b, float* f) {
  if constexpr (sizeof(typename E::raw) == 4) {
    f[0] = __uint_as_float(b.x);
    f[1] = __uint_as_float(b.y);
    f[2] = __uint_as_float(b.z);
    f[3] = __uint_as_float(b.w);
  } else {
    const unsigned int w[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 pr = E::pair_to_f(w[i]);
      f[2 * i] = pr.x;
      f[2 * i + 1] = pr.y;
    }
  }
}

// out = x1*c - x2*s (first half) or x2*c + x1*s (second half), each product and the sum
// rounded separately in fp32: the reference oracle's unfused arithmetic.
__device__ __forceinline__ float rotate_one(float x1, float x2, float c, float s, bool first) {
  return first ? __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s))
               : __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
}

template <typename E, typename Idx, int LPR, int HPB>
__global__ void __launch_bounds__(kAttnThreads)
rope_kv_attention_kernel(const __grid_constant__ KernelParams p,
                         const __grid_constant__ AttentionParams a) {
  using raw = typename E::raw;
  constexpr int ES = static_cast<int>(sizeof(raw));
  constexpr int VL = 16 / ES;                 // dims per lane
  constexpr int DMAX = 32 * VL;               // widest head one warp row covers
  constexpr int PPW = 32 / LPR;               // positions per warp step
  constexpr int STEP = PPW * kAttnWarps;      // positions per CTA step

  const int64_t t = blockIdx.z;
  const int g = static_cast<int>(blockIdx.y);
  const int hb = static_cast<int>(blockIdx.x) % a.nhb;
  const int chunk_id = static_cast<int>(blockIdx.x) / a.nhb;
  const int tid = static_cast<int>(threadIdx.x);
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int sub = lane / LPR;                 // which of the warp's positions
  const int dl = (lane % LPR) * VL;           // this lane's first dim
  const bool dim_lane = dl < p.D;
  const int h0 = g * a.group + hb * HPB;      // first query head of this CTA
  const int nh = min(HPB, a.group - hb * HPB);

  __shared__ float s_q[HPB][DMAX];
  __shared__ __align__(16) uint4 s_kn[DMAX / VL];
  __shared__ __align__(16) uint4 s_vn[DMAX / VL];
  __shared__ float s_m[kAttnWarps][HPB];
  __shared__ float s_l[kAttnWarps][HPB];
  __shared__ float s_acc[kAttnWarps][HPB][DMAX];
  __shared__ int s_last;

  pdl_launch_dependents();
  pdl_wait();
  const int64_t pos = load_index<Idx>(p.positions, t);
  const int64_t ri = load_index<Idx>(p.request_indices, t);
  if (pos < 0 || pos >= p.S || pos >= p.table_rows || ri < 0 || ri >= p.B) {
    if (tid == 0 && blockIdx.x == 0 && g == 0 && p.status != nullptr) {
      uint32_t bad = 0;
      if (pos < 0 || pos >= p.S) bad |= kStatusPosCache;
      if (ri < 0 || ri >= p.B) bad |= kStatusRequest;
      if (pos < 0 || pos >= p.table_rows) bad |= kStatusPosTable;
      atomicOr(p.status, bad);
    }
    return;
  }
  const int64_t npos = pos + 1;
  const int64_t p0 = static_cast<int64_t>(chunk_id) * a.chunk;
  if (p0 >= npos) return;
  const int64_t p1 = min(npos, p0 + a.chunk);
  const int nchunks = static_cast<int>((npos + a.chunk - 1) / a.chunk);
  const int half_r = p.R >> 1;
  const float* crow = p.cos_t + pos * p.table_stride;
  const float* srow = p.sin_t + pos * p.table_stride;
  const bool holds_pos = pos < p1;   // p0 <= pos always holds here

  // ---- rotated queries of the head block (and q_out from chunk 0) ----
  for (int idx = tid; idx < nh * p.D; idx += kAttnThreads) {
    const int hh = idx / p.D, d = idx - hh * p.D;
    const raw* qrow =
        reinterpret_cast<const raw*>(p.q) + t * p.q_ts + static_cast<int64_t>(h0 + hh) * p.q_hs;
    raw y;
    if (d < p.R) {
      const int i = d < half_r ? d : d - half_r;
      y = E::from_f(rotate_one(E::to_f(qrow[i]), E::to_f(qrow[i + half_r]), __ldg(crow + i),
                               __ldg(srow + i), d < half_r));
    } else {
      y = qrow[d];
    }
    s_q[hh][d] = E::to_f(y);
    if (a.q_out != nullptr && chunk_id == 0)
      reinterpret_cast<raw*>(a.q_out)[(t * p.Hq + h0 + hh) * static_cast<int64_t>(p.D) + d] = y;
  }

  // ---- the new token's K and V rows; head block 0 appends them to the cache ----
  if (holds_pos) {
    const raw* krow = reinterpret_cast<const raw*>(p.k) + t * p.k_ts + g * p.k_hs;
    const raw* vrow = reinterpret_cast<const raw*>(p.v) + t * p.v_ts + g * p.v_hs;
    raw* kn = reinterpret_cast<raw*>(s_kn);
    raw* vn = reinterpret_cast<raw*>(s_vn);
    const int64_t slot = ri * p.c_bs + pos * p.c_ss + g * p.c_hs;
    for (int d = tid; d < p.D; d += kAttnThreads) {
      raw kr = krow[d];
      if (d < p.R) {
        const int i = d < half_r ? d : d - half_r;
        kr = E::from_f(rotate_one(E::to_f(krow[i]), E::to_f(krow[i + half_r]), __ldg(crow + i),
                                  __ldg(srow + i), d < half_r));
      }
      const raw vr = vrow[d];
      kn[d] = kr;
      vn[d] = vr;
      if (hb == 0) {
        reinterpret_cast<raw*>(p.k_dst)[slot + d] = kr;
        reinterpret_cast<raw*>(p.v_dst)[slot + d] = vr;
      }
    }
  }
  __syncthreads();

  // ---- this lane's scaled queries ----
  float qr[HPB][VL];
#pragma unroll
  for (int hh = 0; hh < HPB; ++hh)
#pragma unroll
    for (int j = 0; j < VL; ++j)
      qr[hh][j] = (hh < nh && dim_lane) ? s_q[hh][dl + j] * a.scale_log2 : 0.f;

  float m[HPB], l[HPB], acc[HPB][VL];
#pragma unroll
  for (int hh = 0; hh < HPB; ++hh) {
    m[hh] = -INFINITY;
    l[hh] = 0.f;
#pragma unroll
    for (int j = 0; j < VL; ++j) acc[hh][j] = 0.f;
  }

  const int64_t row_step = p.c_ss * ES;
  const char* kbase = p.k_dst + ((ri * p.c_bs + g * p.c_hs) * ES + dl * ES);
  const char* vbase = p.v_dst + ((ri * p.c_bs + g * p.c_hs) * ES + dl * ES);
  const uint4 zero4 = make_uint4(0u, 0u, 0u, 0u);

  // Two positions per lane per iteration (pa and pa + STEP): four 16-byte loads in flight.
  for (int64_t base = p0 + warp * PPW; base < p1; base += 2 * STEP) {
    const int64_t pa = base + sub, pb = pa + STEP;
    const bool va = pa < p1, vb = pb < p1;
    uint4 ka = zero4, xa = zero4, kb = zero4, xb = zero4;
    if (dim_lane) {
      if (va) {
        if (pa == pos) {
          ka = s_kn[dl / VL];
          xa = s_vn[dl / VL];
        } else {
          ka = __ldcs(reinterpret_cast<const uint4*>(kbase + pa * row_step));
          xa = __ldcs(reinterpret_cast<const uint4*>(vbase + pa * row_step));
        }
      }
      if (vb) {
        if (pb == pos) {
          kb = s_kn[dl / VL];
          xb = s_vn[dl / VL];
        } else {
          kb = __ldcs(reinterpret_cast<const uint4*>(kbase + pb * row_step));
          xb = __ldcs(reinterpret_cast<const uint4*>(vbase + pb * row_step));
        }
      }
    }
    float kfa[VL], kfb[VL];
    unpack16<E>(ka, kfa);
    unpack16<E>(kb, kfb);
    float sa[HPB], sb[HPB];
#pragma unroll
    for (int hh = 0; hh < HPB; ++hh) {
      float da = 0.f, db = 0.f;
#pragma unroll
      for (int j = 0; j < VL; ++j) {
        da = fmaf(qr[hh][j], kfa[j], da);
        db = fmaf(qr[hh][j], kfb[j], db);
      }
      sa[hh] = da;
      sb[hh] = db;
    }
#pragma unroll
    for (int off = LPR / 2; off >= 1; off >>= 1) {
#pragma unroll
      for (int hh = 0; hh < HPB; ++hh) {
        sa[hh] += __shfl_xor_sync(0xffffffffu, sa[hh], off);
        sb[hh] += __shfl_xor_sync(0xffffffffu, sb[hh], off);
      }
    }
    if (va) {   // vb implies va
      float vfa[VL], vfb[VL];
      unpack16<E>(xa, vfa);
      unpack16<E>(xb, vfb);
#pragma unroll
      for (int hh = 0; hh < HPB; ++hh) {
        const float sbm = vb ? sb[hh] : -INFINITY;
        const float m_new = fmaxf(m[hh], fmaxf(sa[hh], sbm));
        const float corr = exp2f(m[hh] - m_new);
        const float wa = exp2f(sa[hh] - m_new);
        const float wb = exp2f(sbm - m_new);
        l[hh] = fmaf(l[hh], corr, wa + wb);
#pragma unroll
        for (int j = 0; j < VL; ++j)
          acc[hh][j] = fmaf(wb, vfb[j], fmaf(wa, vfa[j], acc[hh][j] * corr));
        m[hh] = m_new;
      }
    }
  }

  // ---- merge the warp's positions (lanes with the same dims), then the warps ----
#pragma unroll
  for (int off = LPR; off < 32; off <<= 1) {
#pragma unroll
    for (int hh = 0; hh < HPB; ++hh) {
      const float mo = __shfl_xor_sync(0xffffffffu, m[hh], off);
      const float lo = __shfl_xor_sync(0xffffffffu, l[hh], off);
      const float m_new = fmaxf(m[hh], mo);
      const float ca = m[hh] == -INFINITY ? 0.f : exp2f(m[hh] - m_new);
      const float cb = mo == -INFINITY ? 0.f : exp2f(mo - m_new);
#pragma unroll
      for (int j = 0; j < VL; ++j) {
        const float other = __shfl_xor_sync(0xffffffffu, acc[hh][j], off);
        acc[hh][j] = acc[hh][j] * ca + other * cb;
      }
      l[hh] = l[hh] * ca + lo * cb;
      m[hh] = m_new;
    }
  }
  if (sub == 0) {
#pragma unroll
    for (int hh = 0; hh < HPB; ++hh) {
      if (hh >= nh) continue;
      if (lane == 0) {
        s_m[warp][hh] = m[hh];
        s_l[warp][hh] = l[hh];
      }
      if (dim_lane)
#pragma unroll
        for (int j = 0; j < VL; ++j) s_acc[warp][hh][dl + j] = acc[hh][j];
    }
  }
  __syncthreads();

  const int row = p.D + 2;
  float* ws = a.workspace + (t * p.Hq + h0) * static_cast<int64_t>(a.max_chunks) * row;
  const int64_t ws_head = static_cast<int64_t>(a.max_chunks) * row;
  raw* out = reinterpret_cast<raw*>(a.attn_out) + (t * p.Hq + h0) * static_cast<int64_t>(p.D);
  for (int idx = tid; idx < nh * row; idx += kAttnThreads) {
    const int hh = idx / row, d = idx - hh * row;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, s_m[w][hh]);
    float acc_d = 0.f, L = 0.f;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) {
      const float cw = s_m[w][hh] == -INFINITY ? 0.f : exp2f(s_m[w][hh] - M);
      L = fmaf(s_l[w][hh], cw, L);
      if (d < p.D) acc_d = fmaf(s_acc[w][hh][d], cw, acc_d);
    }
    if (nchunks == 1) {
      if (d < p.D) out[hh * static_cast<int64_t>(p.D) + d] = E::from_f(acc_d / L);
    } else {
      ws[hh * ws_head + static_cast<int64_t>(chunk_id) * row + d] =
          d < p.D ? acc_d : (d == p.D ? M : L);
    }
  }
  if (nchunks == 1) return;

  // ---- the last chunk to arrive merges every chunk of this (token, KV head, head block) ----
  __threadfence();
  __syncthreads();
  int* counter = a.counters + (t * p.Hkv + g) * a.nhb + hb;
  if (tid == 0) s_last = atomicAdd(counter, 1) == nchunks - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // The last chunk to arrive merges. Warp w takes heads w, w + kAttnWarps, ...; a lane holds
  // chunk cb + lane of each batch of 32 for the (m, l) reduction and dims lane + 32 i for the
  // sums, with 16 chunks' partial loads in flight at once.
  for (int hh = warp; hh < nh; hh += kAttnWarps) {
    const float* hw = ws + hh * ws_head;
    float M = -INFINITY, Ls = 0.f, O[VL];
#pragma unroll
    for (int i = 0; i < VL; ++i) O[i] = 0.f;
    for (int cb = 0; cb < nchunks; cb += 32) {
      const int c = cb + lane;
      const bool in = c < nchunks;
      const float mc = in ? __ldcg(hw + static_cast<int64_t>(c) * row + p.D) : -INFINITY;
      const float lc = in ? __ldcg(hw + static_cast<int64_t>(c) * row + p.D + 1) : 0.f;
      float mg = fmaxf(M, mc);
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1)
        mg = fmaxf(mg, __shfl_xor_sync(0xffffffffu, mg, off));
      const float rescale = exp2f(M - mg);
      const float wc = in ? exp2f(mc - mg) : 0.f;
      float lg = lc * wc;
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) lg += __shfl_xor_sync(0xffffffffu, lg, off);
      Ls = fmaf(Ls, rescale, lg);
#pragma unroll
      for (int i = 0; i < VL; ++i) O[i] *= rescale;
      const int nc = min(32, nchunks - cb);
#pragma unroll 4
      for (int j = 0; j < nc; ++j) {
        const float wj = __shfl_sync(0xffffffffu, wc, j);
        const float* cp = hw + static_cast<int64_t>(cb + j) * row;
#pragma unroll
        for (int i = 0; i < VL; ++i) {
          const int d = lane + 32 * i;
          if (d < p.D) O[i] = fmaf(__ldcg(cp + d), wj, O[i]);
        }
      }
      M = mg;
    }
#pragma unroll
    for (int i = 0; i < VL; ++i) {
      const int d = lane + 32 * i;
      if (d < p.D) out[hh * static_cast<int64_t>(p.D) + d] = E::from_f(O[i] / Ls);
    }
  }
  if (tid == 0) *counter = 0;
}

}  // namespace drk
