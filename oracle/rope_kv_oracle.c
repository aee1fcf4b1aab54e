/*
 * CPU oracle for the decode-step RoPE + KV-cache append path.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the checker that the CUDA kernels are compared
 * against; it is never part of the product path. Only tests, the smoke check and the CPU
 * baseline leg of the benchmark load it.
 *
 * It restates, element by element, the PyTorch oracle of the reference project:
 *   decode_kernels/reference/rope_cache.py:14-18  rotate_half(x) = cat(-x2, x1)
 *   decode_kernels/reference/rope_cache.py:20-24  apply_rope(x) = x*cos + rotate_half(x)*sin
 *   decode_kernels/reference/rope_cache.py:26-36  fused_rope_kv_append_ref: gather the fp32 table
 *       rows at each token's position, rotate Q and K in fp32, round to the storage dtype,
 *       write K to k_cache[request, position] and raw V to v_cache[request, position].
 * PyTorch evaluates `x*cos + rotate_half(x)*sin` as three separate elementwise kernels, each
 * rounding to fp32, so every output element is
 *       out[i]        = fl( fl(x[i]*cos[i])        + fl(-x[i+h]*sin[i]) )        i <  h
 *       out[i+h]      = fl( fl(x[i+h]*cos[i+h])    + fl( x[i]  *sin[i+h]) )      i <  h
 * with h = rotary_dim/2, followed by one round-to-nearest-even conversion to the storage
 * dtype. This file is compiled with -ffp-contract=off so no multiply-add is fused.
 *
 * Partial rotary (rotary_dim < head_dim) is an extension the reference does not have: the
 * first rotary_dim dims rotate as above with an [P, rotary_dim] table, the rest pass through
 * unchanged (a raw copy, like V).
 *
 * Storage dtypes: 0 = fp32, 1 = fp16, 2 = bf16, 3 = fp64. fp64 goes through fp32 exactly as
 * the reference does (`q.to(torch.float32)` then `.to(q.dtype)`).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

enum { ORC_F32 = 0, ORC_F16 = 1, ORC_BF16 = 2, ORC_F64 = 3 };

/* ---- storage <-> fp32 conversions (IEEE 754 binary16 / bfloat16, round to nearest even) ---- */

static inline uint32_t f32_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float bits_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

static inline float bf16_to_f32(uint16_t h) { return bits_f32((uint32_t)h << 16); }

/* Keeps the top 16 bits, rounding the discarded 16 to nearest, ties to even. A NaN becomes the
 * canonical quiet NaN 0x7FC0, which is what PyTorch's CPU conversion produces. */
static inline uint16_t f32_to_bf16(float f) {
  uint32_t u = f32_bits(f);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return 0x7FC0;
  uint32_t lsb = (u >> 16) & 1u;
  u += 0x7FFFu + lsb;
  return (uint16_t)(u >> 16);
}

static inline float f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1Fu;
  uint32_t man = h & 0x3FFu;
  if (exp == 0x1Fu) return bits_f32(sign | 0x7F800000u | (man << 13));  /* inf / nan */
  if (exp == 0) {
    if (man == 0) return bits_f32(sign);
    /* subnormal: value = man * 2^-24, exact in fp32 */
    float v = (float)man * 5.9604644775390625e-08f;
    return (sign ? -v : v);
  }
  return bits_f32(sign | ((exp + 112u) << 23) | (man << 13));
}

/* fp32 -> binary16, round to nearest even, overflow to inf, gradual underflow. */
static inline uint16_t f32_to_f16(float f) {
  uint32_t u = f32_bits(f);
  uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
  uint32_t a = u & 0x7FFFFFFFu;
  if (a > 0x7F800000u) return (uint16_t)(sign | 0x7E00u);          /* nan */
  if (a >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);         /* rounds to >= 65520: inf */
  int32_t e = (int32_t)(a >> 23) - 127;                            /* unbiased exponent */
  if (e >= -14) {
    /* normal half: keep 10 mantissa bits of the 23 */
    uint32_t man = a & 0x7FFFFFu;
    uint32_t half = ((uint32_t)(e + 15) << 10) | (man >> 13);
    uint32_t rest = man & 0x1FFFu;
    if (rest > 0x1000u || (rest == 0x1000u && (half & 1u))) half += 1u;  /* may carry into exp */
    return (uint16_t)(sign | half);
  }
  if (e < -25) return sign;                                        /* below half the min subnormal */
  /* subnormal half: value / 2^-24 rounded to an integer, ties to even */
  uint32_t man = (a & 0x7FFFFFu) | 0x800000u;                      /* 24-bit significand */
  int shift = -e - 1;                                              /* = (-14 - e) + 13 */
  uint32_t q = man >> shift;
  uint32_t rem = man & ((1u << shift) - 1u);
  uint32_t halfway = 1u << (shift - 1);
  if (rem > halfway || (rem == halfway && (q & 1u))) q += 1u;
  return (uint16_t)(sign | q);
}

static inline float load_f32(const void* base, int dtype, int64_t i) {
  switch (dtype) {
    case ORC_F32: return ((const float*)base)[i];
    case ORC_F16: return f16_to_f32(((const uint16_t*)base)[i]);
    case ORC_BF16: return bf16_to_f32(((const uint16_t*)base)[i]);
    default: return (float)((const double*)base)[i];
  }
}

static inline void store_f32(void* base, int dtype, int64_t i, float x) {
  switch (dtype) {
    case ORC_F32: ((float*)base)[i] = x; break;
    case ORC_F16: ((uint16_t*)base)[i] = f32_to_f16(x); break;
    case ORC_BF16: ((uint16_t*)base)[i] = f32_to_bf16(x); break;
    default: ((double*)base)[i] = (double)x; break;
  }
}

static inline size_t elem_size(int dtype) {
  return dtype == ORC_F32 ? 4 : (dtype == ORC_F64 ? 8 : 2);
}

/* Raw element copy: V and the pass-through dims are never converted. */
static inline void copy_elem(void* dst, int64_t di, const void* src, int64_t si, int dtype) {
  size_t e = elem_size(dtype);
  memcpy((char*)dst + di * (int64_t)e, (const char*)src + si * (int64_t)e, e);
}

/* One head row: rotate the first R dims (pair i with i + R/2), copy dims [R, D) raw.
 * `crow`/`srow` point at the token's table row. */
static void rope_row(const void* src, int64_t s0, void* dst, int64_t d0, int dtype, int D, int R,
                     const float* crow, const float* srow) {
  const int h = R / 2;
  for (int i = 0; i < h; ++i) {
    float x1 = load_f32(src, dtype, s0 + i);
    float x2 = load_f32(src, dtype, s0 + i + h);
    /* rotate_half gives (-x2, x1); each product is rounded before the add (no contraction). */
    float a = x1 * crow[i];
    float b = (-x2) * srow[i];
    float c = x2 * crow[i + h];
    float d = x1 * srow[i + h];
    store_f32(dst, dtype, d0 + i, a + b);
    store_f32(dst, dtype, d0 + i + h, c + d);
  }
  for (int i = R; i < D; ++i) copy_elem(dst, d0 + i, src, s0 + i, dtype);
}

/* Validates the addressing contract the reference enforces with device asserts
 * (csrc/kernel_common.cuh:38-51): every position inside the cache and the table, every request
 * index inside the batch. Returns 0, or -1 position, -2 request index, -3 table row. */
static int check_indices(int64_t T, const int64_t* pos, const int64_t* ri, int64_t B, int64_t S,
                         int64_t table_rows) {
  for (int64_t t = 0; t < T; ++t) {
    if (pos[t] < 0 || (ri && pos[t] >= S)) return -1;
    if (ri && (ri[t] < 0 || ri[t] >= B)) return -2;
    if (pos[t] >= table_rows) return -3;
  }
  return 0;
}

static void set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

int orc_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/*
 * fused_rope_kv_append_ref (decode_kernels/reference/rope_cache.py:26-36).
 * q/k/v: element strides (token, head); last dim contiguous. q_out: contiguous [T, Hq, D].
 * Caches: element strides (batch, position, head); last dim contiguous, which covers the
 * token-major [B, S, Hkv, D] layout and the head-major [B, Hkv, S, D] one.
 * Tokens are processed in order, so a duplicated slot keeps the last token's data.
 */
int orc_fused_rope_kv_append(int dtype, const void* q, const void* k, const void* v,
                             int64_t T, int Hq, int Hkv, int D, int R,
                             int64_t q_st, int64_t q_sh, int64_t k_st, int64_t k_sh,
                             int64_t v_st, int64_t v_sh,
                             const float* cos_t, const float* sin_t, int64_t table_rows,
                             int64_t table_stride,
                             const int64_t* positions, const int64_t* request_indices,
                             void* q_out, void* k_cache, void* v_cache,
                             int64_t B, int64_t S, int64_t c_sb, int64_t c_ss, int64_t c_sh,
                             int nthreads) {
  int rc = check_indices(T, positions, request_indices, B, S, table_rows);
  if (rc) return rc;
  set_threads(nthreads);
  /* Q rows first, then the cache scatter, both parallel over tokens. */
#pragma omp parallel for schedule(static)
  for (int64_t t = 0; t < T; ++t) {
    const float* crow = cos_t + positions[t] * table_stride;
    const float* srow = sin_t + positions[t] * table_stride;
    for (int h = 0; h < Hq; ++h)
      rope_row(q, t * q_st + h * q_sh, q_out, (t * Hq + h) * (int64_t)D, dtype, D, R, crow, srow);
  }
  /* Duplicate (request, position) slots have no defined result in the reference
   * (benchmarks/validation.py:51-53). With nthreads == 1 the last token wins. */
#pragma omp parallel for schedule(static)
  for (int64_t t = 0; t < T; ++t) {
    const float* crow = cos_t + positions[t] * table_stride;
    const float* srow = sin_t + positions[t] * table_stride;
    const int64_t slot = request_indices[t] * c_sb + positions[t] * c_ss;
    for (int h = 0; h < Hkv; ++h) {
      rope_row(k, t * k_st + h * k_sh, k_cache, slot + h * c_sh, dtype, D, R, crow, srow);
      const size_t e = elem_size(dtype);
      memcpy((char*)v_cache + (slot + h * c_sh) * (int64_t)e,
             (const char*)v + (t * v_st + h * v_sh) * (int64_t)e, (size_t)D * e);
    }
  }
  return 0;
}

/* The rope-only rung (csrc/rope.cu semantics): contiguous q_out [T,Hq,D], k_out [T,Hkv,D]. */
int orc_rope_forward(int dtype, const void* q, const void* k, int64_t T, int Hq, int Hkv, int D,
                     int R, int64_t q_st, int64_t q_sh, int64_t k_st, int64_t k_sh,
                     const float* cos_t, const float* sin_t, int64_t table_rows,
                     int64_t table_stride, const int64_t* positions, void* q_out, void* k_out,
                     int nthreads) {
  int rc = check_indices(T, positions, NULL, 0, 0, table_rows);
  if (rc) return rc;
  set_threads(nthreads);
#pragma omp parallel for schedule(static)
  for (int64_t t = 0; t < T; ++t) {
    const float* crow = cos_t + positions[t] * table_stride;
    const float* srow = sin_t + positions[t] * table_stride;
    for (int h = 0; h < Hq; ++h)
      rope_row(q, t * q_st + h * q_sh, q_out, (t * Hq + h) * (int64_t)D, dtype, D, R, crow, srow);
    for (int h = 0; h < Hkv; ++h)
      rope_row(k, t * k_st + h * k_sh, k_out, (t * Hkv + h) * (int64_t)D, dtype, D, R, crow, srow);
  }
  return 0;
}

/* The append-only rung (csrc/kv_append.cu semantics): raw copies of k_rot and v into slots. */
int orc_kv_append(int dtype, const void* k_rot, const void* v, int64_t T, int Hkv, int D,
                  int64_t k_st, int64_t k_sh, int64_t v_st, int64_t v_sh,
                  const int64_t* positions, const int64_t* request_indices, void* k_cache,
                  void* v_cache, int64_t B, int64_t S, int64_t c_sb, int64_t c_ss, int64_t c_sh) {
  int rc = check_indices(T, positions, request_indices, B, S, S);
  if (rc) return rc;
  const size_t e = elem_size(dtype);
  for (int64_t t = 0; t < T; ++t) {
    const int64_t slot = request_indices[t] * c_sb + positions[t] * c_ss;
    for (int h = 0; h < Hkv; ++h) {
      memcpy((char*)k_cache + (slot + h * c_sh) * (int64_t)e,
             (const char*)k_rot + (t * k_st + h * k_sh) * (int64_t)e, (size_t)D * e);
      memcpy((char*)v_cache + (slot + h * c_sh) * (int64_t)e,
             (const char*)v + (t * v_st + h * v_sh) * (int64_t)e, (size_t)D * e);
    }
  }
  return 0;
}

/*
 * Decode attention over the cache after the append (the consumer of this path's writes; the
 * reference prices it with torch SDPA, benchmarks/probe_cache_read.py:26-172):
 *   out[t, h] = sum_p softmax_p(scale * q[t, h] . K[ri, p, g]) V[ri, p, g],  p in [0, pos[t]]
 * with g = h / (Hq / Hkv) (grouped-query attention). q is the rotated query in the storage
 * dtype (what the fused op returns); the dot products, the softmax and the weighted sum are
 * evaluated in double from the stored values, then rounded once to the storage dtype.
 * Returns 0, or -1 / -2 for an out-of-range position / request index.
 */
int orc_decode_attention(int dtype, const void* q, int64_t T, int Hq, int Hkv, int D,
                         const void* k_cache, const void* v_cache, int64_t B, int64_t S,
                         int64_t c_sb, int64_t c_ss, int64_t c_sh, const int64_t* positions,
                         const int64_t* request_indices, double scale, void* out,
                         int nthreads) {
  int rc = check_indices(T, positions, request_indices, B, S, S);
  if (rc) return rc;
  if (Hq % Hkv) return -4;
  set_threads(nthreads);
  const int group = Hq / Hkv;
#pragma omp parallel for schedule(dynamic)
  for (int64_t th = 0; th < T * Hq; ++th) {
    const int64_t t = th / Hq;
    const int h = (int)(th % Hq);
    const int g = h / group;
    const int64_t npos = positions[t] + 1;
    const int64_t base = request_indices[t] * c_sb + (int64_t)g * c_sh;
    double m = -1e300, l = 0.0;
    double acc[1024];
    for (int d = 0; d < D; ++d) acc[d] = 0.0;
    for (int64_t p = 0; p < npos; ++p) {
      double dot = 0.0;
      for (int d = 0; d < D; ++d)
        dot += (double)load_f32(q, dtype, (t * Hq + h) * (int64_t)D + d) *
               (double)load_f32(k_cache, dtype, base + p * c_ss + d);
      const double sc = dot * scale;
      const double m_new = sc > m ? sc : m;
      const double corr = exp(m - m_new);
      const double w = exp(sc - m_new);
      l = l * corr + w;
      for (int d = 0; d < D; ++d)
        acc[d] = acc[d] * corr + w * (double)load_f32(v_cache, dtype, base + p * c_ss + d);
      m = m_new;
    }
    for (int d = 0; d < D; ++d)
      store_f32(out, dtype, (t * Hq + h) * (int64_t)D + d, (float)(acc[d] / l));
  }
  return 0;
}

/* Exposed for the conversion tests. */
uint16_t orc_f32_to_bf16(float f) { return f32_to_bf16(f); }
uint16_t orc_f32_to_f16(float f) { return f32_to_f16(f); }
float orc_f16_to_f32(uint16_t h) { return f16_to_f32(h); }
float orc_bf16_to_f32(uint16_t h) { return bf16_to_f32(h); }
