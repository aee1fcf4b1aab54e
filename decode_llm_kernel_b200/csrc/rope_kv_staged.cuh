// Bandwidth-regime form of the fused RoPE + KV append: TMA bulk copies through shared memory.
//
// Used when many tokens are in one call (the host picks it by token count) and every row
// block the op moves is contiguous: a token's Q heads, K heads and V heads each form one run
// of H*D elements in the source (head stride == D; fused-QKV views qualify), q_out is
// contiguous, and a cache slot [Hkv, D] is contiguous (token-major or paged caches).
//
// Per CTA, a persistent loop over tokens t = blockIdx.x, blockIdx.x + gridDim.x, ... with a
// kStages-deep pipeline in shared memory. Before griddepcontrol.wait (programmatic dependent
// launch) a CTA pulls its first tokens' row blocks toward L2 (cp.async.bulk.prefetch.L2) and
// resolves the positions, request indices, bounds and cache slots of its first 64 tokens into
// shared memory, many threads at once (later blocks of 32 the same way, a block ahead), so no
// token waits on a load of its own index; launched without PDL, its first thread issues the
// first stage-full of copies during that round trip. Then:
//   1. one thread issues cp.async.bulk global->shared copies of the token's Q, K and V row
//      blocks, completing on the stage's mbarrier (expect_tx bytes); the lanes load their
//      cos/sin slice of the token a token ahead, from the position in shared memory;
//   2. every thread waits on the stage's mbarrier (bounded: see below);
//   3. threads rotate only the rotary dims of the Q and K rows, in place in shared memory
//      (lane j: elements [j*VEC, +VEC) and [R/2 + j*VEC, +VEC), the rotate_half pair), with
//      the same per-element roundings as the register kernel (bit-exact to the oracle);
//   4. after a proxy fence and a barrier, one thread issues cp.async.bulk shared->global
//      copies: the Q block to q_out[t], the K and V blocks to the token's cache slots. V rows
//      and the pass-through dims of partial rotary never pass through registers;
//   5. a stage is refilled with the token kStages ahead once the bulk stores that read it
//      have finished reading (cp.async.bulk.wait_group.read).
// No thread-block clusters: every copy moves data between global memory and this CTA's own
// shared memory.
//
// Waits. Each mbarrier wait is bounded (one second of %globaltimer). If a wait runs out -- a
// copy that never lands, which no valid input produces -- the CTA sets DRK_STATUS_TIMEOUT in
// the status word, stops issuing work, waits (bounded) for its own copies in flight and
// returns.
#pragma once

#include "rope_kv_kernels.cuh"

namespace drk {

constexpr int kStagedThreads = kStagedThreadsPerBlock;
constexpr uint32_t kStatusTimeout = 1u << 4;
// A bounded wait gives up after this many nanoseconds of %globaltimer: a second, against the
// microseconds any copy this library issues takes.
#ifndef DRK_WAIT_LIMIT_NS
#define DRK_WAIT_LIMIT_NS 1000000000ull
#endif

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// True once the barrier's phase with this parity has completed; false once limit_ns
// (DRK_WAIT_LIMIT_NS unless given) have passed on %globaltimer since the wait started (read
// every 16 polls: try_wait itself suspends the thread for a while between polls).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          uint64_t limit_ns = DRK_WAIT_LIMIT_NS) {
  const uint32_t addr = smem_u32(bar);
  uint64_t deadline = 0;
  for (uint32_t i = 0;; ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return true;
    if ((i & 15u) == 15u) {
      const uint64_t now = global_ns();
      if (deadline == 0) {
        deadline = now + limit_ns;
      } else if (now >= deadline) {
        return false;
      }
    }
  }
}

// L2 eviction priority of the bulk copies: 0 none; bit 0: loads (q/k/v are read once) marked
// evict-first; bit 1: stores (q_out and the cache slots, not read again in the launch) marked
// evict-first. Measured on B200 (Mistral-shaped batch 4096, 64 GiB caches, 102.8 MB per
// launch): none 19.73 us, loads only 20.18, stores only 19.93, both 19.28.
#ifndef DRK_STAGED_L2_HINT
#define DRK_STAGED_L2_HINT 3
#endif

__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gmem_src, uint32_t bytes,
                                          uint64_t* bar) {
#if DRK_STAGED_L2_HINT & 1
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;"
      ::"r"(smem_u32(smem_dst)), "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar)),
      "l"(evict_first_policy())
      : "memory");
#else
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(smem_u32(smem_dst)), "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
#endif
}

__device__ __forceinline__ void bulk_store(void* gmem_dst, const void* smem_src, uint32_t bytes) {
#if DRK_STAGED_L2_HINT & 2
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group.L2::cache_hint [%0], [%1], %2, %3;"
               ::"l"(gmem_dst), "r"(smem_u32(smem_src)), "r"(bytes), "l"(evict_first_policy())
               : "memory");
#else
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gmem_dst),
               "r"(smem_u32(smem_src)), "r"(bytes)
               : "memory");
#endif
}

// Pulls `bytes` (a multiple of 16, 16-byte aligned) toward L2 without a destination: issued
// before griddepcontrol.wait, so the copies after it hit L2. L2 is the point of coherence, so a
// line the preceding kernel writes after the prefetch is still read fresh.
__device__ __forceinline__ void bulk_prefetch_l2(const void* gmem_src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(gmem_src), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Waits until at most N committed bulk-store groups still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Shared-memory vector access of VB bytes.
template <int VB>
__device__ __forceinline__ typename VecBits<VB>::type lds(const unsigned char* p) {
  return *reinterpret_cast<const typename VecBits<VB>::type*>(p);
}
template <int VB>
__device__ __forceinline__ void sts(unsigned char* p, typename VecBits<VB>::type x) {
  *reinterpret_cast<typename VecBits<VB>::type*>(p) = x;
}

// One token's metadata, resolved once for the CTA's walk (shared memory).
struct StagedTokenMeta {
  int64_t pos;
  int64_t slot;       // element offset of the token's cache slot (valid when cache_ok)
  uint32_t bad;       // DRK_STATUS bits this token reports
  uint32_t ok;        // bit 0: table row in range; bit 1: cache slot in range
};
static_assert(2 * kStagedMetaBlock * sizeof(StagedTokenMeta) == kStagedMetaBytes,
              "the launcher's shared-memory size for the metadata array");
constexpr uint32_t kMetaTableOk = 1u, kMetaCacheOk = 2u;

template <typename E, typename Idx, int VB, Cache C>
__global__ void __launch_bounds__(kStagedThreads)
rope_kv_staged_kernel(const __grid_constant__ KernelParams p,
                      const __grid_constant__ StagedParams sp) {
  using raw = typename E::raw;
  constexpr int VEC = VB / static_cast<int>(sizeof(raw));
  constexpr int64_t ES = static_cast<int64_t>(sizeof(raw));
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(sp.stages) *
                                               sp.stage_bytes);
  StagedTokenMeta* meta = reinterpret_cast<StagedTokenMeta*>(bars + sp.stages);
  __shared__ int s_abort;

  pdl_launch_dependents();

  const int tid = static_cast<int>(threadIdx.x + threadIdx.y * blockDim.x);
  const int nthreads = static_cast<int>(blockDim.x * blockDim.y);
  const int lane = static_cast<int>(threadIdx.x);   // < nrot
  const int grp = static_cast<int>(threadIdx.y);
  const int rot_rows = p.Hq + p.Hkv;
  const int64_t my_tokens = p.T > blockIdx.x ? (p.T - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const int row_bytes = p.D * static_cast<int>(ES);

  // Token j's metadata lives in block (j / kStagedMetaBlock) % 2 of the shared array. Threads
  // first.. resolve a block's tokens at once (one round of dependent index -> slot /
  // block-table loads for the whole block), so no token waits on its own index loads.
  auto meta_at = [&](int64_t jj) {
    return meta + ((jj / kStagedMetaBlock) & 1) * kStagedMetaBlock + jj % kStagedMetaBlock;
  };
  auto fill_meta = [&](int64_t j0, int first) {
    if (tid < first) return;
    for (int i = tid - first; i < kStagedMetaBlock; i += nthreads - first) {
      const int64_t jj = j0 + i;
      if (jj >= my_tokens) break;
      const int64_t t = blockIdx.x + jj * gridDim.x;
      const int64_t pos = load_index<Idx>(p.positions, t);
      const int64_t ri = load_index<Idx>(p.request_indices, t);
      uint32_t bad = 0u;
      int64_t slot = 0;
      const bool table_ok = pos >= 0 && pos < p.table_rows;
      if (!table_ok) bad |= kStatusPosTable;
      const bool pos_ok = pos >= 0 && pos < p.S;
      const bool ri_ok = ri >= 0 && ri < p.B;
      if (!pos_ok) bad |= kStatusPosCache;
      if (!ri_ok) bad |= kStatusRequest;
      bool cache_ok = pos_ok && ri_ok;
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
      // Warm the address translation of the token's cache slots before the bulk stores.
      if (cache_ok) {
        prefetch_l2(p.k_dst + slot * ES);
        prefetch_l2(p.v_dst + slot * ES);
      }
      StagedTokenMeta* m = meta_at(jj);
      m->pos = pos;
      m->slot = slot;
      m->bad = bad;
      m->ok = (table_ok ? kMetaTableOk : 0u) | (cache_ok ? kMetaCacheOk : 0u);
    }
  };

  const uint64_t wait_ns = p.wait_limit_ns > 0 ? static_cast<uint64_t>(p.wait_limit_ns)
                                               : DRK_WAIT_LIMIT_NS;
  int64_t issued = 0;   // tokens whose copies thread 0 has issued
  int64_t skipped = -1; // testing only: the token whose copies were not issued
  // Thread 0: the token's Q, K and V row blocks into its stage (no metadata needed).
  auto issue_load = [&](int64_t j) {
    issued = j + 1;
    const int64_t t = blockIdx.x + j * gridDim.x;
    if (t == p.test_skip_token) {
      skipped = j;        // nothing in flight for it: its stage's wait runs out
      return;
    }
    const int st = static_cast<int>(j % sp.stages);
    unsigned char* stage = smem + static_cast<size_t>(st) * sp.stage_bytes;
    mbar_expect_tx(&bars[st], sp.q_bytes + 2 * sp.kv_bytes);
    bulk_load(stage, p.q + t * p.q_ts * ES, sp.q_bytes, &bars[st]);
    bulk_load(stage + sp.q_bytes, p.k + t * p.k_ts * ES, sp.kv_bytes, &bars[st]);
    bulk_load(stage + sp.q_bytes + sp.kv_bytes, p.v + t * p.v_ts * ES, sp.kv_bytes, &bars[st]);
  };

  // The first two blocks' metadata is never written by the preceding kernel, so it is
  // resolved before waiting on it. Launched as a programmatic dependent, every thread resolves
  // it while the preceding kernel finishes, and thread 0 issues the first copies after the
  // wait. Launched plainly (early_issue), nothing hides that round trip, so thread 0 issues the
  // first stage-full of copies at once while the threads of the other warps resolve the
  // metadata (not warp 0's: its lanes would run their loads only after thread 0's path).
  // Measured on B200 (Mistral-shaped rows, 4096 tokens): either order alone costs 1.4-1.5 us
  // in the other regime. A CTA of fewer than 64 threads always resolves first.
  const int meta_first = (sp.early_issue && nthreads >= 64) ? 32 : 0;
  if (tid == 0) {
    for (int st = 0; st < sp.stages; ++st) mbar_init(&bars[st], 1);
    fence_mbar_init();
    s_abort = 0;
    // The first tokens' Q/K/V row blocks toward L2 while the preceding kernel may still run
    // (launched as a programmatic dependent; otherwise this is simply the first request).
    for (int64_t j = 0; j < my_tokens && j < sp.stages; ++j) {
      const int64_t t = blockIdx.x + j * gridDim.x;
      bulk_prefetch_l2(p.q + t * p.q_ts * ES, sp.q_bytes);
      bulk_prefetch_l2(p.k + t * p.k_ts * ES, sp.kv_bytes);
      bulk_prefetch_l2(p.v + t * p.v_ts * ES, sp.kv_bytes);
    }
    if (meta_first != 0) {
      pdl_wait();    // q/k/v may be written by the preceding kernel
      for (int64_t j = 0; j < my_tokens && j < sp.stages; ++j) issue_load(j);
    }
  }
  fill_meta(0, meta_first);
  if (my_tokens > kStagedMetaBlock) fill_meta(kStagedMetaBlock, meta_first);

  const bool lane_rotates = lane < p.nrot;
  const int off1 = lane * VEC * static_cast<int>(ES);
  const int off2 = off1 + (p.R >> 1) * static_cast<int>(ES);

  // This lane's cos/sin slice of token jj: computed in registers (in-register trig) or loaded
  // a token ahead of its use.
  auto table_slice = [&](int64_t jj, float* c, float* s) {
    const StagedTokenMeta* m = meta_at(jj);
    if (!lane_rotates || !(m->ok & kMetaTableOk)) return;
    const int64_t pos = m->pos;
    if (p.inreg_trig) {
      const float pf = static_cast<float>(pos);
#pragma unroll
      for (int e = 0; e < VEC; ++e) {
        const float ang = __fmul_rn(pf, __ldg(p.inv_freq + lane * VEC + e));
        sincosf(ang, &s[e], &c[e]);
      }
      return;
    }
    const float* crow = p.cos_t + pos * p.table_stride + lane * VEC;
    const float* srow = p.sin_t + pos * p.table_stride + lane * VEC;
    bool vec4 = false;
    if constexpr (VEC % 4 == 0) vec4 = p.table_vec4 != 0;
    if (vec4) {
#pragma unroll
      for (int e = 0; e < VEC; e += 4) {
        const float4 cv = __ldg(reinterpret_cast<const float4*>(crow + e));
        const float4 sv = __ldg(reinterpret_cast<const float4*>(srow + e));
        c[e] = cv.x; c[e + 1] = cv.y; c[e + 2] = cv.z; c[e + 3] = cv.w;
        s[e] = sv.x; s[e + 1] = sv.y; s[e + 2] = sv.z; s[e + 3] = sv.w;
      }
    } else {
#pragma unroll
      for (int e = 0; e < VEC; ++e) { c[e] = __ldg(crow + e); s[e] = __ldg(srow + e); }
    }
  };

  float c_cur[VEC], s_cur[VEC];
#pragma unroll
  for (int e = 0; e < VEC; ++e) c_cur[e] = s_cur[e] = 0.f;
  __syncthreads();   // the barriers are initialised and the first blocks' metadata written
  if (my_tokens > 0) table_slice(0, c_cur, s_cur);
  pdl_wait();        // q/k/v may be written by the preceding kernel
  if (tid == 0 && meta_first == 0) {
    for (int64_t j = 0; j < my_tokens && j < sp.stages; ++j) issue_load(j);
  }

  int64_t j = 0;
  for (; j < my_tokens; ++j) {
    const int64_t t = blockIdx.x + j * gridDim.x;
    const int st = static_cast<int>(j % sp.stages);
    const uint32_t parity = static_cast<uint32_t>((j / sp.stages) & 1);
    unsigned char* stage = smem + static_cast<size_t>(st) * sp.stage_bytes;

    // Every block of metadata but the first two is resolved as the walk enters the block
    // before it (into the array's other half, whose tokens are done): the loads of a whole
    // block share one round trip, and the barriers below order them before their first reader
    // (the next token's table slice, kStagedMetaBlock - 1 tokens later).
    if (j >= kStagedMetaBlock && j % kStagedMetaBlock == 0 && j + kStagedMetaBlock < my_tokens)
      fill_meta(j + kStagedMetaBlock, 0);
    const StagedTokenMeta* curp = meta_at(j);
    const uint32_t cur_ok = curp->ok, cur_bad = curp->bad;
    const int64_t cur_slot = curp->slot;
    const bool table_ok = (cur_ok & kMetaTableOk) != 0;
    // The next token's table slice, in flight while this one is processed.
    float c_nxt[VEC], s_nxt[VEC];
#pragma unroll
    for (int e = 0; e < VEC; ++e) c_nxt[e] = s_nxt[e] = 0.f;
    if (j + 1 < my_tokens) table_slice(j + 1, c_nxt, s_nxt);

    if (!mbar_wait(&bars[st], parity, wait_ns)) {
      atomicOr(&s_abort, 1);
    }
    __syncthreads();
    if (s_abort) break;

    // Rotate the rotary dims of the Q and K rows in place.
    if (lane_rotates && table_ok) {
      for (int r = grp; r < rot_rows; r += blockDim.y) {
        unsigned char* row = stage + static_cast<size_t>(r) * row_bytes;
        Pack<E, VB> x1, x2;
        x1.bits = lds<VB>(row + off1);
        x2.bits = lds<VB>(row + off2);
        rotate_pack<E, VB>(x1, x2, c_cur, s_cur);
        sts<VB>(row + off1, x1.bits);
        sts<VB>(row + off2, x2.bits);
      }
    }
    fence_proxy_async_smem();
    __syncthreads();

    if (tid == 0) {
      if (cur_bad && p.status != nullptr) atomicOr(p.status, cur_bad);
      if (table_ok)
        bulk_store(p.q_out + t * static_cast<int64_t>(sp.q_bytes), stage, sp.q_bytes);
      if (cur_ok & kMetaCacheOk) {
        if (table_ok) bulk_store(p.k_dst + cur_slot * ES, stage + sp.q_bytes, sp.kv_bytes);
        bulk_store(p.v_dst + cur_slot * ES, stage + sp.q_bytes + sp.kv_bytes, sp.kv_bytes);
      }
      bulk_commit();
      // Refill the stage read by the previous token's stores once they have read it.
      if (j >= 1 && j - 1 + sp.stages < my_tokens) {
        bulk_wait_read<1>();
        issue_load(j - 1 + sp.stages);
      }
    }

#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      c_cur[e] = c_nxt[e];
      s_cur[e] = s_nxt[e];
    }
  }

  if (tid == 0) {
    bulk_wait_read<0>();
    if (s_abort) {
      if (p.status != nullptr) atomicOr(p.status, kStatusTimeout);
      // Let copies still landing in this CTA's stages finish before the CTA exits.
      for (int64_t k = j; k < issued; ++k) {
        if (k == skipped) continue;
        mbar_wait(&bars[k % sp.stages], static_cast<uint32_t>((k / sp.stages) & 1), wait_ns);
      }
    }
  }
}

}  // namespace drk
