// Fused RoPE + KV append + decode attention on the 5th-generation tensor cores (tcgen05), for
// 16-bit caches with head_dim 128 or 64: the bandwidth form of rope_kv_attention.cuh.
//
// Work unit: (token t, KV head g, head block hb of up to 16 query heads, chunk of positions).
// A persistent grid (one CTA per SM) takes units from a global atomic counter in the order they
// are numbered (so the chunks and head blocks of one KV head run at about the same time) and
// streams each unit's positions in tiles of 128 through a ring of shared-memory stages (3 deep,
// 6 with 64 dims). Taking units dynamically keeps the CTAs level even though the unit that
// holds the new token, and whichever chunk arrives last and merges, do more work than the
// others.
// Five roles, synchronised by mbarriers only:
//   - warp 4, the producer, takes the units, passes their indices to the other warps through a
//     small queue in shared memory, and refills a stage as soon as the tensor core has finished
//     reading it (an "empty" mbarrier that tcgen05.commit arrives on after the tile's last MMA),
//     so the ring stays full;
//   - warp 6, the aux warp, prepares each unit ahead of the tensor core (the rotated queries
//     into one of two Q buffers, the new token's rotated K and raw V row, the cache-slot append
//     and q_out) and finishes the unit before it (below);
//   - warp 5 issues the QK products (one lane) and patches the new token's row into the tile
//     holding it; warp 7 issues the PV products. Each tcgen05.mma blocks its issuing thread for
//     about as long as the tensor pipe takes to run it, so two issuers keep the pipe fed while
//     the other waits on a barrier;
//   - warps 0-3 (the 128 TMEM lanes) run the softmax and the output correction, and hand each
//     unit's accumulators to the aux warp through shared memory, which writes the unit's
//     output, or its partial, and merges a split KV head's chunks when it sees the last of
//     them arrive.
// So the softmax warps never wait on an MMA issue, a query rotation or a merge.
// Per tile (64 KB: 128 positions of 128 dims, or 256 positions of 64 dims):
//   1. TMA (cp.async.bulk.tensor, 128-byte swizzle) brings the tile's K rows and the V rows of
//      the same positions as boxes of [128 positions][64 dims], completing on the stage's
//      mbarrier;
//   2. one thread issues S^T = K_tile . Q^T on the tensor cores, per 128-position row block
//      (M = 128 positions, N = 16 heads, K = D dims: D / 16 tcgen05.mma of K = 16; A = K rows,
//      K-major; B = the unit's rotated queries, K-major) into TMEM accumulators;
//   3. each softmax thread reads its positions' scores from TMEM (thread = TMEM lane = position
//      within a row block), scales them, masks positions past the unit's end, takes the
//      per-head tile maximum across the consumers, and writes p = 2^(s - m) to shared memory
//      in the storage type (the B operand of the next product, K-major); per-thread partial row
//      sums stay in registers;
//   4. one thread issues O^T = V^T . P^T (M = 128 dims, N = 16 heads, K = the tile's positions;
//      A = the V rows read MN-major, dims past D read from a zero block, B = P) into a second
//      TMEM accumulator;
//   5. each thread (= one dim) reads its head values and folds them into its fp32 accumulator
//      with the online-softmax correction.
// S^T is triple-buffered and O^T and P double-buffered: QKs run up to two tiles ahead of the
// softmax, and a tile's O^T is read after the next tile's softmax. Each tcgen05.mma of these
// shapes holds its issuing thread for ~85-130 cycles whatever N is (the tensor pipe itself is
// active for ~8 of them), so one SM streams ~90 GB/s with 128 dims (16 products per tile) and
// ~45 GB/s with 64 dims (24). Only the HR real heads of a unit (the group size rounded up to a
// power of two, at most 16) go through the softmax; the MMA always runs N = 16 with zero query
// rows.
// At a unit's end the partial (acc, m, l) per head goes to the workspace; the last chunk of a
// (token, KV head, head block) to arrive merges them, exactly as in rope_kv_attention.cuh.
//
// A paged cache ([num_blocks, block_size, Hkv, D] pages and a block table) takes the same kernel:
// a tile is gathered as one TMA box per page slice and lands in shared memory exactly like a
// contiguous tile; entries outside the pool read zeros and set DRK_STATUS_BLOCK_OUT_OF_RANGE.
//
// The new token's rotated K and raw V row is written to the cache slot by head block 0 of the
// unit holding pos and patched into the shared-memory tile that holds pos by every unit that
// reads it, so no unit depends on another's global write (the tile may have been fetched before
// the slot was written).
//
// Waits are bounded (one second of %globaltimer); a wait that runs out -- no valid input
// causes one -- sets DRK_STATUS_TIMEOUT and ends the CTA's walk; the producer waits (bounded)
// for the copies it issued, and the CTA frees its TMEM and returns. No thread-block clusters
// and no cross-CTA waits.
#pragma once

#include <cuda.h>

#include <type_traits>

#include "rope_kv_attention.cuh"
#include "rope_kv_staged.cuh"

namespace drk {

constexpr int kTcThreads = 128;                    // consumers: warps 0-3
constexpr int kTcProducerWarp = 4;
constexpr int kTcMmaWarp = 5;
constexpr int kTcAuxWarp = 6;
constexpr int kTcPvWarp = 7;
// Eight warps: each sub-partition's register file (16K) then holds two warps, so a thread may
// use up to 255 registers.
constexpr int kTcBlock = kTcThreads + 128;         // + producer, QK, aux and PV warps
constexpr int kTcRows = 128;                       // MMA M: positions of S^T, dims of O^T
constexpr int kTcHeads = 16;                       // query heads per unit (MMA N)
constexpr uint32_t kTcBoxBytes = kTcRows * 128;    // [128 rows][64 dims] of 2 bytes: 16 KB
constexpr int kTcStages = 3;
constexpr int kTcSBufs = 3;                        // S^T accumulators in flight

// Tile geometry per head_dim (64 or 128). A tile is 64 KB of K and V rows either way: 128
// positions of 128 dims, or 256 positions of 64 dims, so the softmax, its barrier and the
// output correction are paid once per 64 KB. A stage holds K then V, each as boxes of
// [128 rows][64 dims] (row blocks, then dim halves); Q^T is [D / 64 dim halves][16 heads]
// [128 B]; P is [tile / 64 position quarters][16 heads][128 B]. S^T takes tile / 128
// accumulators of 16 columns (one per 128-position row block), O^T one: three S^T buffers and
// two O^T buffers fill the 128 TMEM columns with 64 dims. O^T = V^T . P^T runs with M = 128
// either way: with 64 dims each product's upper 64 rows are read from a 2 KB zero block after
// the ring (the descriptor's leading-byte offset points there), so the accumulator keeps the
// M = 128 TMEM layout (row i in lane i) and rows 64..127 come out zero.
template <int DIM>
struct TcGeom {
  static_assert(DIM == 64 || DIM == 128, "the tensor-core path takes head_dim 64 or 128");
  static constexpr int kTile = DIM == 64 ? 256 : 128;            // positions per tile
  static constexpr int kRowBlocks = kTile / kTcRows;
  static constexpr int kHalves = DIM / 64;
  static constexpr uint32_t kVOff = kRowBlocks * kHalves * kTcBoxBytes;   // V's offset
  static constexpr uint32_t kStageBytes = 2 * kVOff;
  static constexpr uint32_t kZeroBytes = DIM == 64 ? 2048 : 0;   // two 8-row swizzle atoms
  static constexpr uint32_t kRingBytes = kTcStages * kStageBytes + kZeroBytes;
  static constexpr uint32_t kQBytes = kHalves * kTcHeads * 128;
  static constexpr uint32_t kPBytes = (kTile / 64) * kTcHeads * 128;
  static constexpr uint32_t kSCols = kRowBlocks * kTcHeads;      // columns of an S^T buffer
  static constexpr uint32_t kOCol = kTcSBufs * kSCols;           // first O^T column
  static constexpr uint32_t kTmemCols = 128;
  static_assert(kOCol + 2 * kTcHeads <= kTmemCols, "S^T and O^T exceed the TMEM columns");
};
// Unit queue slots. The producer is at most kTcStages tiles ahead of the MMA warp, the prep
// warp at most two units ahead of it (two Q buffers), the consumers at most two tiles behind it
// and the epilogue warp at most one unit behind the consumers, so fewer than 8 queued units are
// ever unread.
constexpr int kTcQueue = 16;
constexpr int kTcSortMax = 2048;                   // tokens ordered longest-first up to this
constexpr int kTcSortBuckets = 256;                // length buckets of that order

template <int DIM>
struct TcShared {
  using G = TcGeom<DIM>;
  uint8_t ring[G::kRingBytes];                     // stages (K boxes, V boxes), zero block
  uint8_t q[2][G::kQBytes];                        // Q^T operand, double-buffered across units
  uint8_t pm[2][G::kPBytes];                       // P, double-buffered across tiles
  float ep_acc[kTcHeads][DIM];                     // a unit's O accumulators for the epilogue
  float ep_m[kTcHeads];
  float ep_l[kTcHeads];
  float red[2][kTcThreads / 32][kTcHeads];         // per-warp tile maxima, double-buffered
  float lsum[2][kTcThreads / 32][kTcHeads];        // per-warp row sums at a unit's end
  float pend_m[2][kTcHeads];                       // that unit's running maxima
  uint4 kn[2][16];                                 // the new token's K row (storage type)
  uint4 vn[2][16];
  uint64_t full[kTcStages];
  uint64_t empty[kTcStages];
  uint64_t s_bar[kTcSBufs];                        // QK done (tcgen05.commit)
  uint64_t s_free[kTcSBufs];                       // S^T read by the softmax (128 arrivals)
  uint64_t o_bar[2];                               // PV done (tcgen05.commit)
  uint64_t p_bar[2];                               // P written (128 consumer arrivals)
  uint64_t q_full[2];                              // a unit's Q and new K/V row are ready (prep)
  uint64_t q_free[2];                              // its last QK has completed (tcgen05.commit)
  uint64_t ep_full;                                // accumulators handed over (128 arrivals)
  uint64_t ep_empty;                               // the epilogue has read them
  int64_t uq[kTcQueue][3];                         // (unit, position, request) taken by the
                                                   // producer; unit -1 ends the walk
  uint64_t uq_bar[kTcQueue];                       // a queue slot was written (producer)
  uint16_t order[kTcSortMax];                      // tokens, longest first (producer)
  int64_t fin[3];                                  // the CTA's last unit, if it merges
  int fin_merge;
  uint32_t tmem_base;
};
template <int DIM>
constexpr size_t tc_smem_bytes() {
  return sizeof(TcShared<DIM>) + 1024;   // + alignment slack
}

// Shared-memory matrix descriptor (tcgen05): start, leading and stride byte offsets (16-byte
// units), descriptor version 1, swizzle layout in bits 61-63 (2 = 128-byte swizzle).
__device__ __forceinline__ uint64_t tc_sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) |
         (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
         (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor, kind::f16: fp32 accumulator, A/B format (0 fp16, 1 bf16), operand
// majors (0 K-major, 1 MN-major), N >> 3, M >> 4.
__host__ __device__ constexpr uint32_t tc_idesc(uint32_t ab, uint32_t a_mn, uint32_t b_mn,
                                                uint32_t m, uint32_t n) {
  return (1u << 4) | (ab << 7) | (ab << 10) | (a_mn << 15) | (b_mn << 16) | ((n >> 3) << 17) |
         ((m >> 4) << 24);
}

__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u),
      "r"(0u), "r"(0u));
}

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void proxy_fence_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// mbar_wait with a non-blocking first look: a phase that has already completed costs one
// test_wait instead of a try_wait round. Bounded like mbar_wait.
__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0 || mbar_wait(bar, parity);
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Barrier 1 over the 128 consumer threads (the producer warp never joins it).
__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kTcThreads) : "memory");
}
// consumer_sync that also ORs a predicate over the consumers.
__device__ __forceinline__ bool consumer_any(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v)), "n"(kTcThreads)
      : "memory");
  return r != 0;
}

// 32 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tc_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 16 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tc_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int c0, int c1,
                                            int c2, int c3, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2),
      "r"(c3), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_load_5d(void* dst, const CUtensorMap* map, int c0, int c1,
                                            int c2, int c3, int c4, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2),
      "r"(c3), "r"(c4), "r"(smem_u32(bar))
      : "memory");
}

// Byte offset of 16-byte chunk c of row r in a 128-byte-swizzled box (box base 1024-aligned).
__device__ __forceinline__ uint32_t sw128(uint32_t r, uint32_t c) {
  return r * 128u + ((c ^ (r & 7u)) << 4);
}

// One work unit of the CTA's walk, resolved from its linear index.
struct TcUnit {
  int64_t t, ri, pos;
  int g, hb, chunk;
  int64_t p0, p1;      // positions [p0, p1) of this unit
  int ntiles;          // 0: nothing to do (chunk past pos, or invalid indices)
  bool bad;            // invalid position or request index
};

// A unit from its index and its token's position and request index (tiles of TILE positions).
template <int TILE>
__device__ __forceinline__ TcUnit tc_unit_at(const KernelParams& p, const AttentionParams& a,
                                             int64_t u, int64_t pos, int64_t ri) {
  TcUnit w;
  const int64_t per_token_head = static_cast<int64_t>(a.max_chunks) * a.nhb;
  const int64_t tg = u / per_token_head;
  const int64_t rest = u - tg * per_token_head;
  w.chunk = static_cast<int>(rest / a.nhb);
  w.hb = static_cast<int>(rest - static_cast<int64_t>(w.chunk) * a.nhb);
  w.t = tg / p.Hkv;
  w.g = static_cast<int>(tg - w.t * p.Hkv);
  w.pos = pos;
  w.ri = ri;
  w.bad = w.pos < 0 || w.pos >= p.S || w.pos >= p.table_rows || w.ri < 0 || w.ri >= p.B;
  w.p0 = static_cast<int64_t>(w.chunk) * a.chunk;
  w.p1 = w.bad ? w.p0 : min(w.pos + 1, w.p0 + a.chunk);
  w.ntiles = w.p1 > w.p0 ? static_cast<int>((w.p1 - w.p0 + TILE - 1) / TILE) : 0;
  return w;
}

template <int TILE, typename Idx>
__device__ __forceinline__ TcUnit tc_unit(const KernelParams& p, const AttentionParams& a,
                                          int64_t u) {
  const int64_t t = u / (static_cast<int64_t>(a.max_chunks) * a.nhb * p.Hkv);
  return tc_unit_at<TILE>(p, a, u, load_index<Idx>(p.positions, t),
                          load_index<Idx>(p.request_indices, t));
}

template <typename E, typename Idx, int HR, int DIM>
__global__ void __launch_bounds__(kTcBlock, 1)
rope_kv_attention_tc_kernel(const __grid_constant__ KernelParams p,
                            const __grid_constant__ AttentionParams a,
                            const __grid_constant__ CUtensorMap kmap,
                            const __grid_constant__ CUtensorMap vmap, const int64_t units) {
  using raw = typename E::raw;
  using G = TcGeom<DIM>;
  constexpr int kStages = kTcStages;
  constexpr int kTile = G::kTile;
  constexpr uint32_t kAB = std::is_same<E, BF16>::value ? 1u : 0u;
  static_assert(sizeof(raw) == 2, "the tensor-core path takes 16-bit caches");
  static_assert(HR >= 1 && HR <= kTcHeads, "HR real heads per unit, at most the MMA N");
  constexpr uint32_t kIdescQK = tc_idesc(kAB, 0, 0, kTcRows, kTcHeads);
  constexpr uint32_t kIdescPV = tc_idesc(kAB, 1, 0, kTcRows, kTcHeads);

  extern __shared__ uint8_t smem_raw[];
  TcShared<DIM>& sh = *reinterpret_cast<TcShared<DIM>*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int tid = static_cast<int>(threadIdx.x);
  const int warp = tid >> 5, lane = tid & 31;

  pdl_launch_dependents();
  if (tid == kTcProducerWarp * 32) {   // the maps are kernel parameters: fetch them early
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&kmap)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&vmap)) : "memory");
  }
  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sh.full[s], 1);
      mbar_init(&sh.empty[s], 1);
    }
    for (int b = 0; b < kTcSBufs; ++b) {
      mbar_init(&sh.s_bar[b], 1);
      mbar_init(&sh.s_free[b], kTcThreads);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sh.o_bar[b], 1);
      mbar_init(&sh.p_bar[b], kTcThreads);
      mbar_init(&sh.q_full[b], 1);
      mbar_init(&sh.q_free[b], 1);
    }
    mbar_init(&sh.ep_full, kTcThreads);
    mbar_init(&sh.ep_empty, 1);
    for (int i = 0; i < kTcQueue; ++i) mbar_init(&sh.uq_bar[i], 1);
    sh.fin_merge = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // P rows of heads past HR are never written per tile: zero both buffers once; so is the
  // zero block that the upper rows of O^T read with 64 dims.
  for (int i = tid; i < static_cast<int>(2 * G::kPBytes / 16); i += kTcBlock)
    reinterpret_cast<uint4*>(sh.pm)[i] = make_uint4(0u, 0u, 0u, 0u);
  uint8_t* const zero_block = sh.ring + kStages * G::kStageBytes;
  for (int i = tid; i < static_cast<int>(G::kZeroBytes / 16); i += kTcBlock)
    reinterpret_cast<uint4*>(zero_block)[i] = make_uint4(0u, 0u, 0u, 0u);
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_u32(&sh.tmem_base)), "r"(G::kTmemCols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  proxy_fence_shared();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem_base;
  pdl_wait();

  auto stage_at = [&](int s) { return sh.ring + static_cast<uint32_t>(s) * G::kStageBytes; };
  auto stage_of = [&](int64_t c) { return stage_at(static_cast<int>(c % kStages)); };
  // Tile layout in a stage: K in the first half, V in the second, each as 128-byte swizzle
  // atoms of 8 rows x 64 dims. 128 dims, contiguous caches: [half][128 rows] (two 16 KB
  // boxes); paged: [row group][half][8 rows] (one box per page slice). 64 dims, both: [256
  // rows] (two 16 KB boxes, or one per page slice). t_half is the offset of the upper 64 dims,
  // t_group the stride of 8-row groups.
  const bool paged = p.block_table != nullptr;
  const bool interleaved = DIM == 128 && paged;
  const uint32_t t_half = interleaved ? 1024u : kTcBoxBytes;
  const uint32_t t_group = interleaved ? 2048u : 1024u;
  auto full_parity = [&](int64_t c) { return static_cast<uint32_t>((c / kStages) & 1); };
  auto pair_parity = [&](int64_t c) { return static_cast<uint32_t>((c >> 1) & 1); };
  auto sbuf = [&](int64_t c) { return static_cast<int>(c % kTcSBufs); };
  auto s_parity = [&](int64_t c) { return static_cast<uint32_t>((c / kTcSBufs) & 1); };
  // The k-th queued unit index (all lanes of the calling warp poll; -1 ends the walk).
  auto queue_wait = [&](int64_t k) {
    return tc_wait(&sh.uq_bar[k % kTcQueue], static_cast<uint32_t>((k / kTcQueue) & 1));
  };
  const int half_r = p.R >> 1;
  const int row = p.D + 2;

  // Merges every chunk of the unit's (token, KV head, head block): a warp takes heads
  // h_first, h_first + h_step, ...; the (m, l) of 32 chunks at a time go into lanes, then each
  // lane folds its 4 dims of each chunk of the group with the group's loads in flight together.
  auto merge_unit = [&](const TcUnit& w, int h_first, int h_step) {
    __threadfence();
    const int h0 = w.g * a.group + w.hb * kTcHeads;
    const int nh = min(HR, a.group - w.hb * kTcHeads);
    const int nchunks = static_cast<int>((w.pos + a.chunk) / a.chunk);
    const float* ws = a.workspace + (w.t * p.Hq + h0) * static_cast<int64_t>(a.max_chunks) * row;
    const int64_t ws_head = static_cast<int64_t>(a.max_chunks) * row;
    raw* out = reinterpret_cast<raw*>(a.attn_out) + (w.t * p.Hq + h0) * int64_t{DIM};
    constexpr int kPerLane = DIM / 32;   // dims lane + 32 i
    if (h_step == 1 && nchunks <= 32) {
      // One warp, up to 8 heads at a time, with every head's loads in flight together: the
      // (m, l) of chunk `lane` of each head, then chunk by chunk the partial rows of all the
      // heads. The same arithmetic, in the same order per head, as the loop below (whose first
      // pass starts from m = -inf, a rescale of 0).
      constexpr int kG = HR < 8 ? HR : 8;
      for (int hb = 0; hb < nh; hb += kG) {
        float mc[kG], lc[kG], wc[kG], Ls[kG], O[kG][kPerLane];
#pragma unroll
        for (int g = 0; g < kG; ++g) {
          const bool on = hb + g < nh && lane < nchunks;
          const float* hw = ws + (hb + g) * ws_head + static_cast<int64_t>(lane) * row;
          mc[g] = on ? __ldcg(hw + DIM) : -INFINITY;
          lc[g] = on ? __ldcg(hw + DIM + 1) : 0.f;
        }
#pragma unroll
        for (int g = 0; g < kG; ++g) {
          float mg = mc[g];
#pragma unroll
          for (int off = 16; off >= 1; off >>= 1)
            mg = fmaxf(mg, __shfl_xor_sync(0xffffffffu, mg, off));
          wc[g] = (hb + g < nh && lane < nchunks) ? exp2f(mc[g] - mg) : 0.f;
          float lg = lc[g] * wc[g];
#pragma unroll
          for (int off = 16; off >= 1; off >>= 1) lg += __shfl_xor_sync(0xffffffffu, lg, off);
          Ls[g] = lg;
#pragma unroll
          for (int i = 0; i < kPerLane; ++i) O[g][i] = 0.f;
        }
#pragma unroll 2
        for (int j = 0; j < nchunks; ++j) {
#pragma unroll
          for (int g = 0; g < kG; ++g) {
            const float wj = __shfl_sync(0xffffffffu, wc[g], j);
            if (hb + g < nh) {
              const float* cp = ws + (hb + g) * ws_head + static_cast<int64_t>(j) * row + lane;
#pragma unroll
              for (int i = 0; i < kPerLane; ++i) O[g][i] = fmaf(__ldcg(cp + 32 * i), wj, O[g][i]);
            }
          }
        }
#pragma unroll
        for (int g = 0; g < kG; ++g)
          if (hb + g < nh)
#pragma unroll
            for (int i = 0; i < kPerLane; ++i)
              out[(hb + g) * int64_t{DIM} + lane + 32 * i] = E::from_f(O[g][i] / Ls[g]);
      }
      if (lane == 0 && h_first == 0) a.counters[(w.t * p.Hkv + w.g) * a.nhb + w.hb] = 0;
      return;
    }
    for (int h = h_first; h < nh; h += h_step) {
      const float* hw = ws + h * ws_head;
      float M = -INFINITY, Ls = 0.f, O[kPerLane];
#pragma unroll
      for (int i = 0; i < kPerLane; ++i) O[i] = 0.f;
      for (int cb = 0; cb < nchunks; cb += 32) {
        const int c = cb + lane;
        const float mc = c < nchunks ? __ldcg(hw + static_cast<int64_t>(c) * row + DIM)
                                     : -INFINITY;
        const float lc = c < nchunks ? __ldcg(hw + static_cast<int64_t>(c) * row + DIM + 1)
                                     : 0.f;
        float mg = fmaxf(M, mc);
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1)
          mg = fmaxf(mg, __shfl_xor_sync(0xffffffffu, mg, off));
        const float rescale = exp2f(M - mg);
        const float wc = c < nchunks ? exp2f(mc - mg) : 0.f;
        float lg = lc * wc;
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) lg += __shfl_xor_sync(0xffffffffu, lg, off);
        Ls = fmaf(Ls, rescale, lg);
#pragma unroll
        for (int i = 0; i < kPerLane; ++i) O[i] *= rescale;
        const int nc = min(32, nchunks - cb);
#pragma unroll 8
        for (int j = 0; j < nc; ++j) {
          const float wj = __shfl_sync(0xffffffffu, wc, j);
          const float* cp = hw + static_cast<int64_t>(cb + j) * row + lane;
#pragma unroll
          for (int i = 0; i < kPerLane; ++i) O[i] = fmaf(__ldcg(cp + 32 * i), wj, O[i]);
        }
        M = mg;
      }
#pragma unroll
      for (int i = 0; i < kPerLane; ++i)
        out[h * int64_t{DIM} + lane + 32 * i] = E::from_f(O[i] / Ls);
    }
    if (lane == 0 && h_first == 0) a.counters[(w.t * p.Hkv + w.g) * a.nhb + w.hb] = 0;
  };

  if (warp == kTcProducerWarp) {
    // ---- producer: order the tokens longest first, then take units, queue them, and refill
    //      each stage once its last MMA has read it ----
    // Units are handed out in the order of a stable counting sort of the tokens on 256 buckets
    // of position / S, descending, so the grid starts the longest units first and fills the
    // tail with short ones (a longest-processing-time schedule). Every CTA computes the same
    // order. The last stage buffer holds the bucket cursors and keys until its first load.
    const int64_t per_token = static_cast<int64_t>(p.Hkv) * a.nhb * a.max_chunks;
    const bool sorted = p.T > 1 && p.T <= kTcSortMax;
    if (sorted) {
      const int n = static_cast<int>(p.T);
      int* cursor = reinterpret_cast<int*>(stage_at(kStages - 1));
      uint8_t* key = reinterpret_cast<uint8_t*>(cursor + kTcSortBuckets);
      for (int b = lane; b < kTcSortBuckets; b += 32) cursor[b] = 0;
      __syncwarp();
      for (int i = lane; i < n; i += 32) {
        const int64_t pos = load_index<Idx>(p.positions, i);
        const int k = (pos >= 0 && pos < p.S) ? static_cast<int>(pos * kTcSortBuckets / p.S) : 0;
        key[i] = static_cast<uint8_t>(k);
        atomicAdd(&cursor[k], 1);
      }
      __syncwarp();
      // Exclusive prefix over the buckets from the longest down: lane l owns buckets
      // 255 - 8l down to 248 - 8l.
      constexpr int kPer = kTcSortBuckets / 32;
      int cnt[kPer], local = 0;
#pragma unroll
      for (int j = 0; j < kPer; ++j) {
        cnt[j] = cursor[kTcSortBuckets - 1 - kPer * lane - j];
        local += cnt[j];
      }
      int incl = local;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, d);
        if (lane >= d) incl += v;
      }
      int run = incl - local;
#pragma unroll
      for (int j = 0; j < kPer; ++j) {
        cursor[kTcSortBuckets - 1 - kPer * lane - j] = run;
        run += cnt[j];
      }
      __syncwarp();
      // Scatter 32 tokens at a time; lanes with equal keys take consecutive slots in lane
      // order, which keeps the sort stable.
      const uint32_t below = (1u << lane) - 1u;
      for (int i0 = 0; i0 < n; i0 += 32) {
        const int i = i0 + lane;
        const int k = i < n ? key[i] : kTcSortBuckets + lane;   // past-the-end lanes: unique
        const uint32_t grp = __match_any_sync(0xffffffffu, k);
        const int base = i < n ? cursor[k] : 0;
        __syncwarp();
        if (i < n) {
          sh.order[base + __popc(grp & below)] = static_cast<uint16_t>(i);
          if ((grp & below) == 0u) cursor[k] = base + __popc(grp);
        }
        __syncwarp();
      }
      proxy_fence_shared();   // generic writes to the stage before its first TMA load
      __syncwarp();
    }
    // All 32 lanes walk the units: lane 0 takes and queues them; the TMA boxes of a paged
    // tile are issued by as many lanes as there are boxes (one instruction for the K and V
    // boxes of up to 16 page slices), the four boxes of a contiguous tile by lane 0.
    int* next_unit = a.counters + static_cast<int64_t>(p.T) * p.Hkv * a.nhb;
    int64_t issued = 0, queued = 0;
    bool ok = true;
    auto enqueue = [&](int64_t u, int64_t pos, int64_t ri) {   // lane 0
      const int slot = static_cast<int>(queued % kTcQueue);
      sh.uq[slot][0] = u;
      sh.uq[slot][1] = pos;
      sh.uq[slot][2] = ri;
      mbar_arrive(&sh.uq_bar[slot]);
      ++queued;
    };
    // The next unit with work: lane 0 takes it, reporting bad indices on the way, and the
    // warp gets its index, position and request index; t = -1 when none is left. A CTA's
    // first unit is its own index (the grid never exceeds the units); later ones come from
    // the counter, offset by the grid.
    bool first_take = true;
    auto take = [&](int64_t& index) {
      int64_t tu = -1, tpos = 0, tri = 0;
      if (lane == 0) {
        while (true) {
          int64_t u = static_cast<int64_t>(blockIdx.x);
          if (!first_take) {
            const int taken = atomicAdd(next_unit, 1);
            u = static_cast<int64_t>(gridDim.x) + taken;
            // Units gridDim.x.. are taken here once each and every CTA's walk ends with one
            // take past the last unit, so the grid adds `units` times in all: the add that
            // returns units - 1 is the last, and it leaves the counter at zero for the next
            // call on this workspace (a walk cut short by a timeout leaves it set).
            if (taken == static_cast<int>(units) - 1) atomicExch(next_unit, 0);
          }
          first_take = false;
          if (u >= units) break;
          if (sorted) {
            const int64_t r = u / per_token;
            u = static_cast<int64_t>(sh.order[r]) * per_token + (u - r * per_token);
          }
          const TcUnit w = tc_unit<kTile, Idx>(p, a, u);
          if (w.bad) {
            if (w.chunk == 0 && w.hb == 0 && w.g == 0 && p.status != nullptr) {
              uint32_t bad = 0;
              if (w.pos < 0 || w.pos >= p.S) bad |= kStatusPosCache;
              if (w.ri < 0 || w.ri >= p.B) bad |= kStatusRequest;
              if (w.pos < 0 || w.pos >= p.table_rows) bad |= kStatusPosTable;
              atomicOr(p.status, bad);
            }
            continue;
          }
          if (w.ntiles > 0) {
            tu = u;
            tpos = w.pos;
            tri = w.ri;
            break;
          }
        }
      }
      tu = __shfl_sync(0xffffffffu, tu, 0);
      tpos = __shfl_sync(0xffffffffu, tpos, 0);
      tri = __shfl_sync(0xffffffffu, tri, 0);
      index = tu;
      if (tu < 0) return TcUnit{-1, 0, 0, 0, 0, 0, 0, 0, 0, false};
      return tc_unit_at<kTile>(p, a, tu, tpos, tri);
    };
    // Units are queued one ahead of the one being streamed, so the prep warp has a whole
    // unit's time to rotate the next unit's queries.
    int64_t next_index = -1;
    TcUnit next = take(next_index);
    if (lane == 0 && next.t >= 0) enqueue(next_index, next.pos, next.ri);
    while (ok && next.t >= 0) {
      const TcUnit w = next;
      // The unit after w is taken during w's first tile: before the wait for a free stage
      // when the ring is full, after the tile's loads are issued while it is still filling
      // (a CTA's first tiles do not wait for a take).
      bool need_next = true;
      auto take_next = [&]() {
        next = take(next_index);
        if (lane == 0 && next.t >= 0) enqueue(next_index, next.pos, next.ri);
        need_next = false;
      };
      for (int tile = 0; tile < w.ntiles; ++tile) {
        const int s = static_cast<int>(issued % kStages);
        const int64_t z = w.p0 + static_cast<int64_t>(tile) * kTile;
        // Paged cache: box b of the tile holds the K (b even) or V rows of slice b / 2 of the
        // tile, a.box_rows positions (the page size up to 128) that lie in one page, and is
        // issued by lane b % 32 (64 dims: up to 64 boxes, two per lane). A lane loads its
        // slices' block-table entries before the wait for a free stage, so the latency hides
        // behind it. Slice i starts at position z + i * box_rows: page zs / bs, row zs % bs.
        constexpr int64_t kPastTable = INT64_MIN;   // a page past the request's table
        constexpr int kSlots = DIM == 64 ? 2 : 1;   // boxes per lane
        int nbox = 0;
        int64_t blk[kSlots];
        int brow[kSlots];
#pragma unroll
        for (int q = 0; q < kSlots; ++q) {
          blk[q] = kPastTable;
          brow[q] = 0;
          const int b = lane + 32 * q;
          if (p.block_table != nullptr) {
            nbox = kTile / a.box_rows;
            const int64_t zs = z + static_cast<int64_t>(b >> 1) * a.box_rows;
            const int64_t pi = zs / p.block_size;
            brow[q] = static_cast<int>(zs - pi * p.block_size);
            if (b < 2 * nbox && pi < p.bt_stride)
              blk[q] = load_index<Idx>(p.block_table, w.ri * p.bt_stride + pi);
          }
        }
        if (need_next && issued >= kStages) take_next();
        if (issued >= kStages)
          ok = __all_sync(0xffffffffu,
                          tc_wait(&sh.empty[s],
                                  static_cast<uint32_t>(((issued / kStages) + 1) & 1)));
        if (!ok) break;
        uint8_t* st = stage_at(s);
        if (p.block_table == nullptr) {
          if (lane == 0) {
            // Boxes of 128 rows x 64 dims: row blocks, then dim halves.
            mbar_expect_tx(&sh.full[s], G::kStageBytes);
            const int ri = static_cast<int>(w.ri);
#pragma unroll
            for (int rb = 0; rb < G::kRowBlocks; ++rb) {
              const int zi = static_cast<int>(z) + kTcRows * rb;
#pragma unroll
              for (int hf = 0; hf < G::kHalves; ++hf) {
                const uint32_t off = (rb * G::kHalves + hf) * kTcBoxBytes;
                tma_load_4d(st + off, &kmap, 64 * hf, w.g, zi, ri, &sh.full[s]);
                tma_load_4d(st + G::kVOff + off, &vmap, 64 * hf, w.g, zi, ri, &sh.full[s]);
              }
            }
          }
        } else {
          // A slice's box holds its rows' 1024-byte swizzle atoms in the paged tile layout
          // (128 dims: [row group][half][8 rows][128 bytes]; 64 dims: [8 rows][128 bytes] per
          // row group), K at 0 and V at kVOff.
          if (lane == 0) mbar_expect_tx(&sh.full[s], G::kStageBytes);
          __syncwarp();
#pragma unroll
          for (int q = 0; q < kSlots; ++q) {
            const int b = lane + 32 * q;
            if (b >= 2 * nbox) continue;
            const int i = b >> 1, kind = b & 1;
            const int r0 = i * a.box_rows;
            int64_t bk = blk[q];
            if (bk < 0 || bk >= p.num_blocks) {
              // Outside the pool: TMA reads zeros there (coordinate past the last page).
              if (kind == 0 && bk != kPastTable && z + r0 < w.p1 && p.status != nullptr)
                atomicOr(p.status, kStatusBlock);
              bk = p.num_blocks;
            }
            const uint32_t off = static_cast<uint32_t>(kind) * G::kVOff +
                                 static_cast<uint32_t>(r0) * (128u * G::kHalves);
            if constexpr (DIM == 128)
              tma_load_5d(st + off, kind ? &vmap : &kmap, 0, 0, 2 * w.g, brow[q] >> 3,
                          static_cast<int>(bk), &sh.full[s]);
            else
              tma_load_4d(st + off, kind ? &vmap : &kmap, 0, w.g, brow[q],
                          static_cast<int>(bk), &sh.full[s]);
          }
        }
        ++issued;
        if (need_next) take_next();
      }
      if (ok && need_next) take_next();
    }
    if (lane == 0) {
      enqueue(-1, 0, 0);
      if (!ok && p.status != nullptr) atomicOr(p.status, kStatusTimeout);
      // Every copy this CTA issued lands before its shared memory goes away.
      for (int64_t i = issued > kStages ? issued - kStages : 0; i < issued; ++i)
        (void)mbar_wait(&sh.full[i % kStages], static_cast<uint32_t>((i / kStages) & 1));
    }
  } else if (warp == kTcAuxWarp) {
    // ---- aux warp, per queued unit k: prepare unit k, then finish unit k - 1 ----
    // Prep: the unit's rotated queries (Q^T operand, K-major, 128-byte swizzle) and the new
    // token's K/V row into buffer k % 2 once the QKs of unit k - 2 have completed; the
    // cache-slot append (head block 0) and q_out (chunk 0).
    auto prep_unit = [&](int64_t k, const TcUnit& w) {
      const int qb = static_cast<int>(k & 1);
      if (k >= 2 && !__all_sync(0xffffffffu, tc_wait(&sh.q_free[qb],
                                                      static_cast<uint32_t>(((k >> 1) - 1) & 1))))
        return false;
        const int h0 = w.g * a.group + w.hb * kTcHeads;
        const int nh = min(HR, a.group - w.hb * kTcHeads);
        const float* crow = p.cos_t + w.pos * p.table_stride;
        const float* srow = p.sin_t + w.pos * p.table_stride;
        uint8_t* qs = sh.q[qb];
        if (a.q_vec) {
          // Full rotary, 16-byte rows: item = (head, 8-dim chunk of the first half); both halves
          // of the rotate_half pair from one lane. A lane's items share their chunk c (and its
          // cos/sin), for heads lane / kChunks + (32 / kChunks) i; every load is issued before
          // the first store.
          constexpr int kChunks = DIM / 16;                 // 8-dim chunks of a half row
          constexpr int kPasses = kTcHeads * kChunks / 32;  // heads per lane
          const int c = lane % kChunks;
          const float4 c0 = __ldg(reinterpret_cast<const float4*>(crow + 8 * c));
          const float4 c1 = __ldg(reinterpret_cast<const float4*>(crow + 8 * c + 4));
          const float4 s0 = __ldg(reinterpret_cast<const float4*>(srow + 8 * c));
          const float4 s1 = __ldg(reinterpret_cast<const float4*>(srow + 8 * c + 4));
          uint4 xs1[kPasses], xs2[kPasses];
#pragma unroll
          for (int r = 0; r < kPasses; ++r) {
            const int hh = lane / kChunks + (32 / kChunks) * r;
            xs1[r] = xs2[r] = make_uint4(0u, 0u, 0u, 0u);
            if (hh < nh) {
              const raw* qrow = reinterpret_cast<const raw*>(p.q) + w.t * p.q_ts +
                                static_cast<int64_t>(h0 + hh) * p.q_hs;
              xs1[r] = *reinterpret_cast<const uint4*>(qrow + 8 * c);
              xs2[r] = *reinterpret_cast<const uint4*>(qrow + DIM / 2 + 8 * c);
            }
          }
          const float cs[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
          const float sn[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
          for (int r = 0; r < kPasses; ++r) {
            const int hh = lane / kChunks + (32 / kChunks) * r;
            uint4 lo = make_uint4(0u, 0u, 0u, 0u), hi = lo;
            if (hh < nh) {
              float f1[8], f2[8];
              unpack16<E>(xs1[r], f1);
              unpack16<E>(xs2[r], f2);
              uint32_t wl[4], wh[4];
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const int e0 = 2 * i, e1 = 2 * i + 1;
                const raw a0 = E::from_f(rotate_one(f1[e0], f2[e0], cs[e0], sn[e0], true));
                const raw a1 = E::from_f(rotate_one(f1[e1], f2[e1], cs[e1], sn[e1], true));
                const raw b0 = E::from_f(rotate_one(f1[e0], f2[e0], cs[e0], sn[e0], false));
                const raw b1 = E::from_f(rotate_one(f1[e1], f2[e1], cs[e1], sn[e1], false));
                wl[i] = static_cast<uint32_t>(a0) | (static_cast<uint32_t>(a1) << 16);
                wh[i] = static_cast<uint32_t>(b0) | (static_cast<uint32_t>(b1) << 16);
              }
              lo = make_uint4(wl[0], wl[1], wl[2], wl[3]);
              hi = make_uint4(wh[0], wh[1], wh[2], wh[3]);
              if (a.q_out != nullptr && w.chunk == 0) {
                raw* qo =
                    reinterpret_cast<raw*>(a.q_out) + (w.t * p.Hq + h0 + hh) * int64_t{DIM};
                *reinterpret_cast<uint4*>(qo + 8 * c) = lo;
                *reinterpret_cast<uint4*>(qo + DIM / 2 + 8 * c) = hi;
              }
            }
            // Dim d of head hh sits in box d / 64, chunk (d % 64) / 8 of row hh.
            constexpr int kHi = DIM / 2;
            *reinterpret_cast<uint4*>(qs + sw128(hh, c)) = lo;
            *reinterpret_cast<uint4*>(qs + (kHi >> 6) * (kTcHeads * 128) +
                                      sw128(hh, ((kHi & 63) >> 3) + c)) = hi;
          }
        } else {
          for (int idx = lane; idx < kTcHeads * (DIM / 2); idx += 32) {
            const int hh = idx / (DIM / 2);
            const int d = 2 * (idx - hh * (DIM / 2));          // an even dim; pairs d, d + 1
            raw y0 = 0, y1 = 0;
            if (hh < nh) {
              const raw* qrow = reinterpret_cast<const raw*>(p.q) + w.t * p.q_ts +
                                static_cast<int64_t>(h0 + hh) * p.q_hs;
              raw ys[2];
#pragma unroll
              for (int e = 0; e < 2; ++e) {
                const int dd = d + e;
                if (dd < p.R) {
                  const int i = dd < half_r ? dd : dd - half_r;
                  ys[e] = E::from_f(rotate_one(E::to_f(qrow[i]), E::to_f(qrow[i + half_r]),
                                               __ldg(crow + i), __ldg(srow + i), dd < half_r));
                } else {
                  ys[e] = qrow[dd];
                }
              }
              y0 = ys[0];
              y1 = ys[1];
              if (a.q_out != nullptr && w.chunk == 0) {
                raw* qo =
                    reinterpret_cast<raw*>(a.q_out) + (w.t * p.Hq + h0 + hh) * int64_t{DIM};
                qo[d] = y0;
                qo[d + 1] = y1;
              }
            }
            const int box = d >> 6, db = (d & 63) * 2;     // byte within the 128-byte row
            uint8_t* dst = qs + box * (kTcHeads * 128) + sw128(hh, db >> 4) + (db & 15);
            *reinterpret_cast<uint32_t*>(dst) =
                static_cast<uint32_t>(y0) | (static_cast<uint32_t>(y1) << 16);
          }
        }
        if (w.pos < w.p1) {
          const raw* krow = reinterpret_cast<const raw*>(p.k) + w.t * p.k_ts + w.g * p.k_hs;
          const raw* vrow = reinterpret_cast<const raw*>(p.v) + w.t * p.v_ts + w.g * p.v_hs;
          raw* kn = reinterpret_cast<raw*>(sh.kn[qb]);
          raw* vn = reinterpret_cast<raw*>(sh.vn[qb]);
          // The cache slot (through the block table for a paged cache; -1 when that entry is
          // outside the pool, which skips the append and is reported).
          int64_t slot = w.ri * p.c_bs + w.pos * p.c_ss + w.g * p.c_hs;
          if (p.block_table != nullptr) {
            const int64_t blk_i = w.pos / p.block_size;
            const int64_t blk = load_index<Idx>(p.block_table, w.ri * p.bt_stride + blk_i);
            if (blk >= 0 && blk < p.num_blocks) {
              slot = blk * p.c_bs + (w.pos - blk_i * p.block_size) * p.c_ss + w.g * p.c_hs;
            } else {
              slot = -1;
              if (lane == 0 && w.hb == 0 && p.status != nullptr) atomicOr(p.status, kStatusBlock);
            }
          }
          // Dims lane + 32 j: every load is issued before the first store (the cache append
          // could alias the sources as far as the compiler knows).
          constexpr int kPerLane = DIM / 32;
          raw kx[kPerLane], k1[kPerLane], k2[kPerLane], vx[kPerLane];
          float cx[kPerLane], sx[kPerLane];
#pragma unroll
          for (int j = 0; j < kPerLane; ++j) {
            const int d = lane + 32 * j;
            const int i = d < half_r ? d : d - half_r;
            kx[j] = krow[d];
            vx[j] = vrow[d];
            k1[j] = k2[j] = kx[j];
            cx[j] = sx[j] = 0.f;
            if (d < p.R) {
              k1[j] = krow[i];
              k2[j] = krow[i + half_r];
              cx[j] = __ldg(crow + i);
              sx[j] = __ldg(srow + i);
            }
          }
#pragma unroll
          for (int j = 0; j < kPerLane; ++j) {
            const int d = lane + 32 * j;
            raw kr = kx[j];
            if (d < p.R)
              kr = E::from_f(rotate_one(E::to_f(k1[j]), E::to_f(k2[j]), cx[j], sx[j],
                                        d < half_r));
            kn[d] = kr;
            vn[d] = vx[j];
            if (w.hb == 0 && slot >= 0) {
              reinterpret_cast<raw*>(p.k_dst)[slot + d] = kr;
              reinterpret_cast<raw*>(p.v_dst)[slot + d] = vx[j];
            }
          }
        }
        proxy_fence_shared();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sh.q_full[qb]);
      return true;
    };
    // Epilogue: read the unit's accumulators (freeing the hand-over buffer), write its output,
    // or its partial and its arrival; `merge` is set when it arrived last of its chunks.
    auto epilogue_fast = [&](int64_t k, const TcUnit& w, bool& merge) {
      merge = false;
      if (!__all_sync(0xffffffffu, tc_wait(&sh.ep_full, static_cast<uint32_t>(k & 1))))
        return false;
        const int h0 = w.g * a.group + w.hb * kTcHeads;
        const int nh = min(HR, a.group - w.hb * kTcHeads);
        const int nchunks = static_cast<int>((w.pos + a.chunk) / a.chunk);
        constexpr int kPerLane = DIM / 32;   // dims lane + 32 i
        float acc[HR][kPerLane], mh[HR], lh[HR];
#pragma unroll
        for (int h = 0; h < HR; ++h) {
          mh[h] = sh.ep_m[h];
          lh[h] = sh.ep_l[h];
#pragma unroll
          for (int i = 0; i < kPerLane; ++i) acc[h][i] = sh.ep_acc[h][lane + 32 * i];
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&sh.ep_empty);   // the softmax warps may refill the buffer
        raw* out = reinterpret_cast<raw*>(a.attn_out) + (w.t * p.Hq + h0) * int64_t{DIM};
        if (nchunks == 1) {
#pragma unroll
          for (int h = 0; h < HR; ++h)
            if (h < nh)
#pragma unroll
              for (int i = 0; i < kPerLane; ++i)
                out[h * int64_t{DIM} + lane + 32 * i] = E::from_f(acc[h][i] / lh[h]);
          return true;
        }
        float* ws = a.workspace + (w.t * p.Hq + h0) * static_cast<int64_t>(a.max_chunks) * row;
        const int64_t ws_head = static_cast<int64_t>(a.max_chunks) * row;
#pragma unroll
        for (int h = 0; h < HR; ++h) {
          if (h >= nh) continue;
          float* dst = ws + h * ws_head + static_cast<int64_t>(w.chunk) * row;
#pragma unroll
          for (int i = 0; i < kPerLane; ++i) dst[lane + 32 * i] = acc[h][i];
          if (lane == 0) {
            dst[DIM] = mh[h];
            dst[DIM + 1] = lh[h];
          }
        }
        __syncwarp();
        int* counter = a.counters + (w.t * p.Hkv + w.g) * a.nhb + w.hb;
        int last = 0;
        if (lane == 0) {
          __threadfence();
          last = atomicAdd(counter, 1) == nchunks - 1;
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        merge = last != 0;
      return true;
    };
    // Per queued unit k: prepare unit k, then finish unit k - 1 (its merge too, if it
    // arrived last of its chunks).
    // The CTA's last unit, when it arrives last of its chunks, is merged after every role has
    // finished, by all eight warps (a warp per head) instead of this one.
    bool ok = true;
    TcUnit prev{};
    int64_t prev_msg[3] = {0, 0, 0};
    for (int64_t k = 0; ok; ++k) {
      ok = __all_sync(0xffffffffu, queue_wait(k));
      if (!ok) break;
      const int64_t* msg = sh.uq[k % kTcQueue];
      const bool last_unit = msg[0] < 0;
      TcUnit w{};
      if (!last_unit) {
        w = tc_unit_at<kTile>(p, a, msg[0], msg[1], msg[2]);
        ok = prep_unit(k, w);
        if (!ok) break;
      }
      if (k >= 1) {
        bool merge = false;
        ok = epilogue_fast(k - 1, prev, merge);
        if (!ok) break;
        if (merge && last_unit) {
          if (lane == 0) {
            sh.fin[0] = prev_msg[0];
            sh.fin[1] = prev_msg[1];
            sh.fin[2] = prev_msg[2];
            sh.fin_merge = 1;
          }
        } else if (merge) {
          merge_unit(prev, 0, 1);
        }
      }
      if (last_unit) break;
      prev = w;
      prev_msg[0] = msg[0];
      prev_msg[1] = msg[1];
      prev_msg[2] = msg[2];
    }
    if (!ok && lane == 0 && p.status != nullptr) atomicOr(p.status, kStatusTimeout);
  } else if (warp == kTcMmaWarp) {
    // ---- QK issuer: S^T(c) = K . Q^T once tile c has landed and the softmax has read the
    //      S^T buffer's previous tile (c - 3); the tile is patched first if it holds pos ----
    int64_t cj = 0;
    bool ok = true;
    for (int64_t k = 0; ok; ++k) {
      // Wait results are made warp-uniform so the warp never splits at a __syncwarp.
      ok = __all_sync(0xffffffffu, queue_wait(k));
      if (!ok) break;
      const int64_t* msg = sh.uq[k % kTcQueue];
      if (msg[0] < 0) break;
      const TcUnit w = tc_unit_at<kTile>(p, a, msg[0], msg[1], msg[2]);
      const int qb = static_cast<int>(k & 1);
      ok = __all_sync(0xffffffffu, tc_wait(&sh.q_full[qb], static_cast<uint32_t>((k >> 1) & 1)));
      if (!ok) break;
      const bool holds_pos = w.pos < w.p1;
      const uint32_t qaddr = smem_u32(sh.q[qb]);
      for (int j = 0; j < w.ntiles; ++j) {
        const int64_t c = cj + j;
        const int64_t tp0 = w.p0 + static_cast<int64_t>(j) * kTile;
        const bool patch_tile = holds_pos && w.pos >= tp0 && w.pos < tp0 + kTile;
        // Lane 0 alone polls unless every lane is about to write into the tile.
        bool mine = true;
        if (lane == 0 && c >= kTcSBufs)
          mine = tc_wait(&sh.s_free[sbuf(c)], static_cast<uint32_t>(((c / kTcSBufs) - 1) & 1));
        if (mine && (patch_tile || lane == 0))
          mine = tc_wait(&sh.full[c % kStages], full_parity(c));
        ok = __all_sync(0xffffffffu, mine);
        if (!ok) break;
        if (patch_tile) {
          // The new token's K and V row, D / 8 16-byte chunks each, into the staged tile.
          const uint32_t r = static_cast<uint32_t>(w.pos - tp0);
          const int ch = lane & 15;
          const bool is_v = lane >= 16;
          uint8_t* base = stage_of(c) + (is_v ? G::kVOff : 0u);
          const uint32_t at = (r >> 3) * t_group + (ch >> 3) * t_half + sw128(r & 7u, ch & 7);
          if (ch < DIM / 8)
            *reinterpret_cast<uint4*>(base + at) = is_v ? sh.vn[qb][ch] : sh.kn[qb][ch];
          proxy_fence_shared();
          __syncwarp();
        }
        if (lane == 0) {
          tc_fence_after();
          const int b = sbuf(c);
          const uint32_t kb = smem_u32(stage_of(c));
          // One S^T accumulator of 16 columns per 128-position row block of the tile.
#pragma unroll
          for (int rb = 0; rb < G::kRowBlocks; ++rb) {
            const uint32_t kr = kb + rb * (kTcRows / 8) * t_group;
#pragma unroll
            for (int ks = 0; ks < DIM / 16; ++ks) {
              const uint32_t off = static_cast<uint32_t>((ks & 3) * 32);
              const uint64_t ad = tc_sdesc(kr + (ks >> 2) * t_half + off, 16, t_group);
              const uint64_t bd =
                  tc_sdesc(qaddr + (ks >> 2) * (kTcHeads * 128) + off, 16, 1024);
              tc_mma(tmem + b * G::kSCols + rb * kTcHeads, ad, bd, kIdescQK,
                     ks > 0 ? 1u : 0u);
            }
          }
          tc_commit(&sh.s_bar[b]);
          // After the unit's last QK, the prep warp may refill this Q buffer.
          if (j + 1 == w.ntiles) tc_commit(&sh.q_free[qb]);
        }
        __syncwarp();
      }
      cj += w.ntiles;
    }
    if (!ok && lane == 0 && p.status != nullptr) atomicOr(p.status, kStatusTimeout);
  } else if (warp == kTcPvWarp) {
    // ---- PV issuer: O^T(c) = V^T . P^T(c) once the softmax has written P(c); its completion
    //      frees tile c's stage (QK(c) completed before the softmax could write P(c)) ----
    if (lane == 0) {
      int64_t c = 0;
      bool ok = true;
      for (int64_t k = 0; ok; ++k) {
        ok = queue_wait(k);
        if (!ok) break;
        const int64_t* msg = sh.uq[k % kTcQueue];
        if (msg[0] < 0) break;
        const TcUnit w = tc_unit_at<kTile>(p, a, msg[0], msg[1], msg[2]);
        for (int j = 0; j < w.ntiles; ++j, ++c) {
          ok = tc_wait(&sh.p_bar[c & 1], pair_parity(c));
          if (!ok) break;
          tc_fence_after();
          const int b = static_cast<int>(c & 1);
          const uint32_t vb = smem_u32(stage_of(c) + G::kVOff), pb = smem_u32(sh.pm[b]);
          const uint32_t zb = smem_u32(zero_block);
#pragma unroll
          for (int ks = 0; ks < kTile / 16; ++ks) {
            // The second 64-row atom of V^T: the upper dims, or (64 dims) the zero block, the
            // same 16 zero rows for every product: it sits past every stage, so the offset is
            // positive and below 256 KB.
            const uint32_t va = vb + ks * 2 * t_group;
            const uint32_t upper = DIM == 128 ? t_half : zb - va;
            const uint64_t ad = tc_sdesc(va, upper, t_group);
            const uint64_t bd =
                tc_sdesc(pb + (ks >> 2) * (kTcHeads * 128) + (ks & 3) * 32, 16, 1024);
            tc_mma(tmem + G::kOCol + b * kTcHeads, ad, bd, kIdescPV, ks > 0 ? 1u : 0u);
          }
          tc_commit(&sh.o_bar[b]);
          tc_commit(&sh.empty[static_cast<int>(c % kStages)]);
        }
      }
      if (!ok && p.status != nullptr) atomicOr(p.status, kStatusTimeout);
    }
  } else {
    // ---- softmax warps (0-3): scores, P, output correction; hand each unit to the epilogue.
    //      A unit's last O^T is read during the next unit's first tile, so the tile pipeline
    //      runs across unit boundaries. ----
    const uint32_t tmem_lane = static_cast<uint32_t>(warp * 32) << 16;
    int64_t cj = 0;                // tiles of the walk consumed so far
    bool timed_out = false;
    bool ok = true;
    const float scale = a.scale_log2;
    // The previous unit, complete but for its last tile's O^T: its accumulators with the last
    // correction applied (registers), its per-warp row sums and maxima (shared memory, ordered
    // before the hand-over by the next tile's barrier).
    bool pending = false;
    int64_t pend_k = 0, pend_c = 0;
    float pend_acc[HR];
    // O^T buffer ob: this thread's dim for the 16 heads.
    auto read_o = [&](int ob, float* o) {
      tc_ld16(tmem + tmem_lane + G::kOCol + ob * kTcHeads, o);
    };
    // Adds the pending unit's last O^T and hands the unit to the epilogue warp.
    auto hand_over = [&]() {
      ok = tc_wait(&sh.o_bar[pend_c & 1], pair_parity(pend_c)) && ok;
      tc_fence_after();
      float o[kTcHeads];
      read_o(static_cast<int>(pend_c & 1), o);
#pragma unroll
      for (int h = 0; h < HR; ++h) pend_acc[h] += o[h];
      tc_fence_before();
      if (pend_k >= 1) ok = tc_wait(&sh.ep_empty, static_cast<uint32_t>((pend_k - 1) & 1)) && ok;
      if (consumer_any(!ok)) return false;
#pragma unroll
      for (int h = 0; h < HR; ++h) {
        if (tid < DIM) sh.ep_acc[h][tid] = pend_acc[h];   // lanes past D hold zero rows
        if (tid == 0) {
          const int pb = static_cast<int>(pend_k & 1);
          sh.ep_m[h] = sh.pend_m[pb][h];
          sh.ep_l[h] = (sh.lsum[pb][0][h] + sh.lsum[pb][1][h]) +
                       (sh.lsum[pb][2][h] + sh.lsum[pb][3][h]);
        }
      }
      mbar_arrive(&sh.ep_full);
      pending = false;
      return true;
    };

    for (int64_t k = 0; !timed_out; ++k) {
      if (consumer_any(!queue_wait(k))) {
        timed_out = true;
        break;
      }
      const int64_t* msg = sh.uq[k % kTcQueue];
      if (msg[0] < 0) break;
      const TcUnit w = tc_unit_at<kTile>(p, a, msg[0], msg[1], msg[2]);
      const int nh = min(HR, a.group - w.hb * kTcHeads);

      float m_run[HR], lp[HR], acc[HR], corr_prev[HR];
#pragma unroll
      for (int h = 0; h < HR; ++h) {
        m_run[h] = -INFINITY;
        lp[h] = 0.f;
        acc[h] = 0.f;
        corr_prev[h] = 0.f;
      }
      for (int j = 0; j < w.ntiles; ++j) {
        const int64_t c = cj + j;
        const int b = static_cast<int>(c & 1);
        ok = tc_wait(&sh.s_bar[sbuf(c)], s_parity(c)) && ok;
        tc_fence_after();
        // Position rb * 128 + tid of the tile, for each 128-position row block rb.
        float sc[G::kRowBlocks][kTcHeads];
        if constexpr (G::kRowBlocks == 2)
          tc_ld32(tmem + tmem_lane + sbuf(c) * G::kSCols, &sc[0][0]);
        else
          tc_ld16(tmem + tmem_lane + sbuf(c) * G::kSCols, &sc[0][0]);
        tc_fence_before();
        mbar_arrive(&sh.s_free[sbuf(c)]);   // the QK issuer may reuse this S^T buffer
        const int64_t tp0 = w.p0 + static_cast<int64_t>(j) * kTile;
        float mx[HR];
#pragma unroll
        for (int rb = 0; rb < G::kRowBlocks; ++rb) {
          const bool live = tp0 + rb * kTcRows + tid < w.p1;
#pragma unroll
          for (int h = 0; h < HR; ++h) {
            sc[rb][h] = h < nh ? (live ? sc[rb][h] * scale : -INFINITY) : 0.f;
            mx[h] = rb == 0 ? sc[rb][h] : fmaxf(mx[h], sc[rb][h]);
          }
        }
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1)
#pragma unroll
          for (int h = 0; h < HR; ++h)
            mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], off));
        if (lane == 0)
#pragma unroll
          for (int h = 0; h < HR; ++h) sh.red[b][warp][h] = mx[h];
        // One consumer barrier per tile, which also carries the timeout vote.
        if (consumer_any(!ok)) {
          timed_out = true;
          break;
        }
        float corr_cur[HR];
#pragma unroll
        for (int h = 0; h < HR; ++h) {
          const float mt = fmaxf(fmaxf(sh.red[b][0][h], sh.red[b][1][h]),
                                 fmaxf(sh.red[b][2][h], sh.red[b][3][h]));
          const float m_new = fmaxf(m_run[h], mt);
          corr_cur[h] = exp2f(m_run[h] - m_new);
          float es = 0.f;
#pragma unroll
          for (int rb = 0; rb < G::kRowBlocks; ++rb) {
            // P is [position quarter][head][64 positions], K-major for the PV product.
            const int pp = rb * kTcRows + tid, pc = pp & 63;
            uint8_t* pb = sh.pm[b] + (pp >> 6) * (kTcHeads * 128);
            const float e = exp2f(sc[rb][h] - m_new);
            es = rb == 0 ? e : es + e;
            *reinterpret_cast<raw*>(pb + sw128(h, (pc * 2) >> 4) + ((pc * 2) & 15)) =
                E::from_f(e);
          }
          lp[h] = fmaf(lp[h], corr_cur[h], es);
          m_run[h] = m_new;
        }
        // P(c) is ready, and this thread is done with O^T(c - 2).
        proxy_fence_shared();
        tc_fence_before();
        mbar_arrive(&sh.p_bar[b]);
        if (j >= 1) {
          // The previous tile's O^T: its PV ran while this tile's softmax did.
          ok = tc_wait(&sh.o_bar[b ^ 1], pair_parity(c - 1)) && ok;
          tc_fence_after();
          float o[kTcHeads];
          read_o(b ^ 1, o);
#pragma unroll
          for (int h = 0; h < HR; ++h) acc[h] = fmaf(acc[h], corr_prev[h], o[h]);
        } else if (pending && !hand_over()) {
          timed_out = true;
          break;
        }
#pragma unroll
        for (int h = 0; h < HR; ++h) corr_prev[h] = corr_cur[h];
      }
      if (timed_out) break;
      pending = true;
      pend_k = k;
      pend_c = cj + w.ntiles - 1;
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1)
#pragma unroll
        for (int h = 0; h < HR; ++h) lp[h] += __shfl_xor_sync(0xffffffffu, lp[h], off);
#pragma unroll
      for (int h = 0; h < HR; ++h) {
        pend_acc[h] = acc[h] * corr_prev[h];
        // Buffer k % 2: unit k - 1's copy may not have been read yet when a one-tile unit ends.
        if (lane == 0) sh.lsum[k & 1][warp][h] = lp[h];
        if (tid == 0) sh.pend_m[k & 1][h] = m_run[h];
      }
      cj += w.ntiles;
    }
    if (!timed_out && pending && !hand_over()) timed_out = true;
    if (timed_out && tid == 0 && p.status != nullptr) atomicOr(p.status, kStatusTimeout);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(G::kTmemCols) : "memory");
  }
  if (sh.fin_merge) merge_unit(tc_unit_at<kTile>(p, a, sh.fin[0], sh.fin[1], sh.fin[2]), warp,
                               kTcBlock / 32);
}

}  // namespace drk
