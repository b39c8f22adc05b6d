// cu_roaring B200 engine — fused filtered brute-force top-k.
//
// No reference counterpart (the reference only describes feeding
// enumerate_ids into an external SDDMM, README.md:265-285).
//
// One call (cr_filtered_topk), stream-ordered, no host wait:
//   k_pass_words       the shard's pass bitset from the Roaring filter, with
//                      per-256-word counts and the device total
//   k_pass_compact     up to 3/4 pass: indices of the passing rows and a dense
//                      copy of them (TMA-friendly); block 0 writes the plan
//                      (SearchPlan: compacted or dense rows, tiling,
//                      speculative rank)
//   k_topk (prologue)  publish-only tiles: every list's best three scores
//   k_spec             per query, the speculative bound from their union
//   k_topk (main)      the search; rows at or above the query's bound are
//                      appended to per-(query, list) candidate arrays
//   k_merge            per query: radix select of the k-th best, exact rank,
//                      verification of the speculative bound
//   k_redo_gate        the exact per-list search, launched from the device
//                      only when the first pass flagged it
//
// k_topk, one CTA per (128-query tile, database slice), 608 threads:
//   warp 0     TMA producer: the query tile once (A operand, 32 KiB), then
//              database tiles of 256 rows x 128 dims (B operand, 64 KiB)
//              into a 3-stage ring, 128-byte-swizzled K-major tiles
//   warp 1     one thread issues 8 tcgen05.mma (M=128, N=256, K=16, fp16 in,
//              fp32 accumulate) per tile into one of two 256-column TMEM
//              accumulators; tcgen05.commit frees the stage and signals the
//              epilogue
//   warp 2     bound keeper: per query, the minimum over all lists of their
//              published j-th best, raised to the speculative bound, in
//              shared memory
//   warps 3-18 epilogue, one thread per (query, quarter of each tile's
//              rows): one 64-column TMEM load and two 32-row max trees per
//              tile; rows at or above the bound (rare) are appended
//
// Internal score is "larger is better": IP -> q.x; L2 -> 2 q.x - |x|^2
// (distance |q|^2 - score). Ties are broken toward the smaller row id.
#include <cuda.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <vector>

#include "chunk_ops.cuh"
#include "cu_roaring/device/make_view.cuh"
#include "cu_roaring/device/roaring_warp_query.cuh"
#include "tcgen05.cuh"

// The error words of a finished search into its host-visible slot (defined
// with the error ring below; the redo gate tail-launches it).
__global__ void k_export_err(const uint32_t* err0, const uint32_t* err1, uint32_t* slot);

namespace crb {
namespace {

using namespace sm100;

constexpr uint32_t BM = 128;       // queries per CTA (UMMA M, TMEM lanes)
constexpr uint32_t BN = 256;       // database rows per tile (UMMA N)
constexpr uint32_t DIM = 128;      // K
constexpr uint32_t STAGES = 3;
constexpr uint32_t EPI_WARPS = 16;  // four per TMEM lane quarter, each on a quarter of the columns
constexpr uint32_t EPI_PARTS = EPI_WARPS / 4;          // column parts (partial lists per slice)
constexpr uint32_t PART_CHUNKS = (BN / 32) / EPI_PARTS; // 32-row chunks per part
constexpr uint32_t EPI = EPI_WARPS * 32;
constexpr uint32_t BUF = 64;       // candidate buffer entries per (query, half); flushed at >= 32
constexpr uint32_t THREADS = 96 + EPI;  // producer, MMA, bound keeper, 16 epilogue warps
constexpr uint32_t EPI_WARP0 = 3;        // first epilogue warp
constexpr uint32_t KB_BYTES_Q = BM * 128;    // one 64-dim K-block of the query tile
constexpr uint32_t KB_BYTES_DB = BN * 128;   // one 64-dim K-block of a database tile
constexpr uint32_t STAGE_BYTES = 2 * KB_BYTES_DB;
constexpr uint32_t SMEM_Q = 0;
constexpr uint32_t SMEM_DB = SMEM_Q + 2 * KB_BYTES_Q;
constexpr uint32_t SMEM_BUF_S = SMEM_DB + STAGES * STAGE_BYTES;
constexpr uint32_t SMEM_BUF_R = SMEM_BUF_S;
constexpr uint32_t SMEM_BAR = SMEM_BUF_R;
constexpr uint32_t SMEM_BOUND = SMEM_BAR + 128;          // float[BM] + done counter
constexpr uint32_t SMEM_TOTAL = SMEM_BOUND + BM * 4 + 16 + 1024;  // + alignment slack
static_assert(SMEM_TOTAL <= 232448, "shared memory per block");
constexpr uint32_t TMEM_COLS = 512;                     // two 256-column accumulators
constexpr uint32_t kIdesc = idesc_f16_f32(BM, BN);

// The search's shape, decided on the device from the pass count so that the
// host never waits for it: which rows are searched and how they are tiled.
struct SearchPlan {
  uint32_t n_rows;      // rows searched (shard rows when dense, passing rows when compacted)
  uint32_t n_tiles;     // BN-row tiles
  uint32_t tps;         // tiles per slice
  uint32_t dense;       // 1: the shard's rows with the pass bitset; 0: the compacted rows
  uint32_t spec_j;      // rank of the speculative bound in the prologue sample (0: none)
  uint32_t spec_tiles;  // prologue tiles per slice
};

struct TopkParams {
  uint32_t n_queries, k, metric;
  const SearchPlan* plan;
  const uint32_t* pass;  // shard pass bitset (dense plans; null = every row passes)
  const float* norms;    // squared shard row norms (L2, dense plans)
  const float* comp_norms;  // squared norms of the compacted rows (L2, compacted plans)
  const float* chunk_min;   // L2: least squared norm of each 32-row chunk of the searched rows
  const uint32_t* guard; // non-null: run only if this error word has kErrOverflow/kErrSpec set
  uint32_t spec_capable; // the prologue launch and k_spec run before this search
  float* list_s;         // per-query sorted lists: [cta][BM][2][k]
  uint32_t* list_r;
  float* part_s;         // [slice][Q][k] internal scores
  int64_t* part_id;
  uint64_t row_offset;
  uint32_t* err;
  uint32_t* shared_thr;  // [Q] order-preserving bits of the best known k-th score
  uint32_t debug;        // measurement only: 1 = skip the epilogue's score work,
                         // 8 = no database tile loads (MMAs on stale tiles), 9 = both
                         // (7 = the producer loads nothing: every pipeline wait
                         // runs out; failure tests only)
  uint32_t spin_limit;   // polls per pipeline wait before it gives up (kSpinLimit)
  float* buf_s;          // per-CTA candidate buffers: [cta][EPI][BUF] (global, L2-resident)
  uint32_t* buf_r;
  uint32_t* pub;         // [Q][n_lists] published j-th best of every partial list (score keys)
  uint32_t n_lists;      // partial lists per query (2 per slice)
  uint32_t jth;          // ceil(k / n_lists)
  const uint32_t* row_map;  // compacted row -> shard row (compacted plans)
  uint32_t append;       // 1: survivors go to per-query candidate arrays, no list merges
  uint32_t cap;          // candidate slots per (query, list) (append mode)
  uint32_t keeper_ns;    // bound keeper refresh period
  float* cand_s;         // [Q][n_lists][cap]
  uint32_t* cand_r;
  uint32_t* cand_cnt;    // [Q][n_lists] entries appended (may exceed cap: overflow)
  // Speculative bound (append mode, plan spec_j > 0). A prologue launch
  // (prologue_only) runs the publish-only tiles and every list writes its
  // best three scores to pub_top [list * 3 + i][Q]; k_spec turns their union
  // into spec_used [Q]; the main launch starts with that bound and skips its
  // own publish-only tiles. The merge verifies it.
  uint32_t prologue_only;
  uint32_t* pub_top;
  const uint32_t* spec_used;
};

constexpr uint32_t kErrOverflow = 64u;  // a candidate array filled up (append mode)
constexpr uint32_t kErrSpec = 128u;      // a query's speculative bound was above its k-th best
constexpr uint32_t kErrLaunch = 256u;    // the device could not launch the exact redo
constexpr uint32_t kPrologueTiles = 4;  // publish-only tiles at the start of each slice (append mode)

// Order-preserving map float -> uint32 (larger float -> larger key); 0 is
// below every real score and decodes to -inf.
__device__ __forceinline__ uint32_t score_key(float f)
{
  const uint32_t i = __float_as_uint(f);
  return (i & 0x80000000u) ? ~i : (i | 0x80000000u);
}
__device__ __forceinline__ float key_score(uint32_t k)
{
  if (k == 0) return -INFINITY;
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

__device__ __forceinline__ bool better(float as, uint32_t ar, float bs, uint32_t br)
{
  return as > bs || (as == bs && ar < br);
}

// One (score, row) pair held by each lane of a warp.
struct Cand {
  float s;
  uint32_t r;
};

__device__ __forceinline__ Cand shfl_xor(Cand c, int m)
{
  return {__shfl_xor_sync(0xFFFFFFFFu, c.s, m), __shfl_xor_sync(0xFFFFFFFFu, c.r, m)};
}

// Compare-exchange with the lane at distance `stride`: the lower lane keeps
// the better element when `better_low`, else the worse one.
__device__ __forceinline__ Cand cmpx(Cand v, int stride, bool better_low)
{
  const Cand o = shfl_xor(v, stride);
  const bool low = (threadIdx.x & stride) == 0;
  const bool v_better = better(v.s, v.r, o.s, o.r);
  return (low == better_low) == v_better ? v : o;
}

// Warp bitonic sort of 32 candidates, best in lane 0.
__device__ __forceinline__ Cand warp_sort(Cand v)
{
  const uint32_t lane = threadIdx.x & 31;
#pragma unroll
  for (int size = 2; size <= 32; size <<= 1)
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1)
      v = cmpx(v, stride, (lane & size) == 0 || size == 32);
  return v;
}

// Sorts a bitonic 32-sequence across the warp, best in lane 0.
__device__ __forceinline__ Cand warp_bitonic_merge(Cand v)
{
#pragma unroll
  for (int stride = 16; stride > 0; stride >>= 1) v = cmpx(v, stride, true);
  return v;
}

// Merges up to 32 candidates (entries [e0, e1) of one lane's shared buffer)
// into that lane's sorted list, all 32 lanes cooperating: the new entries are
// warp-sorted, then the list is consumed in coalesced 32-entry chunks, each
// bitonically merged with the carried 32 best-not-yet-output candidates.
// Returns the list's new length; *kth gets its k-th entry when full.
__device__ uint32_t warp_merge_into(const float* bs, const uint32_t* br, uint32_t e0, uint32_t e1,
                                    const float* src_s, const uint32_t* src_r, float* dst_s,
                                    uint32_t* dst_r, uint32_t cnt, uint32_t k, Cand* kth,
                                    uint32_t j, Cand* jth)
{
  const uint32_t lane = threadIdx.x & 31;
  const uint32_t total = min(k, cnt + (e1 - e0));
  const uint32_t nch = (total + 31) / 32;  // <= 8 for k <= 256
  // Issue every load first (list chunks and new entries are independent),
  // so the merge pays about one L2 round trip.
  Cand a[8];
#pragma unroll
  for (uint32_t c = 0; c < 8; ++c) {
    a[c] = {-INFINITY, 0xFFFFFFFFu};
    const uint32_t i = c * 32 + lane;
    if (c < nch && i < cnt) a[c] = {__ldcg(src_s + i), __ldcg(src_r + i)};
  }
  Cand b{-INFINITY, 0xFFFFFFFFu};
  if (e0 + lane < e1) b = {__ldcg(bs + e0 + lane), __ldcg(br + e0 + lane)};
  b = warp_sort(b);
#pragma unroll
  for (uint32_t c = 0; c < 8; ++c) {
    if (c >= nch) break;
    const uint32_t i = c * 32 + lane;
    // a[c] is sorted best-first, b reversed -> one bitonic 64-sequence; split it.
    Cand rb{__shfl_sync(0xFFFFFFFFu, b.s, 31 - lane), __shfl_sync(0xFFFFFFFFu, b.r, 31 - lane)};
    const bool a_better = better(a[c].s, a[c].r, rb.s, rb.r);
    Cand top = a_better ? a[c] : rb, bot = a_better ? rb : a[c];
    top = warp_bitonic_merge(top);
    b = warp_bitonic_merge(bot);
    if (i < total) { dst_s[i] = top.s; dst_r[i] = top.r; }
    if (i == k - 1) *kth = top;
    if (i == j - 1) *jth = top;
  }
  return total;
}

// v[j] for a run-time j < 32 without indexing a register array (which would
// put it in local memory): a 5-level select tree on the bits of j.
__device__ __forceinline__ float pick32(const float* v, uint32_t j)
{
  float a[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) a[i] = (j & 16u) ? v[i + 16] : v[i];
#pragma unroll
  for (int w = 8; w >= 1; w >>= 1)
#pragma unroll
    for (int i = 0; i < w; ++i) a[i] = (j & uint32_t(w)) ? a[i + w] : a[i];
  return a[0];
}

// Three-input maximum (sm_100 max.f32 with three sources): a 32-value
// maximum in 16 instructions instead of 31.
__device__ __forceinline__ float fmax3(float a, float b, float c)
{
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

__device__ __forceinline__ float max8(const float* v)
{
  return fmax3(fmax3(v[0], v[1], v[2]), fmax3(v[3], v[4], v[5]), fmaxf(v[6], v[7]));
}

// v[j] for a run-time j < 8 (a 3-level select tree, no local memory).
__device__ __forceinline__ float pick8(const float* v, uint32_t j)
{
  const float a0 = (j & 4u) ? v[4] : v[0], a1 = (j & 4u) ? v[5] : v[1], a2 = (j & 4u) ? v[6] : v[2],
              a3 = (j & 4u) ? v[7] : v[3];
  const float b0 = (j & 2u) ? a2 : a0, b1 = (j & 2u) ? a3 : a1;
  return (j & 1u) ? b1 : b0;
}

__device__ __forceinline__ float max32(const float* v)
{
  float a[12];
#pragma unroll
  for (int j = 0; j < 10; ++j) a[j] = fmax3(v[3 * j], v[3 * j + 1], v[3 * j + 2]);
  a[10] = v[30];
  a[11] = v[31];
  const float b0 = fmax3(a[0], a[1], a[2]), b1 = fmax3(a[3], a[4], a[5]), b2 = fmax3(a[6], a[7], a[8]),
              b3 = fmax3(a[9], a[10], a[11]);
  return fmaxf(fmax3(b0, b1, b2), b3);
}

template <bool APPEND, bool L2>
__global__ void __launch_bounds__(THREADS, 1)
    k_topk(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tdb,
           const __grid_constant__ CUtensorMap tdb_comp, TopkParams p)
{
  // A fallback search runs only when the first pass asked for it.
  if (p.guard && !(*reinterpret_cast<const volatile uint32_t*>(p.guard) & (kErrOverflow | kErrSpec))) return;
  const SearchPlan pl = *p.plan;
  const bool use_spec = APPEND && p.spec_capable && pl.spec_j != 0;
  if (p.prologue_only && !use_spec) return;  // no speculative bound for this plan
  const uint32_t n_rows = pl.n_rows;
  const uint32_t* pass = pl.dense ? p.pass : nullptr;
  const float* norms = pl.dense ? p.norms : p.comp_norms;
  const uint32_t* row_map = pl.dense ? nullptr : p.row_map;
  const CUtensorMap* tdbp = pl.dense ? &tdb : &tdb_comp;
  const uint32_t* spec_used = use_spec ? p.spec_used : nullptr;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sQ = smem + SMEM_Q;
  uint8_t* sDB = smem + SMEM_DB;
  const size_t cta_id = size_t(blockIdx.y) * gridDim.x + blockIdx.x;
  float* buf_s = p.buf_s + cta_id * EPI * BUF;
  uint32_t* buf_r = p.buf_r + cta_id * EPI * BUF;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SMEM_BAR);
  uint64_t* q_full = bars + 0;
  uint64_t* full = bars + 1;                   // [STAGES]
  uint64_t* empty = bars + 1 + STAGES;         // [STAGES]
  uint64_t* acc_full = bars + 1 + 2 * STAGES;  // [2]
  uint64_t* acc_empty = acc_full + 2;          // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  static_assert((1 + 2 * STAGES + 4) * 8 + 8 <= 128, "barrier block");
  float* s_bound = reinterpret_cast<float*>(smem + SMEM_BOUND);
  uint32_t* s_done = reinterpret_cast<uint32_t*>(smem + SMEM_BOUND + BM * 4);

  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t qt = blockIdx.x, slice = blockIdx.y;
  const uint32_t t0 = slice * pl.tps;
  const uint32_t t1 = max(t0, min(pl.n_tiles, t0 + pl.tps));  // slices past the rows get no tiles
  // Tile schedule. In append mode the first D tiles of the slice run first
  // in publish-only mode (their best scores feed the shared bound, nothing is
  // kept), then every tile runs with the bound, those D last.
  const uint32_t T = t1 - t0;
  const uint32_t D = (APPEND && (p.prologue_only || !use_spec))
                         ? min(T, p.prologue_only ? pl.spec_tiles : kPrologueTiles) : 0u;
  const uint32_t n_it = p.prologue_only ? D : T + D;
  auto tile_of = [&](uint32_t it) { return it < T ? t0 + it : t0 + (it - T); };

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (uint32_t s = 0; s < STAGES; ++s) { mbar_init(full + s, 1); mbar_init(empty + s, 1); }
    for (uint32_t a = 0; a < 2; ++a) { mbar_init(acc_full + a, 1); mbar_init(acc_empty + a, EPI_WARPS); }
    fence_mbar_init();
    *s_done = 0;
  }
  // The shared bound starts at the speculative bound when there is one, so
  // the first tiles are filtered before the keeper's first refresh.
  for (uint32_t i = threadIdx.x; i < BM; i += THREADS) {
    const uint32_t q2 = qt * BM + i;
    s_bound[i] = (spec_used && !p.prologue_only && q2 < p.n_queries) ? key_score(__ldcg(spec_used + q2)) : -INFINITY;
  }
  if (warp == 0) tmem_alloc(tmem_slot, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer
    if (lane == 0 && p.debug != 7) {
      prefetch_tmap(&tq);
      prefetch_tmap(tdbp);
      mbar_expect_tx(q_full, 2 * KB_BYTES_Q);
      tma_load_2d(&tq, q_full, sQ, 0, int32_t(qt * BM));
      tma_load_2d(&tq, q_full, sQ + KB_BYTES_Q, 64, int32_t(qt * BM));
      for (uint32_t it = 0; it < n_it; ++it) {
        const uint32_t t = tile_of(it), s = it % STAGES;
        if (!mbar_wait(empty + s, ((it / STAGES) & 1u) ^ 1u, p.err, 1u, p.spin_limit)) break;
        uint8_t* dst = sDB + s * STAGE_BYTES;
        if (p.debug == 8 || p.debug == 9) {  // measurement only: no database loads (stale tiles)
          mbar_arrive(full + s);
          continue;
        }
        mbar_expect_tx(full + s, STAGE_BYTES);
        tma_load_2d(tdbp, full + s, dst, 0, int32_t(t * BN));
        tma_load_2d(tdbp, full + s, dst + KB_BYTES_DB, 64, int32_t(t * BN));
      }
    }
  } else if (warp == 1) {
    // ---------------- UMMA issuer
    if (lane == 0) {
      bool ok = mbar_wait(q_full, 0, p.err, 2u, p.spin_limit);
      const uint32_t aq = smem_addr(sQ);
      for (uint32_t it = 0; it < n_it && ok; ++it) {
        const uint32_t s = it % STAGES, a = it & 1u;
        if (!mbar_wait(full + s, (it / STAGES) & 1u, p.err, 4u, p.spin_limit)) break;
        if (!mbar_wait(acc_empty + a, ((it >> 1) & 1u) ^ 1u, p.err, 8u, p.spin_limit)) break;
        tc_fence_after();
        const uint32_t adb = smem_addr(sDB + s * STAGE_BYTES);
#pragma unroll
        for (uint32_t kk = 0; kk < DIM / 16; ++kk) {
          const uint32_t kb = kk >> 2, ko = (kk & 3u) * 32u;  // K-block, byte offset in 128-B row
          const uint64_t ad = smem_desc_sw128(aq + kb * KB_BYTES_Q + ko);
          const uint64_t bd = smem_desc_sw128(adb + kb * KB_BYTES_DB + ko);
          umma_f16(tmem + a * BN, ad, bd, kIdesc, kk > 0 ? 1u : 0u);
        }
        umma_commit(empty + s);
        umma_commit(acc_full + a);
      }
    }
  } else if (warp == 2) {
    // ---------------- bound keeper: for each query of the tile, the minimum
    // over all partial lists of their published jth best (a lower bound of
    // the k-th best, see the epilogue), kept fresh in shared memory; raised
    // to the speculative bound once that is known.
    float spec[BM / 32];
#pragma unroll
    for (uint32_t i = 0; i < BM / 32; ++i) {
      const uint32_t q2 = qt * BM + lane + 32 * i;
      spec[i] = (spec_used && !p.prologue_only && q2 < p.n_queries) ? key_score(__ldcg(spec_used + q2)) : -INFINITY;
    }
    for (uint32_t iter = 0; iter < kSpinLimit; ++iter) {
#pragma unroll
      for (uint32_t i = 0; i < BM / 32; ++i) {
        const uint32_t qq = lane + 32 * i;
        const uint32_t q2 = qt * BM + qq;
        if (q2 >= p.n_queries) continue;
        uint32_t m0 = 0xFFFFFFFFu, m1 = 0xFFFFFFFFu, m2 = 0xFFFFFFFFu, m3 = 0xFFFFFFFFu;
        uint32_t l = 0;
        for (; l + 4 <= p.n_lists; l += 4) {
          m0 = min(m0, __ldcg(p.pub + size_t(l) * p.n_queries + q2));
          m1 = min(m1, __ldcg(p.pub + size_t(l + 1) * p.n_queries + q2));
          m2 = min(m2, __ldcg(p.pub + size_t(l + 2) * p.n_queries + q2));
          m3 = min(m3, __ldcg(p.pub + size_t(l + 3) * p.n_queries + q2));
        }
        for (; l < p.n_lists; ++l) m0 = min(m0, __ldcg(p.pub + size_t(l) * p.n_queries + q2));
        s_bound[qq] = fmaxf(key_score(min(min(m0, m1), min(m2, m3))), spec[i]);
      }
      if (*reinterpret_cast<volatile uint32_t*>(s_done) >= EPI_WARPS) break;
      __nanosleep(p.keeper_ns);
    }
  } else {
    // ---------------- epilogue: warps 3..18, one thread per (query, quarter of the rows)
    const uint32_t quarter = warp & 3u;               // TMEM lane quarter this warp may access
    const uint32_t chalf = (warp - EPI_WARP0) >> 2;   // which column part (rows of the tile)
    const uint32_t t_local = quarter * 32 + lane;     // query row inside the tile
    const uint32_t e_local = chalf * BM + t_local;    // this thread's (half, query) slot
    const uint32_t qi = qt * BM + t_local;
    const bool valid_q = qi < p.n_queries;
    const size_t cta = size_t(slice) * gridDim.x + qt;
    // This warp's 32 lists: [lane][half][k], contiguous per query.
    float* Lw_s = p.list_s + ((cta * EPI_PARTS + chalf) * BM + quarter * 32) * 2 * p.k;
    uint32_t* Lw_r = p.list_r + ((cta * EPI_PARTS + chalf) * BM + quarter * 32) * 2 * p.k;
    float* mybuf_s = buf_s + e_local * BUF;
    uint32_t* mybuf_r = buf_r + e_local * BUF;
    uint32_t half = 0, cnt = 0, nb = 0, thr_r = 0xFFFFFFFFu;
    float thr_s = -INFINITY;
    constexpr bool l2 = L2;  // the metric is a template parameter: IP code carries no L2 work

    // Warp-cooperative merge of every lane whose buffer holds >= `min_fill`.
    auto flush = [&](uint32_t min_fill) {
      __syncwarp();  // buffer appends (global stores) visible to the whole warp
      uint32_t need = __ballot_sync(0xFFFFFFFFu, nb >= min_fill && nb > 0);
      if (p.debug == 4) { if (nb >= min_fill) nb = 0; need = 0; }
      if (p.debug == 3 && lane == 0 && need) {
        atomicAdd(p.err + 1, __popc(need));
        atomicAdd(p.err + 2, 1u);
      }
      while (need) {
        const uint32_t f = __ffs(need) - 1;
        need &= need - 1;
        const uint32_t f_nb = __shfl_sync(0xFFFFFFFFu, nb, f);
        uint32_t f_cnt = __shfl_sync(0xFFFFFFFFu, cnt, f);
        uint32_t f_half = __shfl_sync(0xFFFFFFFFu, half, f);
        const float* fb_s = buf_s + (chalf * BM + quarter * 32 + f) * BUF;
        const uint32_t* fb_r = buf_r + (chalf * BM + quarter * 32 + f) * BUF;
        float* fl_s = Lw_s + size_t(f) * 2 * p.k;
        uint32_t* fl_r = Lw_r + size_t(f) * 2 * p.k;
        Cand kth{-INFINITY, 0xFFFFFFFFu}, jth{-INFINITY, 0xFFFFFFFFu};
        for (uint32_t e0 = 0; e0 < f_nb; e0 += 32) {
          const uint32_t src = f_half, dst = f_half ^ 1u;
          f_cnt = warp_merge_into(fb_s, fb_r, e0, min(f_nb, e0 + 32), fl_s + src * p.k, fl_r + src * p.k,
                                  fl_s + dst * p.k, fl_r + dst * p.k, f_cnt, p.k, &kth, p.jth, &jth);
          f_half = dst;
          __syncwarp();
        }
        // The lane that wrote entry k-1 (if any) broadcasts the new k-th best.
        const uint32_t owner = (p.k - 1) & 31u;
        kth.s = __shfl_sync(0xFFFFFFFFu, kth.s, owner);
        kth.r = __shfl_sync(0xFFFFFFFFu, kth.r, owner);
        jth.s = __shfl_sync(0xFFFFFFFFu, jth.s, (p.jth - 1) & 31u);
        if (lane == f) {
          if (!(p.jth <= 3) && f_cnt >= p.jth)
            p.pub[size_t(slice * EPI_PARTS + chalf) * p.n_queries + qi] = score_key(jth.s);
          nb = 0;
          cnt = f_cnt;
          half = f_half;
          if (cnt == p.k) {
            thr_s = kth.s;
            thr_r = kth.r;
            atomicMax(p.shared_thr + qi, score_key(thr_s));
          }
        }
      }
    };

    float gthr = -INFINITY;  // bound shared by every slice of this query
    // Best three scores this list has taken in (list + buffer), to publish its
    // jth best every tile when jth <= 3 without waiting for a merge.
    float top1 = -INFINITY, top2 = -INFINITY, top3 = -INFINITY;
    // A main launch after a prologue launch keeps the prologue's published
    // values (valid lower bounds) until this list beats them.
    uint32_t published =
        (use_spec && !p.prologue_only && valid_q) ? __ldcg(p.pub + size_t(slice * EPI_PARTS + chalf) * p.n_queries + qi) : 0u;
    const bool fast_pub = p.jth <= 3;
    const uint32_t my_list = slice * EPI_PARTS + chalf;
    uint32_t nc = 0;  // candidates this (query, list) appended (append mode)
    const size_t cand_base = (size_t(qi) * p.n_lists + my_list) * p.cap;
    for (uint32_t it = 0; it < n_it; ++it) {
      const uint32_t t = tile_of(it), a = it & 1u;
      const bool publish_only = it < D;
      if (valid_q) {
        if (!APPEND) gthr = fmaxf(gthr, key_score(__ldcg(p.shared_thr + qi)));  // written by list merges only
        // Every list holds >= jth entries >= its published jth best, and
        // n_lists * jth >= k: the minimum over lists bounds the k-th best.
        gthr = fmaxf(gthr, reinterpret_cast<volatile float*>(s_bound)[t_local]);
      }
      if (!mbar_wait(acc_full + a, (it >> 1) & 1u, p.err, 16u, p.spin_limit)) break;
      tc_fence_after();
      const uint32_t row0 = t * BN;
      const float bound = fmaxf(gthr, thr_s);
      bool released = false;  // this warp has arrived on acc_empty for this tile
      // Slow path for one 32-row chunk, kept compact (instruction-cache
      // friendly): the lane's candidate rows as a bit mask, then a small loop
      // over the set bits only, each score picked from registers.
      auto slow = [&](const float* v, uint32_t r0, uint32_t m, float lb, bool want) {
        uint32_t c8[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};  // 8 independent OR chains
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          c8[j & 7] |= (v[j] >= lb ? 1u : 0u) << j;
        }
        const uint32_t cm0 = (c8[0] | c8[1]) | (c8[2] | c8[3]);
        uint32_t cm = cm0 | ((c8[4] | c8[5]) | (c8[6] | c8[7]));
        cm = want ? (cm & m) : 0u;
        if (APPEND && !publish_only && p.debug == 3) {
          if (cm) atomicAdd(p.err + 3, __popc(cm));
          if (lane == 0) atomicAdd(p.err + 2, 1u);
        }
#pragma unroll 1
        for (uint32_t x = cm; x; x &= x - 1) {
          const uint32_t j = __ffs(x) - 1;
          const float val = pick32(v, j);
          const uint32_t r = r0 + j;
          if (APPEND) {
            if (!publish_only) {
              if (nc < p.cap) {
                p.cand_s[cand_base + nc] = val;
                p.cand_r[cand_base + nc] = r;
              }
              ++nc;
            }
          } else {
            if (!(val >= gthr && better(val, r, thr_s, thr_r))) continue;
            mybuf_s[nb] = val;
            mybuf_r[nb] = r;
            ++nb;
          }
          // Re-run prologue tiles (it >= T) were already counted in the
          // best three during the prologue; counting them again would let
          // one row stand for two.
          if (fast_pub && it < T && val > top3) {
            if (val > top1) { top3 = top2; top2 = top1; top1 = val; }
            else if (val > top2) { top3 = top2; top2 = val; }
            else { top3 = val; }
          }
        }
      };
      // Candidates among 8 exact scores e[] of rows r0..r0+7 (append mode):
      // every score at or above lb is appended. With `exact_max` (gm is the
      // exact maximum of e) a single candidate's score is gm itself.
      auto group8 = [&](const float* e, uint32_t r0, float lb, bool exact_max, float gm) {
        uint32_t cm = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) cm |= (e[j] >= lb ? 1u : 0u) << j;
        const bool one = exact_max && __popc(cm) == 1;
#pragma unroll 1
        for (uint32_t x = cm; x; x &= x - 1) {
          const uint32_t j = __ffs(x) - 1;
          const float val = one ? gm : pick8(e, j);
          if (nc < p.cap) {
            p.cand_s[cand_base + nc] = val;
            p.cand_r[cand_base + nc] = r0 + j;
          }
          ++nc;
          if (fast_pub && it < T && val > top3) {
            if (val > top1) { top3 = top2; top2 = top1; top1 = val; }
            else if (val > top2) { top3 = top2; top2 = val; }
            else { top3 = val; }
          }
        }
      };
      // Publish-only tiles keep just the list's best three, fed with the
      // maximum of every 32-row chunk (real scores of distinct rows, so each
      // list still holds three rows at or above them).
      auto take_top = [&](float x) {
        if (x > top3) {
          if (x > top1) { top3 = top2; top2 = top1; top1 = x; }
          else if (x > top2) { top3 = top2; top2 = x; }
          else { top3 = x; }
        }
      };
      // Whole-part fast path: every row of the part is searched (no mask, or
      // both of its mask words full).
      const bool whole = APPEND && row0 + BN <= n_rows && (p.debug == 0 || p.debug == 8 || p.debug >= 10) &&
                         (!pass || (__ldg(pass + ((row0 >> 5) + chalf * 2)) & __ldg(pass + ((row0 >> 5) + chalf * 2 + 1))) ==
                                       0xFFFFFFFFu);
      if (whole) {
        // Every row of this part passes: one 64-column TMEM load and one
        // 6-level max tree for the part's two chunks.
        static_assert(PART_CHUNKS == 2, "64-column part");
        float v[64];
        tmem_ld64(tmem + ((quarter * 32u) << 16) + a * BN + chalf * 64, v);
        // The part's scores are in registers: hand the accumulator back to
        // the MMA warp now, so the next-but-one tile's MMAs overlap this
        // warp's selection work.
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acc_empty + a);
        released = true;
        // L2: the internal score is 2 q.x - |x|^2. Publish-only tiles need
        // exact scores of real rows; the other tiles test the bound against
        // 2 max(q.x) - (least |x|^2 of the 32-row chunk), an upper bound of
        // the chunk's best score, and convert a chunk exactly only when that
        // passes (rare), so the common path matches the inner product's.
        const float* nr = norms + row0 + chalf * 64;
        if (l2 && publish_only) {
#pragma unroll
          for (int j = 0; j < 64; ++j) v[j] = 2.f * v[j] - __ldg(nr + j);
        }
        // Maxima of the eight 8-row groups and of the two 32-row halves: a
        // half is opened only when some lane's half maximum reaches the
        // bound, and then only the groups whose maximum reaches it (usually
        // one, holding a single candidate whose score is that maximum).
        float g[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) g[i] = max8(v + 8 * i);
        const float h0 = fmaxf(fmax3(g[0], g[1], g[2]), g[3]), h1 = fmaxf(fmax3(g[4], g[5], g[6]), g[7]);
        if (p.debug == 11) {  // measurement only: TMEM load and max trees, nothing else
          if (h0 == 12345.f && h1 == 12345.f) p.err[3] = 1u;
        } else if (publish_only) {
          if (valid_q) { take_top(h0); take_top(h1); }
        } else {
          const uint32_t ch = (row0 >> 5) + chalf * 2;
          const float cmin0 = l2 ? __ldg(p.chunk_min + ch) : 0.f, cmin1 = l2 ? __ldg(p.chunk_min + ch + 1) : 0.f;
#pragma unroll
          for (uint32_t hh = 0; hh < 2; ++hh) {
            const float cmin = hh ? cmin1 : cmin0;
            const float u = l2 ? 2.f * (hh ? h1 : h0) - cmin : (hh ? h1 : h0);
            const bool want = valid_q && u >= bound && p.debug != 10;
            if (!__any_sync(0xFFFFFFFFu, want)) continue;
#pragma unroll
            for (uint32_t gi = 0; gi < 4; ++gi) {
              const uint32_t gx = 4 * hh + gi;
              const float ug = l2 ? 2.f * g[gx] - cmin : g[gx];
              if (!(want && ug >= bound)) continue;
              float e[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) e[j] = l2 ? 2.f * v[8 * gx + j] - __ldg(nr + 8 * gx + j) : v[8 * gx + j];
              group8(e, row0 + chalf * 64 + 8 * gx, bound, !l2, g[gx]);
            }
          }
        }
      } else {
#pragma unroll 1
        for (uint32_t c = chalf * PART_CHUNKS; c < ((p.debug == 1 || p.debug == 9) ? 0u : (chalf + 1) * PART_CHUNKS); ++c) {
          const uint32_t r0 = row0 + c * 32;
          if (r0 >= n_rows) break;
          uint32_t m = pass ? __ldg(pass + (r0 >> 5)) : 0xFFFFFFFFu;
          const uint32_t left = n_rows - r0;
          if (left < 32) m &= (1u << left) - 1u;
          if (m == 0) continue;
          float v[32];
          tmem_ld32(tmem + ((quarter * 32u) << 16) + a * BN + c * 32, v);
          // L2 as in the whole-part path: exact scores for publish-only
          // tiles, else the chunk's upper bound first and exact scores only
          // when it reaches the bound. Rows past the mask (and n_rows) are
          // never read.
          auto to_l2 = [&]() {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = ((m >> j) & 1u) ? 2.f * v[j] - __ldg(norms + r0 + j) : -INFINITY;
          };
          if (l2 && publish_only) to_l2();
          // Fast path: the best passing score of the chunk against the bound
          // (a 5-level max tree, not a 32-long dependency chain).
          float mx;
          if (m == 0xFFFFFFFFu) {
            mx = max32(v);
          } else {
            float vm[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) vm[j] = ((m >> j) & 1u) ? v[j] : -INFINITY;
            mx = max32(vm);
          }
          if (publish_only) {
            if (valid_q) take_top(mx);
          } else {
            const float u = l2 ? 2.f * mx - __ldg(p.chunk_min + (r0 >> 5)) : mx;
            const bool want = valid_q && u >= bound;
            if (__any_sync(0xFFFFFFFFu, want) && p.debug != 2) {
              if (l2) to_l2();
              slow(v, r0, m, bound, want);
            }
          }
          if (!APPEND) flush(32);  // at most 31 + 32 entries are ever buffered
        }
      }
      if (!released) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acc_empty + a);
      }
      if (APPEND && p.prologue_only && it + 1 == D && valid_q) {
        const size_t base = size_t(my_list) * 3 * p.n_queries + qi;
        p.pub_top[base] = top1 == -INFINITY ? 0u : score_key(top1);
        p.pub_top[base + p.n_queries] = top2 == -INFINITY ? 0u : score_key(top2);
        p.pub_top[base + 2 * size_t(p.n_queries)] = top3 == -INFINITY ? 0u : score_key(top3);
      }
      if (fast_pub && valid_q && p.debug < 10) {
        const float xj = p.jth == 1 ? top1 : (p.jth == 2 ? top2 : top3);
        const uint32_t key = xj == -INFINITY ? 0u : score_key(xj);
        if (key > published) {
          published = key;
          p.pub[size_t(slice * EPI_PARTS + chalf) * p.n_queries + qi] = key;
        }
      }
    }
    if (!APPEND) flush(1);
    if (APPEND && valid_q && !p.prologue_only) {
      p.cand_cnt[size_t(qi) * p.n_lists + my_list] = nc;
      if (nc > p.cap) atomicOr(p.err, kErrOverflow);
    }
    if (lane == 0) atomicAdd(s_done, 1u);
    // Coalesced copy of each lane's final list into this slice's output.
    for (uint32_t f = 0; f < (APPEND ? 0u : 32u); ++f) {
      const uint32_t fq = qt * BM + quarter * 32 + f;
      if (fq >= p.n_queries) break;
      const uint32_t f_cnt = __shfl_sync(0xFFFFFFFFu, cnt, f);
      const uint32_t f_half = __shfl_sync(0xFFFFFFFFu, half, f);
      const float* ls = Lw_s + (size_t(f) * 2 + f_half) * p.k;
      const uint32_t* lr = Lw_r + (size_t(f) * 2 + f_half) * p.k;
      const size_t base = ((size_t(slice) * EPI_PARTS + chalf) * p.n_queries + fq) * p.k;
      for (uint32_t i = lane; i < p.k; i += 32) {
        p.part_s[base + i] = i < f_cnt ? ls[i] : -INFINITY;
        const uint32_t r = i < f_cnt ? lr[i] : 0u;
        p.part_id[base + i] =
            i < f_cnt ? int64_t(row_map ? __ldg(row_map + r) : r) + int64_t(p.row_offset) : int64_t(-1);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, TMEM_COLS);
}

// The search plan from the pass count (`count`, null = every
// shard row passes). Up to 3/4 of the rows passing, the passing rows are compacted and
// searched; otherwise the shard is searched with the pass bitset. Then the
// tiling over `slices`, and the speculative bound's rank: the prologue sees
// about `sample` of the searched rows, and the spec_j-th best of the union
// of every list's best three has fewer than k rows at or above it with
// probability P(Poisson(k * sample / rows) >= spec_j), taken below 1e-9
// (each list's best three only lower the value). spec_override (measurement
// and tests) forces the rank when >= 0; tiles_override the prologue length.
struct PlanArgs {
  uint32_t shard_rows, slices, n_lists, k, spec_capable;
  uint32_t cap_rows;  // the compacted copy holds up to this many rows
  int spec_override, tiles_override;
};
__device__ void make_plan(const uint32_t* count, const PlanArgs a, SearchPlan* plan)
{
  const uint32_t shard_rows = a.shard_rows, slices = a.slices, n_lists = a.n_lists, k = a.k;
  const uint32_t spec_capable = a.spec_capable;
  const int spec_override = a.spec_override, tiles_override = a.tiles_override;
  SearchPlan pl{};
  const uint32_t n_pass = count ? *count : shard_rows;
  pl.dense = (count == nullptr || n_pass > a.cap_rows) ? 1u : 0u;
  pl.n_rows = pl.dense ? shard_rows : n_pass;
  pl.n_tiles = (pl.n_rows + BN - 1) / BN;
  pl.tps = max(1u, (pl.n_tiles + slices - 1) / slices);
  pl.spec_tiles = max(kPrologueTiles, min(24u, pl.tps / 8));  // at most an eighth of a slice
  if (tiles_override > 0) pl.spec_tiles = uint32_t(tiles_override);
  if (spec_capable && pl.n_rows > 0 && 3 * n_lists <= 256) {
    const double sample = double(min(uint64_t(pl.n_rows), uint64_t(slices) * min(pl.tps, pl.spec_tiles) * BN));
    const double f = sample / double(pl.n_rows);
    if (f > 0.5) {
      // Most rows are in the sample: use the union's k-th best, which needs
      // no luck (k distinct rows are at or above it) and is nearly exact.
      if (k <= 3 * n_lists) pl.spec_j = k;
    } else {
      const double lam = double(k) * f;
      // Smallest j >= 1 with P(X >= j) = 1 - P(X < j) below 1e-9, X ~ Poisson(lam).
      double term = exp(-lam), below = 0.0;  // P(X = j), P(X < j)
      uint32_t j = 0;
      for (; j <= 3 * n_lists; ++j) {
        if (j >= 1 && 1.0 - below < 1e-9) break;
        below += term;
        term *= lam / double(j + 1);
      }
      if (j <= 3 * n_lists) pl.spec_j = min(j, k);  // rank k never needs luck
    }
    if (spec_override >= 0) pl.spec_j = min(uint32_t(spec_override), 3 * n_lists);
  }
  *plan = pl;
}

__global__ void k_plan(const uint32_t* count, const PlanArgs a, SearchPlan* plan, uint32_t* err0, uint32_t* err1)
{
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    make_plan(count, a, plan);
    *err0 = 0u;  // this call's error words start clear
    *err1 = 0u;
  }
}

// One warp per query: spec_used[q] = the j-th largest of the n_vals (<= 256)
// published keys pub_top[i][q] (0 when fewer than j are non-zero).
__global__ void __launch_bounds__(128) k_spec(const uint32_t* pub_top, uint32_t n_vals, uint32_t n_queries,
                                              const SearchPlan* plan, uint32_t* spec_used)
{
  const uint32_t q = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (q >= n_queries) return;
  const uint32_t j = plan->spec_j;
  if (j == 0) return;  // no speculative bound: the searches ignore spec_used
  uint32_t v[8];
#pragma unroll
  for (uint32_t e = 0; e < 8; ++e) {
    const uint32_t idx = lane + 32 * e;
    v[e] = idx < n_vals ? __ldg(pub_top + size_t(idx) * n_queries + q) : 0u;
  }
  // Largest key x with at least j keys >= x, one bit at a time.
  uint32_t x = 0;
  for (int bit = 31; bit >= 0; --bit) {
    const uint32_t c = x | (1u << bit);
    uint32_t n = 0;
#pragma unroll
    for (uint32_t e = 0; e < 8; ++e) n += v[e] >= c ? 1u : 0u;
    if (__reduce_add_sync(0xFFFFFFFFu, n) >= j) x = c;
  }
  if (lane == 0) spec_used[q] = x;
}

// L2 only: out[c] = the least squared norm of searched rows [32c, 32c + 32)
// (the plan's rows: the shard's, or the compacted ones), the per-chunk term
// of the epilogue's upper bound 2 max(q.x) - min |x|^2.
__global__ void __launch_bounds__(256) k_chunk_min_norms(const SearchPlan* plan, const float* norms,
                                                         const float* comp_norms, float* out)
{
  const SearchPlan pl = *plan;
  const float* src = pl.dense ? norms : comp_norms;
  const uint32_t n = pl.n_rows, n_chunks = (n + 31) / 32;
  const uint32_t stride = gridDim.x * blockDim.x;
  for (uint32_t c = blockIdx.x * blockDim.x + threadIdx.x; c < n_chunks; c += stride) {
    const uint32_t r1 = min(n, 32 * c + 32);
    float m = INFINITY;
    for (uint32_t r = 32 * c; r < r1; ++r) m = fminf(m, __ldg(src + r));
    out[c] = m;
  }
}

// ------------------------------------------------------------------ merge
constexpr uint32_t MERGE_N = 2048;
constexpr uint32_t MERGE_THREADS = 256;
constexpr uint32_t kMaxListsMerge = 1023;  // partial lists per query in append mode

__device__ __forceinline__ bool better64(float as, int64_t ai, float bs, int64_t bi)
{
  // Valid ids before padding (-1 sorts last on ties at -inf).
  const uint64_t ua = static_cast<uint64_t>(ai), ub = static_cast<uint64_t>(bi);
  return as > bs || (as == bs && ua < ub);
}

// Sorts the first n slots (n a power of two, 2 <= n <= MERGE_N), best first.
__device__ void bitonic_sort(float* s, int64_t* id, uint32_t n = MERGE_N)
{
  for (uint32_t size = 2; size <= n; size <<= 1) {
    for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
      for (uint32_t pr = threadIdx.x; pr < n / 2; pr += MERGE_THREADS) {
        const uint32_t i = (pr / stride) * 2 * stride + (pr % stride), j = i + stride;
        const bool first_better = better64(s[i], id[i], s[j], id[j]);
        const bool want_first_better = (i & size) == 0;
        if (first_better != want_first_better) {
          const float ts = s[i]; s[i] = s[j]; s[j] = ts;
          const int64_t ti = id[i]; id[i] = id[j]; id[j] = ti;
        }
      }
      __syncthreads();
    }
  }
}

// One CTA per query: the best k of `parts` sorted lists. kind 0: inputs are
// internal scores of k_topk; kind 1: inputs are final distances.
__global__ void __launch_bounds__(MERGE_THREADS, 6) k_merge(const float* part_s, const int64_t* part_id,
                                                         uint32_t parts, uint32_t n_queries,
                                                         uint32_t k, int metric, int kind,
                                                         const __half* queries, uint32_t dim,
                                                         float* out_d, int64_t* out_id,
                                                         const uint32_t* cand_cnt, uint32_t cap,
                                                         const uint32_t* cand_r,
                                                         const uint32_t* row_map, uint64_t row_offset,
                                                         const uint32_t* pub, uint32_t n_lists,
                                                         uint32_t n_rows, const uint32_t* spec_used,
                                                         uint32_t* err, const SearchPlan* plan,
                                                         const uint32_t* guard, uint64_t s_stride,
                                                         uint64_t i_stride)
{
  if (guard && !(*reinterpret_cast<const volatile uint32_t*>(guard) & (kErrOverflow | kErrSpec))) return;
  if (plan) {  // a search's candidates: rows and row ids as the plan decided
    n_rows = plan->n_rows;
    if (plan->dense) row_map = nullptr;
    if (plan->spec_j == 0) spec_used = nullptr;
  }
  extern __shared__ uint8_t smem_raw[];
  float* s = reinterpret_cast<float*>(smem_raw);
  int64_t* id = reinterpret_cast<int64_t*>(smem_raw + MERGE_N * 4);
  __shared__ float s_qn;
  const uint32_t q = blockIdx.x;
  const bool l2 = metric == CR_METRIC_L2;
  if (threadIdx.x < 32) {
    float acc = 0.f;
    if (l2 && kind != 1)
      for (uint32_t d = threadIdx.x; d < dim; d += 32) {
        const float x = __half2float(queries[size_t(q) * dim + d]);
        acc += x * x;
      }
#pragma unroll
    for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, o);
    if (threadIdx.x == 0) s_qn = acc;
  }
  // kind 2 (candidate arrays): only candidates at or above the final
  // published bound (min over lists of their jth best) can be in the top k.
  float bound = -INFINITY;
  if (kind == 2 && pub) {
    __shared__ uint32_t s_min;
    if (threadIdx.x == 0) s_min = 0xFFFFFFFFu;
    __syncthreads();
    uint32_t mn = 0xFFFFFFFFu;
    for (uint32_t l = threadIdx.x; l < n_lists; l += MERGE_THREADS) mn = min(mn, pub[size_t(l) * n_queries + q]);
    atomicMin(&s_min, mn);
    __syncthreads();
    bound = key_score(s_min);
  }
  // kind 2 with a speculative bound: rows below it were dropped, which is
  // exact only if the k-th best found is at or above it.
  const uint32_t spec = (kind == 2 && spec_used) ? spec_used[q] : 0u;
  // kind 2: n_lists regions of `cap` slots per query. An overflowed region
  // has unwritten slots; that pass is redone by the caller, so skip it here.
  __shared__ uint32_t s_over;
  if (kind == 2) {
    if (threadIdx.x == 0) s_over = 0;
    __syncthreads();
    for (uint32_t l = threadIdx.x; l < n_lists; l += MERGE_THREADS)
      if (cand_cnt[size_t(q) * n_lists + l] > cap) s_over = 1;
    __syncthreads();
  }
  const uint64_t total = kind == 2 ? (s_over ? 0u : uint64_t(n_lists) * cap) : uint64_t(parts) * k;
  auto load = [&](uint64_t c, uint32_t slot) {
    float v = -INFINITY;
    int64_t i = -1;
    if (kind == 2) {
      if (c < total) {
        const size_t g = size_t(q) * cap + c;
        const float x = part_s[g];
        if (x >= bound) {
          const uint32_t r = cand_r[g];
          v = x;
          i = int64_t(row_map ? __ldg(row_map + r) : r) + int64_t(row_offset);
        }
      }
    } else if (c < total) {
      const uint32_t pidx = static_cast<uint32_t>(c / k), e = static_cast<uint32_t>(c % k);
      const size_t g = size_t(q) * k + e;
      i = part_id[pidx * i_stride + g];
      const float x = part_s[pidx * s_stride + g];
      v = (i < 0) ? -INFINITY : (kind == 0 ? x : (l2 ? -x : x));
    }
    s[slot] = v;
    id[slot] = i;
  };
  // Best k of the n entries in s/id [0, n) (n <= MERGE_N - kSelMax), written
  // to the outputs: radix select of the k-th best score key, then an exact
  // rank (score desc, id asc) of the entries at or above it. False (nothing
  // written) when more than kSelMax entries tie at or above that key.
  constexpr uint32_t kSelMax = MERGE_THREADS;  // selected set ranked one per thread
  __shared__ uint32_t s_hist[256];
  __shared__ uint32_t s_sel[3];
  __shared__ uint32_t s_m;
  __shared__ uint32_t s_ge_spec;
  auto dist_of = [&](float x, int64_t r) {
    if (r < 0) return l2 ? INFINITY : -INFINITY;
    if (!l2) return x;
    return kind != 1 ? s_qn - x : -x;
  };
  // Best k of a set of entries, written to the outputs: radix select of the
  // k-th best score key T (8-bit digits, most significant first), then an
  // exact rank (score desc, id asc) of the entries at or above T. `each(fn)`
  // calls fn(score, id_of) for every entry (all threads, strided); `known_n`
  // is the entry count when known (UINT32_MAX otherwise). False (nothing
  // written) when more than kSelMax entries tie at or above T.
  auto select_k = [&](auto&& each, uint32_t known_n) -> bool {
    uint32_t thr = 0;
    if (known_n > k) {
      uint32_t prefix = 0, mask = 0, rem = k;
      for (int shift = 24; shift >= 0; shift -= 8) {
        for (uint32_t b = threadIdx.x; b < 256; b += MERGE_THREADS) s_hist[b] = 0;
        __syncthreads();
        each([&](float x, auto) {
          const uint32_t key = score_key(x);
          if ((key & mask) == prefix) atomicAdd(&s_hist[(key >> shift) & 255u], 1u);
        });
        __syncthreads();
        if (threadIdx.x < 32) {
          const uint32_t lane = threadIdx.x;
          uint32_t cnt[8], tot = 0;
#pragma unroll
          for (int j = 0; j < 8; ++j) { cnt[j] = s_hist[255 - (8 * lane + j)]; tot += cnt[j]; }
          uint32_t x = tot;
#pragma unroll
          for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, x, o);
            if (lane >= o) x += y;
          }
          // Everything still matching the prefix is selected when it is no
          // more than the rank still wanted.
          const uint32_t matching = __shfl_sync(0xFFFFFFFFu, x, 31);
          if (lane == 0) s_sel[2] = matching <= rem ? 1u : 0u;
          const uint32_t before = x - tot;  // entries in higher digits
          if (matching > rem && before < rem && rem <= x) {
            uint32_t acc = before;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              if (acc + cnt[j] >= rem) {
                s_sel[0] = prefix | (uint32_t(255 - (8 * lane + j)) << shift);
                s_sel[1] = rem - acc;
                break;
              }
              acc += cnt[j];
            }
          }
        }
        __syncthreads();
        if (s_sel[2]) break;  // thr = prefix: every entry at or above it
        prefix = s_sel[0];
        rem = s_sel[1];
        mask |= 255u << shift;
      }
      thr = prefix;
    }
    // Compact key >= T into the tail slots; count the entries at or above a
    // speculative bound (it was safe iff at least k are).
    if (threadIdx.x == 0) { s_m = 0; s_ge_spec = 0; }
    __syncthreads();
    float* cs = s + (MERGE_N - kSelMax);
    int64_t* cid = id + (MERGE_N - kSelMax);
    each([&](float x, auto id_of) {
      if (spec && score_key(x) >= spec) atomicAdd(&s_ge_spec, 1u);
      if (score_key(x) >= thr) {
        const uint32_t slot = atomicAdd(&s_m, 1u);
        if (slot < kSelMax) { cs[slot] = x; cid[slot] = id_of(); }
      }
    });
    __syncthreads();
    if (threadIdx.x == 0 && spec && !s_over && s_ge_spec < k) atomicOr(err, kErrSpec);
    const uint32_t m = s_m;
    if (m <= kSelMax) {
      // Exact rank of each selected entry (score desc, id asc); the best k
      // go straight to their output slots.
      if (threadIdx.x < m) {
        const float x = cs[threadIdx.x];
        const int64_t g = cid[threadIdx.x];
        uint32_t rank = 0;
        for (uint32_t j = 0; j < m; ++j) rank += better64(cs[j], cid[j], x, g) ? 1u : 0u;
        if (rank < k) {
          out_d[size_t(q) * k + rank] = dist_of(x, g);
          out_id[size_t(q) * k + rank] = g;
        }
      }
      for (uint32_t i = m + threadIdx.x; i < k; i += MERGE_THREADS) {
        out_d[size_t(q) * k + i] = l2 ? INFINITY : -INFINITY;
        out_id[size_t(q) * k + i] = -1;
      }
      return true;
    }
    return false;
  };
  // The entries in s/id [0, n) (n <= MERGE_N - kSelMax).
  auto select_out = [&](uint32_t n) -> bool {
    return select_k(
        [&](auto&& fn) {
          for (uint32_t e = threadIdx.x; e < n; e += MERGE_THREADS) fn(s[e], [&] { return id[e]; });
        },
        n);
  };
  if (kind == 2) {
    // Per-list counts -> prefix in shared memory (flattened candidate index
    // -> (list, entry)).
    __shared__ uint32_t s_fill;
    __shared__ uint32_t s_pre[kMaxListsMerge + 1];
    const uint32_t nl = total ? n_lists : 0u;
    if (threadIdx.x < 32) {  // warp scan of the per-list counts, 32 lists per step
      uint32_t carry = 0;
      for (uint32_t l0 = 0; l0 < nl; l0 += 32) {
        const uint32_t l = l0 + threadIdx.x;
        const uint32_t c = l < nl ? cand_cnt[size_t(q) * n_lists + l] : 0u;
        uint32_t x = c;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, x, o);
          if (threadIdx.x >= o) x += y;
        }
        if (l < nl) s_pre[l] = carry + x - c;
        carry += __shfl_sync(0xFFFFFFFFu, x, 31);
      }
      if (threadIdx.x == 0) s_pre[nl] = carry;
    }
    if (threadIdx.x == 0) s_fill = 0;
    __syncthreads();
    const uint32_t n_valid = s_pre[nl];
    // Candidate c: its score and final id; false when below the bound.
    auto fetch = [&](uint32_t c, float& x, int64_t& gid) {
      uint32_t lo = 0, hi = nl;  // last list whose prefix <= c
      while (hi - lo > 1) {
        const uint32_t mid = (lo + hi) >> 1;
        if (s_pre[mid] <= c) lo = mid; else hi = mid;
      }
      const size_t g = (size_t(q) * n_lists + lo) * cap + (c - s_pre[lo]);
      x = part_s[g];
      const uint32_t r = cand_r[g];
      if (!(x >= bound && r < n_rows)) return false;
      gid = int64_t(row_map ? __ldg(row_map + r) : r) + int64_t(row_offset);
      return true;
    };
    // Survivors of the bound into slots [0, MERGE_N); the count may exceed.
    for (uint32_t c = threadIdx.x; c < n_valid; c += MERGE_THREADS) {
      float x;
      int64_t g;
      if (fetch(c, x, g)) {
        const uint32_t slot = atomicAdd(&s_fill, 1u);
        if (slot < MERGE_N) { s[slot] = x; id[slot] = g; }
      }
    }
    __syncthreads();
    const uint32_t n = s_fill;
    __syncthreads();  // every thread has n before the fallback below resets s_fill
    if (n <= MERGE_N - kSelMax && select_out(n)) return;
    if (n > MERGE_N - kSelMax) {
      // More survivors than shared memory holds: select straight from the
      // candidate arrays (one warp per list, lanes over its entries).
      const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
      auto each_candidate = [&](auto&& fn) {
        for (uint32_t l = warp; l < nl; l += MERGE_THREADS / 32) {
          const uint32_t cnt = min(s_pre[l + 1] - s_pre[l], cap);
          const size_t base = (size_t(q) * n_lists + l) * cap;
          for (uint32_t e = lane; e < cnt; e += 32) {
            const float x = part_s[base + e];
            const uint32_t r = cand_r[base + e];
            if (x >= bound && r < n_rows)
              fn(x, [&] { return int64_t(row_map ? __ldg(row_map + r) : r) + int64_t(row_offset); });
          }
        }
      };
      if (select_k(each_candidate, 0xFFFFFFFFu)) return;
    }
    if (n <= MERGE_N) {
      // Too many ties at the k-th score for the rank pass: sort the
      // survivors (already in [0, n)).
      uint32_t n_sort = 2;
      while (n_sort < n) n_sort <<= 1;
      for (uint32_t i = n + threadIdx.x; i < n_sort; i += MERGE_THREADS) { s[i] = -INFINITY; id[i] = -1; }
      __syncthreads();
      bitonic_sort(s, id, n_sort);
    } else {
      // More survivors than shared memory holds: stream them again,
      // compacted into the free slots [k, MERGE_N), sorted when full.
      for (uint32_t i = threadIdx.x; i < MERGE_N; i += MERGE_THREADS) { s[i] = -INFINITY; id[i] = -1; }
      if (threadIdx.x == 0) s_fill = 0;
      __syncthreads();
      constexpr uint32_t B = 2 * MERGE_THREADS;
      for (uint32_t c0 = 0; c0 < n_valid; c0 += B) {
        if (s_fill + B > MERGE_N - k) {
          bitonic_sort(s, id);
          for (uint32_t i = k + threadIdx.x; i < MERGE_N; i += MERGE_THREADS) { s[i] = -INFINITY; id[i] = -1; }
          __syncthreads();
          if (threadIdx.x == 0) s_fill = 0;
          __syncthreads();
        }
        for (uint32_t c = c0 + threadIdx.x; c < min(n_valid, c0 + B); c += MERGE_THREADS) {
          float x;
          int64_t g;
          if (fetch(c, x, g)) {
            const uint32_t slot = k + atomicAdd(&s_fill, 1u);
            s[slot] = x;
            id[slot] = g;
          }
        }
        __syncthreads();
      }
      uint32_t n_sort = 2;
      while (n_sort < k + s_fill) n_sort <<= 1;
      bitonic_sort(s, id, min(n_sort, MERGE_N));
    }
  } else {
    if (total <= MERGE_N - kSelMax) {
      // Valid entries only (padding would tie with padding in the rank pass).
      if (threadIdx.x == 0) s_m = 0;
      __syncthreads();
      for (uint32_t c = threadIdx.x; c < total; c += MERGE_THREADS) {
        const uint32_t pidx = c / k, e = c % k;
        const size_t g = size_t(q) * k + e;
        const int64_t i = part_id[pidx * i_stride + g];
        if (i >= 0) {
          const float x = part_s[pidx * s_stride + g];
          const uint32_t slot = atomicAdd(&s_m, 1u);
          s[slot] = kind == 0 ? x : (l2 ? -x : x);
          id[slot] = i;
        }
      }
      __syncthreads();
      const uint32_t n_ok = s_m;
      __syncthreads();  // every thread has n_ok before select_out resets s_m
      if (select_out(n_ok)) return;
    }
    uint64_t pos = 0;
    for (uint32_t i = threadIdx.x; i < MERGE_N; i += MERGE_THREADS) load(pos + i, i);
    pos += MERGE_N;
    __syncthreads();
    bitonic_sort(s, id);
    while (pos < total) {
      for (uint32_t i = k + threadIdx.x; i < MERGE_N; i += MERGE_THREADS) load(pos + (i - k), i);
      pos += MERGE_N - k;
      __syncthreads();
      bitonic_sort(s, id);
    }
  }
  if (threadIdx.x == 0 && spec && (id[k - 1] < 0 || score_key(s[k - 1]) < spec)) atomicOr(err, kErrSpec);
  const float qn = s_qn;
  for (uint32_t i = threadIdx.x; i < k; i += MERGE_THREADS) {
    const int64_t r = id[i];
    float d;
    if (r < 0) d = l2 ? INFINITY : -INFINITY;
    else if (!l2) d = s[i];
    else d = (kind != 1) ? qn - s[i] : -s[i];
    out_d[size_t(q) * k + i] = d;
    out_id[size_t(q) * k + i] = r;
  }
}

// Shard-local pass bitset: bit i of word w = filter.contains(row_offset + 32w + i).
__global__ void k_pass_bits(cu_roaring::GpuRoaringView v, uint64_t row_offset, uint64_t n_rows,
                            uint32_t* out, uint64_t n_words, uint64_t universe)
{
  const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
  for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n_words * 32; i += stride) {
    const uint64_t id = row_offset + i;
    const bool ok = i < n_rows && id < universe;  // IDs past the universe are never members
    const bool hit = cu_roaring::warp_contains(v, ok ? uint32_t(id) : 0u) && ok;
    const uint32_t bits = __ballot_sync(0xFFFFFFFFu, hit);
    if ((threadIdx.x & 31) == 0) out[i >> 5] = bits;
  }
}

// Same, one thread per output word when row_offset is a multiple of 32 (the
// 32 IDs of a word then share one container): one key lookup per word; a
// BITMAP container gives the word directly, ARRAY and RUN containers are
// searched for the word's 32-ID window.
// 256 threads, one pass word each; the block's popcount lands in
// tile_sums[block] and is added to *count.
__global__ void __launch_bounds__(256) k_pass_words(DevBitmap b, uint64_t row_offset, uint64_t n_rows,
                                                    uint32_t* out, uint64_t n_words, uint32_t* tile_sums,
                                                    uint32_t* err0, uint32_t* err1, uint4* zero,
                                                    uint64_t zero_vec)
{
  if (blockIdx.x == 0 && threadIdx.x == 0) {  // this call's error words start clear
    *err0 = 0u;
    *err1 = 0u;
  }
  // The search's counters and published bounds start at zero (null: the
  // caller clears them).
  for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; zero && i < zero_vec;
       i += uint64_t(gridDim.x) * blockDim.x)
    zero[i] = make_uint4(0u, 0u, 0u, 0u);
  __shared__ uint32_t s_red[32];
  const uint64_t w = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const uint64_t id0 = row_offset + w * 32;
  uint32_t bits = 0;
  if (w < n_words && id0 <= 0xFFFFFFFFull) {
    const uint32_t key = uint32_t(id0 >> 16), low0 = uint32_t(id0 & 0xFFFFu);
    const ContainerRef c = dev_container(b, dev_lookup(b, key));
    if (c.idx >= 0) {
      if (c.type == kBitmap) {
        bits = __ldg(reinterpret_cast<const uint32_t*>(b.bitmap + (c.off >> 3)) + (low0 >> 5));
      } else if (c.type == kArray) {
        const uint16_t* a = b.array + (c.off >> 1);
        uint32_t lo = 0, hi = c.card;  // first element >= low0
        while (lo < hi) {
          const uint32_t mid = (lo + hi) >> 1;
          if (__ldg(a + mid) < low0) lo = mid + 1; else hi = mid;
        }
        for (uint32_t i = lo; i < c.card; ++i) {
          const uint32_t v = __ldg(a + i);
          if (v >= low0 + 32) break;
          bits |= 1u << (v - low0);
        }
      } else {
        const uint16_t* r = b.run + (c.off >> 1);
        uint32_t lo = 0, hi = c.card;  // first run ending at or after low0
        while (lo < hi) {
          const uint32_t mid = (lo + hi) >> 1;
          if (uint32_t(__ldg(r + 2 * mid)) + __ldg(r + 2 * mid + 1) < low0) lo = mid + 1; else hi = mid;
        }
        for (uint32_t i = lo; i < c.card; ++i) {
          const uint32_t st = __ldg(r + 2 * i), en = st + __ldg(r + 2 * i + 1);
          if (st >= low0 + 32) break;
          const uint32_t a0 = max(st, low0) - low0, a1 = min(en, low0 + 31) - low0;
          bits |= (a1 == 31 ? 0xFFFFFFFFu : ((1u << (a1 + 1)) - 1u)) & ~((1u << a0) - 1u);
        }
      }
    }
  }
  if (b.negated) bits = ~bits;
  // IDs at or past the universe are never members; rows past n_rows are cleared.
  const uint64_t U = b.universe;
  for (uint32_t j = 0; j < 32; ++j) {
    const uint64_t id = id0 + j;
    if (w * 32 + j >= n_rows || id >= U) bits &= ~(1u << j);
  }
  if (w < n_words) out[w] = bits;
  const uint32_t t = block_sum<256>(uint32_t(__popc(w < n_words ? bits : 0u)), s_red);
  if (threadIdx.x == 0) tile_sums[blockIdx.x] = t;
}

// Squared norms, 16 lanes per 128-dim row (16 bytes each).
__global__ void k_row_norms(const uint4* db, uint64_t n_rows, float* out)
{
  const uint64_t g = (uint64_t(blockIdx.x) * blockDim.x + threadIdx.x);
  const uint64_t row = g >> 4;
  const uint32_t sub = threadIdx.x & 15;
  float acc = 0.f;
  if (row < n_rows) {
    const uint4 x = __ldcs(db + row * 16 + sub);
    const __half2* h = reinterpret_cast<const __half2*>(&x);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(h[i]);
      acc += f.x * f.x + f.y * f.y;
    }
  }
#pragma unroll
  for (int o = 8; o; o >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, o);
  if (row < n_rows && sub == 0) out[row] = acc;
}

// -------------------------------------------------- pre-filter compaction
constexpr uint32_t kWordTile = 256;  // pass words per block of the count and compaction kernels

__global__ void __launch_bounds__(kWordTile) k_pass_tile_sums(const uint32_t* pass, uint64_t n_words,
                                                              uint32_t* tile_sums, uint32_t* err0, uint32_t* err1)
{
  if (blockIdx.x == 0 && threadIdx.x == 0) {  // this call's error words start clear
    *err0 = 0u;
    *err1 = 0u;
  }
  __shared__ uint32_t s_red[32];
  const uint64_t w = uint64_t(blockIdx.x) * kWordTile + threadIdx.x;
  const uint32_t c = w < n_words ? __popc(pass[w]) : 0u;
  const uint32_t t = block_sum<kWordTile>(c, s_red);
  if (threadIdx.x == 0) tile_sums[blockIdx.x] = t;
}

// idx[] = shard rows whose filter bit is set, ascending; *total = count.
// Nothing is written when the count exceeds cap_rows (the plan then searches
// the shard densely).
// With `comp`, the block then copies its rows: comp[i] = db[idx[i]]
// (16 threads x 16 B per 128-dim row), so the gather needs no launch of its
// own and starts as soon as the block's indices are known.
constexpr uint32_t kCompactThreads = 1024;  // threads past the word tile only copy rows
__global__ void __launch_bounds__(kCompactThreads) k_pass_compact(const uint32_t* pass, uint64_t n_words,
                                                            const uint32_t* tile_sums, uint32_t n_tiles,
                                                            uint32_t* idx, uint32_t* total,
                                                            const float* norms, float* comp_norms,
                                                            const uint4* db, uint4* comp, uint32_t cap_rows,
                                                            const PlanArgs pa, SearchPlan* plan)
{
  __shared__ uint32_t s_red[32];
  // Rows of the earlier word tiles: the block's first output slot.
  uint32_t before = 0, all = 0;
  for (uint32_t j = threadIdx.x; j < n_tiles; j += kCompactThreads) {
    const uint32_t c = tile_sums[j];
    if (j < blockIdx.x) before += c;
    all += c;
  }
  const uint32_t base = block_sum<kCompactThreads>(before, s_red);
  const uint32_t everything = block_sum<kCompactThreads>(all, s_red);
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    *total = everything;
    make_plan(&everything, pa, plan);  // the pass count is final: plan here
  }
  if (everything > cap_rows) return;  // dense plan: the shard is searched with the bitset
  const uint64_t w = uint64_t(blockIdx.x) * kWordTile + threadIdx.x;
  uint32_t x = (threadIdx.x < kWordTile && w < n_words) ? pass[w] : 0u;
  uint32_t tot;
  uint32_t pos = base + block_exclusive_scan<kCompactThreads>(uint32_t(__popc(x)), s_red, &tot);
  while (x) {
    const uint32_t r = uint32_t(w * 32 + __ffs(x) - 1);
    idx[pos] = r;
    if (norms) comp_norms[pos] = __ldg(norms + r);
    ++pos;
    x &= x - 1;
  }
  if (!comp) return;
  __syncthreads();  // the block's idx[] entries are visible to all its threads
  const uint32_t n16 = tot * 16;
  constexpr uint32_t U = 4;  // independent row loads in flight per thread
  for (uint32_t i0 = 0; i0 < n16; i0 += kCompactThreads * U) {
    uint4 v[U];
    uint32_t dst[U];
#pragma unroll
    for (uint32_t u = 0; u < U; ++u) {
      const uint32_t i = i0 + u * kCompactThreads + threadIdx.x;
      dst[u] = i < n16 ? base * 16 + i : 0xFFFFFFFFu;
      if (i < n16) v[u] = __ldcs(db + uint64_t(idx[base + i / 16]) * 16 + (i & 15));
    }
#pragma unroll
    for (uint32_t u = 0; u < U; ++u)
      if (dst[u] != 0xFFFFFFFFu) comp[size_t(dst[u])] = v[u];
  }
}

// ------------------------------------------------------------------- host

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn()
{
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  if (!fn) fail(CR_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
  return fn;
}

// Row-major fp16 matrix [rows x 128] as 2-D tiles of 64 dims x box_rows,
// 128-byte swizzle (the layout the UMMA descriptors expect).
CUtensorMap make_map(const void* base, uint64_t rows, uint32_t box_rows)
{
  CUtensorMap m;
  const cuuint64_t dims[2] = {DIM, rows};
  const cuuint64_t strides[1] = {DIM * 2};
  const cuuint32_t box[2] = {64, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims,
                                 strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                 CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) fail(CR_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string(int(r)));
  return m;
}

void merge_launch(const float* ps, const int64_t* pid, uint32_t parts, uint32_t nq, uint32_t k,
                  int metric, int kind, const __half* queries, uint32_t dim, float* od, int64_t* oi,
                  cudaStream_t s, const uint32_t* cand_cnt = nullptr, uint32_t cap = 0,
                  const uint32_t* cand_r = nullptr, const uint32_t* row_map = nullptr,
                  uint64_t row_offset = 0, const uint32_t* pub = nullptr, uint32_t n_lists = 0,
                  uint32_t n_rows = 0, const uint32_t* spec_used = nullptr, uint32_t* err = nullptr,
                  const SearchPlan* plan = nullptr, const uint32_t* guard = nullptr, uint64_t s_stride = 0,
                  uint64_t i_stride = 0)
{
  // Lists of part p: scores at ps + p * s_stride, ids at pid + p * i_stride
  // (elements; default: parts packed back to back as [parts][nq][k]).
  if (!s_stride) s_stride = uint64_t(nq) * k;
  if (!i_stride) i_stride = uint64_t(nq) * k;
  const size_t smem = MERGE_N * 12;
  set_max_dynamic_smem(reinterpret_cast<const void*>(k_merge), int(smem));
  ProfileScope prof(CR_KERNEL_TOPK_MERGE, s);
  k_merge<<<nq, MERGE_THREADS, smem, s>>>(ps, pid, parts, nq, k, metric, kind, queries, dim, od, oi,
                                          cand_cnt, cap, cand_r, row_map, row_offset, pub, n_lists, n_rows,
                                          spec_used, err, plan, guard, s_stride, i_stride);
  CR_CUDA(cudaGetLastError());
}

// The exact redo (per-list merging: no candidate capacity, no speculative
// bound) launched from the device, and only when the first pass flagged an
// overflowing candidate array or a speculative bound above some query's k-th
// best: one block checks the flag, zeroes the redo's counters and tail-launches
// the search and its merge (they run, in order, once this block has finished).
// `slot` (host-visible, may be null) receives both passes' error words once
// the call's work is done: here when no redo runs, else from a tail launch
// after the redo's search and merge.
__global__ void __launch_bounds__(1024) k_redo_gate(const uint32_t* guard, uint32_t* zero, uint64_t zero_words,
                                                    uint32_t* err, dim3 grid, const __grid_constant__ CUtensorMap tq,
                                                    const __grid_constant__ CUtensorMap tdb,
                                                    const __grid_constant__ CUtensorMap tcomp, TopkParams tp,
                                                    uint32_t n_lists, const __half* queries, float* out_d,
                                                    int64_t* out_id, uint32_t* slot)
{
  if (!(*reinterpret_cast<const volatile uint32_t*>(guard) & (kErrOverflow | kErrSpec))) {
    if (slot && threadIdx.x == 0) {
      slot[0] = *reinterpret_cast<const volatile uint32_t*>(guard);
      slot[1] = *reinterpret_cast<const volatile uint32_t*>(err);
    }
    return;
  }
  for (uint64_t i = threadIdx.x; i < zero_words; i += blockDim.x) zero[i] = 0u;
  __syncthreads();
  if (threadIdx.x == 0) {
    if (tp.metric == CR_METRIC_L2)
      k_topk<false, true><<<grid, THREADS, SMEM_TOTAL, cudaStreamTailLaunch>>>(tq, tdb, tcomp, tp);
    else
      k_topk<false, false><<<grid, THREADS, SMEM_TOTAL, cudaStreamTailLaunch>>>(tq, tdb, tcomp, tp);
    const uint64_t stride = uint64_t(tp.n_queries) * tp.k;
    k_merge<<<tp.n_queries, MERGE_THREADS, MERGE_N * 12, cudaStreamTailLaunch>>>(
        tp.part_s, tp.part_id, n_lists, tp.n_queries, tp.k, tp.metric, 0, queries, DIM, out_d, out_id, nullptr, 0,
        nullptr, nullptr, 0, nullptr, 0, 0, nullptr, err, nullptr, nullptr, stride, stride);
    if (cudaGetLastError() != cudaSuccess) atomicOr(err, kErrLaunch);
    if (slot) ::k_export_err<<<1, 32, 0, cudaStreamTailLaunch>>>(guard, err, slot);
  }
}

void row_norms(const uint16_t* db, uint64_t n_rows, float* out, cudaStream_t s)
{
  const uint64_t threads = n_rows * 16;
  k_row_norms<<<div_up(threads, 256), 256, 0, s>>>(reinterpret_cast<const uint4*>(db), n_rows, out);
  CR_CUDA(cudaGetLastError());
}

}  // namespace
}  // namespace crb

using namespace crb;

extern "C" int cr_row_norms(const uint16_t* d_db, uint64_t n_rows, uint32_t dim, float* d_out,
                            cr_stream_t stream)
{
  CR_API_BEGIN
  CR_REQUIRE(dim == DIM, "cr_row_norms: dim must be 128");
  CR_REQUIRE(d_db && d_out, "cr_row_norms: null buffer");
  CR_REQUIRE((reinterpret_cast<uintptr_t>(d_db) & 15u) == 0, "cr_row_norms: db must be 16-byte aligned");
  if (n_rows) row_norms(d_db, n_rows, d_out, reinterpret_cast<cudaStream_t>(stream));
  CR_API_END
}

// Measurement only (CR_TOPK_TRACE=1): events at the phase boundaries of one
// call, printed as the device time between consecutive marks.
struct Trace {
  bool on = false;
  cudaEvent_t ev[16];
  const char* name[16];
  int n = 0;
  static Trace& get()
  {
    thread_local Trace t;
    return t;
  }
  void mark(const char* what, cudaStream_t s)
  {
    if (!on || n >= 16) return;
    if (!ev[n]) cudaEventCreate(&ev[n]);
    name[n] = what;
    cudaEventRecord(ev[n++], s);
  }
  void print()
  {
    if (!on || n < 2) return;
    cudaEventSynchronize(ev[n - 1]);
    fprintf(stderr, "topk trace:");
    for (int i = 1; i < n; ++i) {
      float ms = 0.f;
      cudaEventElapsedTime(&ms, ev[i - 1], ev[i]);
      fprintf(stderr, " %s %.1f", name[i], ms * 1e3f);
    }
    fprintf(stderr, " (us)\n");
  }
  Trace() { for (auto& e : ev) e = nullptr; }
};

// The tcgen05 search over `n_rows` rows (optionally masked by `pass`, row
// ids optionally translated by `row_map`) plus the per-query merge.
// Scratch of cr_filtered_topk: chunks of device memory kept per (device,
// stream, host thread) and handed out again by every call, so a steady stream
// of searches allocates nothing. Calls on one stream run in stream order, so
// reusing the memory of the previous call is safe; each host thread has its
// own chunks. The memory stays allocated until the thread exits.
struct Arena {
  struct Chunk { char* p; size_t cap; };
  std::vector<Chunk> chunks;
  size_t ci = 0, off = 0;
  cudaStream_t s = nullptr;
  static Arena& get(cudaStream_t st)
  {
    thread_local std::map<std::pair<int, cudaStream_t>, Arena> arenas;
    int dev = 0;
    CR_CUDA(cudaGetDevice(&dev));
    Arena& a = arenas[{dev, st}];
    a.s = st;
    return a;
  }
  void reset() { ci = 0; off = 0; }
  template <class T> T* take(size_t bytes)
  {
    if (bytes == 0) return nullptr;
    bytes = (bytes + 255) & ~size_t(255);
    for (; ci < chunks.size(); ++ci, off = 0)
      if (off + bytes <= chunks[ci].cap) {
        char* r = chunks[ci].p + off;
        off += bytes;
        return reinterpret_cast<T*>(r);
      }
    const size_t cap = std::max(bytes, size_t(64) << 20);
    chunks.push_back({static_cast<char*>(dev_alloc(cap, s)), cap});
    ci = chunks.size() - 1;
    off = bytes;
    return reinterpret_cast<T*>(chunks[ci].p);
  }
};

// The error words of a finished search (and of its exact redo, if any) into
// the host-visible slot.
__global__ void k_export_err(const uint32_t* err0, const uint32_t* err1, uint32_t* slot)
{
  if (threadIdx.x == 0) {
    slot[0] = *err0;
    slot[1] = err1 ? *err1 : 0u;
  }
}

// Device-side failures of a search (bounded waits that ran out) are copied to
// a small ring of page-locked words per host thread and reported by the next
// call on that thread, or by cr_filtered_topk_check, without making the
// search itself wait for the device.
struct ErrorRing {
  static constexpr int kSlots = 8;
  uint32_t* words = nullptr;  // [kSlots][2], mapped page-locked host memory
  uint32_t* d_words = nullptr;  // the same words' device address
  cudaEvent_t ev[kSlots] = {};
  bool pending[kSlots] = {};
  int next = 0;
  static ErrorRing& get()
  {
    thread_local ErrorRing r;
    return r;
  }
  // Reports completed slots; with `wait`, waits for every slot first.
  void check(bool wait)
  {
    for (int i = 0; i < kSlots; ++i) {
      if (!pending[i]) continue;
      if (wait) CR_CUDA(cudaEventSynchronize(ev[i]));
      else if (cudaEventQuery(ev[i]) != cudaSuccess) continue;
      pending[i] = false;
      // First pass: everything but the fallback requests; fallback: everything.
      const uint32_t bad = (words[2 * i] & ~(kErrOverflow | kErrSpec)) | words[2 * i + 1];
      if (bad)
        fail(CR_ERR_DEVICE, "cr_filtered_topk: a pipeline wait timed out on the device (code " +
                                std::to_string(bad) + ")");
    }
  }
  // The next slot's device address (waiting for its previous search when
  // more than kSlots are in flight); the caller has its words written on
  // stream `s`, then calls commit(s).
  uint32_t* acquire()
  {
    if (!words) {
      CR_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&words), kSlots * 2 * 4, cudaHostAllocMapped));
      CR_CUDA(cudaHostGetDevicePointer(reinterpret_cast<void**>(&d_words), words, 0));
      for (auto& e : ev) CR_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    }
    const int i = next;
    if (pending[i]) {
      CR_CUDA(cudaEventSynchronize(ev[i]));
      const uint32_t bad = (words[2 * i] & ~(kErrOverflow | kErrSpec)) | words[2 * i + 1];
      pending[i] = false;
      if (bad) fail(CR_ERR_DEVICE, "cr_filtered_topk: a pipeline wait timed out on the device (code " +
                                       std::to_string(bad) + ")");
    }
    return d_words + 2 * i;
  }
  void commit(cudaStream_t s)
  {
    const int i = next;
    next = (next + 1) % kSlots;
    CR_CUDA(cudaEventRecord(ev[i], s));
    pending[i] = true;
  }
  // A search without a redo gate: one tiny kernel stores its error words
  // straight into the mapped slot (no copy-engine work on the stream).
  void record(const uint32_t* d_err0, const uint32_t* d_err1, cudaStream_t s)
  {
    uint32_t* slot = acquire();
    k_export_err<<<1, 32, 0, s>>>(d_err0, d_err1, slot);
    CR_CUDA(cudaGetLastError());
    commit(s);
  }
};

// What a search reads: the shard (dense plans) and the compacted passing rows
// (compacted plans); the plan on the device says which.
struct SearchInput {
  const uint16_t* db;
  uint64_t shard_rows;
  const float* norms;      // shard norms (L2)
  const uint32_t* pass;    // shard pass bitset, null = every row passes
  const uint16_t* comp;    // compacted rows (null: no compaction)
  uint64_t comp_cap;       // rows comp can hold
  const float* comp_norms;
  const uint32_t* idx;     // compacted row -> shard row
  const SearchPlan* plan;
  const float* chunk_min;  // L2: least norm per 32 searched rows
};

// Bytes of the block a search needs cleared before it runs: per-query shared
// thresholds, published bounds, candidate counts, published best three
// (the same sizing as run_search's).
static size_t search_zero_bytes(uint32_t n_queries, uint32_t k, uint32_t slices, bool allow_append, bool allow_spec)
{
  const uint32_t n_lists = slices * EPI_PARTS;
  const uint32_t jth = (k + n_lists - 1) / n_lists;
  const bool append = allow_append && jth <= 3 && n_lists <= kMaxListsMerge;
  const bool spec_capable = append && allow_spec && 3 * n_lists <= 256;
  const size_t pub_b = size_t(n_queries) * n_lists * 4;
  const size_t cnt_b = append ? size_t(n_queries) * n_lists * 4 : 0;
  const size_t top_b = spec_capable ? size_t(n_queries) * n_lists * 3 * 4 : 0;
  return size_t(n_queries) * 4 + pub_b + cnt_b + top_b;
}

// One search over the planned rows plus the per-query merge, stream-ordered.
// Append mode (candidate arrays, speculative bound) unless disabled; `guard`
// makes every kernel of it a no-op unless that error word asks for a redo;
// device-side failures land in `err` (16 bytes, zeroed by the caller). With
// a guard the search is the exact redo, launched by k_redo_gate.
static void run_search(const SearchInput& in, const uint16_t* d_queries, uint32_t n_queries, uint64_t row_offset,
                       uint32_t k, int metric, float* d_out_dist, int64_t* d_out_ids, cudaStream_t s,
                       bool allow_append, bool allow_spec, const uint32_t* guard, uint32_t* err,
                       bool* used_append, uint32_t* err_slot = nullptr, char* cleared = nullptr)
{
  set_max_dynamic_smem(reinterpret_cast<const void*>(k_topk<true, false>), int(SMEM_TOTAL));
  set_max_dynamic_smem(reinterpret_cast<const void*>(k_topk<false, false>), int(SMEM_TOTAL));
  set_max_dynamic_smem(reinterpret_cast<const void*>(k_topk<true, true>), int(SMEM_TOTAL));
  set_max_dynamic_smem(reinterpret_cast<const void*>(k_topk<false, true>), int(SMEM_TOTAL));
  const bool l2m = metric == CR_METRIC_L2;
  auto* const k_app = l2m ? k_topk<true, true> : k_topk<true, false>;
  auto* const k_exact = l2m ? k_topk<false, true> : k_topk<false, false>;
  // Grid: query tiles x slices, sized for the largest plan (every shard row).
  const uint32_t max_tiles = std::max<uint32_t>(1u, div_up(in.shard_rows, BN));
  const uint32_t qtiles = div_up(n_queries, BM);
  const uint32_t slices = std::min<uint32_t>(std::max(1, sm_count() / int(qtiles)), max_tiles);
  const size_t ctas = size_t(qtiles) * slices;
  const size_t list_b = ctas * EPI_PARTS * 2 * k * BM * 4;
  const size_t part_b = size_t(slices) * EPI_PARTS * n_queries * k;
  const size_t cbuf_b = ctas * EPI * BUF * 4;
  const uint32_t n_lists = slices * EPI_PARTS;
  const size_t pub_b = size_t(n_queries) * n_lists * 4;
  const uint32_t jth = (k + n_lists - 1) / n_lists;
  // Append mode needs the register-tracked list bounds (jth <= 3); its
  // candidate arrays hold up to `cap` survivors per query.
  const bool append = allow_append && jth <= 3 && n_lists <= kMaxListsMerge;
  *used_append = append;
  const uint32_t cap = append ? std::max<uint32_t>(256u, div_up(std::max<uint32_t>(32768u, 128u * k), n_lists)) : 0u;
  const size_t cand_b = append ? size_t(n_queries) * n_lists * cap * 4 : 0;
  const bool spec_capable = append && allow_spec && 3 * n_lists <= 256;
  const size_t spec_b = spec_capable ? size_t(n_queries) * 4 + 16 : 0;
  const size_t top_b = spec_capable ? size_t(n_queries) * n_lists * 3 * 4 : 0;
  const size_t cnt_b = append ? size_t(n_queries) * n_lists * 4 : 0;
  // Everything that must start at zero sits in one block at the front, cleared
  // by one memset: per-query shared thresholds, published bounds, candidate
  // counts, published best three.
  const size_t zero_b = size_t(n_queries) * 4 + pub_b + cnt_b + top_b;
  // `cleared`: the block, already zeroed by the call's first kernel.
  char* p = Arena::get(s).take<char>((cleared ? 0 : zero_b) + 256 + list_b * 2 + cbuf_b * 2 + part_b * 12 +
                                     cand_b * 2 + spec_b + 256);
  char* const rest = p + (cleared ? 0 : zero_b);
  if (cleared) p = cleared;
  TopkParams tp{};
  tp.err = err;
  tp.shared_thr = reinterpret_cast<uint32_t*>(p); p += size_t(n_queries) * 4;
  tp.pub = reinterpret_cast<uint32_t*>(p); p += pub_b;
  if (append) { tp.cand_cnt = reinterpret_cast<uint32_t*>(p); p += cnt_b; }
  if (spec_capable) { tp.pub_top = reinterpret_cast<uint32_t*>(p); p += top_b; }
  if (!guard && !cleared) CR_CUDA(cudaMemsetAsync(tp.shared_thr, 0, zero_b, s));
  p = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(rest) + 255) & ~uintptr_t(255));
  tp.n_queries = n_queries;
  tp.k = k;
  tp.metric = metric;
  tp.plan = in.plan;
  tp.row_offset = row_offset;
  tp.pass = in.pass;
  tp.norms = in.norms;
  tp.comp_norms = in.comp_norms;
  tp.chunk_min = in.chunk_min;
  tp.row_map = in.idx;
  tp.guard = guard;
  tp.spec_capable = spec_capable ? 1u : 0u;
  tp.list_s = reinterpret_cast<float*>(p); p += list_b;
  tp.list_r = reinterpret_cast<uint32_t*>(p); p += list_b;
  tp.buf_s = reinterpret_cast<float*>(p); p += cbuf_b;
  tp.buf_r = reinterpret_cast<uint32_t*>(p); p += cbuf_b;
  tp.n_lists = n_lists;
  tp.jth = jth;
  tp.append = append ? 1u : 0u;
  tp.cap = cap;
  if (append) {
    tp.cand_s = reinterpret_cast<float*>(p); p += cand_b;
    tp.cand_r = reinterpret_cast<uint32_t*>(p); p += cand_b;
  }
  uint32_t* spec_used = nullptr;
  if (spec_capable) { spec_used = reinterpret_cast<uint32_t*>(p); p += spec_b; }
  tp.spec_used = spec_used;
  tp.part_id = reinterpret_cast<int64_t*>(p); p += part_b * 8;
  tp.part_s = reinterpret_cast<float*>(p); p += part_b * 4;
  if (const char* dbg = getenv("CR_TOPK_DEBUG")) tp.debug = uint32_t(atoi(dbg));
  tp.keeper_ns = 2000;
  tp.spin_limit = kSpinLimit;
  // Failure tests only: a short limit for every pipeline wait.
  if (const char* sl = getenv("CR_TOPK_SPIN_LIMIT")) tp.spin_limit = std::max(1, atoi(sl));
  if (const char* kn = getenv("CR_TOPK_KEEPER_NS")) tp.keeper_ns = uint32_t(atoi(kn));
  Trace::get().mark("setup", s);
  const CUtensorMap tq = make_map(d_queries, n_queries, BM);
  const CUtensorMap tdb = make_map(in.db, in.shard_rows, BN);
  const CUtensorMap tcomp = in.comp ? make_map(in.comp, std::max<uint64_t>(1, in.comp_cap), BN) : tdb;
  const dim3 grid(qtiles, slices);
  if (guard) {
    k_redo_gate<<<1, 1024, 0, s>>>(guard, tp.shared_thr, zero_b / 4, err, grid, tq, tdb, tcomp, tp, n_lists,
                                   reinterpret_cast<const __half*>(d_queries), d_out_dist, d_out_ids, err_slot);
    CR_CUDA(cudaGetLastError());
    Trace::get().mark("redo_gate", s);
    return;
  }
  {
    ProfileScope prof(guard ? -1 : CR_KERNEL_TOPK, s);
    if (spec_capable) {
      // Prologue launch (publish-only tiles), the speculative bound per
      // query, then the main launch starting from it (all no-ops when the
      // plan has no speculative bound).
      TopkParams pro = tp;
      pro.prologue_only = 1;
      k_app<<<grid, THREADS, SMEM_TOTAL, s>>>(tq, tdb, tcomp, pro);
      k_spec<<<div_up(n_queries, 4u), 128, 0, s>>>(tp.pub_top, 3 * n_lists, n_queries, in.plan, spec_used);
    }
    Trace::get().mark("prologue_spec", s);
    if (append) k_app<<<grid, THREADS, SMEM_TOTAL, s>>>(tq, tdb, tcomp, tp);
    else k_exact<<<grid, THREADS, SMEM_TOTAL, s>>>(tq, tdb, tcomp, tp);
  }
  CR_CUDA(cudaGetLastError());
  if (append)
    merge_launch(tp.cand_s, nullptr, 0, n_queries, k, metric, 2, reinterpret_cast<const __half*>(d_queries),
                 DIM, d_out_dist, d_out_ids, s, tp.cand_cnt, cap, tp.cand_r, in.idx, row_offset, tp.pub,
                 n_lists, 0, spec_used, err, in.plan, guard);
  else
    merge_launch(tp.part_s, tp.part_id, n_lists, n_queries, k, metric, 0,
                 reinterpret_cast<const __half*>(d_queries), DIM, d_out_dist, d_out_ids, s, nullptr, 0, nullptr,
                 nullptr, 0, nullptr, 0, 0, nullptr, nullptr, nullptr, guard);
  Trace::get().mark(guard ? "fallback" : "main_merge", s);
  if (tp.debug == 3) {  // measurement only: waits
    uint32_t c[4];
    CR_CUDA(cudaMemcpyAsync(c, err, 16, cudaMemcpyDeviceToHost, s));
    CR_CUDA(cudaStreamSynchronize(s));
    fprintf(stderr, "topk debug: lane flushes %u, warp slow paths / flush rounds %u, inserts %u, err %u\n", c[1],
            c[2], c[3], c[0]);
  }
}

namespace crb {

void filtered_topk_enqueue(const uint16_t* d_db, const float* d_db_norms, uint64_t n_rows, uint32_t dim,
                           const uint16_t* d_queries, uint32_t n_queries, const cr_gpu_roaring* filter,
                           uint64_t row_offset, uint32_t k, int metric, float* d_out_dist, int64_t* d_out_ids,
                           cudaStream_t s)
{
  CR_REQUIRE(dim == DIM, "cr_filtered_topk: this build supports dim == 128");
  CR_REQUIRE(k >= 1 && k <= 256, "cr_filtered_topk: k must be in [1, 256]");
  CR_REQUIRE(metric == CR_METRIC_IP || metric == CR_METRIC_L2, "cr_filtered_topk: unknown metric");
  CR_REQUIRE(n_rows >= 1 && n_rows < (1ull << 31), "cr_filtered_topk: n_rows must be in [1, 2^31)");
  CR_REQUIRE(n_queries >= 1, "cr_filtered_topk: no queries");
  CR_REQUIRE(d_db && d_queries && d_out_dist && d_out_ids, "cr_filtered_topk: null buffer");
  CR_REQUIRE((reinterpret_cast<uintptr_t>(d_db) & 15u) == 0 &&
                 (reinterpret_cast<uintptr_t>(d_queries) & 15u) == 0,
             "cr_filtered_topk: db and queries must be 16-byte aligned");
  ErrorRing::get().check(false);  // failures of earlier searches on this thread
  const bool l2 = metric == CR_METRIC_L2;
  Trace& tr = Trace::get();
  tr.on = getenv("CR_TOPK_TRACE") != nullptr;
  tr.n = 0;
  tr.mark("start", s);

  // Control block for the whole call: plan and both searches' error words
  // (the fallback reads the first one). The call's first kernel clears the
  // error words; the plan is written whole.
  Arena& arena = Arena::get(s);
  arena.reset();
  char* ctl = arena.take<char>(256);
  SearchPlan* plan = reinterpret_cast<SearchPlan*>(ctl);
  uint32_t* err0 = reinterpret_cast<uint32_t*>(ctl + 128);
  uint32_t* err1 = reinterpret_cast<uint32_t*>(ctl + 192);

  // Squared norms of the shard rows (L2 only), computed here when not given.
  const float* norms = d_db_norms;
  if (l2 && !norms) {
    float* nb = arena.take<float>(n_rows * 4);
    row_norms(d_db, n_rows, nb, s);
    norms = nb;
  }
  SearchInput in{};
  in.db = d_db;
  in.shard_rows = n_rows;
  in.norms = norms;
  in.plan = plan;
  const uint32_t qtiles = div_up(n_queries, BM);
  const uint32_t slices =
      std::min<uint32_t>(std::max(1, sm_count() / int(qtiles)), std::max<uint32_t>(1u, div_up(n_rows, BN)));
  const int spec_override = getenv("CR_TOPK_SPEC_J") ? atoi(getenv("CR_TOPK_SPEC_J")) : -1;  // tests
  const int tiles_override = getenv("CR_TOPK_SPEC_TILES") ? atoi(getenv("CR_TOPK_SPEC_TILES")) : 0;  // measurement
  const uint32_t jth = (k + slices * EPI_PARTS - 1) / (slices * EPI_PARTS);
  const uint32_t spec_capable = (jth <= 3 && 3 * slices * EPI_PARTS <= 256) ? 1u : 0u;
  // Pass bitset and compaction (filtered searches); their scratch lives to
  // the end of the call.
  const uint64_t pass_words = (n_rows + 31) / 32;
  const uint32_t n_wtiles = div_up(pass_words, kWordTile);
  // Up to 3/4 of the rows passing, copying the passing rows (512 B of HBM
  // traffic each) is cheaper than searching every row with the mask.
  const uint64_t cap_rows = filter ? std::max<uint64_t>(1, n_rows * 3 / 4) : 0;
  // The first search's zeroed block: cleared by k_pass_words when that
  // kernel runs with enough threads (at most 8 16-byte stores each), else
  // by a memset inside the search.
  const size_t zero_bytes = (search_zero_bytes(n_queries, k, slices, true, true) + 15) & ~size_t(15);
  const bool clear_in_pass = filter && row_offset % 32 == 0 && uint64_t(n_wtiles) * 256 * 8 >= zero_bytes / 16;
  char* cleared = clear_in_pass ? arena.take<char>(zero_bytes) : nullptr;
  Scratch kidx_holder;
  const PlanArgs pa{uint32_t(n_rows), slices, slices * EPI_PARTS, k, spec_capable, uint32_t(cap_rows),
                    spec_override, tiles_override};
  if (!filter) {
    k_plan<<<1, 32, 0, s>>>(nullptr, pa, plan, err0, err1);
  } else {
    uint32_t* pass = arena.take<uint32_t>(pass_words * 4 + 16);
    uint32_t* d_total = arena.take<uint32_t>(16);
    uint32_t* tiles = arena.take<uint32_t>(size_t(n_wtiles) * 4);
    if (row_offset % 32 == 0) {
      static_assert(kWordTile == 256, "one pass-word block per word tile");
      const DevBitmap b = make_dev(filter, kidx_holder, s);
      k_pass_words<<<n_wtiles, 256, 0, s>>>(b, row_offset, n_rows, pass, pass_words, tiles, err0, err1,
                                            reinterpret_cast<uint4*>(cleared), zero_bytes / 16);
    } else {
      const cu_roaring::GpuRoaringView v =
          cu_roaring::make_view(*reinterpret_cast<const cu_roaring::GpuRoaring*>(filter));
      const uint64_t threads = pass_words * 32;
      const int grid = static_cast<int>(std::min<uint64_t>(div_up(threads, 256), uint64_t(sm_count()) * 16));
      k_pass_bits<<<grid, 256, 0, s>>>(v, row_offset, n_rows, pass, pass_words, filter->universe_size);
      k_pass_tile_sums<<<n_wtiles, kWordTile, 0, s>>>(pass, pass_words, tiles, err0, err1);
    }
    CR_CUDA(cudaGetLastError());
    tr.mark("pass_bits", s);
    // Pre-filter up to 3/4 density: compact the passing rows' indices (and
    // norms) and copy those rows into a dense block searched with TMA tiles.
    uint32_t* idx = arena.take<uint32_t>(cap_rows * 4);
    float* comp_norms = l2 ? arena.take<float>(cap_rows * 4) : nullptr;
    uint16_t* comp = arena.take<uint16_t>(cap_rows * DIM * 2);
    {
      ProfileScope prof_c(CR_KERNEL_TOPK_COMPACT, s);
      k_pass_compact<<<n_wtiles, kCompactThreads, 0, s>>>(pass, pass_words, tiles, n_wtiles, idx, d_total,
                                                    l2 ? norms : nullptr, comp_norms,
                                                    reinterpret_cast<const uint4*>(d_db),
                                                    reinterpret_cast<uint4*>(comp), uint32_t(cap_rows),
                                                    pa, plan);
      CR_CUDA(cudaGetLastError());
    }
    tr.mark("compact_gather", s);
    in.pass = pass;
    in.comp = comp;
    in.comp_cap = cap_rows;
    in.comp_norms = comp_norms;
    in.idx = idx;
  }
  if (l2) {  // per-chunk least norms of the planned rows (the epilogue's L2 bound)
    const uint64_t chunks = (n_rows + 31) / 32;
    float* cm = arena.take<float>(chunks * 4 + 16);
    k_chunk_min_norms<<<std::max<uint32_t>(1u, std::min<uint32_t>(div_up(chunks, 256), 4 * sm_count())), 256, 0,
                        s>>>(plan, norms, in.comp_norms, cm);
    in.chunk_min = cm;
  }
  CR_CUDA(cudaGetLastError());
  bool appended = false, unused = false;
  run_search(in, d_queries, n_queries, row_offset, k, metric, d_out_dist, d_out_ids, s, true, true, nullptr, err0,
             &appended, nullptr, cleared);
  // The exact redo with per-list merging, which needs neither candidate
  // capacity nor a speculative bound: every kernel of it returns at once
  // unless the first search flagged an overflowing candidate array
  // (degenerate score distributions, e.g. massive ties) or a speculative
  // bound above some query's k-th best.
  ErrorRing& ring = ErrorRing::get();
  if (appended) {
    // The redo gate also hands the error words to the host-visible ring.
    uint32_t* slot = ring.acquire();
    run_search(in, d_queries, n_queries, row_offset, k, metric, d_out_dist, d_out_ids, s, false, false, err0, err1,
               &unused, slot);
    ring.commit(s);
  } else {
    ring.record(err0, nullptr, s);
  }
  tr.mark("search", s);
  tr.print();
}

void topk_merge_enqueue(const float* d_dist, const int64_t* d_ids, uint64_t dist_stride, uint64_t id_stride,
                        uint32_t n_parts, uint32_t n_queries, uint32_t k, int metric, float* d_out_dist,
                        int64_t* d_out_ids, cudaStream_t s)
{
  merge_launch(d_dist, d_ids, n_parts, n_queries, k, metric, 1, nullptr, 0, d_out_dist, d_out_ids, s, nullptr, 0,
               nullptr, nullptr, 0, nullptr, 0, 0, nullptr, nullptr, nullptr, nullptr, dist_stride, id_stride);
}

}  // namespace crb


extern "C" int cr_filtered_topk(const uint16_t* d_db, const float* d_db_norms, uint64_t n_rows,
                                uint32_t dim, const uint16_t* d_queries, uint32_t n_queries,
                                const cr_gpu_roaring* filter, uint64_t row_offset, uint32_t k,
                                int metric, float* d_out_dist, int64_t* d_out_ids,
                                cr_stream_t stream)
{
  CR_API_BEGIN
  filtered_topk_enqueue(d_db, d_db_norms, n_rows, dim, d_queries, n_queries, filter, row_offset, k, metric,
                        d_out_dist, d_out_ids, reinterpret_cast<cudaStream_t>(stream));
  CR_API_END
}

extern "C" int cr_topk_merge_packed(const void* d_parts, uint64_t part_bytes, uint32_t n_parts,
                                    uint32_t n_queries, uint32_t k, int metric, float* d_out_dist,
                                    int64_t* d_out_ids, cr_stream_t stream)
{
  CR_API_BEGIN
  CR_REQUIRE(d_parts && d_out_dist && d_out_ids, "cr_topk_merge_packed: null buffer");
  CR_REQUIRE(k >= 1 && k <= 256 && n_parts >= 1, "cr_topk_merge_packed: bad k or n_parts");
  const uint64_t dist_bytes = uint64_t(n_queries) * k * 4;
  CR_REQUIRE(part_bytes % 8 == 0 && dist_bytes % 8 == 0 && part_bytes >= dist_bytes * 3,
             "cr_topk_merge_packed: each part needs 8-byte aligned dist and id blocks (n_queries * k even)");
  CR_REQUIRE((reinterpret_cast<uintptr_t>(d_parts) & 7u) == 0, "cr_topk_merge_packed: d_parts must be 8-byte aligned");
  const char* base = static_cast<const char*>(d_parts);
  merge_launch(reinterpret_cast<const float*>(base), reinterpret_cast<const int64_t*>(base + dist_bytes), n_parts,
               n_queries, k, metric, 1, nullptr, 0, d_out_dist, d_out_ids, reinterpret_cast<cudaStream_t>(stream),
               nullptr, 0, nullptr, nullptr, 0, nullptr, 0, 0, nullptr, nullptr, nullptr, nullptr, part_bytes / 4,
               part_bytes / 8);
  CR_API_END
}

extern "C" int cr_filtered_topk_check(void)
{
  CR_API_BEGIN
  ErrorRing::get().check(true);
  CR_API_END
}

extern "C" int cr_topk_merge(const float* d_dist_parts, const int64_t* d_id_parts, uint32_t n_parts,
                             uint32_t n_queries, uint32_t k, int metric, float* d_out_dist,
                             int64_t* d_out_ids, cr_stream_t stream)
{
  CR_API_BEGIN
  CR_REQUIRE(d_dist_parts && d_id_parts && d_out_dist && d_out_ids, "cr_topk_merge: null buffer");
  CR_REQUIRE(k >= 1 && k <= 256 && n_parts >= 1, "cr_topk_merge: bad k or n_parts");
  merge_launch(d_dist_parts, d_id_parts, n_parts, n_queries, k, metric, 1, nullptr, 0, d_out_dist,
               d_out_ids, reinterpret_cast<cudaStream_t>(stream));
  CR_API_END
}
