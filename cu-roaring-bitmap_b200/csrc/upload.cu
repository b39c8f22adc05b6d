// cu_roaring B200 engine — construction (upload_from_ids / _bitset).
//
// Replaces reference src/upload_ids.cu (CUB 32-bit radix sort -> unique ->
// RLE -> global-atomic scatter into all-BITMAP containers, 2+ host syncs)
// with a chunk-bitmap pipeline that never sorts:
//
//   ids  --(k_mark, sparse only)--> 65536-bit key presence
//        --(k_assign_slots)-------> one 8 KiB chunk slot per touched key
//        --(k_scatter)------------> red.global.or of every ID into its slot
//   bitset ------------------------> chunk slots are the caller's words
//   chunk slots --(k_analyze)------> per chunk: popcount c, run count r, and
//                                    the same for the complement
//              --(k_plan_tiles, k_plan_emit)--> complement decision
//                                    (|set| > U/2), canonical type per chunk,
//                                    stream-compacted metadata and offsets
//   one 64-byte D2H + sync (the only one) -> packed allocation
//              --(k_emit)---------> BITMAP copy / ARRAY extraction (block
//                                    scan of popcounts) / RUN extraction,
//                                    metadata and key_index in one pass
//
// Duplicates vanish in the OR; IDs >= universe raise a device error flag that
// the host turns into CR_ERR_RANGE.
#include <algorithm>
#include <vector>

#include "common.cuh"

namespace crb {

namespace {

constexpr int kEmitThreads = 256;   // 4 u64 words per thread
constexpr int kPlanTile = 1024;

struct ChunkSrc {
  const uint32_t* words;     // slot s occupies words [s*2048, s*2048+2048)
  uint64_t n_words;          // words at or beyond this index read as zero
  const uint16_t* slot_keys; // null: slot == key (dense)
  const uint32_t* n_slots;   // device count of used slots (sparse only)
  uint32_t universe;
  uint32_t keep_uncomplemented;  // 1: never store the complement (the reference's CRoaring upload without a universe)
};

struct PlanTotals {
  uint32_t n_cont;
  uint32_t nb[2], na[2], nr[2];
  unsigned long long ab[2], rb[2];
};

struct PlanHeader {
  uint32_t n_cont, nb, na, nr;
  unsigned long long array_bytes, run_bytes;
  unsigned long long total_logical;
  uint32_t negated, threshold, err, pad;
};

__device__ __forceinline__ uint32_t slot_count(const ChunkSrc& src, uint32_t max_slots)
{
  return src.slot_keys ? *src.n_slots : max_slots;
}

// Loads this thread's 4 consecutive u64 words (words 4t..4t+3 of the chunk),
// masked to the chunk's valid bits and optionally complemented.
template <bool VEC>
__device__ __forceinline__ void load_chunk_words(const ChunkSrc& src, uint32_t slot,
                                                 uint32_t valid, bool complement,
                                                 uint64_t w[4])
{
  const uint32_t t = threadIdx.x;
  const uint64_t g = uint64_t(slot) * kChunkWords32 + 8ull * t;
  uint32_t v[8];
  if (VEC && g + 8 <= src.n_words) {
    const uint4* p = reinterpret_cast<const uint4*>(src.words + g);
    const uint4 a = __ldg(p), b = __ldg(p + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = (g + i < src.n_words) ? __ldg(src.words + g + i) : 0u;
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint64_t m = word_mask(4 * t + i, valid);
    uint64_t x = uint64_t(v[2 * i]) | (uint64_t(v[2 * i + 1]) << 32);
    w[i] = (complement ? ~x : x) & m;
  }
}

// Top bit of the previous thread's last word (0 for thread 0).
__device__ __forceinline__ uint64_t prev_top_bit(uint64_t last, uint64_t* smem_last)
{
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint64_t p = __shfl_up_sync(0xFFFFFFFFu, last, 1);
  if (lane == 31) smem_last[warp] = last;
  __syncthreads();
  if (lane == 0) p = warp ? smem_last[warp - 1] : 0ull;
  __syncthreads();
  return p >> 63;
}

// Bit 0 of the next thread's first word (0 for the last thread).
__device__ __forceinline__ uint64_t next_low_bit(uint64_t first, uint64_t* smem_first)
{
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint64_t n = __shfl_down_sync(0xFFFFFFFFu, first, 1);
  if (lane == 0) smem_first[warp] = first;
  __syncthreads();
  if (lane == 31) n = (warp + 1 < kEmitThreads / 32) ? smem_first[warp + 1] : 0ull;
  __syncthreads();
  return n & 1ull;
}

__device__ __forceinline__ uint32_t count_run_starts(const uint64_t w[4], uint64_t carry)
{
  uint32_t r = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    r += __popcll(w[i] & ~((w[i] << 1) | carry));
    carry = w[i] >> 63;
  }
  return r;
}

// One CTA per chunk slot: stats[s] = (c, r, c_complement, r_complement).
// Two barriers per chunk: one to pass each warp's top bits (set and
// complement) to the next warp, one for the per-warp sums; the complement's
// count is the chunk's valid bits minus the set's.
template <bool VEC>
__global__ void __launch_bounds__(kEmitThreads) k_analyze(ChunkSrc src, uint32_t max_slots,
                                                          uint4* stats,
                                                          unsigned long long* total)
{
  __shared__ uint32_t s_last[kEmitThreads / 32];
  __shared__ uint4 s_red[kEmitThreads / 32];
  const uint32_t s = blockIdx.x;
  if (s >= slot_count(src, max_slots)) return;
  const uint32_t key = src.slot_keys ? src.slot_keys[s] : s;
  const uint32_t valid = chunk_valid_bits(key, src.universe);
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint64_t w[4], cw[4];
  load_chunk_words<VEC>(src, s, valid, false, w);
#pragma unroll
  for (int i = 0; i < 4; ++i) cw[i] = ~w[i] & word_mask(4 * threadIdx.x + i, valid);
  uint32_t c = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) c += __popcll(w[i]);
  // Top bits of the previous thread's last words: bit 0 set, bit 1 complement.
  const uint32_t mine = uint32_t(w[3] >> 63) | (uint32_t(cw[3] >> 63) << 1);
  uint32_t prev = __shfl_up_sync(0xFFFFFFFFu, mine, 1);
  if (lane == 31) s_last[warp] = mine;
  __syncthreads();
  if (lane == 0) prev = warp ? s_last[warp - 1] : 0u;
  uint32_t r = count_run_starts(w, prev & 1u);
  uint32_t cr = count_run_starts(cw, (prev >> 1) & 1u);
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    c += __shfl_xor_sync(0xFFFFFFFFu, c, o);
    r += __shfl_xor_sync(0xFFFFFFFFu, r, o);
    cr += __shfl_xor_sync(0xFFFFFFFFu, cr, o);
  }
  if (lane == 0) s_red[warp] = make_uint4(c, r, cr, 0u);
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t C = 0, R = 0, CR = 0;
#pragma unroll
    for (int i = 0; i < kEmitThreads / 32; ++i) {
      const uint4 x = s_red[i];
      C += x.x;
      R += x.y;
      CR += x.z;
    }
    stats[s] = make_uint4(C, R, valid - C, CR);
    if (C) atomicAdd(total, static_cast<unsigned long long>(C));
  }
}

__device__ __forceinline__ bool plan_negate(const unsigned long long* total, const ChunkSrc& src)
{
  return !src.keep_uncomplemented && *total > static_cast<unsigned long long>(src.universe / 2u);
}

// Per tile of 1024 chunk slots: totals under the two candidate thresholds.
__global__ void __launch_bounds__(kPlanTile) k_plan_tiles(ChunkSrc src, uint32_t max_slots,
                                                          const uint4* stats,
                                                          const unsigned long long* total,
                                                          uint32_t t0, uint32_t t1,
                                                          PlanTotals* tiles)
{
  __shared__ unsigned long long s_red[kPlanTile / 32];
  const uint32_t i = blockIdx.x * kPlanTile + threadIdx.x;
  const bool neg = plan_negate(total, src);
  uint32_t c = 0, r = 0;
  if (i < slot_count(src, max_slots)) {
    const uint4 st = stats[i];
    c = neg ? st.z : st.x;
    r = neg ? st.w : st.y;
  }
  unsigned long long v;
  PlanTotals out{};
  v = block_sum<kPlanTile, unsigned long long>(c ? 1ull : 0ull, s_red);
  out.n_cont = static_cast<uint32_t>(v);
  const uint32_t ts[2] = {t0, t1};
#pragma unroll
  for (int o = 0; o < 2; ++o) {
    const uint8_t ty = c ? container_type(c, r, ts[o]) : 0xFF;
    out.nb[o] = static_cast<uint32_t>(block_sum<kPlanTile, unsigned long long>(ty == kBitmap, s_red));
    out.na[o] = static_cast<uint32_t>(block_sum<kPlanTile, unsigned long long>(ty == kArray, s_red));
    out.nr[o] = static_cast<uint32_t>(block_sum<kPlanTile, unsigned long long>(ty == kRun, s_red));
    out.ab[o] = block_sum<kPlanTile, unsigned long long>(ty == kArray ? 2ull * c : 0ull, s_red);
    out.rb[o] = block_sum<kPlanTile, unsigned long long>(ty == kRun ? 4ull * r : 0ull, s_red);
  }
  if (threadIdx.x == 0) tiles[blockIdx.x] = out;
}

// Chooses the threshold (AUTO compression guard of reference
// src/upload.cpp:112-118), then writes each slot's final plan record
// (container index, type, byte offset, cardinality field) and the header.
__global__ void __launch_bounds__(kPlanTile) k_plan_emit(ChunkSrc src, uint32_t max_slots,
                                                         const uint4* stats,
                                                         const unsigned long long* total,
                                                         uint32_t t0, uint32_t t1,
                                                         uint32_t auto_guard,
                                                         const PlanTotals* tiles,
                                                         uint32_t n_tiles, uint4* plan,
                                                         PlanHeader* header,
                                                         const uint32_t* err)
{
  __shared__ unsigned long long s_red[kPlanTile / 32];
  __shared__ PlanTotals s_base, s_all;
  __shared__ int s_opt;
  if (threadIdx.x == 0) {
    PlanTotals b{}, a{};
    for (uint32_t j = 0; j < n_tiles; ++j) {
      const PlanTotals& x = tiles[j];
      PlanTotals* dst[2] = {&a, &b};
      for (int d = 0; d < (j < blockIdx.x ? 2 : 1); ++d) {
        PlanTotals& y = *dst[d];
        y.n_cont += x.n_cont;
        for (int o = 0; o < 2; ++o) {
          y.nb[o] += x.nb[o]; y.na[o] += x.na[o]; y.nr[o] += x.nr[o];
          y.ab[o] += x.ab[o]; y.rb[o] += x.rb[o];
        }
      }
    }
    s_base = b;
    s_all = a;
    int opt = 0;
    if (auto_guard) {
      const unsigned long long promoted = 8192ull * a.n_cont;
      const unsigned long long flat = (static_cast<unsigned long long>(src.universe) + 7ull) / 8ull;
      if (promoted * 2ull >= flat) opt = 1;
    }
    s_opt = opt;
  }
  __syncthreads();
  const int o = s_opt;
  const uint32_t t = o ? t1 : t0;
  const bool neg = plan_negate(total, src);
  const uint32_t i = blockIdx.x * kPlanTile + threadIdx.x;
  uint32_t c = 0, r = 0;
  if (i < slot_count(src, max_slots)) {
    const uint4 st = stats[i];
    c = neg ? st.z : st.x;
    r = neg ? st.w : st.y;
  }
  const uint8_t ty = c ? container_type(c, r, t) : 0xFF;
  unsigned long long tot;
  const unsigned long long idx = block_exclusive_scan<kPlanTile, unsigned long long>(c ? 1 : 0, s_red, &tot);
  const unsigned long long bslot = block_exclusive_scan<kPlanTile, unsigned long long>(ty == kBitmap, s_red, &tot);
  const unsigned long long aoff = block_exclusive_scan<kPlanTile, unsigned long long>(ty == kArray ? 2ull * c : 0ull, s_red, &tot);
  const unsigned long long roff = block_exclusive_scan<kPlanTile, unsigned long long>(ty == kRun ? 4ull * r : 0ull, s_red, &tot);
  if (i < max_slots) {
    uint4 rec = make_uint4(kNone, 0xFF, 0, 0);
    if (c) {
      rec.x = static_cast<uint32_t>(s_base.n_cont + idx);
      rec.y = ty;
      if (ty == kBitmap) {
        rec.z = static_cast<uint32_t>((s_base.nb[o] + bslot) * 8192ull);
        rec.w = c & 0xFFFFu;
      } else if (ty == kArray) {
        rec.z = static_cast<uint32_t>(s_base.ab[o] + aoff);
        rec.w = c;
      } else {
        rec.z = static_cast<uint32_t>(s_base.rb[o] + roff);
        rec.w = r;
      }
    }
    plan[i] = rec;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    PlanHeader h{};
    h.n_cont = s_all.n_cont;
    h.nb = s_all.nb[o]; h.na = s_all.na[o]; h.nr = s_all.nr[o];
    h.array_bytes = s_all.ab[o];
    h.run_bytes = s_all.rb[o];
    h.negated = neg;
    h.total_logical = *total;
    h.threshold = t;
    h.err = err ? *err : 0u;
    *header = h;
  }
}

// One CTA per chunk slot: writes the container payload, its metadata and its
// key_index entry at the places the plan assigned.
template <bool VEC>
__global__ void __launch_bounds__(kEmitThreads) k_emit(ChunkSrc src, uint32_t max_slots,
                                                       const uint4* plan,
                                                       const PlanHeader* header,
                                                       cr_gpu_roaring out)
{
  __shared__ uint64_t s_edge[kEmitThreads / 32];
  __shared__ uint32_t s_red[kEmitThreads / 32];
  __shared__ uint16_t s_starts[2048], s_ends[2048];
  const uint32_t s = blockIdx.x;
  if (s >= slot_count(src, max_slots)) return;
  const uint4 rec = plan[s];
  if (rec.x == kNone) return;
  const uint32_t key = src.slot_keys ? src.slot_keys[s] : s;
  const uint32_t valid = chunk_valid_bits(key, src.universe);
  uint64_t w[4];
  load_chunk_words<VEC>(src, s, valid, header->negated != 0, w);
  const uint32_t t = threadIdx.x;
  const uint8_t ty = static_cast<uint8_t>(rec.y);
  if (t == 0) {
    out.keys[rec.x] = static_cast<uint16_t>(key);
    out.types[rec.x] = ty;
    out.offsets[rec.x] = rec.z;
    out.cardinalities[rec.x] = static_cast<uint16_t>(rec.w);
    out.key_index[key] = static_cast<uint16_t>(rec.x);
  }
  if (ty == kBitmap) {
    uint4* dst = reinterpret_cast<uint4*>(out.bitmap_data + (rec.z >> 3)) + 2 * t;
    dst[0] = make_uint4(uint32_t(w[0]), uint32_t(w[0] >> 32), uint32_t(w[1]), uint32_t(w[1] >> 32));
    dst[1] = make_uint4(uint32_t(w[2]), uint32_t(w[2] >> 32), uint32_t(w[3]), uint32_t(w[3] >> 32));
  } else if (ty == kArray) {
    uint32_t cnt = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) cnt += __popcll(w[i]);
    uint32_t total;
    uint32_t pos = block_exclusive_scan<kEmitThreads>(cnt, s_red, &total);
    uint16_t* dst = out.array_data + (rec.z >> 1);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint64_t x = w[i];
      while (x) {
        dst[pos++] = static_cast<uint16_t>((4 * t + i) * 64 + __ffsll(x) - 1);
        x &= x - 1;
      }
    }
  } else {
    const uint64_t prev = prev_top_bit(w[3], s_edge);
    const uint64_t next = next_low_bit(w[0], s_edge);
    uint64_t st[4], en[4];
    uint64_t carry = prev;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      st[i] = w[i] & ~((w[i] << 1) | carry);
      carry = w[i] >> 63;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint64_t nb = (i < 3) ? (w[i + 1] & 1ull) : next;
      en[i] = w[i] & ~((w[i] >> 1) | (nb << 63));
    }
    uint32_t ns = 0, ne = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) { ns += __popcll(st[i]); ne += __popcll(en[i]); }
    uint32_t tot_s, tot_e;
    uint32_t ps = block_exclusive_scan<kEmitThreads>(ns, s_red, &tot_s);
    uint32_t pe = block_exclusive_scan<kEmitThreads>(ne, s_red, &tot_e);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint64_t x = st[i];
      while (x) { s_starts[ps++] = static_cast<uint16_t>((4 * t + i) * 64 + __ffsll(x) - 1); x &= x - 1; }
      x = en[i];
      while (x) { s_ends[pe++] = static_cast<uint16_t>((4 * t + i) * 64 + __ffsll(x) - 1); x &= x - 1; }
    }
    __syncthreads();
    uint16_t* dst = out.run_data + (rec.z >> 1);
    for (uint32_t k = t; k < tot_s; k += kEmitThreads) {
      dst[2 * k] = s_starts[k];
      dst[2 * k + 1] = static_cast<uint16_t>(s_ends[k] - s_starts[k]);
    }
  }
}

// ----------------------------------------------------------- ids -> slots

// Sparse mode: mark the high-16 keys present in the input (8 KiB presence in
// shared memory per CTA, merged into the global presence once per CTA).
__global__ void __launch_bounds__(256) k_mark(const uint32_t* ids, uint64_t n, uint32_t U,
                                              unsigned long long* presence, uint32_t* err)
{
  __shared__ unsigned long long s_pres[1024];
  for (int i = threadIdx.x; i < 1024; i += 256) s_pres[i] = 0;
  __syncthreads();
  bool bad = false;
  const uint64_t stride = uint64_t(gridDim.x) * 256;
  for (uint64_t i = uint64_t(blockIdx.x) * 256 + threadIdx.x; i < n; i += stride) {
    const uint32_t id = __ldg(ids + i);
    if (id >= U) { bad = true; continue; }
    const uint32_t key = id >> 16;
    atomicOr(&s_pres[key >> 6], 1ull << (key & 63));
  }
  if (__any_sync(0xFFFFFFFFu, bad) && (threadIdx.x & 31) == 0) atomicOr(err, 1u);
  __syncthreads();
  for (int i = threadIdx.x; i < 1024; i += 256)
    if (s_pres[i]) atomicOr(presence + i, s_pres[i]);
}

// Sparse mode: slot = rank of the key among present keys (single CTA).
__global__ void __launch_bounds__(1024) k_assign_slots(const unsigned long long* presence,
                                                       uint32_t* chunk_slot,
                                                       uint16_t* slot_keys, uint32_t* n_slots)
{
  __shared__ uint32_t s_red[32];
  const uint64_t w = presence[threadIdx.x];
  uint32_t total;
  uint32_t base = block_exclusive_scan<1024>(static_cast<uint32_t>(__popcll(w)), s_red, &total);
  uint64_t x = w;
  while (x) {
    const uint32_t key = threadIdx.x * 64u + __ffsll(x) - 1;
    chunk_slot[key] = base;
    slot_keys[base] = static_cast<uint16_t>(key);
    ++base;
    x &= x - 1;
  }
  if (threadIdx.x == 0) *n_slots = total;
}

__global__ void k_zero_slots(uint4* words, const uint32_t* n_slots)
{
  const uint64_t n = uint64_t(*n_slots) * (kBitmapBytes / 16);
  const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
  for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
    words[i] = make_uint4(0, 0, 0, 0);
}

__device__ __forceinline__ void scatter_one(uint32_t id, uint32_t U, const uint32_t* chunk_slot,
                                            uint32_t* words, bool& bad, uint32_t slot_lo, uint32_t slot_hi)
{
  if (id >= U) { bad = true; return; }
  const uint32_t key = id >> 16;
  const uint32_t slot = chunk_slot ? __ldg(chunk_slot + key) : key;
  if (slot < slot_lo || slot >= slot_hi) return;  // another pass's slots
  atomicOr(words + uint64_t(slot) * kChunkWords32 + ((id & 0xFFFFu) >> 5), 1u << (id & 31u));
}

// OR every ID whose chunk slot lies in [slot_lo, slot_hi) into that slot.
// Vector loads when the input is 16-byte aligned; the result is independent
// of order and duplicates.
__global__ void __launch_bounds__(256) k_scatter(const uint32_t* ids, uint64_t n, uint32_t U,
                                                 const uint32_t* chunk_slot, uint32_t* words,
                                                 uint32_t* err, int vec, uint32_t slot_lo, uint32_t slot_hi,
                                                 const uint32_t* n_slots)
{
  // Sparse inputs size their passes by the host bound min(n, chunks); a pass
  // whose slot range starts past the slots actually used has nothing to do.
  if (n_slots && slot_lo >= *n_slots) return;
  bool bad = false;
  const uint64_t stride = uint64_t(gridDim.x) * 256;
  const uint64_t tid = uint64_t(blockIdx.x) * 256 + threadIdx.x;
  uint64_t head = 0;
  if (vec) {
    const uint64_t n4 = n / 4;
    const uint4* p = reinterpret_cast<const uint4*>(ids);
    for (uint64_t i = tid; i < n4; i += stride) {
      const uint4 v = __ldg(p + i);
      scatter_one(v.x, U, chunk_slot, words, bad, slot_lo, slot_hi);
      scatter_one(v.y, U, chunk_slot, words, bad, slot_lo, slot_hi);
      scatter_one(v.z, U, chunk_slot, words, bad, slot_lo, slot_hi);
      scatter_one(v.w, U, chunk_slot, words, bad, slot_lo, slot_hi);
    }
    head = n4 * 4;
  }
  for (uint64_t i = head + tid; i < n; i += stride)
    scatter_one(__ldg(ids + i), U, chunk_slot, words, bad, slot_lo, slot_hi);
  if (__any_sync(0xFFFFFFFFu, bad) && (threadIdx.x & 31) == 0) atomicOr(err, 1u);
}

}  // namespace

constexpr size_t kPassBytes = size_t(32) << 20;  // words per scatter pass (well inside L2)

// Runs analyze -> plan -> (sync) -> allocate -> emit over chunk slots.
static void build_from_chunks(const ChunkSrc& src, uint32_t max_slots, uint32_t U, uint32_t thr,
                              const uint32_t* d_err, cudaStream_t s, cr_gpu_roaring* out)
{
  std::memset(out, 0, sizeof(*out));
  out->universe_size = U;
  if (max_slots == 0) return;
  const uint32_t n_tiles = div_up(max_slots, kPlanTile);
  uint32_t t0 = thr, t1 = thr, guard = 0;
  if (thr == kPromoteAuto) {
    t0 = resolve_auto(U, -1);
    t1 = kPromoteKeep;
    guard = t0 < kPromoteKeep;
  }
  const size_t stats_b = size_t(max_slots) * 16, plan_b = stats_b;
  const size_t tiles_b = size_t(n_tiles) * sizeof(PlanTotals);
  Scratch scr(stats_b + plan_b + tiles_b + sizeof(PlanHeader) + 64, s);
  char* base = scr.as<char>();
  uint4* stats = reinterpret_cast<uint4*>(base);
  uint4* plan = reinterpret_cast<uint4*>(base + stats_b);
  PlanTotals* tiles = reinterpret_cast<PlanTotals*>(base + stats_b + plan_b);
  PlanHeader* d_hdr = reinterpret_cast<PlanHeader*>(base + stats_b + plan_b + tiles_b);
  unsigned long long* d_total =
      reinterpret_cast<unsigned long long*>(base + stats_b + plan_b + tiles_b + sizeof(PlanHeader));
  CR_CUDA(cudaMemsetAsync(d_total, 0, 8, s));
  const bool vec = (reinterpret_cast<uintptr_t>(src.words) & 15u) == 0;
  if (vec) k_analyze<true><<<max_slots, kEmitThreads, 0, s>>>(src, max_slots, stats, d_total);
  else k_analyze<false><<<max_slots, kEmitThreads, 0, s>>>(src, max_slots, stats, d_total);
  k_plan_tiles<<<n_tiles, kPlanTile, 0, s>>>(src, max_slots, stats, d_total, t0, t1, tiles);
  k_plan_emit<<<n_tiles, kPlanTile, 0, s>>>(src, max_slots, stats, d_total, t0, t1, guard, tiles,
                                            n_tiles, plan, d_hdr, d_err);
  CR_CUDA(cudaGetLastError());
  PlanHeader* hp = static_cast<PlanHeader*>(pinned_stage(sizeof(PlanHeader)));
  CR_CUDA(cudaMemcpyAsync(hp, d_hdr, sizeof(PlanHeader), cudaMemcpyDeviceToHost, s));
  CR_CUDA(cudaStreamSynchronize(s));
  const PlanHeader h = *hp;
  if (h.err) fail(CR_ERR_RANGE, "upload: an input ID is >= universe_size");
  out->negated = h.negated != 0;
  out->total_cardinality = h.total_logical;
  out->n_containers = h.n_cont;
  out->n_bitmap_containers = h.nb;
  out->n_array_containers = h.na;
  out->n_run_containers = h.nr;
  if (h.array_bytes > 0xFFFFFFFFull || h.run_bytes > 0xFFFFFFFFull)
    fail(CR_ERR_UNSUPPORTED, "upload: array or run pool exceeds 4 GiB");
  out->array_pool_bytes = static_cast<uint32_t>(h.array_bytes);
  out->run_pool_bytes = static_cast<uint32_t>(h.run_bytes);
  if (h.n_cont == 0) return;
  out->max_key = max_key_for(U);
  alloc_result(out, s);
  CR_CUDA(cudaMemsetAsync(out->key_index, 0xFF, (size_t(out->max_key) + 1u) * 2u, s));
  ProfileScope prof(CR_KERNEL_UPLOAD_EMIT, s);
  if (vec) k_emit<true><<<max_slots, kEmitThreads, 0, s>>>(src, max_slots, plan, d_hdr, *out);
  else k_emit<false><<<max_slots, kEmitThreads, 0, s>>>(src, max_slots, plan, d_hdr, *out);
  CR_CUDA(cudaGetLastError());
}

static int grid_for(uint64_t n, int per_sm)
{
  const uint64_t want = (n + 255) / 256;
  const uint64_t cap = uint64_t(sm_count()) * per_sm;
  return static_cast<int>(std::max<uint64_t>(1, std::min(want, cap)));
}

void upload_device_ids(const uint32_t* d_ids, uint64_t n, uint32_t U, uint32_t thr,
                       cudaStream_t s, cr_gpu_roaring* out)
{
  std::memset(out, 0, sizeof(*out));
  out->universe_size = U;
  if (n == 0 || U == 0) {
    // Still reject out-of-range IDs for U == 0 inputs.
    if (n && U == 0) fail(CR_ERR_RANGE, "upload: an input ID is >= universe_size");
    return;
  }
  CR_REQUIRE(d_ids != nullptr, "upload: null ID pointer");
  const uint32_t n_chunks = n_chunks_for(U);
  // Dense: one slot per chunk of the universe (needed whenever the
  // complement could be taken, which requires n > U/2). Sparse: slots only
  // for touched chunks, so tiny inputs in huge universes stay cheap.
  const bool dense = n >= uint64_t(n_chunks) * 1024u || n_chunks <= 64;
  const uint32_t max_slots = dense ? n_chunks : static_cast<uint32_t>(std::min<uint64_t>(n, n_chunks));
  const size_t words_b = size_t(max_slots) * kBitmapBytes;
  const size_t aux_b = dense ? 64 : (8192 + 65536 * 4 + 65536 * 2 + 64);
  Scratch scr(words_b + aux_b, s);
  char* base = scr.as<char>();
  uint32_t* words = reinterpret_cast<uint32_t*>(base);
  char* aux = base + words_b;
  uint32_t* d_err = reinterpret_cast<uint32_t*>(aux);
  ChunkSrc src{};
  src.words = words;
  src.n_words = uint64_t(max_slots) * kChunkWords32;
  src.universe = U;
  const int vec = (reinterpret_cast<uintptr_t>(d_ids) & 15u) == 0;
  // The OR reductions go to L2; a word array much larger than L2 makes each
  // one a DRAM read-modify-write. Above kPassBytes the IDs are streamed once
  // per slot range of kPassBytes of words (reading the IDs again is cheaper
  // than the missed reductions).
  const uint32_t slots_per_pass = std::max<uint32_t>(1u, uint32_t(kPassBytes / kBitmapBytes));
  auto scatter_passes = [&](const uint32_t* chunk_slot, const uint32_t* n_slots) {
    for (uint32_t lo = 0; lo < max_slots; lo += slots_per_pass)
      k_scatter<<<grid_for(n, 8), 256, 0, s>>>(d_ids, n, U, chunk_slot, words, d_err, vec, lo,
                                               std::min<uint64_t>(max_slots, uint64_t(lo) + slots_per_pass),
                                               n_slots);
  };
  if (dense) {
    CR_CUDA(cudaMemsetAsync(base, 0, words_b + 64, s));
    ProfileScope prof(CR_KERNEL_UPLOAD_SCATTER, s);
    scatter_passes(nullptr, nullptr);
  } else {
    unsigned long long* presence = reinterpret_cast<unsigned long long*>(aux + 64);
    uint32_t* chunk_slot = reinterpret_cast<uint32_t*>(aux + 64 + 8192);
    uint16_t* slot_keys = reinterpret_cast<uint16_t*>(aux + 64 + 8192 + 65536 * 4);
    uint32_t* n_slots = d_err + 1;
    CR_CUDA(cudaMemsetAsync(aux, 0, 64 + 8192, s));
    k_mark<<<grid_for(n, 4), 256, 0, s>>>(d_ids, n, U, presence, d_err);
    k_assign_slots<<<1, 1024, 0, s>>>(presence, chunk_slot, slot_keys, n_slots);
    k_zero_slots<<<std::max(1, std::min<int>(sm_count() * 4, div_up(words_b / 16, 256))), 256, 0, s>>>(
        reinterpret_cast<uint4*>(words), n_slots);
    scatter_passes(chunk_slot, n_slots);
    src.slot_keys = slot_keys;
    src.n_slots = n_slots;
  }
  CR_CUDA(cudaGetLastError());
  build_from_chunks(src, max_slots, U, thr, d_err, s, out);
}

void upload_device_bitset(const uint32_t* d_words, uint64_t n_words, uint32_t U, uint32_t thr,
                          cudaStream_t s, cr_gpu_roaring* out, bool keep_uncomplemented)
{
  std::memset(out, 0, sizeof(*out));
  out->universe_size = U;
  if (n_words == 0 || U == 0) return;
  CR_REQUIRE(d_words != nullptr, "upload_from_bitset: null bitset pointer");
  ChunkSrc src{};
  src.words = d_words;
  src.n_words = std::min<uint64_t>(n_words, uint64_t(n_chunks_for(U)) * kChunkWords32);
  src.universe = U;
  src.keep_uncomplemented = keep_uncomplemented ? 1u : 0u;
  build_from_chunks(src, n_chunks_for(U), U, thr, nullptr, s, out);
}

}  // namespace crb

using namespace crb;

extern "C" int cr_upload_from_device_ids(const uint32_t* d_ids, uint64_t n_ids, uint32_t U,
                                         cr_stream_t stream, uint32_t thr, cr_gpu_roaring* out)
{
  CR_API_BEGIN
  CR_REQUIRE(out != nullptr, "cr_upload_from_device_ids: null output");
  upload_device_ids(d_ids, n_ids, U, thr, reinterpret_cast<cudaStream_t>(stream), out);
  CR_API_END
}

extern "C" int cr_upload_from_ids(const uint32_t* host_ids, uint32_t n_ids, uint32_t U,
                                  cr_stream_t stream, uint32_t thr, cr_gpu_roaring* out)
{
  CR_API_BEGIN
  CR_REQUIRE(out != nullptr, "cr_upload_from_ids: null output");
  CR_REQUIRE(host_ids != nullptr || n_ids == 0, "cr_upload_from_ids: null IDs");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  Scratch ids(size_t(n_ids) * 4, s);
  if (n_ids) CR_CUDA(cudaMemcpyAsync(ids.p, host_ids, size_t(n_ids) * 4, cudaMemcpyHostToDevice, s));
  upload_device_ids(ids.as<uint32_t>(), n_ids, U, thr, s, out);
  CR_API_END
}

extern "C" int cr_upload_from_device_bitset(const uint32_t* d_bitset, uint32_t n_words, uint32_t U,
                                            cr_stream_t stream, uint32_t thr, cr_gpu_roaring* out)
{
  CR_API_BEGIN
  CR_REQUIRE(out != nullptr, "cr_upload_from_device_bitset: null output");
  upload_device_bitset(d_bitset, n_words, U, thr, reinterpret_cast<cudaStream_t>(stream), out);
  CR_API_END
}

extern "C" int cr_upload_from_bitset(const uint32_t* host_bitset, uint32_t n_words, uint32_t U,
                                     cr_stream_t stream, uint32_t thr, cr_gpu_roaring* out)
{
  CR_API_BEGIN
  CR_REQUIRE(out != nullptr, "cr_upload_from_bitset: null output");
  CR_REQUIRE(host_bitset != nullptr || n_words == 0, "cr_upload_from_bitset: null bitset");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  Scratch bits(size_t(n_words) * 4, s);
  if (n_words)
    CR_CUDA(cudaMemcpyAsync(bits.p, host_bitset, size_t(n_words) * 4, cudaMemcpyHostToDevice, s));
  upload_device_bitset(bits.as<uint32_t>(), n_words, U, thr, s, out);
  CR_API_END
}
