// cu_roaring B200 engine — set algebra: set_operation, multi_and, multi_or.
//
// Replaces reference src/set_ops.cu, whose pairwise path downloads both
// index arrays, merges keys on the host, classifies pairs on the host and
// launches one kernel per class with 5-7 host syncs (src/set_ops.cu:567-1207).
// Here every operation is ONE k-way combine over the 65536 key space:
//
//   MODE_AND_SUB: result = AND(P) minus OR(N), keys common to every P operand
//   MODE_OR / MODE_XOR: over the union of keys of all P operands
//
// set_operation maps onto it after the reference's DeMorgan rewrite of
// negated operands (src/set_ops.cu:512-565); multi_and puts non-negated
// inputs in P and negated ones in N (so negated inputs never inflate the
// result); multi_or is ~multi_and(~inputs).
//
// Pipeline (2 host syncs, both for sizes the host-side struct must hold):
//   k_plan_tiles/k_plan_work : per key, through each operand's key_index,
//     decide presence, structural output type and a payload bound; compact
//     the work list in key order.                              -> sync 1
//   allocate the packed block (bound sizes)
//   k_execute : one CTA per output container; all-BITMAP operands stream
//     with 16-byte loads, ARRAY/RUN operands expand in shared memory;
//     BITMAP results go straight to their slot, ARRAY results to scratch.
//   k_final_tiles : totals of the non-empty results          -> sync 2
//   k_final_meta + k_final_payload : compact metadata, key_index, array
//     pool (and, only when an empty BITMAP left a hole, a repack into a new
//     exact-size block so BITMAP slot == rank keeps holding).
//
// Output typing rule (structural; the oracle restates it): a key held by a
// single contributing operand is copied through with its type; AND_SUB with an
// ARRAY among the P containers -> ARRAY; OR/XOR of ARRAYs only whose
// cardinalities sum to <= 4096 -> ARRAY; otherwise BITMAP. Empty results are
// dropped (reference src/set_ops.cu:1111-1145).
#include <algorithm>
#include <vector>

#include "chunk_ops.cuh"

namespace crb {
namespace {

constexpr int kMaxOperands = 64;
constexpr int kTile = 1024;
enum { MODE_AND_SUB = 0, MODE_OR = 1, MODE_XOR = 2 };

struct Operands {
  DevBitmap op[kMaxOperands];
  uint32_t np, nn, mode, n_keys;
  uint32_t res_max_key;  // keys above it (IDs beyond the universe) are an error
};

// Per-key decision. Returns false when the key produces no work item.
struct KeyPlan {
  uint8_t type;       // output type
  uint8_t copy;       // 1 = copy-through
  uint8_t src;        // copy-through operand
  int src_idx;        // copy-through container
  uint32_t bound;     // payload bytes upper bound
  uint8_t pair;       // two operands, both BITMAP here: their pool offsets below
  uint32_t a_off, b_off;
};

__device__ __forceinline__ bool plan_key(const Operands& ops, uint32_t key, KeyPlan& kp)
{
  int holders = 0, first = -1, first_idx = -1;
  bool any_array = false, all_array = true;
  uint32_t min_arr = 0xFFFFFFFFu, sum_card = 0;
  for (uint32_t j = 0; j < ops.np; ++j) {
    const int idx = dev_lookup(ops.op[j], key);
    if (idx < 0) { if (ops.mode == MODE_AND_SUB) return false; continue; }
    ++holders;
    if (first < 0) { first = static_cast<int>(j); first_idx = idx; }
    const uint8_t t = __ldg(ops.op[j].types + idx);
    if (t == kArray) {
      const uint32_t c = __ldg(ops.op[j].cards + idx);
      any_array = true;
      min_arr = min(min_arr, c);
      sum_card += c;
    } else {
      all_array = false;
    }
  }
  if (holders == 0) return false;
  bool n_hold = false;
  for (uint32_t j = ops.np; j < ops.np + ops.nn && !n_hold; ++j) n_hold = dev_lookup(ops.op[j], key) >= 0;
  if (holders == 1 && !n_hold) {
    const DevBitmap& b = ops.op[first];
    kp.copy = 1;
    kp.src = static_cast<uint8_t>(first);
    kp.src_idx = first_idx;
    kp.type = __ldg(b.types + first_idx);
    const uint32_t c = __ldg(b.cards + first_idx);
    kp.bound = kp.type == kBitmap ? kBitmapBytes : (kp.type == kArray ? 2u * c : 4u * c);
    return true;
  }
  kp.copy = 0; kp.src = 0; kp.src_idx = -1; kp.pair = 0;
  if (ops.np + ops.nn == 2) {
    // Two operands both holding the key as BITMAP containers: the executor
    // reads their words straight from these pool offsets.
    const int ia = dev_lookup(ops.op[0], key), ib = dev_lookup(ops.op[1], key);
    if (ia >= 0 && ib >= 0) {
      const ContainerRef ca = dev_container(ops.op[0], ia), cb = dev_container(ops.op[1], ib);
      if (ca.type == kBitmap && cb.type == kBitmap) {
        kp.pair = 1;
        kp.a_off = ca.off;
        kp.b_off = cb.off;
      }
    }
  }
  if (ops.mode == MODE_AND_SUB) {
    kp.type = any_array ? kArray : kBitmap;
    kp.bound = any_array ? 2u * min_arr : kBitmapBytes;
  } else {
    const bool arr = all_array && sum_card <= kPromoteKeep;
    kp.type = arr ? kArray : kBitmap;
    kp.bound = arr ? 2u * sum_card : kBitmapBytes;
  }
  return true;
}

struct WorkTotals {
  uint32_t n, nb;
  unsigned long long ab, rb;
  uint32_t err, pad;
};

__global__ void __launch_bounds__(kTile) k_plan_tiles(const Operands* __restrict__ ops_p,
                                                      WorkTotals* tiles)
{
  __shared__ unsigned long long s_red[32];
  const Operands& ops = *ops_p;
  const uint32_t key = blockIdx.x * kTile + threadIdx.x;
  KeyPlan kp{};
  const bool has = key < ops.n_keys && plan_key(ops, key, kp);
  WorkTotals t{};
  t.n = static_cast<uint32_t>(block_sum<kTile, unsigned long long>(has, s_red));
  t.nb = static_cast<uint32_t>(block_sum<kTile, unsigned long long>(has && kp.type == kBitmap, s_red));
  t.ab = block_sum<kTile, unsigned long long>(has && kp.type == kArray ? kp.bound : 0u, s_red);
  t.rb = block_sum<kTile, unsigned long long>(has && kp.type == kRun ? kp.bound : 0u, s_red);
  if (threadIdx.x == 0) tiles[blockIdx.x] = t;
}

// work[w] = (key | type<<16 | copy<<24, bound offset, src operand, src idx);
// for a BITMAP pair (not copy-through): z = first operand's pool offset / 8
// + 1, w = second's / 8 (z = 0 otherwise).
__global__ void __launch_bounds__(kTile) k_plan_work(const Operands* __restrict__ ops_p,
                                                     const WorkTotals* tiles, uint32_t n_tiles,
                                                     uint4* work, WorkTotals* header)
{
  __shared__ unsigned long long s_red[32];
  __shared__ WorkTotals s_base, s_all;
  const Operands& ops = *ops_p;
  if (threadIdx.x == 0) {
    WorkTotals b{}, a{};
    for (uint32_t j = 0; j < n_tiles; ++j) {
      const WorkTotals x = tiles[j];
      a.n += x.n; a.nb += x.nb; a.ab += x.ab; a.rb += x.rb;
      if (j < blockIdx.x) { b.n += x.n; b.nb += x.nb; b.ab += x.ab; b.rb += x.rb; }
    }
    s_base = b;
    s_all = a;
  }
  __syncthreads();
  const uint32_t key = blockIdx.x * kTile + threadIdx.x;
  KeyPlan kp{};
  const bool has = key < ops.n_keys && plan_key(ops, key, kp);
  unsigned long long tot;
  const unsigned long long wi = block_exclusive_scan<kTile, unsigned long long>(has, s_red, &tot);
  const unsigned long long bs = block_exclusive_scan<kTile, unsigned long long>(has && kp.type == kBitmap, s_red, &tot);
  const unsigned long long ao = block_exclusive_scan<kTile, unsigned long long>(has && kp.type == kArray ? kp.bound : 0u, s_red, &tot);
  const unsigned long long ro = block_exclusive_scan<kTile, unsigned long long>(has && kp.type == kRun ? kp.bound : 0u, s_red, &tot);
  if (has && key > ops.res_max_key) atomicOr(&header->err, 1u);
  if (has) {
    uint32_t off;
    if (kp.type == kBitmap) off = static_cast<uint32_t>((s_base.nb + bs) * kBitmapBytes);
    else if (kp.type == kArray) off = static_cast<uint32_t>(s_base.ab + ao);
    else off = static_cast<uint32_t>(s_base.rb + ro);
    work[s_base.n + wi] = make_uint4(key | (uint32_t(kp.type) << 16) | (uint32_t(kp.copy) << 24), off,
                                     kp.pair ? (kp.a_off >> 3) + 1u : kp.src,
                                     kp.pair ? (kp.b_off >> 3) : static_cast<uint32_t>(kp.src_idx));
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    header->n = s_all.n;
    header->nb = s_all.nb;
    header->ab = s_all.ab;
    header->rb = s_all.rb;
  }
}

__device__ __forceinline__ void store4(uint64_t* dst, const uint64_t w[4])
{
  uint4* p = reinterpret_cast<uint4*>(dst) + 2 * threadIdx.x;
  p[0] = make_uint4(uint32_t(w[0]), uint32_t(w[0] >> 32), uint32_t(w[1]), uint32_t(w[1] >> 32));
  p[1] = make_uint4(uint32_t(w[2]), uint32_t(w[2] >> 32), uint32_t(w[3]), uint32_t(w[3] >> 32));
}

// One CTA per work item. counts[w] = element count of the result container.
// Eight resident blocks per SM (32 registers a thread): the block's work is a
// short chain of dependent loads, so latency hiding needs occupancy.
__global__ void __launch_bounds__(256, 8) k_execute(const Operands* __restrict__ ops_p,
                                                 const uint4* __restrict__ work,
                                                 cr_gpu_roaring out, uint16_t* arr_scratch,
                                                 uint32_t* counts)
{
  __shared__ __align__(16) uint64_t sm[1024];
  __shared__ uint32_t s_red[8];
  const Operands& ops = *ops_p;
  const uint4 item = work[blockIdx.x];
  const uint32_t key = item.x & 0xFFFFu;
  const uint8_t type = (item.x >> 16) & 0xFFu;
  const bool copy = (item.x >> 24) != 0;
  const uint32_t off = item.y;
  const uint32_t t = threadIdx.x;
  if (copy) {
    const DevBitmap& b = ops.op[item.z];
    const ContainerRef c = dev_container(b, static_cast<int>(item.w));
    uint32_t count;
    if (type == kBitmap) {
      const uint4* src = reinterpret_cast<const uint4*>(b.bitmap + (c.off >> 3));
      uint4* dst = reinterpret_cast<uint4*>(out.bitmap_data + (off >> 3));
      dst[2 * t] = __ldg(src + 2 * t);
      dst[2 * t + 1] = __ldg(src + 2 * t + 1);
      count = c.card ? c.card : 65536u;
    } else if (type == kArray) {
      const uint16_t* src = b.array + (c.off >> 1);
      for (uint32_t j = t; j < c.card; j += 256) arr_scratch[(off >> 1) + j] = __ldg(src + j);
      count = c.card;
    } else {
      const uint16_t* src = b.run + (c.off >> 1);
      for (uint32_t j = t; j < 2 * c.card; j += 256) out.run_data[(off >> 1) + j] = __ldg(src + j);
      count = c.card;  // only non-zero-ness matters for runs
    }
    if (t == 0) counts[blockIdx.x] = count;
    return;
  }
  uint64_t acc[4], w[4];
  const bool and_sub = ops.mode == MODE_AND_SUB;
#pragma unroll
  for (int i = 0; i < 4; ++i) acc[i] = and_sub ? ~0ull : 0ull;
  // Fast path for two operands that are both BITMAP containers here (every
  // set_operation on promoted layouts): the planner recorded both pool
  // offsets, so the block issues its data loads at once, with no metadata
  // reads in front of them.
  bool done = false;
  if (item.z != 0) {
    const uint4* qa = reinterpret_cast<const uint4*>(ops.op[0].bitmap + (item.z - 1)) + 2 * t;
    const uint4* qb = reinterpret_cast<const uint4*>(ops.op[1].bitmap + item.w) + 2 * t;
    const uint4 a0 = __ldg(qa), a1 = __ldg(qa + 1), b0 = __ldg(qb), b1 = __ldg(qb + 1);
    const uint64_t av[4] = {uint64_t(a0.x) | (uint64_t(a0.y) << 32), uint64_t(a0.z) | (uint64_t(a0.w) << 32),
                            uint64_t(a1.x) | (uint64_t(a1.y) << 32), uint64_t(a1.z) | (uint64_t(a1.w) << 32)};
    const uint64_t bv[4] = {uint64_t(b0.x) | (uint64_t(b0.y) << 32), uint64_t(b0.z) | (uint64_t(b0.w) << 32),
                            uint64_t(b1.x) | (uint64_t(b1.y) << 32), uint64_t(b1.z) | (uint64_t(b1.w) << 32)};
    const bool b_neg = ops.np == 1;  // ANDNOT: the second operand is subtracted
#pragma unroll
    for (int i = 0; i < 4; ++i)
      acc[i] = b_neg ? (av[i] & ~bv[i])
                     : (and_sub ? (av[i] & bv[i]) : (ops.mode == MODE_OR ? (av[i] | bv[i]) : (av[i] ^ bv[i])));
    done = true;
  }
  for (uint32_t j = 0; j < (done ? 0u : ops.np); ++j) {
    const DevBitmap& b = ops.op[j];
    const int idx = dev_lookup(b, key);
    if (idx < 0) continue;
    container_words<256, 4>(b, dev_container(b, idx), sm, w);
#pragma unroll
    for (int i = 0; i < 4; ++i)
      acc[i] = and_sub ? (acc[i] & w[i]) : (ops.mode == MODE_OR ? (acc[i] | w[i]) : (acc[i] ^ w[i]));
  }
  for (uint32_t j = ops.np; j < (done ? 0u : ops.np + ops.nn); ++j) {
    const DevBitmap& b = ops.op[j];
    const int idx = dev_lookup(b, key);
    if (idx < 0) continue;
    container_words<256, 4>(b, dev_container(b, idx), sm, w);
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[i] &= ~w[i];
  }
  uint32_t cnt = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) cnt += __popcll(acc[i]);
  uint32_t total;
  uint32_t pos = block_exclusive_scan<256>(cnt, s_red, &total);
  if (type == kBitmap) {
    store4(out.bitmap_data + (off >> 3), acc);
  } else {
    uint16_t* dst = arr_scratch + (off >> 1);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint64_t x = acc[i];
      while (x) {
        dst[pos++] = static_cast<uint16_t>((4 * t + i) * 64 + __ffsll(x) - 1);
        x &= x - 1;
      }
    }
  }
  if (t == 0) counts[blockIdx.x] = total;
}

struct FinalTotals {
  uint32_t n, nb, na, nr, holes, pad;
  unsigned long long ab, rb, stored;
};

__device__ __forceinline__ void final_item(const uint4& item, uint32_t count, bool& keep,
                                           uint8_t& type, uint32_t& abytes, uint32_t& rbytes)
{
  type = (item.x >> 16) & 0xFFu;
  keep = count > 0;
  abytes = keep && type == kArray ? 2u * count : 0u;
  rbytes = keep && type == kRun ? 4u * count : 0u;
}

__global__ void __launch_bounds__(kTile) k_final_tiles(const uint4* work, const uint32_t* counts,
                                                       uint32_t n_work,
                                                       const Operands* ops_p, FinalTotals* tiles)
{
  __shared__ unsigned long long s_red[32];
  const uint32_t w = blockIdx.x * kTile + threadIdx.x;
  bool keep = false;
  uint8_t type = 0xFF;
  uint32_t ab = 0, rb = 0, count = 0;
  unsigned long long stored = 0;
  if (w < n_work) {
    const uint4 item = work[w];
    count = counts[w];
    final_item(item, count, keep, type, ab, rb);
    if (keep) {
      if (type == kRun) {
        // count holds the run count; the stored element total needs the lengths.
        const DevBitmap& b = ops_p->op[item.z];
        stored = container_count(b, dev_container(b, static_cast<int>(item.w)));
      } else {
        stored = count;
      }
    }
  }
  FinalTotals f{};
  f.n = static_cast<uint32_t>(block_sum<kTile, unsigned long long>(keep, s_red));
  f.nb = static_cast<uint32_t>(block_sum<kTile, unsigned long long>(keep && type == kBitmap, s_red));
  f.na = static_cast<uint32_t>(block_sum<kTile, unsigned long long>(keep && type == kArray, s_red));
  f.nr = static_cast<uint32_t>(block_sum<kTile, unsigned long long>(keep && type == kRun, s_red));
  f.holes = static_cast<uint32_t>(block_sum<kTile, unsigned long long>(!keep && type == kBitmap, s_red));
  f.ab = block_sum<kTile, unsigned long long>(ab, s_red);
  f.rb = block_sum<kTile, unsigned long long>(rb, s_red);
  f.stored = block_sum<kTile, unsigned long long>(stored, s_red);
  if (threadIdx.x == 0) tiles[blockIdx.x] = f;
}

// Writes the final metadata + key_index into `dst`; dst_off[w] = final
// payload byte offset of kept item w.
__global__ void __launch_bounds__(kTile) k_final_meta(const uint4* work, const uint32_t* counts,
                                                      uint32_t n_work, const FinalTotals* tiles,
                                                      uint32_t n_tiles, int repack,
                                                      cr_gpu_roaring dst, uint32_t* dst_off)
{
  __shared__ unsigned long long s_red[32];
  __shared__ FinalTotals s_base;
  if (threadIdx.x == 0) {
    FinalTotals b{};
    for (uint32_t j = 0; j < blockIdx.x && j < n_tiles; ++j) {
      b.n += tiles[j].n; b.nb += tiles[j].nb; b.ab += tiles[j].ab; b.rb += tiles[j].rb;
    }
    s_base = b;
  }
  __syncthreads();
  const uint32_t w = blockIdx.x * kTile + threadIdx.x;
  bool keep = false;
  uint8_t type = 0xFF;
  uint32_t ab = 0, rb = 0, count = 0;
  uint4 item = make_uint4(0, 0, 0, 0);
  if (w < n_work) {
    item = work[w];
    count = counts[w];
    final_item(item, count, keep, type, ab, rb);
  }
  unsigned long long tot;
  const unsigned long long ci = block_exclusive_scan<kTile, unsigned long long>(keep, s_red, &tot);
  const unsigned long long bs = block_exclusive_scan<kTile, unsigned long long>(keep && type == kBitmap, s_red, &tot);
  const unsigned long long ao = block_exclusive_scan<kTile, unsigned long long>(ab, s_red, &tot);
  const unsigned long long ro = block_exclusive_scan<kTile, unsigned long long>(rb, s_red, &tot);
  if (!keep) return;
  const uint32_t i = static_cast<uint32_t>(s_base.n + ci);
  const uint32_t key = item.x & 0xFFFFu;
  uint32_t off;
  uint16_t card;
  if (type == kBitmap) {
    off = repack ? static_cast<uint32_t>((s_base.nb + bs) * kBitmapBytes) : item.y;
    card = static_cast<uint16_t>(count & 0xFFFFu);
  } else if (type == kArray) {
    off = static_cast<uint32_t>(s_base.ab + ao);
    card = static_cast<uint16_t>(count);
  } else {
    off = static_cast<uint32_t>(s_base.rb + ro);
    card = static_cast<uint16_t>(count);
  }
  dst.keys[i] = static_cast<uint16_t>(key);
  dst.types[i] = type;
  dst.offsets[i] = off;
  dst.cardinalities[i] = card;
  if (key <= dst.max_key) dst.key_index[key] = static_cast<uint16_t>(i);
  dst_off[w] = off;
}

// Payload moves: ARRAY results from scratch into the pool; with `repack`,
// BITMAP and RUN payloads from the bound-layout block into the exact one.
__global__ void __launch_bounds__(256) k_final_payload(const uint4* work, const uint32_t* counts,
                                                       const uint32_t* dst_off,
                                                       const uint16_t* arr_scratch,
                                                       cr_gpu_roaring old_block,
                                                       cr_gpu_roaring dst, int repack)
{
  const uint32_t w = blockIdx.x;
  const uint32_t count = counts[w];
  if (count == 0) return;
  const uint4 item = work[w];
  const uint8_t type = (item.x >> 16) & 0xFFu;
  const uint32_t off = dst_off[w];
  if (type == kArray) {
    const uint16_t* src = arr_scratch + (item.y >> 1);
    for (uint32_t j = threadIdx.x; j < count; j += 256) dst.array_data[(off >> 1) + j] = src[j];
  } else if (repack && type == kBitmap) {
    const uint4* src = reinterpret_cast<const uint4*>(old_block.bitmap_data + (item.y >> 3));
    uint4* d = reinterpret_cast<uint4*>(dst.bitmap_data + (off >> 3));
    d[2 * threadIdx.x] = src[2 * threadIdx.x];
    d[2 * threadIdx.x + 1] = src[2 * threadIdx.x + 1];
  } else if (repack && type == kRun) {
    for (uint32_t j = threadIdx.x; j < 2 * count; j += 256)
      dst.run_data[(off >> 1) + j] = old_block.run_data[(item.y >> 1) + j];
  }
}

}  // namespace

// The k-way combine (see the file comment). `P`/`N` are host structs.
void kway(const std::vector<const cr_gpu_roaring*>& P, const std::vector<const cr_gpu_roaring*>& N,
          int mode, bool negated, cudaStream_t s, cr_gpu_roaring* out)
{
  std::memset(out, 0, sizeof(*out));
  uint32_t U = 0;
  for (auto* b : P) U = std::max(U, b->universe_size);
  for (auto* b : N) U = std::max(U, b->universe_size);
  out->universe_size = U;
  out->negated = negated;
  if (negated) out->total_cardinality = U;
  const uint32_t np = static_cast<uint32_t>(P.size()), nn = static_cast<uint32_t>(N.size());
  CR_REQUIRE(np + nn <= kMaxOperands, "set operation: at most 64 operands");
  if (np == 0) return;

  std::vector<Scratch> holders(np + nn);
  Operands h_ops{};
  h_ops.np = np;
  h_ops.nn = nn;
  h_ops.mode = mode;
  uint32_t max_key = max_key_for(U);
  bool any_p_empty = false;
  for (uint32_t j = 0; j < np + nn; ++j) {
    const cr_gpu_roaring* b = j < np ? P[j] : N[j - np];
    h_ops.op[j] = make_dev(b, holders[j], s);
    if (b->n_containers) max_key = std::max(max_key, h_ops.op[j].max_key);
    if (j < np && b->n_containers == 0) any_p_empty = true;
  }
  if (mode == MODE_AND_SUB && any_p_empty) return;
  const uint32_t K = max_key + 1;
  h_ops.n_keys = K;
  h_ops.res_max_key = max_key_for(U);
  max_key = max_key_for(U);
  const uint32_t n_tiles = div_up(K, kTile);

  // scratch: operands | work | counts | dst_off | plan tiles | final tiles | headers
  const size_t ops_b = (sizeof(Operands) + 255) / 256 * 256;
  const size_t work_b = size_t(K) * 16, cnt_b = size_t(K) * 4;
  const size_t tiles_b = size_t(n_tiles) * sizeof(WorkTotals);
  const size_t ftiles_b = size_t(n_tiles) * sizeof(FinalTotals);
  Scratch scr(ops_b + work_b + 2 * cnt_b + tiles_b + ftiles_b + 256, s);
  char* p = scr.as<char>();
  Operands* d_ops = reinterpret_cast<Operands*>(p); p += ops_b;
  uint4* work = reinterpret_cast<uint4*>(p); p += work_b;
  uint32_t* counts = reinterpret_cast<uint32_t*>(p); p += cnt_b;
  uint32_t* dst_off = reinterpret_cast<uint32_t*>(p); p += cnt_b;
  WorkTotals* tiles = reinterpret_cast<WorkTotals*>(p); p += tiles_b;
  FinalTotals* ftiles = reinterpret_cast<FinalTotals*>(p); p += ftiles_b;
  WorkTotals* d_hdr = reinterpret_cast<WorkTotals*>(p);

  CR_CUDA(cudaMemcpyAsync(d_ops, &h_ops, sizeof(Operands), cudaMemcpyHostToDevice, s));
  CR_CUDA(cudaMemsetAsync(d_hdr, 0, sizeof(WorkTotals), s));
  k_plan_tiles<<<n_tiles, kTile, 0, s>>>(d_ops, tiles);
  k_plan_work<<<n_tiles, kTile, 0, s>>>(d_ops, tiles, n_tiles, work, d_hdr);
  CR_CUDA(cudaGetLastError());
  WorkTotals* hp = static_cast<WorkTotals*>(pinned_stage(sizeof(WorkTotals)));
  CR_CUDA(cudaMemcpyAsync(hp, d_hdr, sizeof(WorkTotals), cudaMemcpyDeviceToHost, s));
  CR_CUDA(cudaStreamSynchronize(s));  // sync 1: the work list size
  const WorkTotals h = *hp;
  if (h.err) fail(CR_ERR_RANGE, "set operation: an operand holds IDs beyond the result universe");
  if (h.n == 0) return;

  cr_gpu_roaring blk{};
  blk.universe_size = U;
  blk.n_containers = h.n;
  blk.n_bitmap_containers = h.nb;
  blk.array_pool_bytes = static_cast<uint32_t>(h.ab);
  blk.run_pool_bytes = static_cast<uint32_t>(h.rb);
  blk.max_key = max_key;
  alloc_result(&blk, s);
  Scratch arr(h.ab, s);
  {
    ProfileScope prof(CR_KERNEL_SETOP, s);
    k_execute<<<h.n, 256, 0, s>>>(d_ops, work, blk, arr.as<uint16_t>(), counts);
  }
  const uint32_t f_tiles = div_up(h.n, kTile);
  k_final_tiles<<<f_tiles, kTile, 0, s>>>(work, counts, h.n, d_ops, ftiles);
  CR_CUDA(cudaGetLastError());
  FinalTotals* ft = static_cast<FinalTotals*>(pinned_stage(f_tiles * sizeof(FinalTotals)));
  CR_CUDA(cudaMemcpyAsync(ft, ftiles, f_tiles * sizeof(FinalTotals), cudaMemcpyDeviceToHost, s));
  CR_CUDA(cudaStreamSynchronize(s));  // sync 2: the final sizes
  FinalTotals f{};
  for (uint32_t t = 0; t < f_tiles; ++t) {
    const FinalTotals& x = ft[t];
    f.n += x.n; f.nb += x.nb; f.na += x.na; f.nr += x.nr; f.holes += x.holes; f.ab += x.ab; f.rb += x.rb; f.stored += x.stored;
  }
  out->total_cardinality = negated ? uint64_t(U) - f.stored : f.stored;
  if (f.n == 0) {
    dev_free(blk._alloc_base, s);
    return;
  }
  const int repack = f.holes > 0;
  cr_gpu_roaring dst = blk;
  if (repack) {
    dst = cr_gpu_roaring{};
    dst.universe_size = U;
    dst.n_containers = f.n;
    dst.n_bitmap_containers = f.nb;
    dst.array_pool_bytes = static_cast<uint32_t>(f.ab);
    dst.run_pool_bytes = static_cast<uint32_t>(f.rb);
    dst.max_key = max_key;
    alloc_result(&dst, s);
  }
  CR_CUDA(cudaMemsetAsync(dst.key_index, 0xFF, (size_t(max_key) + 1) * 2, s));
  k_final_meta<<<f_tiles, kTile, 0, s>>>(work, counts, h.n, ftiles, f_tiles, repack, dst, dst_off);
  if (repack || f.na > 0)  // otherwise every payload already sits where the result wants it
    k_final_payload<<<h.n, 256, 0, s>>>(work, counts, dst_off, arr.as<uint16_t>(), blk, dst, repack);
  CR_CUDA(cudaGetLastError());
  if (repack) dev_free(blk._alloc_base, s);
  const uint64_t logical = out->total_cardinality;
  *out = dst;
  out->universe_size = U;
  out->negated = negated;
  out->total_cardinality = logical;
  out->n_containers = f.n;
  out->n_bitmap_containers = f.nb;
  out->n_array_containers = f.na;
  out->n_run_containers = f.nr;
  out->array_pool_bytes = static_cast<uint32_t>(f.ab);
  out->run_pool_bytes = static_cast<uint32_t>(f.rb);
  if (f.ab == 0) out->array_data = nullptr;
  if (f.rb == 0) out->run_data = nullptr;
  if (f.nb == 0) out->bitmap_data = nullptr;
}

}  // namespace crb

using namespace crb;

// DeMorgan rewrite of negated operands (reference src/set_ops.cu:512-565),
// then AND -> AND_SUB{a,b}; ANDNOT -> AND_SUB{a} minus {b}; OR; XOR.
extern "C" int cr_set_operation(const cr_gpu_roaring* a, const cr_gpu_roaring* b, int op,
                                cr_stream_t stream, cr_gpu_roaring* out)
{
  CR_API_BEGIN
  CR_REQUIRE(a && b && out, "cr_set_operation: null argument");
  CR_REQUIRE(op >= CR_OP_AND && op <= CR_OP_XOR, "cr_set_operation: unknown op");
  const bool na = a->negated != 0, nb = b->negated != 0;
  bool neg = false;
  const cr_gpu_roaring* x = a;
  const cr_gpu_roaring* y = b;
  if (na || nb) {
    switch (op) {
      case CR_OP_AND:
        if (na && !nb) { op = CR_OP_ANDNOT; std::swap(x, y); }
        else if (!na && nb) { op = CR_OP_ANDNOT; }
        else { op = CR_OP_OR; neg = true; }
        break;
      case CR_OP_OR:
        if (na && !nb) { op = CR_OP_ANDNOT; neg = true; }
        else if (!na && nb) { op = CR_OP_ANDNOT; std::swap(x, y); neg = true; }
        else { op = CR_OP_AND; neg = true; }
        break;
      case CR_OP_ANDNOT:
        if (na && !nb) { op = CR_OP_OR; neg = true; }
        else if (!na && nb) { op = CR_OP_AND; }
        else { op = CR_OP_ANDNOT; std::swap(x, y); }
        break;
      default:
        neg = na != nb;
        break;
    }
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (op == CR_OP_AND) kway({x, y}, {}, MODE_AND_SUB, neg, s, out);
  else if (op == CR_OP_ANDNOT) kway({x}, {y}, MODE_AND_SUB, neg, s, out);
  else kway({x, y}, {}, op == CR_OP_OR ? MODE_OR : MODE_XOR, neg, s, out);
  CR_API_END
}

static void multi(const cr_gpu_roaring* bms, uint32_t count, bool is_or, cudaStream_t s,
                  cr_gpu_roaring* out)
{
  std::memset(out, 0, sizeof(*out));
  if (count == 0) return;
  CR_REQUIRE(bms != nullptr, "multi_and/multi_or: null input array");
  if (count > uint32_t(kMaxOperands)) {
    // More inputs than one k-way pass takes: the first 64 in one pass, then
    // the running result with the next 63 per pass (any count, like the
    // reference's chained path, src/set_ops.cu:1733-1762).
    cr_gpu_roaring acc{};
    multi(bms, uint32_t(kMaxOperands), is_or, s, &acc);
    std::vector<cr_gpu_roaring> grp;
    for (uint32_t i = uint32_t(kMaxOperands); i < count;) {
      const uint32_t n = std::min<uint32_t>(kMaxOperands - 1, count - i);
      grp.assign(1, acc);
      grp.insert(grp.end(), bms + i, bms + i + n);
      cr_gpu_roaring next{};
      try {
        multi(grp.data(), n + 1, is_or, s, &next);
      } catch (...) {
        if (acc._alloc_base) dev_free(acc._alloc_base, s);
        throw;
      }
      if (acc._alloc_base) dev_free(acc._alloc_base, s);
      acc = next;
      i += n;
    }
    *out = acc;
    return;
  }
  std::vector<const cr_gpu_roaring*> pos, negs;
  for (uint32_t i = 0; i < count; ++i) (bms[i].negated ? negs : pos).push_back(&bms[i]);
  // multi_and: AND(pos) minus OR(stored negs); all negated -> ~OR(stored).
  // multi_or = ~multi_and(~inputs): roles of negated/non-negated swap.
  const auto& P = is_or ? negs : pos;
  const auto& N = is_or ? pos : negs;
  if (!P.empty()) kway(P, N, MODE_AND_SUB, is_or, s, out);
  else kway(N, {}, MODE_OR, !is_or, s, out);
}

extern "C" int cr_multi_and(const cr_gpu_roaring* bitmaps, uint32_t count, cr_stream_t stream,
                            cr_gpu_roaring* out)
{
  CR_API_BEGIN
  CR_REQUIRE(out != nullptr, "cr_multi_and: null output");
  multi(bitmaps, count, false, reinterpret_cast<cudaStream_t>(stream), out);
  CR_API_END
}

extern "C" int cr_multi_or(const cr_gpu_roaring* bitmaps, uint32_t count, cr_stream_t stream,
                           cr_gpu_roaring* out)
{
  CR_API_BEGIN
  CR_REQUIRE(out != nullptr, "cr_multi_or: null output");
  multi(bitmaps, count, true, reinterpret_cast<cudaStream_t>(stream), out);
  CR_API_END
}
