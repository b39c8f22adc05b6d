// cu_roaring B200 engine — key-range sharding of bitmaps across GPUs.
//
// No reference counterpart (the reference has no multi-GPU path). Set
// operations, multi_and / multi_or, uploads and point queries work key by
// key (one 65536-ID chunk at a time), so a bitmap splits across G ranks at
// chunk boundaries with no communication: rank g holds the containers whose
// key lies in [g * K / G, (g + 1) * K / G) of every operand (K = chunks of
// the universe), runs the operation on its slices, and the result slices
// laid end to end are the unsharded result, container for container: the
// engine's output typing is decided per key from that key's operand
// containers alone.
//
//   cr_key_slice          one rank's containers of a bitmap (same types,
//                         universe and complement flag), one packed block
//   cr_concat_key_slices  slices with ascending, disjoint key ranges -> one
//                         bitmap: metadata concatenated, per-type pool
//                         offsets rebased, key index rebuilt
//
// A slice of a complement-stored bitmap keeps the flag; its logical set is
// the complement within its key range. total_cardinality of a slice (and of
// a concatenation) counts as if it were the whole bitmap: its stored
// members, or U minus them when the complement is stored.
//
// Both are host helpers: they read the (small) container metadata back to
// the host, plan the copy there, and move every container's payload with one
// kernel (one block per container).
#include <algorithm>
#include <vector>

#include "common.cuh"

namespace crb {
namespace {

struct CopyItem {
  const uint8_t* src;  // payload start
  uint64_t dst_off;    // byte offset in the output's pool of the same type
  uint32_t bytes;
  uint32_t type;
};

__global__ void __launch_bounds__(256) k_copy_containers(const CopyItem* items, uint8_t* bitmap_pool,
                                                         uint8_t* array_pool, uint8_t* run_pool)
{
  const CopyItem it = items[blockIdx.x];
  uint8_t* dst = (it.type == kBitmap ? bitmap_pool : (it.type == kArray ? array_pool : run_pool)) + it.dst_off;
  if (it.type == kBitmap) {  // 8 KiB, 16-byte aligned on both sides
    const uint4* s = reinterpret_cast<const uint4*>(it.src);
    uint4* d = reinterpret_cast<uint4*>(dst);
    for (uint32_t i = threadIdx.x; i < it.bytes / 16; i += blockDim.x) d[i] = s[i];
  } else {  // u16 payloads, 2-byte aligned
    const uint16_t* s = reinterpret_cast<const uint16_t*>(it.src);
    uint16_t* d = reinterpret_cast<uint16_t*>(dst);
    for (uint32_t i = threadIdx.x; i < it.bytes / 2; i += blockDim.x) d[i] = s[i];
  }
}

struct HostMeta {
  std::vector<uint16_t> keys, cards;
  std::vector<uint8_t> types;
  std::vector<uint32_t> offsets;
};

HostMeta read_meta(const cr_gpu_roaring* b, cudaStream_t s)
{
  HostMeta m;
  const uint32_t n = b->n_containers;
  m.keys.resize(n);
  m.cards.resize(n);
  m.types.resize(n);
  m.offsets.resize(n);
  if (n) {
    CR_REQUIRE(b->keys && b->types && b->offsets && b->cardinalities, "key slicing: bitmap without metadata");
    CR_CUDA(cudaMemcpyAsync(m.keys.data(), b->keys, n * 2, cudaMemcpyDeviceToHost, s));
    CR_CUDA(cudaMemcpyAsync(m.cards.data(), b->cardinalities, n * 2, cudaMemcpyDeviceToHost, s));
    CR_CUDA(cudaMemcpyAsync(m.types.data(), b->types, n, cudaMemcpyDeviceToHost, s));
    CR_CUDA(cudaMemcpyAsync(m.offsets.data(), b->offsets, n * 4, cudaMemcpyDeviceToHost, s));
    CR_CUDA(cudaStreamSynchronize(s));
  }
  return m;
}

uint64_t payload_bytes(uint8_t type, uint16_t card)
{
  if (type == kBitmap) return kBitmapBytes;
  if (type == kArray) return uint64_t(card) * 2;
  return uint64_t(card) * 4;  // RUN: card counts runs, (start, length) u16 pairs
}

// Stored members of the assembled containers (BITMAP: card, 65536 stored as
// 0; ARRAY: card; RUN: the sum of run lengths, read from the payload).
__global__ void __launch_bounds__(256) k_stored_members(cr_gpu_roaring b, unsigned long long* total)
{
  const uint32_t i = blockIdx.x;
  const uint8_t t = b.types[i];
  const uint32_t c = b.cardinalities[i];
  unsigned long long v = 0;
  if (t == kRun) {
    const uint16_t* r = b.run_data + (b.offsets[i] >> 1);
    for (uint32_t j = threadIdx.x; j < c; j += blockDim.x) v += uint32_t(r[2 * j + 1]) + 1u;
  } else if (threadIdx.x == 0) {
    v = (t == kBitmap && c == 0) ? 65536u : c;
  }
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  if ((threadIdx.x & 31) == 0 && v) atomicAdd(total, v);
}

// Assembles `out` from the selected containers of several sources, in order.
struct Pick {
  const cr_gpu_roaring* b;
  const HostMeta* m;
  uint32_t i;
};

void assemble(const std::vector<Pick>& picks, uint32_t U, bool negated, cudaStream_t s, cr_gpu_roaring* out)
{
  std::memset(out, 0, sizeof(*out));
  out->universe_size = U;
  out->negated = negated;
  out->total_cardinality = negated ? U : 0;
  const uint32_t n = uint32_t(picks.size());
  if (n == 0) return;
  std::vector<uint16_t> keys(n), cards(n);
  std::vector<uint8_t> types(n);
  std::vector<uint32_t> offsets(n);
  std::vector<CopyItem> items(n);
  uint64_t nb = 0, ab = 0, rb = 0;
  uint32_t na = 0, nr = 0;
  for (uint32_t j = 0; j < n; ++j) {
    const Pick& p = picks[j];
    const uint8_t t = p.m->types[p.i];
    const uint16_t c = p.m->cards[p.i];
    keys[j] = p.m->keys[p.i];
    types[j] = t;
    cards[j] = c;
    const uint64_t bytes = payload_bytes(t, c);
    const uint8_t* pool = t == kBitmap ? reinterpret_cast<const uint8_t*>(p.b->bitmap_data)
                                       : (t == kArray ? reinterpret_cast<const uint8_t*>(p.b->array_data)
                                                      : reinterpret_cast<const uint8_t*>(p.b->run_data));
    CR_REQUIRE(pool != nullptr || bytes == 0, "key slicing: container without its pool");
    uint64_t& cur = t == kBitmap ? nb : (t == kArray ? ab : rb);
    offsets[j] = uint32_t(cur);
    items[j] = CopyItem{pool + p.m->offsets[p.i], cur, uint32_t(bytes), t};
    cur += bytes;
    if (t == kArray) ++na;
    if (t == kRun) ++nr;
  }
  CR_REQUIRE(ab <= 0xFFFFFFFFull && rb <= 0xFFFFFFFFull, "key slicing: pool exceeds 4 GiB");
  out->n_containers = n;
  out->n_bitmap_containers = uint32_t(nb / kBitmapBytes);
  out->n_array_containers = na;
  out->n_run_containers = nr;
  out->array_pool_bytes = uint32_t(ab);
  out->run_pool_bytes = uint32_t(rb);
  out->max_key = max_key_for(U);
  alloc_result(out, s);
  CR_CUDA(cudaMemcpyAsync(out->keys, keys.data(), n * 2, cudaMemcpyHostToDevice, s));
  CR_CUDA(cudaMemcpyAsync(out->cardinalities, cards.data(), n * 2, cudaMemcpyHostToDevice, s));
  CR_CUDA(cudaMemcpyAsync(out->types, types.data(), n, cudaMemcpyHostToDevice, s));
  CR_CUDA(cudaMemcpyAsync(out->offsets, offsets.data(), n * 4, cudaMemcpyHostToDevice, s));
  Scratch plan(sizeof(CopyItem) * n, s);
  CR_CUDA(cudaMemcpyAsync(plan.p, items.data(), sizeof(CopyItem) * n, cudaMemcpyHostToDevice, s));
  k_copy_containers<<<n, 256, 0, s>>>(plan.as<CopyItem>(), reinterpret_cast<uint8_t*>(out->bitmap_data),
                                      reinterpret_cast<uint8_t*>(out->array_data),
                                      reinterpret_cast<uint8_t*>(out->run_data));
  CR_CUDA(cudaGetLastError());
  build_key_index(out->keys, n, out->key_index, out->max_key + 1, s);
  Scratch tot(8, s);
  CR_CUDA(cudaMemsetAsync(tot.p, 0, 8, s));
  k_stored_members<<<n, 256, 0, s>>>(*out, tot.as<unsigned long long>());
  CR_CUDA(cudaGetLastError());
  unsigned long long stored = 0;
  CR_CUDA(cudaMemcpyAsync(&stored, tot.p, 8, cudaMemcpyDeviceToHost, s));
  CR_CUDA(cudaStreamSynchronize(s));  // also completes the pageable host copies above
  // As if the result were the whole bitmap: stored members, or U minus them
  // when the complement is stored.
  out->total_cardinality = negated ? uint64_t(U) - stored : stored;
}

}  // namespace
}  // namespace crb

using namespace crb;

extern "C" int cr_key_range(uint32_t universe_size, uint32_t rank, uint32_t n_ranks, uint32_t* key_lo,
                            uint32_t* key_hi)
{
  CR_API_BEGIN
  CR_REQUIRE(key_lo && key_hi && n_ranks >= 1 && rank < n_ranks, "cr_key_range: bad argument");
  const uint64_t K = n_chunks_for(universe_size);
  *key_lo = uint32_t(K * rank / n_ranks);
  *key_hi = uint32_t(K * (rank + 1) / n_ranks);
  CR_API_END
}

extern "C" int cr_key_slice(const cr_gpu_roaring* bm, uint32_t key_lo, uint32_t key_hi, cr_stream_t stream,
                            cr_gpu_roaring* out)
{
  CR_API_BEGIN
  CR_REQUIRE(bm && out, "cr_key_slice: null argument");
  CR_REQUIRE(key_lo <= key_hi && key_hi <= 65536u, "cr_key_slice: bad key range");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const HostMeta m = read_meta(bm, s);
  std::vector<Pick> picks;
  for (uint32_t i = 0; i < bm->n_containers; ++i)
    if (m.keys[i] >= key_lo && m.keys[i] < key_hi) picks.push_back({bm, &m, i});
  assemble(picks, bm->universe_size, bm->negated != 0, s, out);
  CR_API_END
}

extern "C" int cr_concat_key_slices(const cr_gpu_roaring* slices, uint32_t n, cr_stream_t stream,
                                    cr_gpu_roaring* out)
{
  CR_API_BEGIN
  CR_REQUIRE(out != nullptr && (n == 0 || slices != nullptr), "cr_concat_key_slices: null argument");
  std::memset(out, 0, sizeof(*out));
  if (n == 0) return CR_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const uint32_t U = slices[0].universe_size;
  const bool neg = slices[0].negated != 0;
  std::vector<HostMeta> metas(n);
  std::vector<Pick> picks;
  int32_t last_key = -1;
  for (uint32_t j = 0; j < n; ++j) {
    CR_REQUIRE(slices[j].universe_size == U, "cr_concat_key_slices: slices of different universes");
    CR_REQUIRE((slices[j].negated != 0) == neg, "cr_concat_key_slices: slices disagree on the complement flag");
    metas[j] = read_meta(&slices[j], s);
    for (uint32_t i = 0; i < slices[j].n_containers; ++i) {
      CR_REQUIRE(int32_t(metas[j].keys[i]) > last_key,
                 "cr_concat_key_slices: slices must hold ascending, disjoint key ranges");
      last_key = metas[j].keys[i];
      picks.push_back({&slices[j], &metas[j], i});
    }
  }
  assemble(picks, U, neg, s, out);
  CR_API_END
}
