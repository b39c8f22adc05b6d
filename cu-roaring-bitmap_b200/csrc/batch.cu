// cu_roaring B200 engine — batches of bitmaps (the reference's v2 API,
// v2/include/cu_roaring_v2/api.hpp, v2/src/*).
//
// Layout: one device block per batch, sections aligned to 256 bytes:
// container_starts, key_index_starts, keys, types, offsets, cardinalities,
// key_indices, bitmap pool, array pool, run pool (the cr_roaring_batch
// pointers point into it); one host block for the per-bitmap mirrors.
// Ingest assembles the whole block on the host from portable Roaring
// serializations and copies it once. Promotion, AND and decompress run one
// block per container.
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "common.cuh"
#include "cu_roaring_v2/query.cuh"

namespace crb {
namespace {

constexpr uint8_t kTArray = 0, kTBitmap = 1, kTRun = 2;

struct BatchSizes {
  uint32_t n = 0, containers = 0, kidx = 0, bitmaps = 0;
  uint64_t array_bytes = 0, run_bytes = 0;
};
struct BatchLayout {
  size_t cstart, kstart, keys, types, offsets, cards, kidx, bitmap, array, run, total;
};

size_t up256(size_t x) { return (x + 255) & ~size_t(255); }

BatchLayout layout_of(const BatchSizes& z)
{
  BatchLayout L{};
  size_t o = 0;
  L.cstart = o; o = up256(o + (size_t(z.n) + 1) * 4);
  L.kstart = o; o = up256(o + (size_t(z.n) + 1) * 4);
  L.keys = o; o = up256(o + size_t(z.containers) * 2);
  L.types = o; o = up256(o + size_t(z.containers));
  L.offsets = o; o = up256(o + size_t(z.containers) * 4);
  L.cards = o; o = up256(o + size_t(z.containers) * 2);
  L.kidx = o; o = up256(o + size_t(z.kidx) * 2);
  L.bitmap = o; o = up256(o + size_t(z.bitmaps) * 8192);
  L.array = o; o = up256(o + z.array_bytes);
  L.run = o; o = up256(o + z.run_bytes);
  L.total = o;
  return L;
}

// Points every device field of `b` into `base` and fills the counts.
void point(cr_roaring_batch* b, char* base, const BatchLayout& L, const BatchSizes& z)
{
  b->n_bitmaps = z.n;
  b->total_containers = z.containers;
  b->n_bitmap_containers_total = z.bitmaps;
  b->array_pool_bytes = uint32_t(z.array_bytes);
  b->run_pool_bytes = uint32_t(z.run_bytes);
  b->container_starts = reinterpret_cast<uint32_t*>(base + L.cstart);
  b->key_index_starts = reinterpret_cast<uint32_t*>(base + L.kstart);
  b->keys = reinterpret_cast<uint16_t*>(base + L.keys);
  b->types = reinterpret_cast<uint8_t*>(base + L.types);
  b->offsets = reinterpret_cast<uint32_t*>(base + L.offsets);
  b->cardinalities = reinterpret_cast<uint16_t*>(base + L.cards);
  b->key_indices = reinterpret_cast<uint16_t*>(base + L.kidx);
  b->bitmap_data = reinterpret_cast<uint64_t*>(base + L.bitmap);
  b->array_data = reinterpret_cast<uint16_t*>(base + L.array);
  b->run_data = reinterpret_cast<uint16_t*>(base + L.run);
  b->_alloc_base = base;
}

// Host mirrors in one malloc block.
struct HostMeta {
  uint64_t* total_card;
  uint32_t *universe, *cstart, *kstart, *nbmp;
};
HostMeta alloc_meta(cr_roaring_batch* b, uint32_t n)
{
  const size_t bytes = size_t(n) * 8 + size_t(n) * 4 + (size_t(n) + 1) * 8 + size_t(n) * 4 + 16;
  char* h = static_cast<char*>(std::calloc(1, bytes));
  if (!h) fail(CR_ERR_OOM, "batch: host allocation failed");
  HostMeta m{};
  m.total_card = reinterpret_cast<uint64_t*>(h);
  m.universe = reinterpret_cast<uint32_t*>(h + size_t(n) * 8);
  m.cstart = m.universe + n;
  m.kstart = m.cstart + n + 1;
  m.nbmp = m.kstart + n + 1;
  b->host_total_cardinalities = m.total_card;
  b->host_universe_sizes = m.universe;
  b->host_container_starts = m.cstart;
  b->host_key_index_starts = m.kstart;
  b->host_n_bitmap_containers = m.nbmp;
  b->_host_meta_base = h;
  return m;
}

void check_batch(const cr_roaring_batch* b, const char* who)
{
  if (!b) fail(CR_ERR_INVALID, std::string(who) + ": null batch");
  if (b->n_bitmaps && (!b->_alloc_base || !b->_host_meta_base))
    fail(CR_ERR_INVALID, std::string(who) + ": batch without memory (freed?)");
}

// A batch as a GpuRoaringBatch for the device queries (same layout).
__host__ __device__ inline const cu_roaring::v2::GpuRoaringBatch& as_v2(const cr_roaring_batch& b)
{
  return *reinterpret_cast<const cu_roaring::v2::GpuRoaringBatch*>(&b);
}

// Container gid of a batch -> its 2048 words in shared memory.
__device__ void container_to_smem(const cr_roaring_batch& b, uint32_t gid, uint32_t* w)
{
  for (uint32_t i = threadIdx.x; i < 2048; i += blockDim.x) w[i] = 0u;
  __syncthreads();
  const uint8_t t = b.types[gid];
  const uint32_t off = b.offsets[gid], n = b.cardinalities[gid];
  if (t == kTBitmap) {
    const uint32_t* src = reinterpret_cast<const uint32_t*>(b.bitmap_data) + (off >> 2);
    for (uint32_t i = threadIdx.x; i < 2048; i += blockDim.x) w[i] = __ldg(src + i);
  } else if (t == kTArray) {
    const uint16_t* a = b.array_data + (off >> 1);
    for (uint32_t e = threadIdx.x; e < n; e += blockDim.x) {
      const uint32_t v = __ldg(a + e);
      atomicOr(&w[v >> 5], 1u << (v & 31));
    }
  } else {
    const uint16_t* r = b.run_data + (off >> 1);
    for (uint32_t k = threadIdx.x; k < n; k += blockDim.x) {
      const uint32_t start = __ldg(r + 2 * k), last = start + __ldg(r + 2 * k + 1);
      for (uint32_t wi = start >> 5; wi <= (last >> 5); ++wi) {
        const uint32_t lo = max(start, wi * 32) - wi * 32, hi = min(last, wi * 32 + 31) - wi * 32;
        atomicOr(&w[wi], (hi == 31 ? 0xFFFFFFFFu : ((1u << (hi + 1)) - 1u)) & ~((1u << lo) - 1u));
      }
    }
  }
  __syncthreads();
}

// Promotion: container gid -> BITMAP slot gid of `out` (card = popcount,
// 65536 stored as 0).
__global__ void __launch_bounds__(256) k_batch_promote(cr_roaring_batch in, cr_roaring_batch out)
{
  __shared__ uint32_t w[2048];
  __shared__ uint32_t s_pop;
  const uint32_t gid = blockIdx.x;
  if (threadIdx.x == 0) s_pop = 0;
  container_to_smem(in, gid, w);
  uint32_t* dst = reinterpret_cast<uint32_t*>(out.bitmap_data) + size_t(gid) * 2048;
  uint32_t pop = 0;
  for (uint32_t i = threadIdx.x; i < 2048; i += blockDim.x) {
    dst[i] = w[i];
    pop += __popc(w[i]);
  }
  atomicAdd(&s_pop, pop);
  __syncthreads();
  if (threadIdx.x == 0) {
    out.types[gid] = kTBitmap;
    out.offsets[gid] = gid * 8192u;
    out.cardinalities[gid] = uint16_t(s_pop & 0xFFFFu);
  }
}

// Decompress: container gid of bitmap b -> window key * 1024 of row b.
__global__ void __launch_bounds__(256) k_batch_decompress(cr_roaring_batch in, uint64_t* out, uint64_t words_each)
{
  __shared__ uint32_t w[2048];
  const uint32_t gid = blockIdx.x;
  uint32_t lo = 0, hi = in.n_bitmaps;  // bitmap owning gid: last start <= gid
  while (hi - lo > 1) {
    const uint32_t mid = (lo + hi) >> 1;
    if (in.container_starts[mid] <= gid) lo = mid; else hi = mid;
  }
  container_to_smem(in, gid, w);
  uint32_t* dst = reinterpret_cast<uint32_t*>(out + size_t(lo) * words_each + size_t(in.keys[gid]) * 1024);
  for (uint32_t i = threadIdx.x; i < 2048; i += blockDim.x) dst[i] = w[i];
}

// AND of n all-BITMAP containers per common key: gids[k * n + j] is input j's
// container for key k; words into tmp[k], popcount into pops[k].
__global__ void __launch_bounds__(256) k_batch_and(cr_roaring_batch in, const uint32_t* gids, uint32_t n,
                                                   uint4* tmp, uint32_t* pops)
{
  __shared__ uint32_t s_pop;
  if (threadIdx.x == 0) s_pop = 0;
  __syncthreads();
  const uint32_t k = blockIdx.x;
  uint32_t pop = 0;
  for (uint32_t i = threadIdx.x; i < 512; i += blockDim.x) {
    uint4 acc = make_uint4(~0u, ~0u, ~0u, ~0u);
    for (uint32_t j = 0; j < n; ++j) {
      const uint4* src = reinterpret_cast<const uint4*>(in.bitmap_data) + (in.offsets[gids[size_t(k) * n + j]] >> 4);
      const uint4 x = __ldg(src + i);
      acc.x &= x.x; acc.y &= x.y; acc.z &= x.z; acc.w &= x.w;
    }
    tmp[size_t(k) * 512 + i] = acc;
    pop += __popc(acc.x) + __popc(acc.y) + __popc(acc.z) + __popc(acc.w);
  }
  atomicAdd(&s_pop, pop);
  __syncthreads();
  if (threadIdx.x == 0) pops[k] = s_pop;
}

// Kept containers: tmp[src[i]] -> bitmap slot i of out.
__global__ void __launch_bounds__(256) k_batch_gather(const uint4* tmp, const uint32_t* src, uint4* dst)
{
  const uint32_t i = blockIdx.x;
  for (uint32_t t = threadIdx.x; t < 512; t += blockDim.x) dst[size_t(i) * 512 + t] = tmp[size_t(src[i]) * 512 + t];
}

__global__ void k_batch_contains(cr_roaring_batch in, const uint32_t* bidx, const uint32_t* ids, uint64_t n,
                                 uint32_t* out_bits)
{
  const uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const bool hit = i < n && cu_roaring::v2::contains(as_v2(in), bidx[i], ids[i]);
  const uint32_t m = __ballot_sync(0xFFFFFFFFu, hit);
  if ((threadIdx.x & 31) == 0 && i < n) out_bits[i >> 5] = m;
}

}  // namespace
}  // namespace crb

using namespace crb;

extern "C" int cr_batch_upload_portable(const void* const* buffers, const uint64_t* sizes, uint32_t n,
                                        cr_stream_t stream, cr_roaring_batch* out)
{
  CR_API_BEGIN
  CR_REQUIRE(out != nullptr, "cr_batch_upload_portable: null output");
  CR_REQUIRE(n == 0 || (buffers && sizes), "cr_batch_upload_portable: null buffer list");
  std::memset(out, 0, sizeof(*out));
  std::vector<PortableImage> ims(n);
  BatchSizes z{};
  z.n = n;
  for (uint32_t b = 0; b < n; ++b) {
    CR_REQUIRE(buffers[b] != nullptr, "cr_batch_upload_portable: null buffer");
    ims[b] = parse_portable(buffers[b], sizes[b], 0, "cr_batch_upload_portable");
    for (const PortableContainer& c : ims[b].cs) {
      if (c.kind == kPortableBitmap) ++z.bitmaps;
      else if (c.kind == kPortableArray) z.array_bytes += 2 * uint64_t(c.count);
      else z.run_bytes += 4 * uint64_t(c.count);
    }
    z.containers += uint32_t(ims[b].cs.size());
    z.kidx += ims[b].cs.empty() ? 0u : ims[b].cs.back().key + 1u;
  }
  CR_REQUIRE(z.array_bytes < (1ull << 32) && z.run_bytes < (1ull << 32) && uint64_t(z.bitmaps) * 8192 < (1ull << 32),
             "cr_batch_upload_portable: a pool would pass 4 GiB (32-bit offsets)");
  const BatchLayout L = layout_of(z);
  std::vector<char> h(L.total, 0);
  HostMeta meta = alloc_meta(out, n);
  auto* cstart = reinterpret_cast<uint32_t*>(h.data() + L.cstart);
  auto* kstart = reinterpret_cast<uint32_t*>(h.data() + L.kstart);
  auto* keys = reinterpret_cast<uint16_t*>(h.data() + L.keys);
  auto* types = reinterpret_cast<uint8_t*>(h.data() + L.types);
  auto* offs = reinterpret_cast<uint32_t*>(h.data() + L.offsets);
  auto* cards = reinterpret_cast<uint16_t*>(h.data() + L.cards);
  auto* kidx = reinterpret_cast<uint16_t*>(h.data() + L.kidx);
  char* bpool = h.data() + L.bitmap;
  char* apool = h.data() + L.array;
  char* rpool = h.data() + L.run;
  uint32_t g = 0, kk = 0, nb = 0;
  uint64_t ab = 0, rb = 0;
  try {
    for (uint32_t b = 0; b < n; ++b) {
      const auto* src = static_cast<const uint8_t*>(buffers[b]);
      const auto& cs = ims[b].cs;
      cstart[b] = meta.cstart[b] = g;
      kstart[b] = meta.kstart[b] = kk;
      const uint32_t klen = cs.empty() ? 0u : cs.back().key + 1u;
      std::fill(kidx + kk, kidx + kk + klen, uint16_t(0xFFFF));
      uint64_t total = 0;
      uint32_t bitmaps_here = 0;
      for (uint32_t i = 0; i < cs.size(); ++i, ++g) {
        const PortableContainer& c = cs[i];
        keys[g] = uint16_t(c.key);
        kidx[kk + c.key] = uint16_t(i);
        const uint8_t* p = src + c.offset;
        if (c.kind == kPortableBitmap) {
          types[g] = kTBitmap;
          offs[g] = nb * 8192u;
          std::memcpy(bpool + size_t(nb) * 8192, p, 8192);
          uint32_t pop = 0;
          for (uint32_t w = 0; w < 2048; ++w) {
            uint32_t x;
            std::memcpy(&x, p + 4 * w, 4);
            pop += uint32_t(__builtin_popcount(x));
          }
          CR_REQUIRE(pop == c.card, "cr_batch_upload_portable: a container's members do not match its declared cardinality");
          cards[g] = uint16_t(pop & 0xFFFFu);
          total += pop;
          ++nb;
          ++bitmaps_here;
        } else if (c.kind == kPortableArray) {
          types[g] = kTArray;
          offs[g] = uint32_t(ab);
          std::memcpy(apool + ab, p, 2 * size_t(c.count));
          for (uint32_t e = 1; e < c.count; ++e)
            CR_REQUIRE((p[2 * e] | (p[2 * e + 1] << 8)) > (p[2 * e - 2] | (p[2 * e - 1] << 8)),
                       "cr_batch_upload_portable: array container not strictly increasing");
          cards[g] = uint16_t(c.count);
          total += c.count;
          ab += 2 * uint64_t(c.count);
        } else {
          types[g] = kTRun;
          offs[g] = uint32_t(rb);
          std::memcpy(rpool + rb, p + 2, 4 * size_t(c.count));
          uint64_t members = 0;
          int64_t prev_last = -1;  // runs must be sorted and disjoint (the lookup bisects them)
          for (uint32_t r = 0; r < c.count; ++r) {
            const uint32_t start = p[2 + 4 * r] | (p[3 + 4 * r] << 8), len = p[4 + 4 * r] | (p[5 + 4 * r] << 8);
            CR_REQUIRE(start + len <= 0xFFFFu, "cr_batch_upload_portable: a run passes the end of its container");
            CR_REQUIRE(int64_t(start) > prev_last, "cr_batch_upload_portable: runs not sorted and disjoint");
            prev_last = int64_t(start) + len;
            members += len + 1;
          }
          CR_REQUIRE(members == c.card, "cr_batch_upload_portable: a container's members do not match its declared cardinality");
          cards[g] = uint16_t(c.count);
          total += members;
          rb += 4 * uint64_t(c.count);
        }
      }
      kk += klen;
      meta.total_card[b] = total;
      meta.universe[b] = cs.empty() ? 0u : uint32_t((uint64_t(cs.back().key) + 1) << 16);
      meta.nbmp[b] = bitmaps_here;
    }
    cstart[n] = meta.cstart[n] = g;
    kstart[n] = meta.kstart[n] = kk;
  } catch (...) {
    std::free(out->_host_meta_base);
    std::memset(out, 0, sizeof(*out));
    throw;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  char* d = static_cast<char*>(dev_alloc(L.total, s));
  CR_CUDA(cudaMemcpyAsync(d, h.data(), L.total, cudaMemcpyHostToDevice, s));
  CR_CUDA(cudaStreamSynchronize(s));  // the staging block is released on return
  point(out, d, L, z);
  CR_API_END
}

extern "C" int cr_batch_free(cr_roaring_batch* batch)
{
  CR_API_BEGIN
  CR_REQUIRE(batch != nullptr, "cr_batch_free: null batch");
  if (batch->_alloc_base) CR_CUDA(cudaFree(batch->_alloc_base));
  std::free(batch->_host_meta_base);
  std::memset(batch, 0, sizeof(*batch));
  CR_API_END
}

extern "C" int cr_batch_promote(const cr_roaring_batch* in, cr_stream_t stream, cr_roaring_batch* out)
{
  CR_API_BEGIN
  check_batch(in, "cr_batch_promote");
  CR_REQUIRE(out != nullptr && out != in, "cr_batch_promote: bad output");
  std::memset(out, 0, sizeof(*out));
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const uint32_t n = in->n_bitmaps;
  BatchSizes z{};
  z.n = n;
  z.containers = in->total_containers;
  z.kidx = n ? in->host_key_index_starts[n] : 0;
  z.bitmaps = in->total_containers;
  const BatchLayout L = layout_of(z);
  const BatchLayout Li = [&] {
    BatchSizes zi{};
    zi.n = n;
    zi.containers = in->total_containers;
    zi.kidx = z.kidx;
    zi.bitmaps = in->n_bitmap_containers_total;
    zi.array_bytes = in->array_pool_bytes;
    zi.run_bytes = in->run_pool_bytes;
    return layout_of(zi);
  }();
  HostMeta meta = alloc_meta(out, n);
  for (uint32_t b = 0; b < n; ++b) {
    meta.total_card[b] = in->host_total_cardinalities[b];
    meta.universe[b] = in->host_universe_sizes[b];
    meta.nbmp[b] = in->host_container_starts[b + 1] - in->host_container_starts[b];
  }
  for (uint32_t b = 0; b <= n; ++b) {
    meta.cstart[b] = in->host_container_starts[b];
    meta.kstart[b] = in->host_key_index_starts[b];
  }
  char* d = static_cast<char*>(dev_alloc(L.total, s));
  point(out, d, L, z);
  // CSR starts, keys and key indices are unchanged (the sections before the
  // types have the same layout in both blocks).
  const char* src = static_cast<const char*>(in->_alloc_base);
  CR_CUDA(cudaMemcpyAsync(d + L.cstart, src + Li.cstart, L.types - L.cstart, cudaMemcpyDeviceToDevice, s));
  CR_CUDA(cudaMemcpyAsync(d + L.kidx, src + Li.kidx, size_t(z.kidx) * 2, cudaMemcpyDeviceToDevice, s));
  if (z.containers) k_batch_promote<<<z.containers, 256, 0, s>>>(*in, *out);
  CR_CUDA(cudaGetLastError());
  CR_API_END
}

extern "C" int cr_batch_decompress(const cr_roaring_batch* in, uint64_t* d_bitsets, uint64_t words_each,
                                   cr_stream_t stream)
{
  CR_API_BEGIN
  check_batch(in, "cr_batch_decompress");
  for (uint32_t b = 0; b < in->n_bitmaps; ++b)
    CR_REQUIRE(uint64_t(in->host_key_index_starts[b + 1] - in->host_key_index_starts[b]) * 1024 <= words_each,
               "cr_batch_decompress: words_each does not cover a bitmap's universe");
  CR_REQUIRE(d_bitsets != nullptr || in->total_containers == 0, "cr_batch_decompress: null output");
  if (in->total_containers)
    k_batch_decompress<<<in->total_containers, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(*in, d_bitsets,
                                                                                                 words_each);
  CR_CUDA(cudaGetLastError());
  CR_API_END
}

extern "C" int cr_batch_contains(const cr_roaring_batch* in, const uint32_t* d_bitmap_idx, const uint32_t* d_ids,
                                 uint64_t n, uint32_t* d_out_bits, cr_stream_t stream)
{
  CR_API_BEGIN
  check_batch(in, "cr_batch_contains");
  CR_REQUIRE(n == 0 || (d_bitmap_idx && d_ids && d_out_bits), "cr_batch_contains: null buffer");
  if (n)
    k_batch_contains<<<div_up(n, 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(*in, d_bitmap_idx, d_ids, n,
                                                                                        d_out_bits);
  CR_CUDA(cudaGetLastError());
  CR_API_END
}

extern "C" int cr_batch_multi_and(const cr_roaring_batch* in, const uint32_t* indices, uint32_t n_in,
                                  cr_stream_t stream, cr_roaring_batch* out)
{
  CR_API_BEGIN
  check_batch(in, "cr_batch_multi_and");
  CR_REQUIRE(out != nullptr && out != in, "cr_batch_multi_and: bad output");
  CR_REQUIRE(indices != nullptr && n_in >= 1, "cr_batch_multi_and: no inputs");
  std::memset(out, 0, sizeof(*out));
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // Keys of every input (host copies of their key slices).
  std::vector<std::vector<uint16_t>> keys(n_in);
  std::vector<uint32_t> first(n_in);
  for (uint32_t j = 0; j < n_in; ++j) {
    const uint32_t b = indices[j];
    CR_REQUIRE(b < in->n_bitmaps, "cr_batch_multi_and: bitmap index out of range");
    const uint32_t c0 = in->host_container_starts[b], c1 = in->host_container_starts[b + 1];
    CR_REQUIRE(in->host_n_bitmap_containers[b] == c1 - c0,
               "cr_batch_multi_and: every input must be all-BITMAP (run cr_batch_promote first)");
    first[j] = c0;
    keys[j].resize(c1 - c0);
    if (c1 > c0) CR_CUDA(cudaMemcpyAsync(keys[j].data(), in->keys + c0, size_t(c1 - c0) * 2, cudaMemcpyDeviceToHost, s));
  }
  CR_CUDA(cudaStreamSynchronize(s));
  // Common keys and, per key, each input's container.
  std::vector<uint32_t> common, gids;
  {
    std::vector<size_t> pos(n_in, 0);
    for (size_t i0 = 0; i0 < keys[0].size(); ++i0) {
      const uint16_t key = keys[0][i0];
      bool all = true;
      for (uint32_t j = 1; j < n_in && all; ++j) {
        auto& v = keys[j];
        while (pos[j] < v.size() && v[pos[j]] < key) ++pos[j];
        all = pos[j] < v.size() && v[pos[j]] == key;
      }
      if (!all) continue;
      common.push_back(key);
      gids.push_back(first[0] + uint32_t(i0));
      for (uint32_t j = 1; j < n_in; ++j) gids.push_back(first[j] + uint32_t(pos[j]));
    }
  }
  const uint32_t m = uint32_t(common.size());
  std::vector<uint32_t> pops(m);
  Scratch work(size_t(m) * 8192 + size_t(m) * 4 * (n_in + 1) + 256, s);
  uint4* tmp = work.as<uint4>();
  uint32_t* d_gids = reinterpret_cast<uint32_t*>(work.as<char>() + size_t(m) * 8192);
  uint32_t* d_pops = d_gids + size_t(m) * n_in;
  if (m) {
    CR_CUDA(cudaMemcpyAsync(d_gids, gids.data(), gids.size() * 4, cudaMemcpyHostToDevice, s));
    k_batch_and<<<m, 256, 0, s>>>(*in, d_gids, n_in, tmp, d_pops);
    CR_CUDA(cudaGetLastError());
    CR_CUDA(cudaMemcpyAsync(pops.data(), d_pops, size_t(m) * 4, cudaMemcpyDeviceToHost, s));
    CR_CUDA(cudaStreamSynchronize(s));
  }
  // One bitmap: the non-empty results.
  std::vector<uint32_t> keep;
  uint64_t total = 0;
  for (uint32_t i = 0; i < m; ++i)
    if (pops[i]) { keep.push_back(i); total += pops[i]; }
  BatchSizes z{};
  z.n = 1;
  z.containers = uint32_t(keep.size());
  z.kidx = keep.empty() ? 0u : common[keep.back()] + 1u;
  z.bitmaps = z.containers;
  const BatchLayout L = layout_of(z);
  std::vector<char> h(L.bitmap, 0);  // metadata sections only
  auto* cstart = reinterpret_cast<uint32_t*>(h.data() + L.cstart);
  auto* kstart = reinterpret_cast<uint32_t*>(h.data() + L.kstart);
  auto* hk = reinterpret_cast<uint16_t*>(h.data() + L.keys);
  auto* ht = reinterpret_cast<uint8_t*>(h.data() + L.types);
  auto* ho = reinterpret_cast<uint32_t*>(h.data() + L.offsets);
  auto* hc = reinterpret_cast<uint16_t*>(h.data() + L.cards);
  auto* hx = reinterpret_cast<uint16_t*>(h.data() + L.kidx);
  cstart[0] = 0; cstart[1] = z.containers;
  kstart[0] = 0; kstart[1] = z.kidx;
  std::fill(hx, hx + z.kidx, uint16_t(0xFFFF));
  for (uint32_t i = 0; i < keep.size(); ++i) {
    hk[i] = uint16_t(common[keep[i]]);
    ht[i] = kTBitmap;
    ho[i] = i * 8192u;
    hc[i] = uint16_t(pops[keep[i]] & 0xFFFFu);
    hx[common[keep[i]]] = uint16_t(i);
  }
  HostMeta meta = alloc_meta(out, 1);
  meta.total_card[0] = total;
  meta.universe[0] = z.kidx ? uint32_t(uint64_t(z.kidx) << 16) : 0u;
  meta.cstart[0] = 0; meta.cstart[1] = z.containers;
  meta.kstart[0] = 0; meta.kstart[1] = z.kidx;
  meta.nbmp[0] = z.containers;
  char* d = static_cast<char*>(dev_alloc(L.total, s));
  CR_CUDA(cudaMemcpyAsync(d, h.data(), L.bitmap, cudaMemcpyHostToDevice, s));
  if (!keep.empty()) {
    Scratch src_idx(keep.size() * 4, s);
    CR_CUDA(cudaMemcpyAsync(src_idx.p, keep.data(), keep.size() * 4, cudaMemcpyHostToDevice, s));
    k_batch_gather<<<uint32_t(keep.size()), 256, 0, s>>>(tmp, src_idx.as<uint32_t>(),
                                                         reinterpret_cast<uint4*>(d + L.bitmap));
    CR_CUDA(cudaGetLastError());
  }
  CR_CUDA(cudaStreamSynchronize(s));  // the host staging vectors go out of scope
  point(out, d, L, z);
  CR_API_END
}
