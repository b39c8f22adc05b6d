// cu_roaring B200 engine — bulk point queries, decompress, enumerate_ids,
// promotion.
//
// decompress: one CTA per 65536-bit chunk of the OUTPUT (not per container,
// as reference src/decompress.cu:8-87 does after a full memset), so every
// output word is written exactly once with 16-byte stores, absent chunks
// and the complement/tail mask included; no global atomics.
// enumerate_ids: count -> tile scan -> one CTA per unit writes sorted IDs;
// negated bitmaps enumerate the complement (the reference ignores
// `negated`, src/to_csr.cu:36-131).
#include <cuda.h>

#include <algorithm>
#include <mutex>
#include <string>

#include "chunk_ops.cuh"
#include "cu_roaring/device/make_view.cuh"
#include "cu_roaring/device/roaring_warp_query.cuh"

namespace crb {
namespace {

static_assert(sizeof(cr_gpu_roaring) == sizeof(cu_roaring::GpuRoaring), "ABI layout");
static_assert(offsetof(cr_gpu_roaring, negated) == offsetof(cu_roaring::GpuRoaring, negated), "ABI");
static_assert(offsetof(cr_gpu_roaring, _alloc_base) == offsetof(cu_roaring::GpuRoaring, _alloc_base), "ABI");
static_assert(offsetof(cr_gpu_roaring, key_index) == offsetof(cu_roaring::GpuRoaring, key_index), "ABI");

constexpr int kUnroll = 4;

// Bulk contains: each warp answers 32*kUnroll consecutive candidates per
// step (coalesced 128-byte ID loads, kUnroll independent lookups in flight)
// and writes one 32-bit result word per 32 candidates via __ballot_sync.
template <int MODE>
__global__ void __launch_bounds__(256) k_contains(cu_roaring::GpuRoaringView v,
                                                  const uint32_t* __restrict__ ids, uint64_t n,
                                                  uint32_t* __restrict__ out)
{
  const uint32_t lane = threadIdx.x & 31;
  const uint64_t n_words = (n + 31) / 32;
  const uint64_t warp = (uint64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const uint64_t n_warps = (uint64_t(gridDim.x) * blockDim.x) >> 5;
  for (uint64_t w0 = warp * kUnroll; w0 < n_words; w0 += n_warps * kUnroll) {
    uint32_t id[kUnroll];
    bool in[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const uint64_t i = (w0 + u) * 32 + lane;
      in[u] = i < n;
      id[u] = in[u] ? __ldcs(ids + i) : 0u;
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      // Every lane calls the query (tail lanes on a dummy ID, result masked):
      // warp_contains is warp-synchronous and must not sit in a lane branch.
      const bool hit = (MODE ? cu_roaring::warp_contains(v, id[u]) : v.contains(id[u])) && in[u];
      const uint32_t bits = __ballot_sync(0xFFFFFFFFu, hit);
      if (lane == 0 && w0 + u < n_words) __stcs(out + w0 + u, bits);
    }
  }
}

// Bulk contains for an all-BITMAP layout (key_index present, container i at
// slot i): branch-free, kMLP candidates per thread with all key_index loads
// issued before all bitmap-word loads, so each thread keeps 2 x kMLP
// independent memory accesses in flight instead of a dependent pair.
constexpr int kMLP = 8;

__global__ void __launch_bounds__(256) k_contains_bitmap(const uint16_t* __restrict__ key_index,
                                                         uint32_t max_key,
                                                         const uint64_t* __restrict__ bitmap,
                                                         uint32_t negated,
                                                         const uint32_t* __restrict__ ids, uint64_t n,
                                                         uint32_t* __restrict__ out)
{
  const uint32_t lane = threadIdx.x & 31;
  const uint64_t n_words = (n + 31) / 32;
  const uint64_t warp = (uint64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const uint64_t n_warps = (uint64_t(gridDim.x) * blockDim.x) >> 5;
  for (uint64_t w0 = warp * kMLP; w0 < n_words; w0 += n_warps * kMLP) {
    uint32_t id[kMLP], idx[kMLP];
    uint64_t word[kMLP];
#pragma unroll
    for (int u = 0; u < kMLP; ++u) {
      const uint64_t i = (w0 + u) * 32 + lane;
      id[u] = i < n ? __ldcs(ids + i) : 0u;
    }
#pragma unroll
    for (int u = 0; u < kMLP; ++u) {
      const uint32_t key = id[u] >> 16;
      idx[u] = key <= max_key ? uint32_t(__ldg(key_index + key)) : 0xFFFFu;
    }
#pragma unroll
    for (int u = 0; u < kMLP; ++u)
      word[u] = idx[u] != 0xFFFFu ? __ldg(bitmap + (size_t(idx[u]) << 10) + ((id[u] & 0xFFFFu) >> 6)) : 0ull;
#pragma unroll
    for (int u = 0; u < kMLP; ++u) {
      const uint64_t i = (w0 + u) * 32 + lane;
      const bool in = (idx[u] != 0xFFFFu) && ((word[u] >> (id[u] & 63u)) & 1ull);
      const uint32_t bits = __ballot_sync(0xFFFFFFFFu, (in != (negated != 0)) && i < n);
      if (lane == 0 && w0 + u < n_words) __stcs(out + w0 + u, bits);
    }
  }
}

// Bulk contains for mixed layouts (ARRAY / BITMAP / RUN, key_index present):
// kMix candidates per thread move through the lookup in phases (key index;
// type, offset and cardinality; the first data probe; the ARRAY search), each
// phase issuing its loads for all kMix candidates before any is consumed, so
// a thread keeps kMix dependent chains in flight instead of one. ARRAY
// containers are probed with the view's 64-entry interpolation window; RUN
// containers (rare in bulk filters) take the view's run search.
constexpr int kMix = 4;
__global__ void __launch_bounds__(256) k_contains_mixed(cu_roaring::GpuRoaringView v,
                                                        const uint32_t* __restrict__ ids, uint64_t n,
                                                        uint32_t* __restrict__ out)
{
  const uint32_t lane = threadIdx.x & 31;
  const uint64_t n_words = (n + 31) / 32;
  const uint64_t warp = (uint64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const uint64_t n_warps = (uint64_t(gridDim.x) * blockDim.x) >> 5;
  const uint8_t* types = reinterpret_cast<const uint8_t*>(v.types);
  for (uint64_t w0 = warp * kMix; w0 < n_words; w0 += n_warps * kMix) {
    uint32_t id[kMix], idx[kMix], off[kMix], card[kMix], base[kMix], cnt[kMix];
    uint8_t ty[kMix];
    bool hit[kMix];
#pragma unroll
    for (int u = 0; u < kMix; ++u) {
      const uint64_t i = (w0 + u) * 32 + lane;
      id[u] = i < n ? __ldcs(ids + i) : 0u;
    }
#pragma unroll
    for (int u = 0; u < kMix; ++u) {
      const uint32_t key = id[u] >> 16;
      idx[u] = key <= v.max_key ? uint32_t(__ldg(v.key_index + key)) : 0xFFFFu;
    }
#pragma unroll
    for (int u = 0; u < kMix; ++u) {
      const uint32_t j = idx[u] != 0xFFFFu ? idx[u] : 0u;
      ty[u] = idx[u] != 0xFFFFu ? __ldg(types + j) : uint8_t(0xFF);
      off[u] = __ldg(v.offsets + j);
      card[u] = __ldg(v.cardinalities + j);
    }
    // First data probe: the BITMAP word, or the ARRAY window's two ends.
    uint64_t word[kMix];
    uint32_t first[kMix], last[kMix];
#pragma unroll
    for (int u = 0; u < kMix; ++u) {
      const uint32_t low = id[u] & 0xFFFFu;
      word[u] = 0;
      first[u] = 0;
      last[u] = 0xFFFFu;
      base[u] = 0;
      cnt[u] = card[u];
      if (ty[u] == uint8_t(cu_roaring::ContainerTypeD::BITMAP)) {
        word[u] = __ldg(v.bitmap_data + (off[u] >> 3) + (low >> 6));
      } else if (ty[u] == uint8_t(cu_roaring::ContainerTypeD::ARRAY) && card[u] > 64) {
        const uint32_t g = (low * card[u]) >> 16;
        const uint32_t ws = g >= 32 ? min(g - 32, card[u] - 64) : 0u;
        const uint16_t* a = v.array_data + (off[u] >> 1);
        first[u] = __ldg(a + ws);
        last[u] = __ldg(a + ws + 63);
        base[u] = ws;
        cnt[u] = 64;
      }
    }
#pragma unroll
    for (int u = 0; u < kMix; ++u) {
      const uint32_t low = id[u] & 0xFFFFu;
      bool in = false;
      if (ty[u] == uint8_t(cu_roaring::ContainerTypeD::BITMAP)) {
        in = (word[u] >> (low & 63u)) & 1ull;
      } else if (ty[u] == uint8_t(cu_roaring::ContainerTypeD::ARRAY) && card[u] > 0) {
        uint32_t b = base[u], m = cnt[u];
        if (card[u] > 64) {  // narrow to the window or to the side of it that must hold `low`
          if (low < first[u]) { b = 0; m = base[u]; }
          else if (low > last[u]) { b = base[u] + 64; m = card[u] - b; }
        }
        const uint16_t* a = v.array_data + (off[u] >> 1);
        if (m > 0) {
          while (m > 1) {
            const uint32_t h = m >> 1;
            b = (__ldg(a + b + h - 1) < low) ? b + h : b;
            m -= h;
          }
          in = __ldg(a + b) == low;
        }
      } else if (ty[u] == uint8_t(cu_roaring::ContainerTypeD::RUN)) {
        in = v.run_contains(off[u], uint16_t(card[u]), uint16_t(low));
      }
      hit[u] = in != v.negated;
    }
#pragma unroll
    for (int u = 0; u < kMix; ++u) {
      const uint64_t i = (w0 + u) * 32 + lane;
      const uint32_t bits = __ballot_sync(0xFFFFFFFFu, hit[u] && i < n);
      if (lane == 0 && w0 + u < n_words) __stcs(out + w0 + u, bits);
    }
  }
}

// One CTA (256 threads) per output chunk.
__global__ void __launch_bounds__(256) k_decompress(DevBitmap b, uint32_t* out, uint64_t out_words)
{
  __shared__ __align__(16) uint64_t sm[1024];
  const uint32_t key = blockIdx.x;
  const ContainerRef c = dev_container(b, dev_lookup(b, key));
  uint64_t w[4];
  container_words<256, 4>(b, c, sm, w);
  const uint32_t valid = chunk_valid_bits(key, b.universe);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint64_t m = word_mask(4 * threadIdx.x + i, valid);
    w[i] = (b.negated ? ~w[i] : w[i]) & m;
  }
  const uint64_t g = uint64_t(key) * kChunkWords32 + 8ull * threadIdx.x;
  if (g + 8 <= out_words && (reinterpret_cast<uintptr_t>(out) & 15u) == 0) {
    uint4* p = reinterpret_cast<uint4*>(out + g);
    p[0] = make_uint4(uint32_t(w[0]), uint32_t(w[0] >> 32), uint32_t(w[1]), uint32_t(w[1] >> 32));
    p[1] = make_uint4(uint32_t(w[2]), uint32_t(w[2] >> 32), uint32_t(w[3]), uint32_t(w[3] >> 32));
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (g + i < out_words) out[g + i] = uint32_t(w[i >> 1] >> (32 * (i & 1)));
  }
}

// Units: containers (plain) or every chunk of the universe (negated).
__device__ __forceinline__ uint32_t unit_key(const DevBitmap& b, uint32_t u)
{
  return b.negated ? u : __ldg(b.keys + u);
}

__global__ void k_enum_count(DevBitmap b, uint32_t n_units, uint32_t* counts)
{
  const uint32_t u = blockIdx.x * blockDim.x + threadIdx.x;
  if (u >= n_units) return;
  const uint32_t key = unit_key(b, u);
  const int idx = b.negated ? dev_lookup(b, key) : static_cast<int>(u);
  const uint32_t stored = container_count(b, dev_container(b, idx));
  counts[u] = b.negated ? chunk_valid_bits(key, b.universe) - stored : stored;
}

constexpr int kScanTile = 1024;

__global__ void __launch_bounds__(kScanTile) k_scan_tiles(const uint32_t* v, uint32_t n,
                                                          unsigned long long* tile_sums)
{
  __shared__ unsigned long long s_red[32];
  const uint32_t i = blockIdx.x * kScanTile + threadIdx.x;
  const unsigned long long x = i < n ? v[i] : 0u;
  const unsigned long long t = block_sum<kScanTile, unsigned long long>(x, s_red);
  if (threadIdx.x == 0) tile_sums[blockIdx.x] = t;
}

__global__ void __launch_bounds__(kScanTile) k_scan_apply(const uint32_t* v, uint32_t n,
                                                          const unsigned long long* tile_sums,
                                                          unsigned long long* prefix)
{
  __shared__ unsigned long long s_red[32];
  __shared__ unsigned long long s_base;
  if (threadIdx.x == 0) {
    unsigned long long b = 0;
    for (uint32_t j = 0; j < blockIdx.x; ++j) b += tile_sums[j];
    s_base = b;
  }
  __syncthreads();
  const uint32_t i = blockIdx.x * kScanTile + threadIdx.x;
  const unsigned long long x = i < n ? v[i] : 0u;
  unsigned long long tot;
  const unsigned long long p = block_exclusive_scan<kScanTile, unsigned long long>(x, s_red, &tot);
  if (i < n) prefix[i] = s_base + p;
}

template <class T>
__global__ void __launch_bounds__(256) k_enum_emit(DevBitmap b, const unsigned long long* prefix,
                                                   T* out)
{
  __shared__ __align__(16) uint64_t sm[1024];
  __shared__ uint32_t s_red[8];
  const uint32_t u = blockIdx.x;
  const uint32_t key = unit_key(b, u);
  const int idx = b.negated ? dev_lookup(b, key) : static_cast<int>(u);
  const ContainerRef c = dev_container(b, idx);
  T* dst = out + prefix[u];
  const uint32_t hi = key << 16;
  if (!b.negated && c.type == kArray) {
    const uint16_t* a = b.array + (c.off >> 1);
    for (uint32_t j = threadIdx.x; j < c.card; j += 256) dst[j] = static_cast<T>(hi | __ldg(a + j));
    return;
  }
  uint64_t w[4];
  container_words<256, 4>(b, c, sm, w);
  if (b.negated) {
    const uint32_t valid = chunk_valid_bits(key, b.universe);
#pragma unroll
    for (int i = 0; i < 4; ++i) w[i] = ~w[i] & word_mask(4 * threadIdx.x + i, valid);
  }
  uint32_t cnt = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) cnt += __popcll(w[i]);
  uint32_t total;
  uint32_t pos = block_exclusive_scan<256>(cnt, s_red, &total);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint64_t x = w[i];
    while (x) {
      dst[pos++] = static_cast<T>(hi | ((4 * threadIdx.x + i) * 64 + __ffsll(x) - 1));
      x &= x - 1;
    }
  }
}

// Promotion: container i becomes BITMAP slot i.
__global__ void __launch_bounds__(256) k_promote(DevBitmap b, cr_gpu_roaring out)
{
  __shared__ __align__(16) uint64_t sm[1024];
  __shared__ uint32_t s_red[8];
  const uint32_t i = blockIdx.x;
  const ContainerRef c = dev_container(b, static_cast<int>(i));
  uint64_t w[4];
  container_words<256, 4>(b, c, sm, w);
  uint4* dst = reinterpret_cast<uint4*>(out.bitmap_data + size_t(i) * 1024) + 2 * threadIdx.x;
  dst[0] = make_uint4(uint32_t(w[0]), uint32_t(w[0] >> 32), uint32_t(w[1]), uint32_t(w[1] >> 32));
  dst[1] = make_uint4(uint32_t(w[2]), uint32_t(w[2] >> 32), uint32_t(w[3]), uint32_t(w[3] >> 32));
  uint32_t cnt = 0;
#pragma unroll
  for (int k = 0; k < 4; ++k) cnt += __popcll(w[k]);
  const uint32_t total = block_sum<256>(cnt, s_red);
  if (threadIdx.x == 0) {
    const uint16_t key = __ldg(b.keys + i);
    out.keys[i] = key;
    out.types[i] = kBitmap;
    out.offsets[i] = i * kBitmapBytes;
    out.cardinalities[i] = static_cast<uint16_t>(total & 0xFFFFu);
    if (key <= out.max_key) out.key_index[key] = static_cast<uint16_t>(i);
  }
}

cu_roaring::GpuRoaringView view_of(const cr_gpu_roaring* bm)
{
  return cu_roaring::make_view(*reinterpret_cast<const cu_roaring::GpuRoaring*>(bm));
}

template <class T>
void enumerate(const cr_gpu_roaring* bm, T* out, cudaStream_t s)
{
  if (bm->total_cardinality == 0) return;
  CR_REQUIRE(out != nullptr, "enumerate_ids: null output");
  Scratch holder;
  const DevBitmap b = make_dev(bm, holder, s);
  const uint32_t n_units = bm->negated ? n_chunks_for(bm->universe_size) : bm->n_containers;
  if (n_units == 0) return;
  const uint32_t n_tiles = div_up(n_units, kScanTile);
  Scratch scr(size_t(n_units) * 4 + size_t(n_units) * 8 + size_t(n_tiles) * 8 + 16, s);
  unsigned long long* prefix = scr.as<unsigned long long>();
  unsigned long long* tiles = prefix + n_units;
  uint32_t* counts = reinterpret_cast<uint32_t*>(tiles + n_tiles);
  k_enum_count<<<div_up(n_units, 256), 256, 0, s>>>(b, n_units, counts);
  k_scan_tiles<<<n_tiles, kScanTile, 0, s>>>(counts, n_units, tiles);
  k_scan_apply<<<n_tiles, kScanTile, 0, s>>>(counts, n_units, tiles, prefix);
  k_enum_emit<T><<<n_units, 256, 0, s>>>(b, prefix, out);
  CR_CUDA(cudaGetLastError());
}

void promote_to_bitmap(const cr_gpu_roaring* in, cr_gpu_roaring* out, cudaStream_t s)
{
  cr_gpu_roaring r{};
  r.universe_size = in->universe_size;
  r.total_cardinality = in->total_cardinality;
  r.negated = in->negated;
  r.n_containers = in->n_containers;
  r.n_bitmap_containers = in->n_containers;
  if (in->n_containers == 0) { *out = r; return; }
  uint32_t max_key = max_key_for(in->universe_size);
  if (in->key_index == nullptr) max_key = 65535;  // keys not checked on the host
  r.max_key = max_key;
  alloc_result(&r, s);
  Scratch holder;
  const DevBitmap b = make_dev(in, holder, s);
  CR_CUDA(cudaMemsetAsync(r.key_index, 0xFF, (size_t(max_key) + 1) * 2, s));
  k_promote<<<in->n_containers, 256, 0, s>>>(b, r);
  CR_CUDA(cudaGetLastError());
  *out = r;
}

}  // namespace
}  // namespace crb

using namespace crb;

extern "C" int cr_contains_batch(const cr_gpu_roaring* bm, const uint32_t* d_ids, uint64_t n,
                                 uint32_t* d_out_bits, int mode, cr_stream_t stream)
{
  CR_API_BEGIN
  CR_REQUIRE(bm != nullptr, "cr_contains_batch: null bitmap");
  CR_REQUIRE(mode == 0 || mode == 1, "cr_contains_batch: mode must be 0 or 1");
  if (n == 0) return CR_OK;
  CR_REQUIRE(d_ids && d_out_bits, "cr_contains_batch: null buffer");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const cu_roaring::GpuRoaringView v = view_of(bm);
  const uint64_t words = (n + 31) / 32;
  const uint64_t want = (words + 8 * kUnroll - 1) / (8 * kUnroll);
  const int grid = static_cast<int>(std::max<uint64_t>(1, std::min<uint64_t>(want, uint64_t(sm_count()) * 8)));
  ProfileScope prof(CR_KERNEL_CONTAINS, s);
  if (mode == 0 && v.all_bitmap) {
    const uint64_t want_b = (words + 8 * kMLP - 1) / (8 * kMLP);
    const int grid_b = static_cast<int>(std::max<uint64_t>(1, std::min<uint64_t>(want_b, uint64_t(sm_count()) * 8)));
    k_contains_bitmap<<<grid_b, 256, 0, s>>>(v.key_index, v.max_key, v.bitmap_data, v.negated ? 1u : 0u,
                                             d_ids, n, d_out_bits);
  } else if (mode == 0 && v.key_index != nullptr && v.n_containers > 0) {
    const uint64_t want_m = (words + 8 * kMix - 1) / (8 * kMix);
    const int grid_m = static_cast<int>(std::max<uint64_t>(1, std::min<uint64_t>(want_m, uint64_t(sm_count()) * 8)));
    k_contains_mixed<<<grid_m, 256, 0, s>>>(v, d_ids, n, d_out_bits);
  } else if (mode) {
    k_contains<1><<<grid, 256, 0, s>>>(v, d_ids, n, d_out_bits);
  } else {
    k_contains<0><<<grid, 256, 0, s>>>(v, d_ids, n, d_out_bits);
  }
  CR_CUDA(cudaGetLastError());
  CR_API_END
}

extern "C" int cr_decompress_to_bitset(const cr_gpu_roaring* bm, uint32_t* d_output,
                                       uint32_t output_words, cr_stream_t stream)
{
  CR_API_BEGIN
  CR_REQUIRE(bm != nullptr, "cr_decompress_to_bitset: null bitmap");
  if (output_words == 0) return CR_OK;
  CR_REQUIRE(d_output != nullptr, "cr_decompress_to_bitset: null output");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  Scratch holder;
  const DevBitmap b = make_dev(bm, holder, s);
  ProfileScope prof(CR_KERNEL_DECOMPRESS, s);
  k_decompress<<<div_up(output_words, kChunkWords32), 256, 0, s>>>(b, d_output, output_words);
  CR_CUDA(cudaGetLastError());
  CR_API_END
}

extern "C" int cr_decompress_to_bitset_alloc(const cr_gpu_roaring* bm, cr_stream_t stream,
                                             uint32_t** d_out)
{
  CR_API_BEGIN
  CR_REQUIRE(bm && d_out, "cr_decompress_to_bitset_alloc: null argument");
  *d_out = nullptr;
  const uint32_t words = div_up(bm->universe_size, 32);
  if (words == 0) return CR_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  uint32_t* p = static_cast<uint32_t*>(dev_alloc(size_t(words) * 4, s));
  const int rc = cr_decompress_to_bitset(bm, p, words, stream);
  if (rc != CR_OK) { cudaFreeAsync(p, s); return rc; }
  *d_out = p;
  CR_API_END
}

extern "C" int cr_enumerate_ids_i64(const cr_gpu_roaring* bm, int64_t* d_output, cr_stream_t stream)
{
  CR_API_BEGIN
  CR_REQUIRE(bm != nullptr, "cr_enumerate_ids: null bitmap");
  enumerate<long long>(bm, reinterpret_cast<long long*>(d_output), reinterpret_cast<cudaStream_t>(stream));
  CR_API_END
}

extern "C" int cr_enumerate_ids_u32(const cr_gpu_roaring* bm, uint32_t* d_output, cr_stream_t stream)
{
  CR_API_BEGIN
  CR_REQUIRE(bm != nullptr, "cr_enumerate_ids: null bitmap");
  enumerate<uint32_t>(bm, d_output, reinterpret_cast<cudaStream_t>(stream));
  CR_API_END
}

extern "C" int cr_enumerate_ids_alloc(const cr_gpu_roaring* bm, cr_stream_t stream, int64_t** d_out)
{
  CR_API_BEGIN
  CR_REQUIRE(bm && d_out, "cr_enumerate_ids_alloc: null argument");
  *d_out = nullptr;
  if (bm->total_cardinality == 0) return CR_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int64_t* p = static_cast<int64_t*>(dev_alloc(bm->total_cardinality * 8, s));
  const int rc = cr_enumerate_ids_i64(bm, p, stream);
  if (rc != CR_OK) { cudaFreeAsync(p, s); return rc; }
  *d_out = p;
  CR_API_END
}

extern "C" int cr_promote_to_bitmap(const cr_gpu_roaring* bm, cr_stream_t stream, cr_gpu_roaring* out)
{
  CR_API_BEGIN
  CR_REQUIRE(bm && out, "cr_promote_to_bitmap: null argument");
  promote_to_bitmap(bm, out, reinterpret_cast<cudaStream_t>(stream));
  CR_API_END
}

// Reference src/promote.cu:369-385: promote iff AUTO resolves to ALL and the
// input has non-bitmap containers, else an independent deep copy.
extern "C" int cr_promote_auto(const cr_gpu_roaring* bm, cr_stream_t stream, int device_id,
                               cr_gpu_roaring* out)
{
  CR_API_BEGIN
  CR_REQUIRE(bm && out, "cr_promote_auto: null argument");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const uint32_t t = resolve_auto(bm->universe_size, device_id);
  if (t == 0 && (bm->n_array_containers || bm->n_run_containers)) promote_to_bitmap(bm, out, s);
  else deep_copy(bm, out, s);
  CR_API_END
}

// ---------------------------------------------------------------------------
// Allocation-free enumerate_ids (no counterpart in the reference).
//
// For callers that may not allocate device memory while they run: engines
// that hand all of a GPU's memory to their own pool at start-up, or
// latency-critical paths where a cudaMallocAsync (and the pool growth or
// synchronisation it can cause) is not allowed. The scratch that
// cr_enumerate_ids_u32 takes from the stream-ordered allocator (per-unit
// counts, the tile scan, the output prefix, and a key index for bitmaps that
// lack one) lives instead in one file-scope device array of
// kNoAllocScratchBytes, which every GPU that loads this library holds until
// the process exits.
// ---------------------------------------------------------------------------

namespace {
constexpr uint32_t kNoAllocMaxUnits = 65536;  // containers or chunks: every valid bitmap
constexpr size_t kNoAllocPrefixOff = 0;                                   // u64[65536]
constexpr size_t kNoAllocTilesOff = kNoAllocPrefixOff + kNoAllocMaxUnits * 8;  // u64[64]
constexpr size_t kNoAllocCountsOff = kNoAllocTilesOff + 64 * 8;           // u32[65536]
constexpr size_t kNoAllocKidxOff = kNoAllocCountsOff + kNoAllocMaxUnits * 4;   // u16[65536]
constexpr size_t kNoAllocScratchBytes = kNoAllocKidxOff + kNoAllocMaxUnits * 2;
}  // namespace

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch on the current device. The first call
// on each device resolves it with cudaGetSymbolAddress (with that device
// current); later calls reuse the cached address as long as the device's
// context is the same one. A context created anew (after cudaDeviceReset, or
// a release and re-creation of the primary context) reloads the module, so
// its address is looked up again.
static unsigned char* noalloc_scratch()
{
  using CtxGetCurrentFn = CUresult (*)(CUcontext*);
  static std::mutex mu;
  static unsigned char* addr[64] = {};
  static CUcontext ctx_of[64] = {};
  static CtxGetCurrentFn ctx_get = nullptr;
  int dev = 0;
  CR_CUDA(cudaGetDevice(&dev));
  CR_REQUIRE(dev >= 0 && dev < 64, "cr_enumerate_ids_u32_noalloc: device ordinal out of range");
  std::lock_guard<std::mutex> lock(mu);
  if (!ctx_get) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || fn == nullptr)
      fail(CR_ERR_CUDA, "cr_enumerate_ids_u32_noalloc: cuCtxGetCurrent is not available");
    ctx_get = reinterpret_cast<CtxGetCurrentFn>(fn);
  }
  CUcontext ctx = nullptr;
  if (ctx_get(&ctx) != CUDA_SUCCESS) fail(CR_ERR_CUDA, "cr_enumerate_ids_u32_noalloc: cuCtxGetCurrent failed");
  if (!addr[dev] || ctx == nullptr || ctx_of[dev] != ctx) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      fail(CR_ERR_CUDA, std::string("cr_enumerate_ids_u32_noalloc: cudaGetSymbolAddress failed: ") +
                            cudaGetErrorString(e));
    }
    addr[dev] = static_cast<unsigned char*>(p);
    // The lookup made the device's context current if nothing had yet.
    if (ctx == nullptr && ctx_get(&ctx) != CUDA_SUCCESS) ctx = nullptr;
    ctx_of[dev] = ctx;
  }
  return addr[dev];
}

extern "C" int cr_enumerate_ids_u32_noalloc(const cr_gpu_roaring* bm, uint32_t* d_output,
                                            cr_stream_t stream)
{
  CR_API_BEGIN
  CR_REQUIRE(bm != nullptr, "cr_enumerate_ids_u32_noalloc: null bitmap");
  if (bm->total_cardinality == 0) return CR_OK;
  CR_REQUIRE(d_output != nullptr, "cr_enumerate_ids_u32_noalloc: null output");
  const uint32_t n_units = bm->negated ? n_chunks_for(bm->universe_size) : bm->n_containers;
  if (n_units == 0) return CR_OK;
  if (n_units > kNoAllocMaxUnits)
    fail(CR_ERR_INVALID, "cr_enumerate_ids_u32_noalloc: " + std::to_string(n_units) +
                             " containers exceed the fixed scratch limit of 65536");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  unsigned char* scratch = noalloc_scratch();
  unsigned long long* prefix = reinterpret_cast<unsigned long long*>(scratch + kNoAllocPrefixOff);
  unsigned long long* tiles = reinterpret_cast<unsigned long long*>(scratch + kNoAllocTilesOff);
  uint32_t* counts = reinterpret_cast<uint32_t*>(scratch + kNoAllocCountsOff);
  DevBitmap b{};
  b.keys = bm->keys;
  b.types = bm->types;
  b.offsets = bm->offsets;
  b.cards = bm->cardinalities;
  b.bitmap = bm->bitmap_data;
  b.array = bm->array_data;
  b.run = bm->run_data;
  b.n = bm->n_containers;
  b.universe = bm->universe_size;
  b.negated = bm->negated ? 1u : 0u;
  b.key_index = bm->key_index;
  b.max_key = bm->max_key;
  if (bm->n_containers == 0) {
    b.key_index = nullptr;
    b.max_key = 0;
  } else if (bm->key_index == nullptr) {
    // No index on the input: build a full one in the static scratch.
    uint16_t* kidx = reinterpret_cast<uint16_t*>(scratch + kNoAllocKidxOff);
    build_key_index(bm->keys, bm->n_containers, kidx, kNoAllocMaxUnits, s);
    b.key_index = kidx;
    b.max_key = kNoAllocMaxUnits - 1;
  }
  // counts, tile sums and prefixes are fully rewritten below, so the
  // previous call's contents never leak into this one.
  const uint32_t n_tiles = div_up(n_units, kScanTile);
  k_enum_count<<<div_up(n_units, 256), 256, 0, s>>>(b, n_units, counts);
  k_scan_tiles<<<n_tiles, kScanTile, 0, s>>>(counts, n_units, tiles);
  k_scan_apply<<<n_tiles, kScanTile, 0, s>>>(counts, n_units, tiles, prefix);
  k_enum_emit<uint32_t><<<n_units, 256, 0, s>>>(b, prefix, d_output);
  CR_CUDA(cudaGetLastError());
  CR_API_END
}
