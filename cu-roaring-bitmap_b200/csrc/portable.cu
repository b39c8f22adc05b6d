// cu_roaring B200 engine — ingest of the portable Roaring serialization.
//
// The portable format is the published, implementation-independent layout
// of a 32-bit Roaring bitmap (the "RoaringFormatSpec"): a cookie (12346 = no
// run containers, followed by the container count; or 12347 in the low 16
// bits with count - 1 in the high 16 bits, followed by a bitset marking the
// run containers), one (key, cardinality - 1) pair of little-endian u16 per
// container, a u32 byte offset per container (always with cookie 12346, and
// with 12347 when there are at least 4 containers), then the containers:
// ARRAY = cardinality sorted u16 values (cardinality <= 4096), BITMAP = 1024
// little-endian u64 words, RUN = u16 run count then (start, length - 1) u16
// pairs.
//
// The reference loads such files only through CRoaring on the host
// (bench/bench_from_disk.cu, not in the tree, feeding upload(roaring_bitmap_t*),
// src/upload.cpp:89-225). Here the header is checked on the host, the bytes
// go to the device once, one block per container rebuilds its 65536-bit chunk
// of a flat bitset, and the bitset upload builds the canonical image
// (container types under bitmap_threshold, complement above half density).
#include <algorithm>
#include <cstring>
#include <string>
#include <vector>

#include "common.cuh"

namespace crb {
namespace {

constexpr uint32_t kCookieNoRun = 12346u;
constexpr uint32_t kCookieRun = 12347u;
constexpr uint32_t kNoOffsetThreshold = 4u;
constexpr uint32_t kErrPastUniverse = 1u;
constexpr uint32_t kErrBadRun = 2u;
constexpr uint32_t kErrCardinality = 4u;

enum : uint32_t { kKindArray = kPortableArray, kKindBitmap = kPortableBitmap, kKindRun = kPortableRun };

__device__ __forceinline__ uint32_t ld_u16(const uint8_t* p) { return uint32_t(p[0]) | (uint32_t(p[1]) << 8); }

// One block per container: its 2048 words, then a check of the declared
// cardinality and of the universe bound; the chunk is written in full.
__global__ void __launch_bounds__(256) k_portable_expand(const uint8_t* buf, const PortableContainer* cs,
                                                         uint32_t* words, uint64_t n_words, uint32_t U,
                                                         uint32_t* err)
{
  __shared__ uint32_t w[2048];
  __shared__ uint32_t s_pop;
  const PortableContainer c = cs[blockIdx.x];
  const uint8_t* p = buf + c.offset;
  for (uint32_t i = threadIdx.x; i < 2048; i += blockDim.x) w[i] = 0u;
  if (threadIdx.x == 0) s_pop = 0;
  __syncthreads();
  if (c.kind == kKindBitmap) {
    for (uint32_t i = threadIdx.x; i < 2048; i += blockDim.x) {
      const uint8_t* q = p + 4 * i;  // payload offsets need not be aligned
      w[i] = uint32_t(q[0]) | (uint32_t(q[1]) << 8) | (uint32_t(q[2]) << 16) | (uint32_t(q[3]) << 24);
    }
  } else if (c.kind == kKindArray) {
    for (uint32_t e = threadIdx.x; e < c.count; e += blockDim.x) {
      const uint32_t v = ld_u16(p + 2 * e);
      atomicOr(&w[v >> 5], 1u << (v & 31));
    }
  } else {
    for (uint32_t r = threadIdx.x; r < c.count; r += blockDim.x) {
      const uint32_t start = ld_u16(p + 2 + 4 * r), last = start + ld_u16(p + 4 + 4 * r);
      if (last > 0xFFFFu) { atomicOr(err, kErrBadRun); continue; }
      for (uint32_t wi = start >> 5; wi <= (last >> 5); ++wi) {
        const uint32_t lo = max(start, wi * 32) - wi * 32, hi = min(last, wi * 32 + 31) - wi * 32;
        const uint32_t m = (hi == 31 ? 0xFFFFFFFFu : ((1u << (hi + 1)) - 1u)) & ~((1u << lo) - 1u);
        atomicOr(&w[wi], m);
      }
    }
  }
  __syncthreads();
  const uint64_t base = uint64_t(c.key) * 2048;
  uint32_t pop = 0;
  for (uint32_t i = threadIdx.x; i < 2048; i += blockDim.x) {
    const uint32_t x = w[i];
    pop += __popc(x);
    const uint64_t gw = base + i, lo_bit = gw * 32;
    uint32_t valid = 0xFFFFFFFFu;  // bits below the universe
    if (lo_bit >= U) valid = 0u;
    else if (U - lo_bit < 32) valid = (1u << (U - lo_bit)) - 1u;
    if (x & ~valid) atomicOr(err, kErrPastUniverse);
    if (gw < n_words) words[gw] = x;
  }
  atomicAdd(&s_pop, pop);
  __syncthreads();
  if (threadIdx.x == 0 && s_pop != c.card) atomicOr(err, kErrCardinality);
}

}  // namespace

namespace {
struct Reader {
  const uint8_t* p;
  uint64_t n;
  uint32_t u16(uint64_t at) const
  {
    CR_REQUIRE(at + 2 <= n, "cr_upload_portable: truncated buffer");
    return uint32_t(p[at]) | (uint32_t(p[at + 1]) << 8);
  }
  uint32_t u32(uint64_t at) const
  {
    CR_REQUIRE(at + 4 <= n, "cr_upload_portable: truncated buffer");
    return u16(at) | (u16(at + 2) << 16);
  }
};

}  // namespace

PortableImage parse_portable(const void* data, uint64_t n_bytes, uint32_t universe_size, const char* who)
{
  const std::string w(who);
  if (!(data != nullptr && n_bytes >= 4)) fail(CR_ERR_INVALID, w + ": empty buffer");
  const Reader rd{static_cast<const uint8_t*>(data), n_bytes};
  // Header.
  const uint32_t cookie = rd.u32(0);
  uint32_t n = 0;
  uint64_t pos = 0, run_flags = 0;
  bool has_runs = false;
  if ((cookie & 0xFFFFu) == kCookieRun) {
    has_runs = true;
    n = (cookie >> 16) + 1;
    run_flags = 4;
    pos = 4 + (uint64_t(n) + 7) / 8;
  } else if (cookie == kCookieNoRun) {
    n = rd.u32(4);
    pos = 8;
  } else {
    fail(CR_ERR_INVALID, w + ": not a portable Roaring bitmap (unknown cookie)");
  }
  if (n > 65536) fail(CR_ERR_INVALID, w + ": more than 65536 containers");
  const uint64_t desc = pos;
  pos += uint64_t(n) * 4;
  const bool has_offsets = !has_runs || n >= kNoOffsetThreshold;
  const uint64_t offs = pos;
  if (has_offsets) pos += uint64_t(n) * 4;
  if (pos > n_bytes) fail(CR_ERR_INVALID, w + ": truncated buffer");
  const uint32_t n_chunks = universe_size ? n_chunks_for(universe_size) : 65536u;
  PortableImage im;
  im.cs.resize(n);
  uint64_t end = pos, cursor = pos;
  for (uint32_t i = 0; i < n; ++i) {
    PortableContainer& c = im.cs[i];
    c.key = rd.u16(desc + 4 * uint64_t(i));
    c.card = rd.u16(desc + 4 * uint64_t(i) + 2) + 1;
    if (!(i == 0 || c.key > im.cs[i - 1].key)) fail(CR_ERR_INVALID, w + ": container keys not strictly increasing");
    if (c.key >= n_chunks) fail(CR_ERR_RANGE, w + ": a container lies past universe_size");
    const bool run = has_runs && ((rd.p[run_flags + i / 8] >> (i % 8)) & 1u);
    c.offset = has_offsets ? rd.u32(offs + 4 * uint64_t(i)) : cursor;
    uint64_t bytes;
    if (run) {
      c.kind = kKindRun;
      c.count = rd.u16(c.offset);
      bytes = 2 + 4 * uint64_t(c.count);
    } else if (c.card <= 4096) {
      c.kind = kKindArray;
      c.count = c.card;
      bytes = 2 * uint64_t(c.card);
    } else {
      c.kind = kKindBitmap;
      c.count = c.card;
      bytes = 8192;
    }
    if (!(c.offset >= pos && c.offset + bytes <= n_bytes)) fail(CR_ERR_INVALID, w + ": container payload out of bounds");
    cursor = c.offset + bytes;
    end = std::max<uint64_t>(end, cursor);
  }
  im.end = end;
  return im;
}

}  // namespace crb

using namespace crb;

static void upload_portable(const void* data, uint64_t n_bytes, uint32_t universe_size, cr_stream_t stream,
                            uint32_t bitmap_threshold, uint32_t flags, cr_gpu_roaring* out)
{
  CR_REQUIRE(out != nullptr, "cr_upload_portable: null output");
  CR_REQUIRE((flags & ~uint32_t(CR_PORTABLE_KEEP_UNCOMPLEMENTED)) == 0, "cr_upload_portable_ex: unknown flag");
  const PortableImage im = parse_portable(data, n_bytes, universe_size, "cr_upload_portable");
  const std::vector<PortableContainer>& cs = im.cs;
  const uint32_t n = uint32_t(cs.size());
  const uint64_t end = im.end;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const uint64_t n_words = (uint64_t(universe_size) + 31) / 32;
  Scratch buf(end + sizeof(PortableContainer) * std::max<uint32_t>(n, 1) + 16 + 256, s);
  Scratch bits(n_words * 4, s);
  uint8_t* d_buf = buf.as<uint8_t>();
  auto* d_cs = reinterpret_cast<PortableContainer*>(
      (reinterpret_cast<uintptr_t>(d_buf + end) + 15) & ~uintptr_t(15));
  uint32_t* d_err = reinterpret_cast<uint32_t*>(d_cs + std::max<uint32_t>(n, 1));
  CR_CUDA(cudaMemcpyAsync(d_buf, data, end, cudaMemcpyHostToDevice, s));
  if (n) CR_CUDA(cudaMemcpyAsync(d_cs, cs.data(), sizeof(PortableContainer) * n, cudaMemcpyHostToDevice, s));
  CR_CUDA(cudaMemsetAsync(d_err, 0, 4, s));
  if (n_words) CR_CUDA(cudaMemsetAsync(bits.p, 0, n_words * 4, s));
  if (n) k_portable_expand<<<n, 256, 0, s>>>(d_buf, d_cs, bits.as<uint32_t>(), n_words, universe_size, d_err);
  CR_CUDA(cudaGetLastError());
  uint32_t h_err = 0;
  CR_CUDA(cudaMemcpyAsync(&h_err, d_err, 4, cudaMemcpyDeviceToHost, s));
  CR_CUDA(cudaStreamSynchronize(s));
  if (h_err & kErrPastUniverse) fail(CR_ERR_RANGE, "cr_upload_portable: a member is >= universe_size");
  if (h_err & kErrBadRun) fail(CR_ERR_INVALID, "cr_upload_portable: a run passes the end of its container");
  if (h_err & kErrCardinality)
    fail(CR_ERR_INVALID, "cr_upload_portable: a container's members do not match its declared cardinality");
  upload_device_bitset(bits.as<uint32_t>(), n_words, universe_size, bitmap_threshold, s, out,
                       (flags & CR_PORTABLE_KEEP_UNCOMPLEMENTED) != 0);
}

extern "C" int cr_upload_portable(const void* data, uint64_t n_bytes, uint32_t universe_size, cr_stream_t stream,
                                  uint32_t bitmap_threshold, cr_gpu_roaring* out)
{
  CR_API_BEGIN
  upload_portable(data, n_bytes, universe_size, stream, bitmap_threshold, 0u, out);
  CR_API_END
}

extern "C" int cr_upload_portable_ex(const void* data, uint64_t n_bytes, uint32_t universe_size, cr_stream_t stream,
                                     uint32_t bitmap_threshold, uint32_t flags, cr_gpu_roaring* out)
{
  CR_API_BEGIN
  upload_portable(data, n_bytes, universe_size, stream, bitmap_threshold, flags, out);
  CR_API_END
}

extern "C" int cr_portable_meta(const void* data, uint64_t n_bytes, cr_roaring_meta* out)
{
  CR_API_BEGIN
  CR_REQUIRE(out != nullptr, "cr_portable_meta: null output");
  std::memset(out, 0, sizeof(*out));
  const PortableImage im = parse_portable(data, n_bytes, 0, "cr_portable_meta");
  uint64_t array_elems = 0, run_pairs = 0, card = 0;
  for (const PortableContainer& c : im.cs) {
    if (c.kind == kKindBitmap) ++out->n_bitmap_containers;
    else if (c.kind == kKindArray) { ++out->n_array_containers; array_elems += c.count; }
    else { ++out->n_run_containers; run_pairs += c.count; }
    card += c.card;
  }
  out->n_containers = uint32_t(im.cs.size());
  out->total_cardinality = card;
  if (!im.cs.empty()) {
    const uint64_t mk = im.cs.back().key;
    out->max_key = uint32_t(mk);
    out->universe_size = uint32_t((mk + 1) << 16);  // the reference's u32 arithmetic: 0 for key 65535
  }
  // Device bytes of the containers as the reference counts them
  // (src/upload.cpp:60-68): per container key u16, type u8, offset u32 and
  // cardinality u16; 8 KiB per BITMAP; 2 B per ARRAY member; 4 B per run.
  out->total_bytes = uint64_t(out->n_containers) * (2 + 1 + 4 + 2) + uint64_t(out->n_bitmap_containers) * 8192 +
                     array_elems * 2 + run_pairs * 4;
  CR_API_END
}
