// cu_roaring B200 engine — per-container device helpers shared by the
// export, promotion and set-algebra kernels.
//
// A CTA of NT threads (NT = 256: 4 u64 words per thread, 1024 = 1 word per
// thread) materialises one 65536-bit container. BITMAP containers are read
// straight from HBM with 16-byte loads; ARRAY and RUN containers are expanded
// into an 8 KiB shared-memory bitmap (shared atomics, word-granular run fill)
// and read back.
#pragma once
#include "common.cuh"

namespace crb {

struct ContainerRef {
  int idx;        // -1 = absent
  uint8_t type;
  uint32_t off;   // byte offset
  uint32_t card;  // raw cardinality field
};

__device__ __forceinline__ int dev_lookup(const DevBitmap& b, uint32_t key)
{
  if (b.key_index == nullptr || key > b.max_key) return -1;
  const uint16_t i = __ldg(b.key_index + key);
  return i == 0xFFFFu ? -1 : static_cast<int>(i);
}

__device__ __forceinline__ ContainerRef dev_container(const DevBitmap& b, int idx)
{
  ContainerRef r{idx, 0xFF, 0, 0};
  if (idx >= 0) {
    r.type = __ldg(b.types + idx);
    r.off = __ldg(b.offsets + idx);
    r.card = __ldg(b.cards + idx);
  }
  return r;
}

// Number of elements of a container (BITMAP 0 means 65536; RUN sums lengths).
__device__ __forceinline__ uint32_t container_count(const DevBitmap& b, const ContainerRef& c)
{
  if (c.idx < 0) return 0;
  if (c.type == kArray) return c.card;
  if (c.type == kBitmap) return c.card ? c.card : 65536u;
  const uint16_t* r = b.run + (c.off >> 1);
  uint32_t n = 0;
  for (uint32_t j = 0; j < c.card; ++j) n += uint32_t(__ldg(r + 2 * j + 1)) + 1u;
  return n;
}

// Expands an ARRAY or RUN container into the shared bitmap `sm` (1024 u64,
// zeroed by this call). All NT threads must call it.
template <int NT>
__device__ __forceinline__ void expand_to_smem(const DevBitmap& b, const ContainerRef& c,
                                               uint64_t* sm)
{
  for (int i = threadIdx.x; i < 1024; i += NT) sm[i] = 0ull;
  __syncthreads();
  if (c.idx >= 0 && c.type == kArray) {
    const uint16_t* a = b.array + (c.off >> 1);
    for (uint32_t j = threadIdx.x; j < c.card; j += NT) {
      const uint32_t v = __ldg(a + j);
      atomicOr(reinterpret_cast<unsigned long long*>(sm + (v >> 6)), 1ull << (v & 63));
    }
  } else if (c.idx >= 0 && c.type == kRun && c.card <= 64) {
    // Few (typically long) runs: the whole block fills each run's words
    // together instead of one thread walking a run word by word.
    __shared__ uint32_t s_runs[64];
    const uint16_t* r = b.run + (c.off >> 1);
    if (threadIdx.x < c.card) {
      const uint32_t s = __ldg(r + 2 * threadIdx.x);
      s_runs[threadIdx.x] = (s << 16) | min(65535u, s + __ldg(r + 2 * threadIdx.x + 1));
    }
    __syncthreads();
    for (uint32_t j = 0; j < c.card; ++j) {
      const uint32_t s = s_runs[j] >> 16, e = s_runs[j] & 0xFFFFu;
      const uint32_t ws = s >> 6, we = e >> 6;
      for (uint32_t w = ws + threadIdx.x; w <= we; w += NT) {
        uint64_t m = ~0ull;
        if (w == ws) m &= ~0ull << (s & 63);
        if (w == we) m &= (~0ull) >> (63 - (e & 63));
        if (m == ~0ull) sm[w] = ~0ull;
        else atomicOr(reinterpret_cast<unsigned long long*>(sm + w), m);
      }
    }
  } else if (c.idx >= 0 && c.type == kRun) {
    const uint16_t* r = b.run + (c.off >> 1);
    for (uint32_t j = threadIdx.x; j < c.card; j += NT) {
      const uint32_t s = __ldg(r + 2 * j);
      const uint32_t e = min(65535u, s + __ldg(r + 2 * j + 1));
      const uint32_t ws = s >> 6, we = e >> 6;
      for (uint32_t w = ws; w <= we; ++w) {
        uint64_t m = ~0ull;
        if (w == ws) m &= ~0ull << (s & 63);
        if (w == we) m &= (~0ull) >> (63 - (e & 63));
        if (m == ~0ull) sm[w] = ~0ull;
        else atomicOr(reinterpret_cast<unsigned long long*>(sm + w), m);
      }
    }
  }
  __syncthreads();
}

// This thread's words of a container: NT=256 -> words 4t..4t+3 (W=4);
// NT=1024 -> word t (W=1). Absent containers read as zero. Uniform call.
template <int NT, int W>
__device__ __forceinline__ void container_words(const DevBitmap& b, const ContainerRef& c,
                                                uint64_t* sm, uint64_t w[W])
{
  static_assert(NT * W == 1024, "one chunk per CTA");
  if (c.idx >= 0 && c.type == kBitmap) {
    const uint64_t* src = b.bitmap + (c.off >> 3) + W * threadIdx.x;
    if (W == 4) {
      const uint4* p = reinterpret_cast<const uint4*>(src);
      const uint4 x = __ldg(p), y = __ldg(p + 1);
      w[0] = uint64_t(x.x) | (uint64_t(x.y) << 32);
      w[1 % W] = uint64_t(x.z) | (uint64_t(x.w) << 32);
      w[2 % W] = uint64_t(y.x) | (uint64_t(y.y) << 32);
      w[3 % W] = uint64_t(y.z) | (uint64_t(y.w) << 32);
    } else {
#pragma unroll
      for (int i = 0; i < W; ++i) w[i] = __ldg(src + i);
    }
    return;
  }
  if (c.idx < 0) {
#pragma unroll
    for (int i = 0; i < W; ++i) w[i] = 0ull;
    return;
  }
  expand_to_smem<NT>(b, c, sm);
#pragma unroll
  for (int i = 0; i < W; ++i) w[i] = sm[W * threadIdx.x + i];
  __syncthreads();
}

}  // namespace crb
