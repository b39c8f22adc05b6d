// cu_roaring B200 engine — batch membership tests in device code (drop-in for
// the reference v2/include/cu_roaring_v2/query.cuh): contains(view, id) for
// one bitmap of a batch, contains(batch, b, id) for bitmap b (two more reads
// for the CSR bounds).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "cu_roaring_v2/types.cuh"

namespace cu_roaring::v2 {
namespace detail {

// Member `low` of container `cid` (an index into types / offsets / cards).
__device__ __forceinline__ bool container_has(const ContainerType* types, const uint32_t* offsets,
                                              const uint16_t* cards, const uint64_t* bitmap_data,
                                              const uint16_t* array_data, const uint16_t* run_data, uint32_t cid,
                                              uint32_t low)
{
  const uint32_t off = __ldg(offsets + cid);
  const ContainerType t = types[cid];
  if (t == ContainerType::BITMAP) {
    const uint64_t* w = bitmap_data + (off >> 3);
    return (__ldg(w + (low >> 6)) >> (low & 63u)) & 1u;
  }
  const uint32_t n = __ldg(cards + cid);
  if (t == ContainerType::ARRAY) {
    const uint16_t* a = array_data + (off >> 1);
    uint32_t lo = 0, hi = n;  // first element >= low
    while (lo < hi) {
      const uint32_t mid = (lo + hi) >> 1;
      if (__ldg(a + mid) < low) lo = mid + 1; else hi = mid;
    }
    return lo < n && __ldg(a + lo) == low;
  }
  const uint16_t* r = run_data + (off >> 1);  // (start, length - 1) pairs
  uint32_t lo = 0, hi = n;                    // runs starting at or before low
  while (lo < hi) {
    const uint32_t mid = (lo + hi) >> 1;
    if (__ldg(r + 2 * mid) <= low) lo = mid + 1; else hi = mid;
  }
  if (lo == 0) return false;
  return low <= uint32_t(__ldg(r + 2 * (lo - 1))) + __ldg(r + 2 * (lo - 1) + 1);
}

}  // namespace detail

__device__ __forceinline__ bool contains(const GpuRoaringView& v, uint32_t id)
{
  const uint32_t key = id >> 16;
  if (v.n_containers == 0 || key > v.max_key) return false;
  const uint32_t cid = __ldg(v.key_index + key);
  if (cid == 0xFFFFu) return false;
  return detail::container_has(v.types, v.offsets, v.cardinalities, v.bitmap_data, v.array_data, v.run_data, cid,
                               id & 0xFFFFu);
}

__device__ __forceinline__ bool contains(const GpuRoaringBatch& batch, uint32_t b, uint32_t id)
{
  if (b >= batch.n_bitmaps) return false;
  const uint32_t c0 = __ldg(batch.container_starts + b), c1 = __ldg(batch.container_starts + b + 1);
  const uint32_t k0 = __ldg(batch.key_index_starts + b), k1 = __ldg(batch.key_index_starts + b + 1);
  const uint32_t key = id >> 16;
  if (c1 == c0 || key >= k1 - k0) return false;
  const uint32_t local = __ldg(batch.key_indices + k0 + key);
  if (local == 0xFFFFu) return false;
  return detail::container_has(batch.types, batch.offsets, batch.cardinalities, batch.bitmap_data,
                               batch.array_data, batch.run_data, c0 + local, id & 0xFFFFu);
}

}  // namespace cu_roaring::v2
