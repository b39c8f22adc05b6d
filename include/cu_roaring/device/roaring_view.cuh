// cu_roaring B200 engine — header-only device view and point query.
//
// Drop-in for include/cu_roaring/device/roaring_view.cuh:14-172 of the
// reference: same struct name, field names/order/types and member function
// names, because user kernels (and the cuVS roaring_filter functor) capture a
// GpuRoaringView by value and call contains() inside their own code; a C ABI
// cannot export device functions, so this stays header-only.
//
// Semantics (reference roaring_view.cuh:39-76, :152-157):
//   contains(id) = (id's container holds id's low 16 bits) XOR negated,
//   where an absent container holds nothing and a run (start, len) covers
//   start..start+len inclusive.
//
// The searches here are branchless lower-bound loops (a fixed number of
// steps, no early exit) so that lanes of a warp querying the same container
// stay converged; the reference uses classic early-exit binary search.
#pragma once
#include <cstdint>

namespace cu_roaring {

enum class ContainerTypeD : uint8_t {
  ARRAY  = 0,
  BITMAP = 1,
  RUN    = 2
};

struct GpuRoaringView {
  const uint16_t*       keys;
  const ContainerTypeD* types;
  const uint32_t*       offsets;
  const uint16_t*       cardinalities;
  uint32_t              n_containers;

  const uint64_t* bitmap_data;
  const uint16_t* array_data;
  const uint16_t* run_data;

  const uint16_t* key_index;   // key -> container index, 0xFFFF = absent
  uint32_t        max_key;     // last valid key_index entry

  // Every container is a BITMAP stored at slot == container index, and
  // key_index is present: the query is two dependent loads.
  bool            all_bitmap;
  bool            negated;

  __device__ __forceinline__ bool contains(uint32_t id) const
  {
    const uint32_t key = id >> 16;
    const uint32_t low = id & 0xFFFFu;
    if (all_bitmap) {
      if (key > max_key) return negated;
      const uint32_t idx = __ldg(key_index + key);
      if (idx == 0xFFFFu) return negated;
      const uint64_t w = __ldg(bitmap_data + (static_cast<size_t>(idx) << 10) + (low >> 6));
      return static_cast<bool>((w >> (low & 63u)) & 1u) != negated;
    }
    const int idx = lookup_key(static_cast<uint16_t>(key));
    if (idx < 0) return negated;
    return contains_in(load_type(idx), load_offset(idx), load_cardinality(idx),
                       static_cast<uint16_t>(low)) != negated;
  }

  // Membership of `low` inside one container whose metadata is known.
  __device__ __forceinline__ bool contains_in(ContainerTypeD t, uint32_t off,
                                              uint16_t card, uint16_t low) const
  {
    if (t == ContainerTypeD::BITMAP) return bitmap_contains(off, low);
    if (t == ContainerTypeD::ARRAY) return array_contains(off, card, low);
    if (t == ContainerTypeD::RUN) return run_contains(off, card, low);
    return false;
  }

  __device__ __forceinline__ int lookup_key(uint16_t key) const
  {
    if (key_index != nullptr) {
      if (key > max_key) return -1;
      const uint16_t idx = __ldg(key_index + key);
      return idx == 0xFFFFu ? -1 : static_cast<int>(idx);
    }
    return binary_search_keys(key);
  }

  __device__ __forceinline__ ContainerTypeD load_type(int idx) const
  {
    return static_cast<ContainerTypeD>(__ldg(reinterpret_cast<const uint8_t*>(types) + idx));
  }
  __device__ __forceinline__ uint32_t load_offset(int idx) const { return __ldg(offsets + idx); }
  __device__ __forceinline__ uint16_t load_cardinality(int idx) const
  {
    return __ldg(cardinalities + idx);
  }

  // Lower bound over the sorted key array; -1 when the key is absent.
  __device__ __forceinline__ int binary_search_keys(uint16_t key) const
  {
    uint32_t n = n_containers;
    if (n == 0) return -1;
    uint32_t base = 0;
    while (n > 1) {
      const uint32_t half = n >> 1;
      base = (__ldg(keys + base + half - 1) < key) ? base + half : base;
      n -= half;
    }
    return __ldg(keys + base) == key ? static_cast<int>(base) : -1;
  }

  // Offsets are BYTE offsets into the pool of the container's type.
  __device__ __forceinline__ bool bitmap_contains(uint32_t byte_offset, uint16_t low) const
  {
    const uint64_t w = __ldg(bitmap_data + (byte_offset >> 3) + (low >> 6));
    return (w >> (low & 63u)) & 1u;
  }

  __device__ __forceinline__ bool array_contains(uint32_t byte_offset, uint16_t card,
                                                 uint16_t low) const
  {
    if (card == 0) return false;
    const uint16_t* a = array_data + (byte_offset >> 1);
    // The sorted lows of a chunk sit near index low * card / 65536 when they
    // are spread out: look at a 64-entry window around that estimate first
    // (its two ends in one or two cache lines, so the search inside is cheap)
    // and narrow the search to the window or to the side of it that must
    // hold `low`. Exact for any data; only the speed depends on the spread.
    uint32_t base = 0, n = card;
    if (card > 64) {
      const uint32_t g = (static_cast<uint32_t>(low) * card) >> 16;
      const uint32_t w0 = g >= 32 ? min(g - 32, static_cast<uint32_t>(card) - 64) : 0u;
      const uint16_t first = __ldg(a + w0), last = __ldg(a + w0 + 63);
      if (low < first) n = w0;
      else if (low > last) { base = w0 + 64; n = card - base; }
      else { base = w0; n = 64; }
      if (n == 0) return false;
    }
    while (n > 1) {
      const uint32_t half = n >> 1;
      base = (__ldg(a + base + half - 1) < low) ? base + half : base;
      n -= half;
    }
    return __ldg(a + base) == low;
  }

  // Finds the last run whose start is <= low, then tests its end.
  __device__ __forceinline__ bool run_contains(uint32_t byte_offset, uint16_t n_runs,
                                               uint16_t low) const
  {
    if (n_runs == 0) return false;
    const uint16_t* r = run_data + (byte_offset >> 1);
    if (low < __ldg(r)) return false;
    uint32_t n = n_runs, base = 0;   // invariant: start[base] <= low
    while (n > 1) {
      const uint32_t half = n >> 1;
      base = (__ldg(r + 2 * (base + half)) <= low) ? base + half : base;
      n -= half;
    }
    const uint32_t start = __ldg(r + 2 * base), len = __ldg(r + 2 * base + 1);
    return static_cast<uint32_t>(low) <= start + len;
  }
};

}  // namespace cu_roaring
