// cu_roaring B200 engine — warp-cooperative point query.
//
// Drop-in for include/cu_roaring/device/roaring_warp_query.cuh:16-78 of the
// reference (same name and signature). Lanes whose IDs share a high-16 key
// elect one leader (__match_any_sync); only the leader resolves the key and
// reads the container metadata, which it broadcasts with __shfl_sync. Every
// lane then reads its own payload word / searches its own container.
//
// Warp-synchronous: call it from converged code. In a kernel with a bounds
// check, let every lane call it (out-of-range lanes on any valid ID, result
// discarded) instead of calling it inside `if (i < n)`: __activemask() does
// not guarantee that the lanes it reports execute the following *_sync
// intrinsics together, and on sm_100 a mismatch raises an illegal
// instruction.
#pragma once
#include "roaring_view.cuh"

namespace cu_roaring {

__device__ __forceinline__ bool warp_contains(const GpuRoaringView& r, uint32_t id)
{
  const uint32_t key    = id >> 16;
  const uint16_t low    = static_cast<uint16_t>(id & 0xFFFFu);
  const unsigned active = __activemask();
  const unsigned peers  = __match_any_sync(active, key);
  const int leader      = __ffs(peers) - 1;
  const bool i_lead     = (static_cast<int>(threadIdx.x & 31u) == leader);

  // Leader packs (container index | type << 16) and (offset) and (card).
  int idx = -1;
  uint32_t meta_off = 0, meta_tc = 0;
  if (i_lead) {
    if (r.all_bitmap) {
      if (key <= r.max_key) {
        const uint16_t k = __ldg(r.key_index + key);
        idx = (k == 0xFFFFu) ? -1 : static_cast<int>(k);
      }
    } else {
      idx = r.lookup_key(static_cast<uint16_t>(key));
      if (idx >= 0) {
        meta_off = r.load_offset(idx);
        meta_tc  = static_cast<uint32_t>(r.load_type(idx)) |
                   (static_cast<uint32_t>(r.load_cardinality(idx)) << 8);
      }
    }
  }
  // Every lane of `active` takes part in all three broadcasts before any
  // lane branches on the result: a __shfl_sync whose mask names a lane that
  // has already returned is undefined (it faults on sm_100).
  idx      = __shfl_sync(active, idx, leader);
  meta_off = __shfl_sync(active, meta_off, leader);
  meta_tc  = __shfl_sync(active, meta_tc, leader);
  if (idx < 0) return r.negated;
  if (r.all_bitmap) {
    const uint64_t w = __ldg(r.bitmap_data + (static_cast<size_t>(idx) << 10) + (low >> 6));
    return static_cast<bool>((w >> (low & 63u)) & 1u) != r.negated;
  }
  const bool hit = r.contains_in(static_cast<ContainerTypeD>(meta_tc & 0xFFu), meta_off,
                                 static_cast<uint16_t>(meta_tc >> 8), low);
  return hit != r.negated;
}

}  // namespace cu_roaring
