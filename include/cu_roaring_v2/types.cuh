// cu_roaring B200 engine — batch types (drop-in for the reference
// v2/include/cu_roaring_v2/types.cuh). Field names, order and types are those
// of the reference, so kernels written against it compile unchanged.
//
// A batch packs N Roaring bitmaps into one device allocation, CSR style:
// containers of bitmap b are [container_starts[b], container_starts[b+1]) in
// the concatenated keys / types / offsets / cardinalities arrays; its
// direct-map key index is key_indices[key_index_starts[b] ..
// key_index_starts[b+1]) (max_key + 1 entries holding the LOCAL container
// index, 0xFFFF = absent); offsets are byte offsets into the pool of the
// container's type, shared by the batch. Cardinalities: ARRAY = members,
// BITMAP = popcount (65536 stored as 0), RUN = number of runs. No complement:
// every bitmap stores its members. Per-bitmap scalars are mirrored in host
// memory (readable without a device read).
#pragma once
#include <cstddef>
#include <cstdint>

namespace cu_roaring::v2 {

enum class ContainerType : uint8_t { ARRAY = 0, BITMAP = 1, RUN = 2 };

struct GpuRoaringBatch {
  uint32_t n_bitmaps = 0;
  uint32_t total_containers = 0;
  uint32_t n_bitmap_containers_total = 0;
  uint32_t array_pool_bytes = 0;
  uint32_t run_pool_bytes = 0;

  uint32_t* container_starts = nullptr;  // [n_bitmaps + 1]
  uint32_t* key_index_starts = nullptr;  // [n_bitmaps + 1]

  uint16_t* keys = nullptr;              // [total_containers]
  ContainerType* types = nullptr;
  uint32_t* offsets = nullptr;
  uint16_t* cardinalities = nullptr;

  uint16_t* key_indices = nullptr;       // concatenated per-bitmap key indices (local ids)

  uint64_t* bitmap_data = nullptr;
  uint16_t* array_data = nullptr;
  uint16_t* run_data = nullptr;

  // Host mirrors: total cardinality and universe ((max_key + 1) << 16) per
  // bitmap, the two CSR arrays, BITMAP-container count per bitmap.
  const uint64_t* host_total_cardinalities = nullptr;
  const uint32_t* host_universe_sizes = nullptr;
  const uint32_t* host_container_starts = nullptr;
  const uint32_t* host_key_index_starts = nullptr;
  const uint32_t* host_n_bitmap_containers = nullptr;

  void* _alloc_base = nullptr;      // the device block
  void* _host_meta_base = nullptr;  // the host mirrors
};

// One bitmap of a batch, by value into kernels (aliases the batch's memory).
struct GpuRoaringView {
  uint32_t n_containers = 0;
  uint32_t max_key = 0;

  uint16_t* keys = nullptr;
  ContainerType* types = nullptr;
  uint32_t* offsets = nullptr;
  uint16_t* cardinalities = nullptr;
  uint16_t* key_index = nullptr;

  uint64_t* bitmap_data = nullptr;
  uint16_t* array_data = nullptr;
  uint16_t* run_data = nullptr;
};

}  // namespace cu_roaring::v2
