// cu_roaring B200 engine — public data model.
//
// Drop-in for the reference's include/cu_roaring/types.cuh:7-63. Field names,
// order and types are kept identical on purpose: existing user kernels and
// the cuVS roaring_filter adapter read these structs directly, so any change
// would break them at compile time (or silently, at the byte level).
//
// Layout produced by this engine (all pointers are device pointers inside one
// packed cudaMallocAsync block whose base is `_alloc_base`):
//   keys[n]          u16  high 16 bits of every container, strictly increasing
//   types[n]         u8   ContainerType
//   offsets[n]       u32  BYTE offset into the pool of the container's type
//   cardinalities[n] u16  ARRAY: element count; BITMAP: popcount (65536 -> 0);
//                         RUN: number of runs
//   key_index[max_key+1] u16 container index of each key, 0xFFFF if absent
//   bitmap_data      1024 x u64 per BITMAP container, slot i at byte 8192*i,
//                    slots assigned in key order (dense, no holes)
//   array_data       sorted u16 values, containers packed in key order
//   run_data         (start, length) u16 pairs; a run covers start..start+length
#pragma once
#include <cstddef>
#include <cstdint>

namespace cu_roaring {

enum class ContainerType : uint8_t {
    ARRAY  = 0,
    BITMAP = 1,
    RUN    = 2
};

struct GpuRoaring {
    uint16_t*      keys          = nullptr;
    ContainerType* types         = nullptr;
    uint32_t*      offsets       = nullptr;
    uint16_t*      cardinalities = nullptr;
    uint32_t       n_containers      = 0;
    uint32_t       universe_size     = 0;   // IDs live in [0, universe_size)
    uint64_t       total_cardinality = 0;   // cardinality of the LOGICAL set

    uint64_t* bitmap_data         = nullptr;
    uint32_t  n_bitmap_containers = 0;

    uint16_t* array_data          = nullptr;
    uint32_t  n_array_containers  = 0;
    uint32_t  array_pool_bytes    = 0;

    uint16_t* run_data            = nullptr;
    uint32_t  n_run_containers    = 0;
    uint32_t  run_pool_bytes      = 0;

    uint16_t* key_index           = nullptr;
    uint32_t  max_key             = 0;

    // When true the stored containers hold the complement of the logical set
    // within [0, universe_size).
    bool      negated             = false;

    // Base of the single packed device allocation (freed by gpu_roaring_free).
    void*     _alloc_base         = nullptr;
};

struct GpuRoaringMeta {
    uint32_t n_containers         = 0;
    uint32_t n_bitmap_containers  = 0;
    uint32_t n_array_containers   = 0;
    uint32_t n_run_containers     = 0;
    uint32_t universe_size        = 0;
    size_t   total_bytes          = 0;
};

}  // namespace cu_roaring
