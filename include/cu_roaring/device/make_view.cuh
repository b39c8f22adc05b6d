// cu_roaring B200 engine — host-side view construction.
//
// Drop-in for include/cu_roaring/device/make_view.cuh:9-27 of the reference.
// all_bitmap (the two-load fast path) is enabled when there are no ARRAY/RUN
// containers and key_index exists; this engine always stores BITMAP container
// i at bitmap slot i in that case, which the fast path relies on.
#pragma once
#include "cu_roaring/device/roaring_view.cuh"
#include "cu_roaring/types.cuh"

namespace cu_roaring {

inline GpuRoaringView make_view(const GpuRoaring& bitmap)
{
  GpuRoaringView v{};
  v.keys          = bitmap.keys;
  v.types         = reinterpret_cast<const ContainerTypeD*>(bitmap.types);
  v.offsets       = bitmap.offsets;
  v.cardinalities = bitmap.cardinalities;
  v.n_containers  = bitmap.n_containers;
  v.bitmap_data   = bitmap.bitmap_data;
  v.array_data    = bitmap.array_data;
  v.run_data      = bitmap.run_data;
  v.key_index     = bitmap.key_index;
  v.max_key       = bitmap.max_key;
  v.all_bitmap    = bitmap.n_array_containers == 0 && bitmap.n_run_containers == 0 &&
                    bitmap.key_index != nullptr && bitmap.n_containers > 0;
  v.negated       = bitmap.negated;
  return v;
}

}  // namespace cu_roaring
