// cu_roaring B200 engine — sample filter for graph-based ANN search.
//
// The reference describes (README.md:267-285) a cuVS `roaring_filter` built
// directly from a GpuRoaring and queried during CAGRA graph traversal with
// warp-cooperative lookups. That adapter lives in an external cuVS fork; this
// header provides the same shape for any traversal kernel: construct it on the
// host from a GpuRoaring (one line, no make_view), pass it by value into the
// kernel, and test candidate rows with it.
//
//   operator()(query_ix, sample_ix)  one row, one thread (the cuVS sample
//                                    filter signature; the query is ignored:
//                                    one filter serves every query)
//   warp_test(sample_ix)             one row per lane, all 32 lanes calling
//                                    (converged code), the warp-cooperative
//                                    lookup of warp_contains
//
// `id_offset` maps a shard's local row index to the bitmap's global ID space
// (row r of the shard is ID id_offset + r).
#pragma once
#include <cstdint>

#include "cu_roaring/device/make_view.cuh"
#include "cu_roaring/device/roaring_view.cuh"
#include "cu_roaring/device/roaring_warp_query.cuh"
#include "cu_roaring/types.cuh"

namespace cu_roaring {
namespace filtering {

struct roaring_filter {
  GpuRoaringView view;
  uint32_t id_offset;

  explicit roaring_filter(const GpuRoaring& bitmap, uint32_t offset = 0)
      : view(make_view(bitmap)), id_offset(offset)
  {
  }

  __device__ __forceinline__ bool operator()(uint32_t /*query_ix*/, uint32_t sample_ix) const
  {
    return view.contains(sample_ix + id_offset);
  }

  __device__ __forceinline__ bool warp_test(uint32_t sample_ix) const
  {
    return warp_contains(view, sample_ix + id_offset);
  }
};

}  // namespace filtering
}  // namespace cu_roaring
