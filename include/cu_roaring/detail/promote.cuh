// cu_roaring B200 engine — promotion policy (drop-in for the reference
// include/cu_roaring/detail/promote.cuh:38-83; same names and defaults).
#pragma once
#include "cu_roaring/detail/utils.cuh"

namespace cu_roaring {

// Threshold N: containers with cardinality > N become BITMAP.
static constexpr uint32_t PROMOTE_KEEP_DEFAULT = 4096;        // Roaring's own cut-off
static constexpr uint32_t PROMOTE_ALL          = 0;           // every container BITMAP
static constexpr uint32_t PROMOTE_AUTO         = UINT32_MAX;  // decided against the L2 size

inline GpuRoaring promote_to_bitmap(const GpuRoaring& bm, cudaStream_t stream = 0)
{
  GpuRoaring out{};
  detail::check(cr_promote_to_bitmap(detail::c(bm), detail::s(stream), detail::c(out)),
                "promote_to_bitmap");
  return out;
}

inline GpuRoaring promote_auto(const GpuRoaring& bm, cudaStream_t stream = 0, int device_id = -1)
{
  GpuRoaring out{};
  detail::check(cr_promote_auto(detail::c(bm), detail::s(stream), device_id, detail::c(out)),
                "promote_auto");
  return out;
}

inline uint32_t resolve_auto_threshold(uint32_t universe_size, int device_id = -1)
{
  uint32_t t = 0;
  detail::check(cr_resolve_auto_threshold(universe_size, device_id, &t), "resolve_auto_threshold");
  return t;
}

inline GpuRoaring gpu_roaring_deep_copy(const GpuRoaring& bm, cudaStream_t stream = 0)
{
  GpuRoaring out{};
  detail::check(cr_deep_copy(detail::c(bm), detail::s(stream), detail::c(out)), "gpu_roaring_deep_copy");
  return out;
}

}  // namespace cu_roaring
