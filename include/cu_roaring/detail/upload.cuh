// cu_roaring B200 engine — upload of CRoaring bitmaps, freeing, metadata
// (drop-in for the reference include/cu_roaring/detail/upload.cuh:19-41).
// The CRoaring-typed upload() / get_meta() overloads are compiled only when a
// CRoaring header is on the include path (__has_include(<roaring/roaring.h>));
// they hand the bitmap to the engine in its portable serialization, written
// by CRoaring's own public roaring_bitmap_portable_serialize.
#pragma once
#include <vector>

#include "cu_roaring/detail/promote.cuh"
#if __has_include(<roaring/roaring.h>)
#include <roaring/roaring.h>
#define CU_ROARING_HAS_CROARING 1
#endif

namespace cu_roaring {

inline void gpu_roaring_free(GpuRoaring& bitmap)
{
  detail::check(cr_gpu_roaring_free(detail::c(bitmap)), "gpu_roaring_free");
}

inline void gpu_roaring_free_async(GpuRoaring& bitmap, cudaStream_t stream)
{
  detail::check(cr_gpu_roaring_free_async(detail::c(bitmap), detail::s(stream)),
                "gpu_roaring_free_async");
}

// A bitmap in the portable Roaring serialization (the format other Roaring
// libraries write to disk), loaded straight into device memory: the
// replacement for the CRoaring-typed upload() path. No reference counterpart.
inline GpuRoaring upload_portable(const void* data, size_t n_bytes, uint32_t universe_size,
                                  cudaStream_t stream = 0, uint32_t bitmap_threshold = PROMOTE_AUTO)
{
  GpuRoaring out{};
  detail::check(cr_upload_portable(data, n_bytes, universe_size, detail::s(stream), bitmap_threshold,
                                   detail::c(out)),
                "upload_portable");
  return out;
}

#ifdef CU_ROARING_HAS_CROARING
namespace detail {
inline std::vector<char> portable_bytes(const roaring_bitmap_t* bm)
{
  std::vector<char> buf(roaring_bitmap_portable_size_in_bytes(bm));
  if (!buf.empty()) roaring_bitmap_portable_serialize(bm, buf.data());
  return buf;
}
inline cr_roaring_meta portable_meta(const std::vector<char>& buf)
{
  cr_roaring_meta m{};
  check(cr_portable_meta(buf.data(), buf.size(), &m), "get_meta");
  return m;
}
}  // namespace detail

// Universe inferred as (max key + 1) << 16 and the set stored as given, never
// complemented (reference src/upload.cpp:290-294). A bitmap whose max key is
// 65535 gets universe 2^32 - 1 (the reference's u32 arithmetic gives 0).
inline GpuRoaring upload(const roaring_bitmap_t* cpu_bitmap, cudaStream_t stream = 0,
                         uint32_t bitmap_threshold = PROMOTE_AUTO)
{
  const std::vector<char> buf = detail::portable_bytes(cpu_bitmap);
  const cr_roaring_meta m = detail::portable_meta(buf);
  GpuRoaring out{};
  if (m.n_containers == 0) return out;
  const uint32_t U = m.max_key == 65535u ? 0xFFFFFFFFu : m.universe_size;
  detail::check(cr_upload_portable_ex(buf.data(), buf.size(), U, detail::s(stream), bitmap_threshold,
                                      CR_PORTABLE_KEEP_UNCOMPLEMENTED, detail::c(out)),
                "upload");
  return out;
}

// Explicit universe: the complement is stored when more than half of it is
// set (reference src/upload.cpp:296-316).
inline GpuRoaring upload(const roaring_bitmap_t* cpu_bitmap, uint32_t universe_size, cudaStream_t stream = 0,
                         uint32_t bitmap_threshold = PROMOTE_AUTO)
{
  const std::vector<char> buf = detail::portable_bytes(cpu_bitmap);
  GpuRoaring out{};
  detail::check(cr_upload_portable(buf.data(), buf.size(), universe_size, detail::s(stream), bitmap_threshold,
                                   detail::c(out)),
                "upload");
  return out;
}

// Host-side counts of a CRoaring bitmap (reference src/upload.cpp:31-71).
inline GpuRoaringMeta get_meta(const roaring_bitmap_t* cpu_bitmap)
{
  const cr_roaring_meta m = detail::portable_meta(detail::portable_bytes(cpu_bitmap));
  GpuRoaringMeta out{};
  out.n_containers = m.n_containers;
  out.n_bitmap_containers = m.n_bitmap_containers;
  out.n_array_containers = m.n_array_containers;
  out.n_run_containers = m.n_run_containers;
  out.universe_size = m.universe_size;
  out.total_bytes = m.total_bytes;
  return out;
}
#endif  // CU_ROARING_HAS_CROARING

// Counts and device footprint of an uploaded bitmap (an addition: the
// reference's get_meta takes only the CRoaring bitmap).
inline GpuRoaringMeta get_meta(const GpuRoaring& b)
{
  GpuRoaringMeta m{};
  m.n_containers = b.n_containers;
  m.n_bitmap_containers = b.n_bitmap_containers;
  m.n_array_containers = b.n_array_containers;
  m.n_run_containers = b.n_run_containers;
  m.universe_size = b.universe_size;
  m.total_bytes = size_t(b.n_containers) * 9 + size_t(b.n_bitmap_containers) * 8192 +
                  b.array_pool_bytes + b.run_pool_bytes + (b.key_index ? (size_t(b.max_key) + 1) * 2 : 0);
  return m;
}

}  // namespace cu_roaring
