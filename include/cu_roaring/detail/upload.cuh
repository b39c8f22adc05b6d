// cu_roaring B200 engine — freeing (drop-in for the reference
// include/cu_roaring/detail/upload.cuh:34-41). The CRoaring-typed upload()
// overloads (:19-33) exist only when a CRoaring header is available; they
// would serialise the CRoaring bitmap's members, which this build cannot
// test because CRoaring is absent.
#pragma once
#include "cu_roaring/detail/promote.cuh"

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
