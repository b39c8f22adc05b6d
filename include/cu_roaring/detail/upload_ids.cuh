// cu_roaring B200 engine — construction from IDs / bitsets (drop-in for the
// reference include/cu_roaring/detail/upload_ids.cuh:19-56). The bitset
// overloads gain a trailing, defaulted bitmap_threshold.
#pragma once
#include "cu_roaring/detail/promote.cuh"

namespace cu_roaring {

inline GpuRoaring upload_from_ids(const uint32_t* ids, uint32_t n_ids, uint32_t universe_size,
                                  cudaStream_t stream = 0, uint32_t bitmap_threshold = PROMOTE_AUTO)
{
  GpuRoaring out{};
  detail::check(cr_upload_from_ids(ids, n_ids, universe_size, detail::s(stream), bitmap_threshold,
                                   detail::c(out)),
                "upload_from_ids");
  return out;
}

inline GpuRoaring upload_from_sorted_ids(const uint32_t* ids, uint32_t n_ids, uint32_t universe_size,
                                         cudaStream_t stream = 0,
                                         uint32_t bitmap_threshold = PROMOTE_AUTO)
{
  return upload_from_ids(ids, n_ids, universe_size, stream, bitmap_threshold);
}

// Device-resident IDs (addition; no host copy).
inline GpuRoaring upload_from_device_ids(const uint32_t* d_ids, uint64_t n_ids, uint32_t universe_size,
                                         cudaStream_t stream = 0,
                                         uint32_t bitmap_threshold = PROMOTE_AUTO)
{
  GpuRoaring out{};
  detail::check(cr_upload_from_device_ids(d_ids, n_ids, universe_size, detail::s(stream),
                                          bitmap_threshold, detail::c(out)),
                "upload_from_device_ids");
  return out;
}

inline GpuRoaring upload_from_bitset(const uint32_t* host_bitset, uint32_t n_words,
                                     uint32_t universe_size, cudaStream_t stream = 0,
                                     uint32_t bitmap_threshold = PROMOTE_AUTO)
{
  GpuRoaring out{};
  detail::check(cr_upload_from_bitset(host_bitset, n_words, universe_size, detail::s(stream),
                                      bitmap_threshold, detail::c(out)),
                "upload_from_bitset");
  return out;
}

inline GpuRoaring upload_from_device_bitset(const uint32_t* d_bitset, uint32_t n_words,
                                            uint32_t universe_size, cudaStream_t stream = 0,
                                            uint32_t bitmap_threshold = PROMOTE_AUTO)
{
  GpuRoaring out{};
  detail::check(cr_upload_from_device_bitset(d_bitset, n_words, universe_size, detail::s(stream),
                                             bitmap_threshold, detail::c(out)),
                "upload_from_device_bitset");
  return out;
}

}  // namespace cu_roaring
