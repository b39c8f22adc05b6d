// cu_roaring B200 engine — flat bitset export (drop-in for the reference
// include/cu_roaring/detail/decompress.cuh:10-17).
#pragma once
#include "cu_roaring/detail/utils.cuh"

namespace cu_roaring {

// Allocates ceil(U/32) words; free with cudaFree.
inline uint32_t* decompress_to_bitset(const GpuRoaring& bitmap, cudaStream_t stream = 0)
{
  uint32_t* out = nullptr;
  detail::check(cr_decompress_to_bitset_alloc(detail::c(bitmap), detail::s(stream), &out),
                "decompress_to_bitset");
  return out;
}

inline void decompress_to_bitset(const GpuRoaring& bitmap, uint32_t* output,
                                 uint32_t output_size_words, cudaStream_t stream = 0)
{
  detail::check(cr_decompress_to_bitset(detail::c(bitmap), output, output_size_words,
                                        detail::s(stream)),
                "decompress_to_bitset");
}

}  // namespace cu_roaring
