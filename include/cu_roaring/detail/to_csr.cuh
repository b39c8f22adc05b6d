// cu_roaring B200 engine — sorted ID export (drop-in for the reference
// include/cu_roaring/detail/to_csr.cuh:35-46), negation-aware; the uint32_t
// overload is an addition.
#pragma once
#include "cu_roaring/detail/utils.cuh"

namespace cu_roaring {

inline void enumerate_ids(const GpuRoaring& bitmap, int64_t* output, cudaStream_t stream = 0)
{
  detail::check(cr_enumerate_ids_i64(detail::c(bitmap), output, detail::s(stream)), "enumerate_ids");
}

inline void enumerate_ids(const GpuRoaring& bitmap, uint32_t* output, cudaStream_t stream = 0)
{
  detail::check(cr_enumerate_ids_u32(detail::c(bitmap), output, detail::s(stream)), "enumerate_ids");
}

// Allocates total_cardinality int64 values; free with cudaFree.
inline int64_t* enumerate_ids(const GpuRoaring& bitmap, cudaStream_t stream = 0)
{
  int64_t* out = nullptr;
  detail::check(cr_enumerate_ids_alloc(detail::c(bitmap), detail::s(stream), &out), "enumerate_ids");
  return out;
}

}  // namespace cu_roaring
