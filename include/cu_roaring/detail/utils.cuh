// cu_roaring B200 engine — error convention of the C++ API.
// Drop-in for the reference include/cu_roaring/detail/utils.cuh:9-21: CUDA and
// library failures surface as std::runtime_error.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>
#include <stdexcept>
#include <string>

#include "cu_roaring_b200.h"
#include "cu_roaring/types.cuh"

namespace cu_roaring {

#ifndef CUDA_CHECK
#define CUDA_CHECK(call)                                                              \
  do {                                                                                \
    cudaError_t cr_err_ = (call);                                                     \
    if (cr_err_ != cudaSuccess)                                                       \
      throw std::runtime_error(std::string("CUDA error at ") + __FILE__ + ":" +       \
                               std::to_string(__LINE__) + ": " +                      \
                               cudaGetErrorString(cr_err_));                          \
  } while (0)
#endif

inline __host__ __device__ uint32_t div_ceil(uint32_t a, uint32_t b) { return (a + b - 1) / b; }

namespace detail {

static_assert(sizeof(GpuRoaring) == sizeof(cr_gpu_roaring), "GpuRoaring must match the C ABI");

// Converts a C-ABI status into the reference's exception convention.
inline void check(int rc, const char* what)
{
  if (rc != CR_OK)
    throw std::runtime_error(std::string(what) + ": " + cr_last_error_string());
}

inline cr_gpu_roaring* c(GpuRoaring& b) { return reinterpret_cast<cr_gpu_roaring*>(&b); }
inline const cr_gpu_roaring* c(const GpuRoaring& b)
{
  return reinterpret_cast<const cr_gpu_roaring*>(&b);
}
inline cr_stream_t s(cudaStream_t st) { return reinterpret_cast<cr_stream_t>(st); }

}  // namespace detail
}  // namespace cu_roaring
