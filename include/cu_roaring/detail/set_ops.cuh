// cu_roaring B200 engine — set algebra (drop-in for the reference
// include/cu_roaring/detail/set_ops.cuh:7-29).
#pragma once
#include "cu_roaring/detail/utils.cuh"

namespace cu_roaring {

enum class SetOp : uint8_t { AND = 0, OR = 1, ANDNOT = 2, XOR = 3 };

inline GpuRoaring set_operation(const GpuRoaring& a, const GpuRoaring& b, SetOp op,
                                cudaStream_t stream = 0)
{
  GpuRoaring out{};
  detail::check(cr_set_operation(detail::c(a), detail::c(b), static_cast<int>(op), detail::s(stream),
                                 detail::c(out)),
                "set_operation");
  return out;
}

inline GpuRoaring multi_and(const GpuRoaring* bitmaps, uint32_t count, cudaStream_t stream = 0)
{
  GpuRoaring out{};
  detail::check(cr_multi_and(reinterpret_cast<const cr_gpu_roaring*>(bitmaps), count,
                             detail::s(stream), detail::c(out)),
                "multi_and");
  return out;
}

inline GpuRoaring multi_or(const GpuRoaring* bitmaps, uint32_t count, cudaStream_t stream = 0)
{
  GpuRoaring out{};
  detail::check(cr_multi_or(reinterpret_cast<const cr_gpu_roaring*>(bitmaps), count,
                            detail::s(stream), detail::c(out)),
                "multi_or");
  return out;
}

}  // namespace cu_roaring
