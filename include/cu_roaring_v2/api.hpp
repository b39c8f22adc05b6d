// cu_roaring B200 engine — batch host API (drop-in for the reference
// v2/include/cu_roaring_v2/api.hpp). Inline shims over the C ABI; errors
// throw std::runtime_error. The reference builds a batch from CRoaring
// bitmaps (upload_batch), which this build cannot take (CRoaring is absent);
// upload_batch_portable takes the same bitmaps in the portable Roaring
// serialization that CRoaring writes.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>
#include <stdexcept>
#include <string>

#include "cu_roaring_b200.h"
#include "cu_roaring_v2/types.cuh"

namespace cu_roaring::v2 {
namespace detail {
static_assert(sizeof(GpuRoaringBatch) == sizeof(cr_roaring_batch), "batch layout");
inline cr_roaring_batch* c(GpuRoaringBatch& b) { return reinterpret_cast<cr_roaring_batch*>(&b); }
inline const cr_roaring_batch* c(const GpuRoaringBatch& b) { return reinterpret_cast<const cr_roaring_batch*>(&b); }
inline cr_stream_t s(cudaStream_t st) { return reinterpret_cast<cr_stream_t>(st); }
inline void check(int rc, const char* what)
{
  if (rc != CR_OK) throw std::runtime_error(std::string(what) + ": " + cr_last_error_string());
}
}  // namespace detail

inline GpuRoaringBatch upload_batch_portable(const void* const* buffers, const size_t* sizes, uint32_t n,
                                             cudaStream_t stream = 0)
{
  static_assert(sizeof(size_t) == sizeof(uint64_t), "64-bit sizes");
  GpuRoaringBatch out{};
  detail::check(cr_batch_upload_portable(buffers, reinterpret_cast<const uint64_t*>(sizes), n, detail::s(stream),
                                         detail::c(out)),
                "upload_batch_portable");
  return out;
}

inline void free_batch(GpuRoaringBatch& batch) { detail::check(cr_batch_free(detail::c(batch)), "free_batch"); }

inline GpuRoaringBatch promote_batch(const GpuRoaringBatch& batch, cudaStream_t stream = 0)
{
  GpuRoaringBatch out{};
  detail::check(cr_batch_promote(detail::c(batch), detail::s(stream), detail::c(out)), "promote_batch");
  return out;
}

// Host-only: the view of bitmap `b` (aliases the batch).
inline GpuRoaringView make_view(const GpuRoaringBatch& batch, uint32_t b)
{
  GpuRoaringView v{};
  if (b >= batch.n_bitmaps) throw std::runtime_error("make_view: bitmap index out of range");
  const uint32_t c0 = batch.host_container_starts[b], c1 = batch.host_container_starts[b + 1];
  const uint32_t k0 = batch.host_key_index_starts[b], k1 = batch.host_key_index_starts[b + 1];
  v.n_containers = c1 - c0;
  v.max_key = k1 > k0 ? k1 - k0 - 1 : 0;
  v.keys = batch.keys + c0;
  v.types = batch.types + c0;
  v.offsets = batch.offsets + c0;
  v.cardinalities = batch.cardinalities + c0;
  v.key_index = batch.key_indices + k0;
  v.bitmap_data = batch.bitmap_data;
  v.array_data = batch.array_data;
  v.run_data = batch.run_data;
  return v;
}

inline GpuRoaringBatch multi_and(const GpuRoaringBatch& batch, const uint32_t* input_indices, uint32_t n_inputs,
                                 cudaStream_t stream = 0)
{
  GpuRoaringBatch out{};
  detail::check(cr_batch_multi_and(detail::c(batch), input_indices, n_inputs, detail::s(stream), detail::c(out)),
                "multi_and");
  return out;
}

inline void decompress_batch(const GpuRoaringBatch& batch, uint64_t* device_bitsets, uint64_t words_each,
                             cudaStream_t stream = 0)
{
  detail::check(cr_batch_decompress(detail::c(batch), device_bitsets, words_each, detail::s(stream)),
                "decompress_batch");
}

}  // namespace cu_roaring::v2
