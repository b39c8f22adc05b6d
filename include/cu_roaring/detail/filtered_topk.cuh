// cu_roaring B200 engine — fused filtered brute-force top-k (no reference
// counterpart: the reference only describes the cuVS pipeline,
// README.md:265-285).
#pragma once
#include <cuda_fp16.h>

#include "cu_roaring/detail/utils.cuh"

namespace cu_roaring {

enum class Metric : int { InnerProduct = CR_METRIC_IP, L2 = CR_METRIC_L2 };

// filter == nullptr searches every row.
inline void filtered_topk(const __half* db, const float* db_norms, uint64_t n_rows, uint32_t dim,
                          const __half* queries, uint32_t n_queries, const GpuRoaring* filter,
                          uint32_t k, Metric metric, float* out_dist, int64_t* out_ids,
                          cudaStream_t stream = 0, uint64_t row_offset = 0)
{
  detail::check(cr_filtered_topk(reinterpret_cast<const uint16_t*>(db), db_norms, n_rows, dim,
                                 reinterpret_cast<const uint16_t*>(queries), n_queries,
                                 filter ? detail::c(*filter) : nullptr, row_offset, k,
                                 static_cast<int>(metric), out_dist, out_ids, detail::s(stream)),
                "filtered_topk");
}

// Row-sharded search over several GPUs, one process per GPU: each rank passes
// its own rows (row_offset = global ID of its first row); `root` receives the
// merged top-k. The communicator comes from cr_topk_comm_init.
inline void filtered_topk_sharded(cr_topk_comm comm, int root, const __half* db, const float* db_norms,
                                  uint64_t shard_rows, uint32_t dim, const __half* queries, uint32_t n_queries,
                                  const GpuRoaring* filter, uint64_t row_offset, uint32_t k, Metric metric,
                                  float* out_dist, int64_t* out_ids, cudaStream_t stream = 0)
{
  detail::check(cr_filtered_topk_sharded(comm, root, reinterpret_cast<const uint16_t*>(db), db_norms, shard_rows,
                                         dim, reinterpret_cast<const uint16_t*>(queries), n_queries,
                                         filter ? detail::c(*filter) : nullptr, row_offset, k,
                                         static_cast<int>(metric), out_dist, out_ids, detail::s(stream)),
                "filtered_topk_sharded");
}

}  // namespace cu_roaring
