// Test-only C entry points over the REFERENCE's own CUDA implementation
// (maxwbuckley/cu-roaring-bitmap src/upload_ids.cu, promote.cu, set_ops.cu,
// decompress.cu, to_csr.cu, compiled unmodified where they lie by
// oracle/build_ref.py into oracle/_ref/libref_cu_roaring.so).
//
// TEST INFRASTRUCTURE ONLY: tests use it to pin this engine's results to
// the reference's on the same inputs. The reference's CRoaring-based
// upload.cpp is not built (CRoaring is absent); its two free functions, which
// set_ops.cu calls, are restated here from their documented behaviour
// (reference src/upload.cpp:318-350: free the packed block if `_alloc_base`
// is set, else every pool pointer).
#include <cuda_runtime.h>

#include <cstring>
#include <stdexcept>
#include <string>

#include "cu_roaring/types.cuh"
#include "cu_roaring/detail/decompress.cuh"
#include "cu_roaring/detail/promote.cuh"
#include "cu_roaring/detail/set_ops.cuh"
#include "cu_roaring/detail/to_csr.cuh"
#include "cu_roaring/detail/upload_ids.cuh"

namespace cu_roaring {

void gpu_roaring_free(GpuRoaring& b)
{
  if (b._alloc_base) {
    cudaFree(b._alloc_base);
  } else {
    void* ptrs[] = {b.keys, b.types, b.offsets, b.cardinalities, b.bitmap_data, b.array_data,
                    b.run_data, b.key_index};
    for (void* p : ptrs)
      if (p) cudaFree(p);
  }
  b = GpuRoaring{};
}

void gpu_roaring_free_async(GpuRoaring& b, cudaStream_t s)
{
  if (b._alloc_base) {
    cudaFreeAsync(b._alloc_base, s);
  } else {
    void* ptrs[] = {b.keys, b.types, b.offsets, b.cardinalities, b.bitmap_data, b.array_data,
                    b.run_data, b.key_index};
    for (void* p : ptrs)
      if (p) cudaFreeAsync(p, s);
  }
  b = GpuRoaring{};
}

}  // namespace cu_roaring

using namespace cu_roaring;

static thread_local std::string g_err;

#define REF_TRY(body)                   \
  try {                                 \
    body;                               \
    return 0;                           \
  } catch (const std::exception& e) {   \
    g_err = e.what();                   \
    return -1;                          \
  }

extern "C" {

const char* ref_last_error() { return g_err.c_str(); }

int ref_upload_from_ids(const uint32_t* host_ids, uint32_t n, uint32_t U, uint32_t thr, GpuRoaring* out)
{
  REF_TRY(*out = upload_from_ids(host_ids, n, U, 0, thr))
}

int ref_upload_from_bitset(const uint32_t* host_words, uint32_t n_words, uint32_t U, GpuRoaring* out)
{
  REF_TRY(*out = upload_from_bitset(host_words, n_words, U, 0))
}

int ref_set_operation(const GpuRoaring* a, const GpuRoaring* b, int op, GpuRoaring* out)
{
  REF_TRY(*out = set_operation(*a, *b, static_cast<SetOp>(op), 0))
}

int ref_multi_and(const GpuRoaring* in, uint32_t count, GpuRoaring* out)
{
  REF_TRY(*out = multi_and(in, count, 0))
}

int ref_multi_or(const GpuRoaring* in, uint32_t count, GpuRoaring* out)
{
  REF_TRY(*out = multi_or(in, count, 0))
}

int ref_promote_to_bitmap(const GpuRoaring* in, GpuRoaring* out)
{
  REF_TRY(*out = promote_to_bitmap(*in, 0); cudaStreamSynchronize(0))
}

int ref_decompress(const GpuRoaring* in, uint32_t* host_out, uint32_t n_words)
{
  REF_TRY({
    uint32_t* d = nullptr;
    if (cudaMalloc(&d, size_t(n_words) * 4) != cudaSuccess) throw std::runtime_error("cudaMalloc");
    decompress_to_bitset(*in, d, n_words, 0);
    cudaMemcpy(host_out, d, size_t(n_words) * 4, cudaMemcpyDeviceToHost);
    cudaFree(d);
  })
}

int ref_enumerate(const GpuRoaring* in, int64_t* host_out)
{
  REF_TRY({
    const uint64_t n = in->total_cardinality;
    int64_t* d = nullptr;
    if (n && cudaMalloc(&d, n * 8) != cudaSuccess) throw std::runtime_error("cudaMalloc");
    if (n) enumerate_ids(*in, d, 0);
    cudaDeviceSynchronize();
    if (n) cudaMemcpy(host_out, d, n * 8, cudaMemcpyDeviceToHost);
    if (d) cudaFree(d);
  })
}

int ref_free(GpuRoaring* b) { REF_TRY(gpu_roaring_free(*b)) }

uint32_t ref_resolve_auto_threshold(uint32_t U) { return resolve_auto_threshold(U, -1); }

}  // extern "C"
