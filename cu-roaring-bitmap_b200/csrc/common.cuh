// cu_roaring B200 engine — shared host/device infrastructure.
//
// Error model: every C-ABI entry point returns a cr_status and records a
// message in a thread-local buffer (cr_last_error_string). Internally a
// CrError exception carries (status, message) up to the entry point, where
// CR_API_BEGIN/CR_API_END convert it; nothing throws across the C ABI.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include "cu_roaring_b200.h"

namespace crb {

constexpr uint32_t kChunkWords64 = 1024;   // u64 words per 65536-bit chunk
constexpr uint32_t kChunkWords32 = 2048;
constexpr uint32_t kBitmapBytes = 8192;
constexpr uint8_t kArray = 0, kBitmap = 1, kRun = 2;
constexpr uint32_t kPromoteKeep = 4096u, kPromoteAuto = 0xFFFFFFFFu;
constexpr uint32_t kNone = 0xFFFFFFFFu;

struct CrError {
  int status;
  std::string msg;
};

void set_last_error(const std::string& m);
[[noreturn]] void fail(int status, const std::string& m);
void check_cuda(cudaError_t e, const char* what, const char* file, int line);

#define CR_CUDA(call) ::crb::check_cuda((call), #call, __FILE__, __LINE__)
#define CR_REQUIRE(cond, msg)                                  \
  do {                                                         \
    if (!(cond)) ::crb::fail(CR_ERR_INVALID, (msg));           \
  } while (0)

#define CR_API_BEGIN try {
#define CR_API_END                                             \
  return CR_OK;                                                \
  }                                                            \
  catch (const ::crb::CrError& e) {                            \
    ::crb::set_last_error(e.msg);                              \
    return e.status;                                           \
  }                                                            \
  catch (const std::exception& e) {                            \
    ::crb::set_last_error(e.what());                           \
    return CR_ERR_INVALID;                                     \
  }

// ---------------------------------------------------------------- memory
void* dev_alloc(size_t bytes, cudaStream_t s);   // cudaMallocAsync, fails loudly
void dev_free(void* p, cudaStream_t s);

// RAII scratch that is released stream-ordered.
struct Scratch {
  void* p = nullptr;
  cudaStream_t s = nullptr;
  Scratch() = default;
  Scratch(size_t bytes, cudaStream_t st) : s(st) { p = bytes ? dev_alloc(bytes, st) : nullptr; }
  ~Scratch() { if (p) cudaFreeAsync(p, s); }
  Scratch(const Scratch&) = delete;
  Scratch& operator=(const Scratch&) = delete;
  template <class T> T* as() const { return static_cast<T*>(p); }
};

// Byte layout of the single packed block behind one GpuRoaring.
struct PackedLayout {
  size_t keys, types, offsets, cards, kidx, bitmap, array, run, total;
};
PackedLayout make_layout(uint32_t n, uint32_t kidx_len, uint32_t n_bitmap,
                         uint64_t array_bytes, uint64_t run_bytes);

// Allocates the packed block and points every field of `out` into it.
// Counts/sizes in `out` must be filled first; key_index gets max_key+1 entries.
void alloc_result(cr_gpu_roaring* out, cudaStream_t s);

inline uint32_t max_key_for(uint32_t U) { return U == 0 ? 0u : ((U - 1u) >> 16); }
inline uint32_t n_chunks_for(uint32_t U) { return static_cast<uint32_t>((uint64_t(U) + 65535u) >> 16); }
inline uint32_t div_up(uint64_t a, uint64_t b) { return static_cast<uint32_t>((a + b - 1) / b); }

void deep_copy(const cr_gpu_roaring* in, cr_gpu_roaring* out, cudaStream_t s);
void build_key_index(const uint16_t* keys, uint32_t n, uint16_t* kidx, uint32_t kidx_len,
                     cudaStream_t s);

int sm_count();
// Page-locked staging for the small device-to-host readbacks a call waits
// on (a pageable destination costs a staged copy). Per host thread, grown on
// demand; the contents are valid until this thread's next call of it.
void* pinned_stage(size_t bytes);
// Raises the dynamic shared memory limit of `fn` on the current device.
// Function attributes are per device, so every device a process launches on
// gets its own call; later calls on that device are free.
void set_max_dynamic_smem(const void* fn, int bytes);

// The fused filtered top-k of one shard (topk.cu), stream-ordered, and the
// merge of per-shard lists that sit at fixed strides (elements) apart.
void filtered_topk_enqueue(const uint16_t* d_db, const float* d_db_norms, uint64_t n_rows, uint32_t dim,
                           const uint16_t* d_queries, uint32_t n_queries, const cr_gpu_roaring* filter,
                           uint64_t row_offset, uint32_t k, int metric, float* d_out_dist, int64_t* d_out_ids,
                           cudaStream_t s);
void topk_merge_enqueue(const float* d_dist, const int64_t* d_ids, uint64_t dist_stride, uint64_t id_stride,
                        uint32_t n_parts, uint32_t n_queries, uint32_t k, int metric, float* d_out_dist,
                        int64_t* d_out_ids, cudaStream_t s);

// One container of a portable Roaring serialization (portable.cu).
enum : uint32_t { kPortableArray = 0, kPortableBitmap = 1, kPortableRun = 2 };
struct PortableContainer {
  uint64_t offset;  // byte offset of the payload in the serialized buffer
  uint32_t key;
  uint32_t kind;    // kPortableArray / kPortableBitmap / kPortableRun
  uint32_t count;   // ARRAY/BITMAP: cardinality; RUN: number of runs
  uint32_t card;    // declared cardinality
};
struct PortableImage {
  std::vector<PortableContainer> cs;
  uint64_t end = 0;  // bytes of the buffer the containers use
};
// Checks the header of a portable Roaring serialization and locates every
// container's payload (keys must lie below universe_size; 0 = any key).
// Errors are raised as CR_ERR_INVALID / CR_ERR_RANGE naming `who`.
PortableImage parse_portable(const void* data, uint64_t n_bytes, uint32_t universe_size, const char* who);

// Roaring image of a flat device bitset (upload.cu): canonical container
// types under `thr`, complement above half density, bits >= U ignored.
void upload_device_bitset(const uint32_t* d_words, uint64_t n_words, uint32_t U, uint32_t thr,
                          cudaStream_t s, cr_gpu_roaring* out, bool keep_uncomplemented = false);
uint64_t l2_bytes(int device);
uint32_t resolve_auto(uint32_t U, int device);

// The canonical container rule (prose in DESIGN and the oracle):
//   t < 4096: BITMAP if c > t else ARRAY;
//   else ARRAY if c <= 4096; RUN if r < 2048 and (c > t or 4r < 2c);
//   ARRAY if c <= t; else BITMAP.
__host__ __device__ __forceinline__ uint8_t container_type(uint32_t c, uint32_t r, uint32_t t)
{
  if (t < kPromoteKeep) return c > t ? kBitmap : kArray;
  if (c <= kPromoteKeep) return kArray;
  if (r < 2048u && (c > t || 4ull * r < 2ull * c)) return kRun;
  if (c <= t) return kArray;
  return kBitmap;
}

__host__ __device__ __forceinline__ uint32_t chunk_valid_bits(uint32_t key, uint32_t U)
{
  const uint64_t lo = uint64_t(key) << 16;
  if (lo >= U) return 0;
  const uint64_t rem = uint64_t(U) - lo;
  return rem >= 65536u ? 65536u : static_cast<uint32_t>(rem);
}

// Mask of the valid bits of u64 word `w` (0..1023) of a chunk with `valid` bits.
__host__ __device__ __forceinline__ uint64_t word_mask(uint32_t w, uint32_t valid)
{
  const uint32_t lo = w * 64u;
  if (lo >= valid) return 0ull;
  const uint32_t n = valid - lo;
  return n >= 64u ? ~0ull : ((1ull << n) - 1ull);
}

// Device-side view of one operand (all pointers device-resident).
struct DevBitmap {
  const uint16_t* keys;
  const uint8_t* types;
  const uint32_t* offsets;
  const uint16_t* cards;
  const uint64_t* bitmap;
  const uint16_t* array;
  const uint16_t* run;
  const uint16_t* key_index;  // never null inside the engine (temp index built)
  uint32_t n;
  uint32_t max_key;
  uint32_t universe;
  uint32_t negated;
};

// Device view of an operand. When the operand has no key_index (a GpuRoaring
// assembled by other code) a full 65536-entry index is built into `holder`.
DevBitmap make_dev(const cr_gpu_roaring* b, Scratch& holder, cudaStream_t s);

// Optional CUDA-event bracketing of the dominant kernels (cr_profile_enable).
struct ProfileScope {
  int kind;
  cudaStream_t s;
  bool on;
  ProfileScope(int k, cudaStream_t st);
  ~ProfileScope();
};

// ------------------------------------------------------- block primitives
// Exclusive scan over a block of BLOCK threads (multiple of 32). Returns the
// exclusive prefix; *total gets the block sum. `smem` holds BLOCK/32 values.
template <int BLOCK, class T>
__device__ __forceinline__ T block_exclusive_scan(T v, T* smem, T* total)
{
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  T x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    T y = __shfl_up_sync(0xFFFFFFFFu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) smem[warp] = x;
  __syncthreads();
  if (warp == 0) {
    T s = lane < BLOCK / 32 ? smem[lane] : T(0);
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      T y = __shfl_up_sync(0xFFFFFFFFu, s, o);
      if (lane >= o) s += y;
    }
    if (lane < BLOCK / 32) smem[lane] = s;
  }
  __syncthreads();
  const T warp_base = warp ? smem[warp - 1] : T(0);
  *total = smem[BLOCK / 32 - 1];
  __syncthreads();
  return warp_base + x - v;
}

template <int BLOCK, class T>
__device__ __forceinline__ T block_sum(T v, T* smem)
{
  T total;
  block_exclusive_scan<BLOCK, T>(v, smem, &total);
  return total;
}

}  // namespace crb
