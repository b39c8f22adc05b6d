// cu_roaring B200 engine — errors, packed allocation, device queries, free,
// deep copy, threshold resolution.
#include <algorithm>
#include <atomic>
#include <map>
#include <mutex>
#include <vector>


#include "common.cuh"

namespace crb {

static thread_local std::string g_last_error;

void set_last_error(const std::string& m) { g_last_error = m; }

void fail(int status, const std::string& m) { throw CrError{status, m}; }

void check_cuda(cudaError_t e, const char* what, const char* file, int line)
{
  if (e == cudaSuccess) return;
  const int st = (e == cudaErrorMemoryAllocation) ? CR_ERR_OOM : CR_ERR_CUDA;
  fail(st, std::string("CUDA error ") + cudaGetErrorString(e) + " in " + what + " at " + file +
               ":" + std::to_string(line));
}

// The stream-ordered allocator's default pool hands memory back to the driver
// at every synchronisation (release threshold 0), which makes each call that
// takes scratch re-map it. Keep freed memory cached in this process's pool
// instead (once per device; the setting belongs to the process, not the GPU).
static void keep_pool_memory()
{
  static std::mutex mu;
  static bool done[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) { cudaGetLastError(); return; }
  std::lock_guard<std::mutex> lock(mu);
  if (done[dev]) return;
  done[dev] = true;
  cudaMemPool_t pool;
  if (cudaDeviceGetDefaultMemPool(&pool, dev) == cudaSuccess) {
    uint64_t keep = ~0ull;
    cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
  }
  cudaGetLastError();
}

// Allocation-failure injection for tests (cr_test_fail_allocations): the
// number of device allocations still allowed to succeed, -1 = no injection.
static std::atomic<int64_t> g_allocs_left{-1};

void* dev_alloc(size_t bytes, cudaStream_t s)
{
  void* p = nullptr;
  if (bytes == 0) return nullptr;
  for (int64_t left = g_allocs_left.load(); left >= 0;) {
    if (left == 0) fail(CR_ERR_OOM, "cudaMallocAsync(" + std::to_string(bytes) + " bytes) failed: injected failure");
    if (g_allocs_left.compare_exchange_weak(left, left - 1)) break;
  }
  keep_pool_memory();
  const cudaError_t e = cudaMallocAsync(&p, bytes, s);
  if (e != cudaSuccess) {
    cudaGetLastError();
    fail(e == cudaErrorMemoryAllocation ? CR_ERR_OOM : CR_ERR_CUDA,
         "cudaMallocAsync(" + std::to_string(bytes) + " bytes) failed: " + cudaGetErrorString(e));
  }
  return p;
}

void dev_free(void* p, cudaStream_t s)
{
  if (p) CR_CUDA(cudaFreeAsync(p, s));
}

static size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

PackedLayout make_layout(uint32_t n, uint32_t kidx_len, uint32_t n_bitmap, uint64_t array_bytes,
                         uint64_t run_bytes)
{
  PackedLayout L{};
  size_t off = 0;
  L.bitmap = off;  off = align_up(off + size_t(n_bitmap) * kBitmapBytes, 256);
  L.keys = off;    off = align_up(off + size_t(n) * 2, 16);
  L.types = off;   off = align_up(off + size_t(n), 16);
  L.offsets = off; off = align_up(off + size_t(n) * 4, 16);
  L.cards = off;   off = align_up(off + size_t(n) * 2, 16);
  L.kidx = off;    off = align_up(off + size_t(kidx_len) * 2, 16);
  L.array = off;   off = align_up(off + array_bytes, 16);
  L.run = off;     off = align_up(off + run_bytes, 16);
  L.total = off ? off : 16;
  return L;
}

void alloc_result(cr_gpu_roaring* out, cudaStream_t s)
{
  if (out->array_pool_bytes > 0xFFFFFFFFull || out->run_pool_bytes > 0xFFFFFFFFull)
    fail(CR_ERR_UNSUPPORTED, "pool exceeds 4 GiB");
  const uint32_t kidx_len = out->max_key + 1u;
  const PackedLayout L = make_layout(out->n_containers, kidx_len, out->n_bitmap_containers,
                                     out->array_pool_bytes, out->run_pool_bytes);
  char* base = static_cast<char*>(dev_alloc(L.total, s));
  out->_alloc_base = base;
  out->keys = reinterpret_cast<uint16_t*>(base + L.keys);
  out->types = reinterpret_cast<uint8_t*>(base + L.types);
  out->offsets = reinterpret_cast<uint32_t*>(base + L.offsets);
  out->cardinalities = reinterpret_cast<uint16_t*>(base + L.cards);
  out->key_index = reinterpret_cast<uint16_t*>(base + L.kidx);
  out->bitmap_data = out->n_bitmap_containers ? reinterpret_cast<uint64_t*>(base + L.bitmap) : nullptr;
  out->array_data = out->array_pool_bytes ? reinterpret_cast<uint16_t*>(base + L.array) : nullptr;
  out->run_data = out->run_pool_bytes ? reinterpret_cast<uint16_t*>(base + L.run) : nullptr;
}

void* pinned_stage(size_t bytes)
{
  struct Stage {
    void* p = nullptr;
    size_t cap = 0;
    ~Stage() { if (p) cudaFreeHost(p); }
  };
  thread_local Stage st;
  if (bytes > st.cap) {
    if (st.p) CR_CUDA(cudaFreeHost(st.p));  // every earlier readback has been waited for
    st.p = nullptr;
    st.cap = 0;
    const size_t cap = std::max<size_t>(bytes, 4096);
    CR_CUDA(cudaHostAlloc(&st.p, cap, cudaHostAllocPortable));
    st.cap = cap;
  }
  return st.p;
}

int sm_count()
{
  static int cached[64] = {0};
  int dev = 0;
  CR_CUDA(cudaGetDevice(&dev));
  if (dev < 64 && cached[dev]) return cached[dev];
  int n = 0;
  CR_CUDA(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
  if (dev < 64) cached[dev] = n;
  return n;
}

void set_max_dynamic_smem(const void* fn, int bytes)
{
  static std::mutex mu;
  static std::map<std::pair<int, const void*>, int> done;
  int dev = 0;
  CR_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(mu);
  int& have = done[{dev, fn}];
  if (have >= bytes) return;
  CR_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  have = bytes;
}

uint64_t l2_bytes(int device)
{
  int dev = device;
  if (dev < 0 && cudaGetDevice(&dev) != cudaSuccess) dev = 0;
  int l2 = 0;
  if (cudaDeviceGetAttribute(&l2, cudaDevAttrL2CacheSize, dev) != cudaSuccess || l2 <= 0) {
    cudaGetLastError();
    l2 = 4 << 20;  // conservative fallback, as the reference does
  }
  return static_cast<uint64_t>(l2);
}

// Reference src/promote.cu:334-367: PROMOTE_ALL iff 2 * ceil(U/8) > L2.
uint32_t resolve_auto(uint32_t U, int device)
{
  if (U == 0) return kPromoteKeep;
  const uint64_t flat = (uint64_t(U) + 7u) / 8u;
  return flat * 2u > l2_bytes(device) ? 0u : kPromoteKeep;
}

static void copy_field(void* dst, const void* src, size_t bytes, cudaStream_t s)
{
  if (bytes && src) CR_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, s));
}

// Deep copy into one packed block (reference src/promote.cu:173-236).
void deep_copy(const cr_gpu_roaring* in, cr_gpu_roaring* out, cudaStream_t s)
{
  cr_gpu_roaring r = *in;
  r.keys = nullptr; r.types = nullptr; r.offsets = nullptr; r.cardinalities = nullptr;
  r.bitmap_data = nullptr; r.array_data = nullptr; r.run_data = nullptr;
  r.key_index = nullptr; r._alloc_base = nullptr;
  if (in->n_containers == 0) { *out = r; return; }
  const bool has_index = in->key_index != nullptr;
  r.max_key = has_index ? in->max_key : max_key_for(in->universe_size);
  alloc_result(&r, s);
  const uint32_t n = in->n_containers;
  copy_field(r.keys, in->keys, n * 2u, s);
  copy_field(r.types, in->types, n, s);
  copy_field(r.offsets, in->offsets, n * 4u, s);
  copy_field(r.cardinalities, in->cardinalities, n * 2u, s);
  copy_field(r.bitmap_data, in->bitmap_data, size_t(in->n_bitmap_containers) * kBitmapBytes, s);
  copy_field(r.array_data, in->array_data, in->array_pool_bytes, s);
  copy_field(r.run_data, in->run_data, in->run_pool_bytes, s);
  if (has_index) {
    copy_field(r.key_index, in->key_index, (size_t(in->max_key) + 1u) * 2u, s);
  } else {
    build_key_index(r.keys, n, r.key_index, r.max_key + 1u, s);
  }
  *out = r;
}

__global__ void k_scatter_key_index(const uint16_t* keys, uint32_t n, uint16_t* kidx,
                                    uint32_t kidx_len)
{
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n && keys[i] < kidx_len) kidx[keys[i]] = static_cast<uint16_t>(i);
}

void build_key_index(const uint16_t* keys, uint32_t n, uint16_t* kidx, uint32_t kidx_len,
                     cudaStream_t s)
{
  CR_CUDA(cudaMemsetAsync(kidx, 0xFF, size_t(kidx_len) * 2u, s));
  if (n) k_scatter_key_index<<<div_up(n, 256), 256, 0, s>>>(keys, n, kidx, kidx_len);
  CR_CUDA(cudaGetLastError());
}

DevBitmap make_dev(const cr_gpu_roaring* b, Scratch& holder, cudaStream_t s)
{
  DevBitmap d{};
  d.keys = b->keys;
  d.types = b->types;
  d.offsets = b->offsets;
  d.cards = b->cardinalities;
  d.bitmap = b->bitmap_data;
  d.array = b->array_data;
  d.run = b->run_data;
  d.n = b->n_containers;
  d.universe = b->universe_size;
  d.negated = b->negated ? 1u : 0u;
  d.key_index = b->key_index;
  d.max_key = b->max_key;
  if (b->n_containers > 0 && b->key_index == nullptr) {
    void* p = dev_alloc(65536 * 2, s);
    holder.p = p;
    holder.s = s;
    build_key_index(b->keys, b->n_containers, static_cast<uint16_t*>(p), 65536, s);
    d.key_index = static_cast<uint16_t*>(p);
    d.max_key = 65535;
  }
  if (b->n_containers == 0) d.max_key = 0, d.key_index = nullptr;
  return d;
}

namespace {
constexpr int kProfileKinds = 8;
bool g_profile = false;
uint32_t g_profile_kinds = 0xFFFFFFFFu;  // which kernel ids cr_profile_enable brackets
// Every profiled launch since cr_profile_enable(1), as (start, stop) event
// pairs; the events are kept and reused across enables.
struct ProfileEvents {
  std::vector<cudaEvent_t> start[kProfileKinds], stop[kProfileKinds];
  size_t n[kProfileKinds] = {};
};
thread_local ProfileEvents g_prof;
}  // namespace

ProfileScope::ProfileScope(int k, cudaStream_t st) : kind(k), s(st), on(g_profile)
{
  if (!on || kind < 0 || kind >= kProfileKinds || !((g_profile_kinds >> kind) & 1u)) { on = false; return; }
  const size_t i = g_prof.n[kind];
  if (i == g_prof.start[kind].size()) {
    cudaEvent_t a, b;
    CR_CUDA(cudaEventCreate(&a));
    CR_CUDA(cudaEventCreate(&b));
    g_prof.start[kind].push_back(a);
    g_prof.stop[kind].push_back(b);
  }
  CR_CUDA(cudaEventRecord(g_prof.start[kind][i], s));
}

ProfileScope::~ProfileScope()
{
  if (!on) return;
  cudaEventRecord(g_prof.stop[kind][g_prof.n[kind]], s);
  ++g_prof.n[kind];
}

}  // namespace crb

using namespace crb;

extern "C" int cr_profile_kinds(uint32_t mask)
{
  g_profile_kinds = mask;
  return CR_OK;
}

extern "C" int cr_profile_enable(int on)
{
  if (on && !g_profile)
    for (int k = 0; k < kProfileKinds; ++k) g_prof.n[k] = 0;
  g_profile = on != 0;
  return CR_OK;
}

extern "C" int cr_profile_last_ms(int kernel, float* ms)
{
  CR_API_BEGIN
  CR_REQUIRE(ms != nullptr && kernel >= 0 && kernel < kProfileKinds, "cr_profile_last_ms: bad argument");
  const size_t n = g_prof.n[kernel];
  CR_REQUIRE(n > 0, "cr_profile_last_ms: no profiled launch of this kernel");
  CR_CUDA(cudaEventSynchronize(g_prof.stop[kernel][n - 1]));
  CR_CUDA(cudaEventElapsedTime(ms, g_prof.start[kernel][n - 1], g_prof.stop[kernel][n - 1]));
  CR_API_END
}

extern "C" int cr_profile_sum_ms(int kernel, float* total_ms, uint32_t* count)
{
  CR_API_BEGIN
  CR_REQUIRE(total_ms != nullptr && count != nullptr && kernel >= 0 && kernel < kProfileKinds,
             "cr_profile_sum_ms: bad argument");
  const size_t n = g_prof.n[kernel];
  double sum = 0.0;
  for (size_t i = 0; i < n; ++i) {
    float ms = 0.f;
    CR_CUDA(cudaEventSynchronize(g_prof.stop[kernel][i]));
    CR_CUDA(cudaEventElapsedTime(&ms, g_prof.start[kernel][i], g_prof.stop[kernel][i]));
    sum += ms;
  }
  *total_ms = float(sum);
  *count = uint32_t(n);
  CR_API_END
}

extern "C" const char* cr_last_error_string(void) { return g_last_error.c_str(); }

extern "C" const char* cr_version(void) { return "cu_roaring_b200 0.1.0 sm_100a"; }

static void reset(cr_gpu_roaring* bm)
{
  const uint32_t U = bm->universe_size;
  std::memset(bm, 0, sizeof(*bm));
  bm->universe_size = U;
}

extern "C" int cr_gpu_roaring_free(cr_gpu_roaring* bm)
{
  CR_API_BEGIN
  CR_REQUIRE(bm != nullptr, "cr_gpu_roaring_free: null bitmap");
  if (bm->_alloc_base) {
    CR_CUDA(cudaFree(bm->_alloc_base));
  } else {
    void* ptrs[] = {bm->keys, bm->types, bm->offsets, bm->cardinalities, bm->bitmap_data,
                    bm->array_data, bm->run_data, bm->key_index};
    for (void* p : ptrs)
      if (p) CR_CUDA(cudaFree(p));
  }
  reset(bm);
  CR_API_END
}

extern "C" int cr_gpu_roaring_free_async(cr_gpu_roaring* bm, cr_stream_t stream)
{
  CR_API_BEGIN
  CR_REQUIRE(bm != nullptr, "cr_gpu_roaring_free_async: null bitmap");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (bm->_alloc_base) {
    CR_CUDA(cudaFreeAsync(bm->_alloc_base, s));
  } else {
    void* ptrs[] = {bm->keys, bm->types, bm->offsets, bm->cardinalities, bm->bitmap_data,
                    bm->array_data, bm->run_data, bm->key_index};
    for (void* p : ptrs)
      if (p) CR_CUDA(cudaFreeAsync(p, s));
  }
  reset(bm);
  CR_API_END
}

extern "C" int cr_resolve_auto_threshold(uint32_t universe_size, int device_id, uint32_t* out)
{
  CR_API_BEGIN
  CR_REQUIRE(out != nullptr, "cr_resolve_auto_threshold: null output");
  *out = resolve_auto(universe_size, device_id);
  CR_API_END
}

extern "C" int cr_deep_copy(const cr_gpu_roaring* bm, cr_stream_t stream, cr_gpu_roaring* out)
{
  CR_API_BEGIN
  CR_REQUIRE(bm && out, "cr_deep_copy: null argument");
  deep_copy(bm, out, reinterpret_cast<cudaStream_t>(stream));
  CR_API_END
}

extern "C" int cr_test_fail_allocations(int64_t after)
{
  crb::g_allocs_left.store(after < 0 ? -1 : after);
  return CR_OK;
}
