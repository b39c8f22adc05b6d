// C++ drop-in test: a user program written against the reference's public
// C++ API (cu_roaring::upload_from_ids, set_operation, multi_and,
// decompress_to_bitset, enumerate_ids, make_view + GpuRoaringView::contains /
// warp_contains inside user kernels), compiled against this engine's headers
// and linked to libcuroaring_b200.so. Cases follow the reference's
// test/test_promote.cu, test/test_complement.cu, test/test_device_query.cu and
// test/test_decompress.cu, plus a graph-traversal harness for the
// roaring_filter adapter. Prints one line per check and exits non-zero on
// any failure.
#include <algorithm>
#include <cstdio>
#include <random>
#include <set>
#include <vector>

#include "cu_roaring/cu_roaring.cuh"
#include "cu_roaring_v2/api.hpp"
#include "cu_roaring_v2/query.cuh"

static int g_fail = 0, g_pass = 0;
#define EXPECT(cond, msg)                                   \
  do {                                                      \
    if (cond) { ++g_pass; }                                 \
    else { ++g_fail; std::printf("FAIL %s (%s:%d)\n", msg, __FILE__, __LINE__); } \
  } while (0)

__global__ void user_contains(cu_roaring::GpuRoaringView v, const uint32_t* q, uint8_t* out, uint32_t n)
{
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = v.contains(q[i]);
}

__global__ void user_warp_contains(cu_roaring::GpuRoaringView v, const uint32_t* q, uint8_t* out,
                                   uint32_t n)
{
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  const bool hit = cu_roaring::warp_contains(v, i < n ? q[i] : 0u);  // all lanes call it
  if (i < n) out[i] = hit;
}

// Graph-traversal harness for cu_roaring::filtering::roaring_filter: a
// deterministic walk over a fixed-degree graph, one warp per query. At every
// hop the warp scores the current node's 32 neighbours, records the best one
// the filter passes (or 0xFFFFFFFF) and moves to the best neighbour overall
// (traversal ignores the filter, as graph search does).
__host__ __device__ inline uint32_t mix32(uint32_t x)
{
  x ^= x >> 16; x *= 0x7feb352du; x ^= x >> 15; x *= 0x846ca68bu; x ^= x >> 16;
  return x;
}
__host__ __device__ inline uint32_t walk_start(uint32_t q, uint32_t n) { return mix32(q * 2654435761u + 1u) % n; }
__host__ __device__ inline uint32_t walk_score(uint32_t q, uint32_t nb) { return mix32(nb ^ (q * 0x9e3779b9u)) | 1u; }

__global__ void graph_walk(cu_roaring::filtering::roaring_filter f, const uint32_t* adj, uint32_t n_nodes,
                           uint32_t n_queries, uint32_t hops, uint32_t* out, int warp_form)
{
  const uint32_t q = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (q >= n_queries) return;  // whole warps
  uint32_t cur = walk_start(q, n_nodes);
  for (uint32_t h = 0; h < hops; ++h) {
    const uint32_t nb = adj[size_t(cur) * 32 + lane];
    const uint32_t sc = walk_score(q, nb);
    const bool pass = warp_form ? f.warp_test(nb) : f(q, nb);
    const uint32_t m_all = __reduce_max_sync(0xFFFFFFFFu, sc);
    const uint32_t next = __reduce_min_sync(0xFFFFFFFFu, sc == m_all ? nb : 0xFFFFFFFFu);
    const uint32_t m_pass = __reduce_max_sync(0xFFFFFFFFu, pass ? sc : 0u);
    const uint32_t best = m_pass ? __reduce_min_sync(0xFFFFFFFFu, (pass && sc == m_pass) ? nb : 0xFFFFFFFFu)
                                 : 0xFFFFFFFFu;
    if (lane == 0) out[size_t(q) * hops + h] = best;
    cur = next;
  }
}

static void check_graph_walk(const cu_roaring::GpuRoaring& bm, const std::vector<bool>& truth, uint32_t offset,
                             const char* what)
{
  const uint32_t n_nodes = 1u << 20, n_queries = 2048, hops = 24;
  std::vector<uint32_t> adj(size_t(n_nodes) * 32);
  std::mt19937 gen(7);
  for (auto& a : adj) a = gen() % n_nodes;
  // Host replay with plain membership.
  std::vector<uint32_t> want(size_t(n_queries) * hops);
  for (uint32_t q = 0; q < n_queries; ++q) {
    uint32_t cur = walk_start(q, n_nodes);
    for (uint32_t h = 0; h < hops; ++h) {
      uint32_t m_all = 0, next = 0xFFFFFFFFu, m_pass = 0, best = 0xFFFFFFFFu;
      for (uint32_t j = 0; j < 32; ++j) {
        const uint32_t nb = adj[size_t(cur) * 32 + j], sc = walk_score(q, nb);
        if (sc > m_all || (sc == m_all && nb < next)) { m_all = sc; next = nb; }
        if (truth[nb + offset] && (sc > m_pass || (sc == m_pass && nb < best))) { m_pass = sc; best = nb; }
      }
      want[size_t(q) * hops + h] = best;
      cur = next;
    }
  }
  uint32_t *d_adj = nullptr, *d_out = nullptr;
  cudaMalloc(&d_adj, adj.size() * 4);
  cudaMalloc(&d_out, want.size() * 4);
  cudaMemcpy(d_adj, adj.data(), adj.size() * 4, cudaMemcpyHostToDevice);
  const cu_roaring::filtering::roaring_filter f(bm, offset);  // one line, no make_view
  for (int warp_form = 0; warp_form < 2; ++warp_form) {
    cudaMemset(d_out, 0, want.size() * 4);
    graph_walk<<<n_queries * 32 / 256, 256>>>(f, d_adj, n_nodes, n_queries, hops, d_out, warp_form);
    std::vector<uint32_t> got(want.size());
    cudaMemcpy(got.data(), d_out, got.size() * 4, cudaMemcpyDeviceToHost);
    char msg[160];
    std::snprintf(msg, sizeof msg, "%s (%s form)", what, warp_form ? "warp" : "per-thread");
    EXPECT(got == want, msg);
  }
  cudaFree(d_adj);
  cudaFree(d_out);
}

// Batch API (cu_roaring::v2): a user kernel testing membership through a
// view and through the batch itself.
__global__ void user_batch_contains(cu_roaring::v2::GpuRoaringBatch batch, cu_roaring::v2::GpuRoaringView v0,
                                    const uint32_t* q, uint8_t* out, uint32_t n)
{
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = uint8_t(cu_roaring::v2::contains(v0, q[i]) | (cu_roaring::v2::contains(batch, 1, q[i]) << 1));
}

// Portable serialization of sorted distinct IDs with at most 4096 per
// 65536-ID chunk (ARRAY containers only, cookie 12346 with offsets).
static std::vector<uint8_t> portable_arrays(const std::vector<uint32_t>& ids)
{
  std::vector<std::pair<uint16_t, std::vector<uint16_t>>> cs;
  for (uint32_t x : ids) {
    if (cs.empty() || cs.back().first != (x >> 16)) cs.push_back({uint16_t(x >> 16), {}});
    cs.back().second.push_back(uint16_t(x & 0xFFFF));
  }
  std::vector<uint8_t> out;
  auto put16 = [&](uint32_t v) { out.push_back(uint8_t(v)); out.push_back(uint8_t(v >> 8)); };
  auto put32 = [&](uint32_t v) { put16(v & 0xFFFF); put16(v >> 16); };
  put32(12346);
  put32(uint32_t(cs.size()));
  for (auto& c : cs) { put16(c.first); put16(uint32_t(c.second.size() - 1)); }
  uint32_t off = 8 + 8 * uint32_t(cs.size());
  for (auto& c : cs) { put32(off); off += 2 * uint32_t(c.second.size()); }
  for (auto& c : cs)
    for (uint16_t v : c.second) put16(v);
  return out;
}

static std::vector<uint8_t> query(const cu_roaring::GpuRoaring& bm, const std::vector<uint32_t>& q,
                                  bool warp)
{
  uint32_t* dq = nullptr;
  uint8_t* dr = nullptr;
  const uint32_t n = static_cast<uint32_t>(q.size());
  CUDA_CHECK(cudaMalloc(&dq, n * 4));
  CUDA_CHECK(cudaMalloc(&dr, n));
  CUDA_CHECK(cudaMemcpy(dq, q.data(), n * 4, cudaMemcpyHostToDevice));
  auto v = cu_roaring::make_view(bm);
  if (warp) user_warp_contains<<<(n + 255) / 256, 256>>>(v, dq, dr, n);
  else user_contains<<<(n + 255) / 256, 256>>>(v, dq, dr, n);
  CUDA_CHECK(cudaGetLastError());
  std::vector<uint8_t> r(n);
  CUDA_CHECK(cudaMemcpy(r.data(), dr, n, cudaMemcpyDeviceToHost));
  cudaFree(dq);
  cudaFree(dr);
  return r;
}

static std::vector<uint32_t> to_host_bitset(const cu_roaring::GpuRoaring& bm)
{
  const uint32_t words = (bm.universe_size + 31) / 32;
  std::vector<uint32_t> h(words);
  if (!words) return h;
  uint32_t* d = cu_roaring::decompress_to_bitset(bm);
  CUDA_CHECK(cudaDeviceSynchronize());
  CUDA_CHECK(cudaMemcpy(h.data(), d, words * 4, cudaMemcpyDeviceToHost));
  cudaFree(d);
  return h;
}

static void check_against(const cu_roaring::GpuRoaring& bm, const std::vector<bool>& truth,
                          const std::vector<uint32_t>& q, const char* what)
{
  for (int warp = 0; warp < 2; ++warp) {
    auto r = query(bm, q, warp);
    bool ok = true;
    for (size_t i = 0; i < q.size(); ++i)
      ok &= (r[i] != 0) == (q[i] < truth.size() && truth[q[i]]);
    EXPECT(ok, what);
  }
}

int main()
{
  using namespace cu_roaring;
  {  // test/test_promote.cu:387-416
    std::vector<uint32_t> ids = {200, 5, 100000, 42, 65536, 0, 100000, 5};
    auto bm = upload_from_ids(ids.data(), ids.size(), 200000, 0, PROMOTE_KEEP_DEFAULT);
    EXPECT(bm.total_cardinality == 6, "unsorted: cardinality 6");
    std::vector<bool> t(200000, false);
    for (auto i : ids) t[i] = true;
    check_against(bm, t, {0, 5, 42, 200, 65536, 100000, 1, 100, 65535}, "unsorted: membership");
    gpu_roaring_free(bm);
  }
  {  // test/test_complement.cu:129-150 (U=10, 90%)
    std::vector<uint32_t> ids = {0, 1, 2, 3, 4, 5, 6, 8, 9};
    auto bm = upload_from_ids(ids.data(), ids.size(), 10);
    EXPECT(bm.negated, "complement: negated");
    std::vector<bool> t(10, false);
    for (auto i : ids) t[i] = true;
    std::vector<uint32_t> q(10);
    for (uint32_t i = 0; i < 10; ++i) q[i] = i;
    check_against(bm, t, q, "complement: contains");
    // NOT({7}) AND {4,6,7} = {4,6}  (test/test_complement.cu:320-353)
    std::vector<uint32_t> bids = {4, 6, 7};
    auto b = upload_from_ids(bids.data(), 3, 10);
    auto r = set_operation(bm, b, SetOp::AND);
    EXPECT(r.total_cardinality == 2, "user example: cardinality");
    int64_t* d = enumerate_ids(r);
    int64_t h[2] = {0, 0};
    CUDA_CHECK(cudaDeviceSynchronize());
    CUDA_CHECK(cudaMemcpy(h, d, 16, cudaMemcpyDeviceToHost));
    EXPECT(h[0] == 4 && h[1] == 6, "user example: {4,6}");
    cudaFree(d);
    gpu_roaring_free(r);
    gpu_roaring_free(b);
    gpu_roaring_free(bm);
  }
  {  // test/test_device_query.cu:83-99 dense random, queries i*20; promoted too
    std::mt19937 gen(42);
    std::uniform_real_distribution<double> dist(0.0, 1.0);
    std::vector<uint32_t> ids;
    std::vector<bool> t(200000, false);
    for (uint32_t i = 0; i < 200000; ++i)
      if (dist(gen) < 0.5) { ids.push_back(i); t[i] = true; }
    std::vector<uint32_t> q;
    for (uint32_t i = 0; i < 10000; ++i) q.push_back(i * 20);
    for (uint32_t thr : {PROMOTE_KEEP_DEFAULT, PROMOTE_ALL}) {
      auto bm = upload_from_ids(ids.data(), ids.size(), 200000, 0, thr);
      check_against(bm, t, q, "dense random: contains / warp_contains");
      auto p = promote_to_bitmap(bm);
      CUDA_CHECK(cudaDeviceSynchronize());
      check_against(p, t, q, "promoted: contains");
      EXPECT(to_host_bitset(p) == to_host_bitset(bm), "promote keeps the set");
      auto c = gpu_roaring_deep_copy(bm);
      CUDA_CHECK(cudaDeviceSynchronize());
      EXPECT(to_host_bitset(c) == to_host_bitset(bm), "deep copy keeps the set");
      gpu_roaring_free(c);
      gpu_roaring_free(p);
      gpu_roaring_free(bm);
    }
  }
  {  // test/test_device_query.cu:137-169 clustered + run containers
    std::vector<uint32_t> ids;
    std::vector<bool> t(200000, false);
    for (uint32_t i = 1000; i <= 5000; ++i) { ids.push_back(i); t[i] = true; }
    for (uint32_t i = 70000; i <= 80000; ++i) { ids.push_back(i); t[i] = true; }
    auto bm = upload_from_ids(ids.data(), ids.size(), 200000, 0, PROMOTE_KEEP_DEFAULT);
    EXPECT(bm.n_run_containers == 1 && bm.n_array_containers == 1, "runs: container types");
    std::vector<uint32_t> q;
    for (uint32_t i = 0; i < 100000; i += 3) q.push_back(i);
    check_against(bm, t, q, "runs: contains");
    gpu_roaring_free(bm);
  }
  {  // multi_and with a negated input (test/test_complement.cu:503-545)
    std::mt19937 gen(42);
    std::vector<uint32_t> a, b, c;
    std::vector<bool> t(50000, false);
    std::vector<bool> ta(50000), tb(50000), tc(50000);
    for (uint32_t i = 0; i < 50000; ++i) {
      if (gen() % 3 == 0) { a.push_back(i); ta[i] = true; }
      if (gen() % 2 == 0) { b.push_back(i); tb[i] = true; }
      if (gen() % 4 != 0) { c.push_back(i); tc[i] = true; }
      t[i] = ta[i] && tb[i] && tc[i];
    }
    GpuRoaring in[3] = {upload_from_ids(a.data(), a.size(), 50000),
                        upload_from_ids(b.data(), b.size(), 50000),
                        upload_from_ids(c.data(), c.size(), 50000)};
    EXPECT(in[2].negated, "multi_and: third input negated");
    auto r = multi_and(in, 3);
    std::vector<uint32_t> q(50000);
    for (uint32_t i = 0; i < 50000; ++i) q[i] = i;
    check_against(r, t, q, "multi_and with negation");
    gpu_roaring_free(r);
    for (auto& x : in) gpu_roaring_free(x);
  }
  {  // roaring_filter in a graph walk: mixed containers, shard offset, negation
    const uint32_t offset = 3 * 65536 + 5, U = (1u << 20) + offset + 1000;
    std::vector<uint32_t> ids;
    std::vector<bool> t(U, false);
    std::mt19937 gen(11);
    for (uint32_t i = 0; i < U; ++i) {
      const uint32_t chunk = i >> 16;
      bool in = false;
      if (chunk % 3 == 0) in = gen() % 100 == 0;            // sparse: ARRAY
      else if (chunk % 3 == 1) in = gen() % 2 == 0;         // dense: BITMAP
      else in = (i / 2000) % 2 == 0;                        // long runs: RUN
      if (in) { ids.push_back(i); t[i] = true; }
    }
    auto bm = upload_from_ids(ids.data(), ids.size(), U);
    EXPECT(bm.n_array_containers > 0 && bm.n_bitmap_containers > 0 && bm.n_run_containers > 0,
           "roaring_filter: mixed container types");
    check_graph_walk(bm, t, offset, "roaring_filter graph walk, offset shard");
    gpu_roaring_free(bm);
    std::vector<uint32_t> dense;
    std::vector<bool> td(U, false);
    for (uint32_t i = 0; i < U; ++i)
      if (gen() % 10 != 0) { dense.push_back(i); td[i] = true; }
    auto neg = upload_from_ids(dense.data(), dense.size(), U);
    EXPECT(neg.negated, "roaring_filter: complement-stored filter");
    check_graph_walk(neg, td, 0, "roaring_filter graph walk, negated");
    gpu_roaring_free(neg);
  }
  {  // batch API: upload, views, contains(batch, b, id), promote, multi_and, decompress
    std::vector<uint32_t> a, c;
    std::vector<bool> ta(3 * 65536, false), tc(3 * 65536, false);
    for (uint32_t i = 0; i < 3 * 65536; i += 37) { a.push_back(i); ta[i] = true; }
    for (uint32_t i = 5; i < 3 * 65536; i += 91) { c.push_back(i); tc[i] = true; }
    const auto sa = portable_arrays(a), sc = portable_arrays(c);
    const void* bufs[2] = {sa.data(), sc.data()};
    const size_t sizes[2] = {sa.size(), sc.size()};
    auto batch = cu_roaring::v2::upload_batch_portable(bufs, sizes, 2);
    EXPECT(batch.n_bitmaps == 2 && batch.host_total_cardinalities[0] == a.size(), "batch: upload counts");
    std::vector<uint32_t> q(3 * 65536 + 100);
    for (uint32_t i = 0; i < q.size(); ++i) q[i] = i;
    uint32_t* dq = nullptr;
    uint8_t* dout = nullptr;
    cudaMalloc(&dq, q.size() * 4);
    cudaMalloc(&dout, q.size());
    cudaMemcpy(dq, q.data(), q.size() * 4, cudaMemcpyHostToDevice);
    user_batch_contains<<<(q.size() + 255) / 256, 256>>>(batch, cu_roaring::v2::make_view(batch, 0), dq, dout,
                                                          uint32_t(q.size()));
    std::vector<uint8_t> got(q.size());
    cudaMemcpy(got.data(), dout, got.size(), cudaMemcpyDeviceToHost);
    bool ok = true;
    for (uint32_t i = 0; i < q.size(); ++i) {
      const bool wa = i < ta.size() && ta[i], wc = i < tc.size() && tc[i];
      ok = ok && ((got[i] & 1) != 0) == wa && ((got[i] & 2) != 0) == wc;
    }
    EXPECT(ok, "batch: contains(view) and contains(batch, b, id) in a user kernel");
    auto prom = cu_roaring::v2::promote_batch(batch);
    const uint32_t both[2] = {0, 1};
    auto r = cu_roaring::v2::multi_and(prom, both, 2);
    uint64_t* dbits = nullptr;
    cudaMalloc(&dbits, 3 * 1024 * 8);
    cudaMemset(dbits, 0, 3 * 1024 * 8);
    cu_roaring::v2::decompress_batch(r, dbits, 3 * 1024);
    std::vector<uint64_t> w(3 * 1024);
    cudaMemcpy(w.data(), dbits, w.size() * 8, cudaMemcpyDeviceToHost);
    ok = true;
    for (uint32_t i = 0; i < 3 * 65536; ++i) ok = ok && (((w[i >> 6] >> (i & 63)) & 1) != 0) == (ta[i] && tc[i]);
    EXPECT(ok, "batch: promote + multi_and + decompress");
    cudaFree(dq);
    cudaFree(dout);
    cudaFree(dbits);
    cu_roaring::v2::free_batch(r);
    cu_roaring::v2::free_batch(prom);
    cu_roaring::v2::free_batch(batch);
  }
  {  // error convention: an ID outside the universe throws std::runtime_error
    std::vector<uint32_t> ids = {5, 500};
    bool threw = false;
    try {
      auto bm = upload_from_ids(ids.data(), 2, 100);
      gpu_roaring_free(bm);
    } catch (const std::runtime_error&) {
      threw = true;
    }
    EXPECT(threw, "out-of-universe ID throws");
  }
  std::printf("api_test: %d passed, %d failed\n", g_pass, g_fail);
  return g_fail ? 1 : 0;
}
