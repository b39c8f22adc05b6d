// C++ drop-in test of the CRoaring-typed overloads of the public headers:
// cu_roaring::upload(const roaring_bitmap_t*, ...) (both overloads) and
// cu_roaring::get_meta(const roaring_bitmap_t*), compiled with
// tests/cpp/croaring_stub on the include path so that the headers'
// __has_include(<roaring/roaring.h>) block is built. Checks follow the
// reference's semantics (src/upload.cpp:31-71, 290-316): without a universe
// the universe is (max key + 1) << 16 and the set is never complemented;
// with one, the complement is stored above half density. Prints one line per
// failed check and exits non-zero on any failure.
#include <cstdio>
#include <random>
#include <set>
#include <vector>

#include "cu_roaring/cu_roaring.cuh"

#ifndef CU_ROARING_HAS_CROARING
#error "the CRoaring-typed overloads were not compiled"
#endif

static int g_fail = 0, g_pass = 0;
#define EXPECT(cond, msg)                                                         \
  do {                                                                            \
    if (cond) { ++g_pass; }                                                       \
    else { ++g_fail; std::printf("FAIL %s (%s:%d)\n", msg, __FILE__, __LINE__); } \
  } while (0)

static std::vector<uint32_t> ids_of(const cu_roaring::GpuRoaring& b)
{
  std::vector<uint32_t> h(b.total_cardinality);
  if (h.empty()) return h;
  int64_t* d = cu_roaring::enumerate_ids(b);
  std::vector<int64_t> t(h.size());
  cudaMemcpy(t.data(), d, t.size() * 8, cudaMemcpyDeviceToHost);
  cudaFree(d);
  for (size_t i = 0; i < h.size(); ++i) h[i] = uint32_t(t[i]);
  return h;
}

int main()
{
  std::mt19937 rng(7);
  // Sparse: 3 chunks, arrays and a run.
  std::set<uint32_t> s;
  for (int i = 0; i < 3000; ++i) s.insert(rng() % 200000u);
  for (uint32_t v = 300000; v < 305000; ++v) s.insert(v);
  std::vector<uint32_t> ids(s.begin(), s.end());
  roaring_bitmap_t bm{ids.data(), ids.size()};

  cu_roaring::GpuRoaring a = cu_roaring::upload(&bm);
  EXPECT(!a.negated, "no-universe upload is never complemented");
  EXPECT(a.universe_size == ((300000u >> 16) + 1) << 16, "universe inferred from the max key");
  EXPECT(a.total_cardinality == ids.size(), "cardinality");
  EXPECT(ids_of(a) == ids, "members (no universe)");

  cu_roaring::GpuRoaringMeta m = cu_roaring::get_meta(&bm);
  EXPECT(m.n_containers == 5, "get_meta: containers");
  EXPECT(m.n_array_containers + m.n_bitmap_containers + m.n_run_containers == m.n_containers,
         "get_meta: types add up");
  EXPECT(m.n_run_containers >= 1, "get_meta: the 5000-long run is a RUN container");
  EXPECT(m.universe_size == ((300000u >> 16) + 1) << 16, "get_meta: universe");
  cu_roaring::gpu_roaring_free(a);

  // Dense: 80% of a 2^20 universe.
  std::vector<uint32_t> dense;
  for (uint32_t v = 0; v < (1u << 20); ++v)
    if (rng() % 10 < 8) dense.push_back(v);
  roaring_bitmap_t dm{dense.data(), dense.size()};
  cu_roaring::GpuRoaring b = cu_roaring::upload(&dm);
  EXPECT(!b.negated, "dense, no universe: stored as given");
  EXPECT(ids_of(b) == dense, "dense members (no universe)");
  cu_roaring::GpuRoaring c = cu_roaring::upload(&dm, 1u << 20);
  EXPECT(c.negated, "dense, explicit universe: complement stored");
  EXPECT(c.universe_size == (1u << 20) && c.total_cardinality == dense.size(), "dense: universe, cardinality");
  EXPECT(ids_of(c) == dense, "dense members (explicit universe)");
  cu_roaring::GpuRoaring p = cu_roaring::upload(&dm, 1u << 20, 0, cu_roaring::PROMOTE_ALL);
  EXPECT(p.n_array_containers == 0 && p.n_run_containers == 0, "PROMOTE_ALL: every container a BITMAP");
  EXPECT(ids_of(p) == dense, "dense members (PROMOTE_ALL)");
  cu_roaring::gpu_roaring_free(b);
  cu_roaring::gpu_roaring_free(c);
  cu_roaring::gpu_roaring_free(p);

  // Empty.
  roaring_bitmap_t em{nullptr, 0};
  cu_roaring::GpuRoaring e = cu_roaring::upload(&em);
  EXPECT(e.n_containers == 0 && e.universe_size == 0 && e.total_cardinality == 0, "empty, no universe");
  cu_roaring::GpuRoaring e2 = cu_roaring::upload(&em, 5000u);
  EXPECT(e2.n_containers == 0 && e2.universe_size == 5000u, "empty, explicit universe");
  EXPECT(cu_roaring::get_meta(&em).n_containers == 0, "empty get_meta");

  std::printf("croaring_test: %d passed, %d failed\n", g_pass, g_fail);
  return g_fail ? 1 : 0;
}
