// Regenerates the input sets of the reference's own unit tests, with the same
// std::mt19937 seeds and the same libstdc++ distributions, so the cases of
//   test/test_set_ops.cu, test/test_complement.cu, test/test_promote.cu,
//   test/test_decompress.cu, test/test_device_query.cu
// (maxwbuckley/cu-roaring-bitmap) can be replayed against this engine and
// its oracle. Each set is written as a u32 bitset (bit i of word i/32) to
// <outdir>/<name>.bin; <outdir>/manifest.txt lists "name universe".
//
// Build: g++ -O2 -std=c++17 make_ref_sets.cpp -o make_ref_sets
// Run:   ./make_ref_sets <outdir>
#include <cstdint>
#include <cstdio>
#include <fstream>
#include <random>
#include <string>
#include <vector>

struct Set {
  std::string name;
  uint32_t universe;
  std::vector<uint32_t> words;
  explicit Set(std::string n, uint32_t u) : name(std::move(n)), universe(u), words((u + 31) / 32, 0) {}
  void add(uint32_t i) { words[i / 32] |= 1u << (i % 32); }
  void remove(uint32_t i) { words[i / 32] &= ~(1u << (i % 32)); }
};

static std::vector<Set> g_sets;

// test/test_set_ops.cu:15-25 make_random (uniform_real_distribution < density).
static void make_random(const std::string& name, uint32_t universe, double density, uint64_t seed)
{
  Set s(name, universe);
  std::mt19937 gen(seed);
  std::uniform_real_distribution<double> dist(0.0, 1.0);
  for (uint32_t i = 0; i < universe; ++i)
    if (dist(gen) < density) s.add(i);
  g_sets.push_back(std::move(s));
}

int main(int argc, char** argv)
{
  if (argc < 2) {
    std::fprintf(stderr, "usage: %s outdir\n", argv[0]);
    return 2;
  }
  const std::string out = argv[1];

  // test/test_set_ops.cu:84-342
  make_random("setops_bb_a", 200000, 0.6, 100);
  make_random("setops_bb_b", 200000, 0.4, 200);
  make_random("setops_aa_a", 200000, 0.02, 300);
  make_random("setops_aa_b", 200000, 0.01, 400);
  make_random("setops_ba_a", 200000, 0.5, 500);
  make_random("setops_ba_b", 200000, 0.02, 600);
  make_random("setops_ident", 100000, 0.3, 700);
  make_random("setops_or_a", 200000, 0.5, 800);
  make_random("setops_or_b", 200000, 0.3, 900);
  make_random("setops_andnot_a", 200000, 0.5, 1000);
  make_random("setops_andnot_b", 200000, 0.3, 1100);
  make_random("setops_xor_a", 200000, 0.5, 1200);
  make_random("setops_xor_b", 200000, 0.3, 1300);
  make_random("setops_xor_ident", 100000, 0.4, 1400);
  make_random("setops_mand_a", 200000, 0.6, 1500);
  make_random("setops_mand_b", 200000, 0.5, 1600);
  make_random("setops_mand_c", 200000, 0.4, 1700);
  make_random("setops_mor_a", 200000, 0.1, 1800);
  make_random("setops_mor_b", 200000, 0.1, 1900);
  make_random("setops_mor_c", 200000, 0.1, 2000);
  {  // AND_EmptyResult / OR_NonOverlapping: [0,1000) vs [65536,66536)
    Set a("setops_disjoint_a", 131072), b("setops_disjoint_b", 131072);
    for (uint32_t i = 0; i < 1000; ++i) a.add(i);
    for (uint32_t i = 65536; i < 66536; ++i) b.add(i);
    g_sets.push_back(std::move(a));
    g_sets.push_back(std::move(b));
  }
  // test/test_complement.cu:372-462 DeMorgan operands
  make_random("demorgan_a", 100000, 0.3, 42);
  make_random("demorgan_b", 100000, 0.4, 99);
  {  // test/test_complement.cu:151-170 NegatedContains_AbsentKey
    Set s("compl_absent_key", 200000);
    std::mt19937 gen(42);
    for (uint32_t i = 0; i < 200000; ++i)
      if (gen() % 10 != 0) s.add(i);
    g_sets.push_back(std::move(s));
  }
  {  // :184-200 LargeGPUPath
    Set s("compl_large", 100000);
    std::mt19937 gen(123);
    for (uint32_t i = 0; i < 100000; ++i)
      if (gen() % 5 != 0) s.add(i);
    g_sets.push_back(std::move(s));
  }
  {  // :212-225 NoNegate_LowDensity
    Set s("compl_low", 100000);
    std::mt19937 gen(42);
    for (uint32_t i = 0; i < 100000; ++i)
      if (gen() % 10 == 0) s.add(i);
    g_sets.push_back(std::move(s));
  }
  {  // :503-545 MultiAnd_WithNegated (interleaved draws)
    Set r1("mand_neg_1", 50000), r2("mand_neg_2", 50000), r3("mand_neg_3", 50000);
    std::mt19937 gen(42);
    for (uint32_t i = 0; i < 50000; ++i) {
      if (gen() % 3 == 0) r1.add(i);
      if (gen() % 2 == 0) r2.add(i);
      if (gen() % 4 != 0) r3.add(i);
    }
    g_sets.push_back(std::move(r1));
    g_sets.push_back(std::move(r2));
    g_sets.push_back(std::move(r3));
  }
  {  // :548-600 MultiAnd_AllNegated
    Set r1("mand_allneg_1", 50000), r2("mand_allneg_2", 50000), r3("mand_allneg_3", 50000);
    std::mt19937 gen(77);
    for (uint32_t i = 0; i < 50000; ++i) {
      if (gen() % 4 != 0) r1.add(i);
      if (gen() % 3 != 0) r2.add(i);
      if (gen() % 5 != 0) r3.add(i);
    }
    g_sets.push_back(std::move(r1));
    g_sets.push_back(std::move(r2));
    g_sets.push_back(std::move(r3));
  }
  {  // :605-680 FusedMultiAnd_AbsentKeyInNegatedInput
    const uint32_t U = 3u * 65536u;
    Set a("absent_A", U), b("absent_B", U), c("absent_C", U);
    std::mt19937 gen(1001);
    for (uint32_t k = 0; k < 3; ++k)
      for (uint32_t i = 0; i < 65536u; ++i)
        if ((gen() % 5u) == 0) a.add(k * 65536u + i);
    for (uint32_t i = 0; i < U; ++i) b.add(i);
    for (uint32_t gap : {70000u, 70001u, 70005u, 70100u, 70200u}) b.remove(gap);
    for (uint32_t i = 0; i < 65536u; ++i) {
      if ((gen() % 7u) == 0) c.add(i);
      if ((gen() % 7u) == 0) c.add(131072u + i);
    }
    g_sets.push_back(std::move(a));
    g_sets.push_back(std::move(b));
    g_sets.push_back(std::move(c));
  }
  {  // :683-745 FusedMultiAnd_MixedNegation_ManyContainers (5 inputs)
    const uint32_t U = 16u * 65536u;
    std::mt19937 gen(2002);
    const double dens[5] = {0.30, 0.90, 0.15, 0.75, 0.25};
    for (int j = 0; j < 5; ++j) {
      Set s("mixed5_" + std::to_string(j), U);
      for (uint32_t i = 0; i < U; ++i)
        if ((gen() & 0xFFFFu) < static_cast<uint32_t>(dens[j] * 65536.0)) s.add(i);
      g_sets.push_back(std::move(s));
    }
  }
  {  // :748-790 eight inputs, alternating 20% / 85%
    const uint32_t U = 8u * 65536u;
    std::mt19937 gen(3003);
    for (int j = 0; j < 8; ++j) {
      Set s("alt8_" + std::to_string(j), U);
      const double d = (j % 2 == 0) ? 0.20 : 0.85;
      for (uint32_t i = 0; i < U; ++i)
        if ((gen() & 0xFFFFu) < static_cast<uint32_t>(d * 65536.0)) s.add(i);
      g_sets.push_back(std::move(s));
    }
  }
  {  // test/test_decompress.cu:89-107 and test/test_device_query.cu:101-117:
     // 1000 draws of uniform_int_distribution(0, 999999), seed 42
    Set s("uniform_int_1e6", 1000000);
    std::mt19937 gen(42);
    std::uniform_int_distribution<uint32_t> dist(0, 999999);
    for (int i = 0; i < 1000; ++i) s.add(dist(gen));
    g_sets.push_back(std::move(s));
  }
  {  // test/test_device_query.cu:83-99 dense random (uniform_real, seed 42)
    make_random("query_dense", 200000, 0.5, 42);
  }

  std::ofstream man(out + "/manifest.txt");
  for (const Set& s : g_sets) {
    std::ofstream f(out + "/" + s.name + ".bin", std::ios::binary);
    f.write(reinterpret_cast<const char*>(s.words.data()), s.words.size() * 4);
    man << s.name << " " << s.universe << "\n";
  }
  return 0;
}
