// CPU baseline: the reference's host-side upload path, restated.
//
// TEST / BASELINE INFRASTRUCTURE ONLY (bench.py times it as the CPU
// baseline of BASELINE config 2; nothing in the product links it).
// Follows the steps of the reference's small-input CPU path,
// src/upload_ids.cu:421-561: std::sort of the raw IDs, std::unique, the
// complement when more than half the universe is set, a partition of the
// sorted IDs into 65536-ID chunks, and per chunk an ARRAY (sorted lows) or a
// BITMAP (1024 u64 words) by the threshold, plus the direct-map key index.
// The device copies of that path are left out: this times the host work.
#include <algorithm>
#include <cstdint>
#include <vector>

extern "C" uint64_t or_cpu_upload_sorted(const uint32_t* ids, uint64_t n, uint32_t universe, uint32_t threshold,
                                         uint64_t* out_counts /* [4]: containers, bitmaps, arrays, card */)
{
  std::vector<uint32_t> v(ids, ids + n);
  std::sort(v.begin(), v.end());
  v.erase(std::unique(v.begin(), v.end()), v.end());
  const uint64_t card = v.size();
  if (card > uint64_t(universe) / 2) {  // store the complement
    std::vector<uint32_t> c;
    c.reserve(universe - card);
    size_t j = 0;
    for (uint64_t x = 0; x < universe; ++x) {
      if (j < v.size() && v[j] == x) ++j;
      else c.push_back(uint32_t(x));
    }
    v.swap(c);
  }
  std::vector<uint16_t> keys, cards, kidx;
  std::vector<uint8_t> types;
  std::vector<uint32_t> offsets;
  std::vector<uint64_t> bitmap_pool;
  std::vector<uint16_t> array_pool;
  uint64_t nb = 0, na = 0;
  for (size_t i = 0; i < v.size();) {
    const uint32_t key = v[i] >> 16;
    size_t e = i;
    while (e < v.size() && (v[e] >> 16) == key) ++e;
    const uint32_t c = uint32_t(e - i);
    keys.push_back(uint16_t(key));
    cards.push_back(uint16_t(c > 65535 ? 0 : c));
    if (c > threshold) {
      types.push_back(1);
      offsets.push_back(uint32_t(bitmap_pool.size() * 8));
      const size_t base = bitmap_pool.size();
      bitmap_pool.resize(base + 1024, 0);
      for (size_t t = i; t < e; ++t) bitmap_pool[base + ((v[t] & 0xFFFFu) >> 6)] |= 1ull << (v[t] & 63u);
      ++nb;
    } else {
      types.push_back(0);
      offsets.push_back(uint32_t(array_pool.size() * 2));
      for (size_t t = i; t < e; ++t) array_pool.push_back(uint16_t(v[t] & 0xFFFFu));
      ++na;
    }
    i = e;
  }
  if (!keys.empty()) {
    kidx.assign(size_t(keys.back()) + 1, 0xFFFF);
    for (size_t i = 0; i < keys.size(); ++i) kidx[keys[i]] = uint16_t(i);
  }
  if (out_counts) {
    out_counts[0] = keys.size();
    out_counts[1] = nb;
    out_counts[2] = na;
    out_counts[3] = card;
  }
  return keys.size();
}
