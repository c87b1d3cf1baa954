// Host-side synthetic data generation for the data loader.
//
// Filling 448x448x3 uint8 frames for 12 images per sample from numpy's
// generator costs ~10 ms per sample, which starves a multi-GPU job of batches.
// This fills a caller-provided (ideally pinned) buffer with uniform bytes from
// xoshiro256** streams seeded per (seed, sample index, chunk) via splitmix64,
// split across host threads. Output depends only on (seed, index), never on
// the thread count.
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <thread>
#include <vector>

#include "nfb_api.h"

#define NFB_HOST_API extern "C" __attribute__((visibility("default")))

namespace {

inline uint64_t splitmix64(uint64_t& x) {
  uint64_t z = (x += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

inline uint64_t rotl(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }

struct Xoshiro256 {
  uint64_t s[4];
  explicit Xoshiro256(uint64_t seed) {
    for (auto& v : s) v = splitmix64(seed);
  }
  inline uint64_t next() {
    const uint64_t r = rotl(s[1] * 5, 7) * 9;
    const uint64_t t = s[1] << 17;
    s[2] ^= s[0]; s[3] ^= s[1]; s[1] ^= s[2]; s[0] ^= s[3];
    s[2] ^= t;
    s[3] = rotl(s[3], 45);
    return r;
  }
};

constexpr int64_t kChunk = 1 << 20;  // bytes per independent stream

void fill_range(uint8_t* dst, int64_t n, uint64_t seed, uint64_t index, int64_t c0, int64_t c1) {
  for (int64_t c = c0; c < c1; ++c) {
    uint64_t k = seed * 0x100000001B3ull ^ (index * 0x9E3779B97F4A7C15ull) ^ (uint64_t)c;
    Xoshiro256 g(splitmix64(k));
    const int64_t lo = c * kChunk;
    const int64_t hi = std::min(n, lo + kChunk);
    int64_t i = lo;
    for (; i + 8 <= hi; i += 8) {
      uint64_t v = g.next();
      memcpy(dst + i, &v, 8);
    }
    if (i < hi) {
      uint64_t v = g.next();
      memcpy(dst + i, &v, (size_t)(hi - i));
    }
  }
}

}  // namespace

// Fill dst[0:n) with uniform bytes for sample `index` of a dataset seeded `seed`.
NFB_HOST_API int nfb_synth_fill_u8(uint8_t* dst, int64_t n, uint64_t seed, uint64_t index, int threads) {
  if (n <= 0) return 0;
  const int64_t chunks = (n + kChunk - 1) / kChunk;
  int nt = std::max(1, std::min<int>(threads, (int)chunks));
  if (nt == 1) {
    fill_range(dst, n, seed, index, 0, chunks);
    return 0;
  }
  std::vector<std::thread> pool;
  pool.reserve(nt);
  for (int t = 0; t < nt; ++t) {
    const int64_t c0 = chunks * t / nt, c1 = chunks * (t + 1) / nt;
    pool.emplace_back(fill_range, dst, n, seed, index, c0, c1);
  }
  for (auto& th : pool) th.join();
  return 0;
}
