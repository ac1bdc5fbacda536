// Host generators: a counter-based stream (splitmix64 of seed ^ index) so
// each element depends only on (seed, index); normals by the Box-Muller
// transform (G. E. P. Box and M. E. Muller, 1958); float -> bf16 by
// round-to-nearest-even on the upper 16 bits of the IEEE-754 binary32 value.
#include "host_ops.h"

#include <cmath>
#include <cstring>
#include <thread>
#include <vector>

namespace ppb {
namespace {

inline uint64_t splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

inline uint16_t to_bf16(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7F800000u) == 0x7F800000u) return static_cast<uint16_t>((u >> 16) | ((u & 0xFFFFu) ? 0x40u : 0u));
  const uint32_t lsb = (u >> 16) & 1u;
  u += 0x7FFFu + lsb;
  return static_cast<uint16_t>(u >> 16);
}

template <typename F>
void parallel(uint64_t n, int threads, F&& body) {
  unsigned t = threads > 0 ? unsigned(threads) : std::thread::hardware_concurrency();
  if (t == 0) t = 1;
  if (n < (1ull << 20)) t = 1;
  std::vector<std::thread> th;
  for (unsigned i = 1; i < t; ++i) th.emplace_back(body, n * i / t, n * (i + 1) / t);
  body(0, n / t);
  for (auto& x : th) x.join();
}

}  // namespace

void fill_normal_bf16(void* dst, uint64_t n, float mean, float stddev, uint64_t seed, int threads) {
  uint16_t* out = static_cast<uint16_t*>(dst);
  const uint64_t pairs = (n + 1) / 2;
  const double two_pi = 6.283185307179586476925286766559;
  parallel(pairs, threads, [&](uint64_t p0, uint64_t p1) {
    for (uint64_t p = p0; p < p1; ++p) {
      const uint64_t r = splitmix64(seed ^ (p * 0xD1B54A32D192ED03ull));
      // two 32-bit uniforms in (0, 1]
      const double u1 = (double((r >> 32) & 0xFFFFFFFFull) + 1.0) * (1.0 / 4294967296.0);
      const double u2 = double(r & 0xFFFFFFFFull) * (1.0 / 4294967296.0);
      const double rad = std::sqrt(-2.0 * std::log(u1));
      const float z0 = static_cast<float>(rad * std::cos(two_pi * u2));
      const float z1 = static_cast<float>(rad * std::sin(two_pi * u2));
      out[2 * p] = to_bf16(mean + stddev * z0);
      if (2 * p + 1 < n) out[2 * p + 1] = to_bf16(mean + stddev * z1);
    }
  });
}

void fill_random_bytes(void* dst, uint64_t n, uint64_t seed, int threads) {
  uint8_t* out = static_cast<uint8_t*>(dst);
  const uint64_t words = n / 8;
  parallel(words, threads, [&](uint64_t w0, uint64_t w1) {
    for (uint64_t w = w0; w < w1; ++w) {
      const uint64_t v = splitmix64(seed ^ (w * 0xA0761D6478BD642Full));
      std::memcpy(out + 8 * w, &v, 8);
    }
  });
  if (n % 8) {
    const uint64_t v = splitmix64(seed ^ (words * 0xA0761D6478BD642Full));
    std::memcpy(out + 8 * words, &v, n % 8);
  }
}

}  // namespace ppb
