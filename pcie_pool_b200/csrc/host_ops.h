// Multithreaded host-side generators for synthetic workloads (weights, KV
// caches, byte patterns) written straight into pinned host memory.
#pragma once

#include <cstdint>

namespace ppb {

// bf16 values ~ N(mean, std) at dst[0..n), counter-based and deterministic
// for a given seed regardless of the thread count.
void fill_normal_bf16(void* dst, uint64_t n, float mean, float stddev, uint64_t seed, int threads);

// Uniform random bytes at dst[0..n), deterministic for a seed.
void fill_random_bytes(void* dst, uint64_t n, uint64_t seed, int threads);

}  // namespace ppb
