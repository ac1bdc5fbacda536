// Host-side native core under sanitizers: the planner (legacy and
// earliest-finish policies, makespan, chunk choice, concurrent caps) and the
// multithreaded generators.  Built and run by tests/test_native_sanitizers.py
// with -fsanitize=address,undefined and, separately, -fsanitize=thread.
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <vector>

#include "host_ops.h"
#include "planner.h"

static int failures = 0;
#define CHECK(cond)                                                        \
  do {                                                                     \
    if (!(cond)) {                                                         \
      std::fprintf(stderr, "CHECK failed at line %d: %s\n", __LINE__, #cond); \
      ++failures;                                                          \
    }                                                                      \
  } while (0)

static std::vector<int> counts(const std::vector<int32_t>& idx, int lanes) {
  std::vector<int> c(lanes, 0);
  for (int32_t i : idx) c.at(i)++;
  return c;
}

int main() {
  using namespace ppb;
  const uint64_t MiB = 1ull << 20;
  // the reference's pinned splits: 14 x 16 MiB over bw {20, 40, 10} -> 4/8/2
  std::vector<uint64_t> c14(14, 16 * MiB);
  CHECK((counts(assign_chunks(c14, {20, 40, 10}, {0, 0, 0}, kLegacyGreedy), 3) == std::vector<int>{4, 8, 2}));
  // 12 x 16 MiB over {10, 20, 30} -> 2/4/6
  std::vector<uint64_t> c12(12, 16 * MiB);
  CHECK((counts(assign_chunks(c12, {10, 20, 30}, {0, 0, 0}, kLegacyGreedy), 3) == std::vector<int>{2, 4, 6}));
  // earliest-finish with latency prefers the fast lanes
  auto ef = counts(assign_chunks(std::vector<uint64_t>(64, 4 * MiB), {50, 25, 5}, {0, 0, 0.01}, kEarliestFinish), 3);
  CHECK(ef[0] > ef[1] && ef[1] > ef[2]);
  // uneven and empty inputs
  CHECK(assign_chunks({}, {1, 2}, {0, 0}, kEarliestFinish).empty());
  auto one = assign_chunks({1}, {1}, {0}, kLegacyGreedy);
  CHECK(one.size() == 1 && one[0] == 0);
  // concurrent caps: two lanes in one group of capacity 60 scale to sum 60
  auto cap = concurrent_bandwidth({50, 50, 40}, {0, 0, -1}, {60});
  CHECK(std::fabs(cap[0] + cap[1] - 60.0) < 1e-9 && cap[2] == 40.0);
  // chunk choice is one of the candidates and makespan is positive
  std::vector<uint64_t> cands{1 * MiB, 4 * MiB, 16 * MiB, 64 * MiB};
  uint64_t ch = choose_chunk_bytes(4096 * MiB, cands, {50, 30, 30}, {2e-5, 2e-5, 2e-5});
  CHECK(ch == 1 * MiB || ch == 4 * MiB || ch == 16 * MiB || ch == 64 * MiB);
  CHECK(estimate_makespan(4096 * MiB, 16 * MiB, {50, 30}, {1e-5, 1e-5}) > 0.0);
  // generators: thread-count invariant, odd sizes, no out-of-bounds writes
  const uint64_t n = (1ull << 21) + 3;
  std::vector<uint16_t> a(n + 8, 0xAAAA), b(n + 8, 0xAAAA);
  fill_normal_bf16(a.data(), n, 0.f, 0.02f, 9, 0);
  fill_normal_bf16(b.data(), n, 0.f, 0.02f, 9, 5);
  CHECK(std::memcmp(a.data(), b.data(), n * 2) == 0);
  CHECK(a[n] == 0xAAAA && a[n + 7] == 0xAAAA);
  std::vector<uint8_t> r(1000003 + 16, 0x55);
  fill_random_bytes(r.data(), 1000003, 3, 7);
  CHECK(r[1000003] == 0x55 && r[1000003 + 15] == 0x55);
  std::printf("host_core_test: %s\n", failures ? "FAILED" : "ok");
  return failures ? 1 : 0;
}
