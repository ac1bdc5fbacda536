// Native planner core: the per-chunk lane assignment loop and the chunk-size
// choice, the two parts of planning whose cost grows with the chunk count.
//
// Policies
//   kLegacyGreedy  -- each chunk goes to argmin_i(assigned_bytes_i / bw_i),
//                     ties to the lower lane index (the reference's rule,
//                     cpp/src/planner.cpp:166-211).
//   kEarliestFinish -- each chunk goes to the lane whose finish time after
//                     taking it, assigned_time_i + latency_i + bytes / bw_i,
//                     is smallest (ties to the lower index).  With per-chunk
//                     latency this also prefers fewer, larger pieces on slow
//                     lanes.
#pragma once

#include <cstdint>
#include <vector>

namespace ppb {

enum PlanPolicy : int { kLegacyGreedy = 0, kEarliestFinish = 1 };

std::vector<int32_t> assign_chunks(const std::vector<uint64_t>& chunk_bytes,
                                   const std::vector<double>& bw_gibps,
                                   const std::vector<double>& latency_s, int policy);

// Scale lane bandwidths so lanes that share an uplink group never sum above the
// group's measured concurrent capacity (group id < 0: no sharing).
std::vector<double> concurrent_bandwidth(const std::vector<double>& bw_gibps,
                                         const std::vector<int32_t>& group,
                                         const std::vector<double>& group_capacity_gibps);

// Estimated makespan (seconds) of moving `total` bytes in `chunk` pieces over
// the lanes with the earliest-finish assignment, including one chunk of
// pipeline fill on the slowest used lane.
double estimate_makespan(uint64_t total, uint64_t chunk, const std::vector<double>& bw_gibps,
                         const std::vector<double>& latency_s);

// Pick the candidate chunk size with the smallest estimated makespan.
uint64_t choose_chunk_bytes(uint64_t total, const std::vector<uint64_t>& candidates,
                            const std::vector<double>& bw_gibps,
                            const std::vector<double>& latency_s);

}  // namespace ppb
