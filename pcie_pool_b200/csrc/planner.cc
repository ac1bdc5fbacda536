#include "planner.h"

#include <algorithm>
#include <limits>
#include <map>
#include <stdexcept>

namespace ppb {

namespace {
constexpr double kGiB = 1024.0 * 1024.0 * 1024.0;
}

std::vector<int32_t> assign_chunks(const std::vector<uint64_t>& chunk_bytes,
                                   const std::vector<double>& bw_gibps,
                                   const std::vector<double>& latency_s, int policy) {
  const size_t lanes = bw_gibps.size();
  if (lanes == 0) throw std::invalid_argument("no lanes to assign to");
  for (double b : bw_gibps)
    if (!(b > 0.0)) throw std::invalid_argument("lane bandwidth must be positive");
  if (!latency_s.empty() && latency_s.size() != lanes)
    throw std::invalid_argument("latency vector must match the lane count");
  std::vector<int32_t> out(chunk_bytes.size(), 0);
  if (policy == kLegacyGreedy) {
    std::vector<double> assigned(lanes, 0.0);
    for (size_t c = 0; c < chunk_bytes.size(); ++c) {
      size_t best = 0;
      double best_score = std::numeric_limits<double>::infinity();
      for (size_t i = 0; i < lanes; ++i) {
        const double score = assigned[i] / bw_gibps[i];
        if (score < best_score) {
          best_score = score;
          best = i;
        }
      }
      out[c] = static_cast<int32_t>(best);
      assigned[best] += static_cast<double>(chunk_bytes[c]);
    }
    return out;
  }
  if (policy != kEarliestFinish) throw std::invalid_argument("unknown plan policy");
  std::vector<double> finish(lanes, 0.0);
  for (size_t c = 0; c < chunk_bytes.size(); ++c) {
    size_t best = 0;
    double best_t = std::numeric_limits<double>::infinity();
    const double gib = static_cast<double>(chunk_bytes[c]) / kGiB;
    for (size_t i = 0; i < lanes; ++i) {
      const double lat = latency_s.empty() ? 0.0 : latency_s[i];
      const double t = finish[i] + lat + gib / bw_gibps[i];
      if (t < best_t) {
        best_t = t;
        best = i;
      }
    }
    out[c] = static_cast<int32_t>(best);
    finish[best] = best_t;
  }
  return out;
}

std::vector<double> concurrent_bandwidth(const std::vector<double>& bw,
                                         const std::vector<int32_t>& group,
                                         const std::vector<double>& cap) {
  if (group.size() != bw.size()) throw std::invalid_argument("group vector must match lanes");
  std::map<int32_t, double> sum;
  for (size_t i = 0; i < bw.size(); ++i)
    if (group[i] >= 0) sum[group[i]] += bw[i];
  std::vector<double> out(bw);
  for (size_t i = 0; i < bw.size(); ++i) {
    const int32_t g = group[i];
    if (g < 0) continue;
    if (static_cast<size_t>(g) >= cap.size()) throw std::invalid_argument("group id without capacity");
    const double s = sum[g];
    if (cap[g] > 0.0 && s > cap[g]) out[i] = bw[i] * (cap[g] / s);
  }
  return out;
}

double estimate_makespan(uint64_t total, uint64_t chunk, const std::vector<double>& bw,
                         const std::vector<double>& lat) {
  if (chunk == 0) throw std::invalid_argument("chunk must be positive");
  std::vector<uint64_t> chunks;
  for (uint64_t off = 0; off < total; off += chunk) chunks.push_back(std::min(chunk, total - off));
  const auto a = assign_chunks(chunks, bw, lat, kEarliestFinish);
  std::vector<double> finish(bw.size(), 0.0);
  double slowest_fill = 0.0;
  for (size_t c = 0; c < chunks.size(); ++c) {
    const size_t i = static_cast<size_t>(a[c]);
    const double t = (lat.empty() ? 0.0 : lat[i]) + (double(chunks[c]) / kGiB) / bw[i];
    finish[i] += t;
    slowest_fill = std::max(slowest_fill, t);
  }
  double mk = 0.0;
  for (double f : finish) mk = std::max(mk, f);
  // A staged lane needs one more chunk-time to drain the last slot.
  return mk + slowest_fill * 0.5;
}

uint64_t choose_chunk_bytes(uint64_t total, const std::vector<uint64_t>& candidates,
                            const std::vector<double>& bw, const std::vector<double>& lat) {
  if (candidates.empty()) throw std::invalid_argument("no chunk-size candidates");
  uint64_t best = candidates.front();
  double best_t = std::numeric_limits<double>::infinity();
  for (uint64_t c : candidates) {
    if (c == 0) continue;
    const double t = estimate_makespan(total, c, bw, lat);
    if (t < best_t * (1.0 - 1e-9)) {
      best_t = t;
      best = c;
    }
  }
  return best;
}

}  // namespace ppb
