// Summary statistics of timing samples, as the reference's benchmark reports
// them (benchmark::summarizeTimings / Statistics, Benchmark.hpp:12-18,
// Benchmark.cpp:10-25): sample count, median (the mean of the two middle
// samples for an even count), the 90th percentile by linear interpolation
// between the samples at ranks floor(0.9 (n-1)) and the next, minimum and
// maximum. Host only.
#pragma once

#include <algorithm>
#include <cstddef>
#include <optional>
#include <vector>

namespace tensor::planner {

struct TimingStatistics {
  std::size_t samples = 0;
  double medianUs = 0.0;
  double p90Us = 0.0;
  double minUs = 0.0;
  double maxUs = 0.0;
};

// Empty input has no statistics.
inline std::optional<TimingStatistics> summarizeTimings(std::vector<double> values) {
  if (values.empty()) return std::nullopt;
  std::sort(values.begin(), values.end());
  const std::size_t n = values.size();
  TimingStatistics s;
  s.samples = n;
  s.medianUs = n % 2 ? values[n / 2] : 0.5 * (values[n / 2 - 1] + values[n / 2]);
  const double rank = 0.9 * static_cast<double>(n - 1);
  const std::size_t below = static_cast<std::size_t>(rank);
  const std::size_t above = std::min(below + 1, n - 1);
  const double t = rank - static_cast<double>(below);
  s.p90Us = values[below] + (values[above] - values[below]) * t;
  s.minUs = values.front();
  s.maxUs = values.back();
  return s;
}

}  // namespace tensor::planner
