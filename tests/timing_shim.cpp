// Test-only C wrapper over the timing statistics
// (aicompiler-test_b200/csrc/timing_stats.hpp), compiled with g++ by
// tests/test_timing_stats.py.
#include <cstddef>
#include <vector>

#include "timing_stats.hpp"

extern "C" int summarize(const double *values, std::size_t n, double *out /* samples, median, p90, min, max */) {
  const auto s = tensor::planner::summarizeTimings(std::vector<double>(values, values + n));
  if (!s) return 0;
  out[0] = double(s->samples);
  out[1] = s->medianUs;
  out[2] = s->p90Us;
  out[3] = s->minUs;
  out[4] = s->maxUs;
  return 1;
}
