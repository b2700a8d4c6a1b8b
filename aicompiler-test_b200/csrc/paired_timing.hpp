// Paired A/B timing for the tuners: alternating baseline / candidate launches,
// each bracketed by CUDA events on the launching stream, summarised per arm
// (timing_stats.hpp) and compared by medians (benchmark::measurePair,
// Benchmark.cpp:68-96).
#pragma once

#include <cuda_runtime.h>

#include <algorithm>
#include <functional>
#include <string>
#include <vector>

#include "timing_stats.hpp"

namespace tensor::planner {

struct PairedTiming {
  bool passed = false;
  TimingStatistics baseline, candidate;           // per arm
  double baselineUs = 0.0, candidateUs = 0.0;     // the medians
  double speedup = 0.0;                           // baseline / candidate median
  std::string errorMessage;
};

// Each launcher enqueues one dispatch on `stream` and returns "" on success.
inline PairedTiming measurePair(const std::function<std::string()> &baseline,
                                const std::function<std::string()> &candidate, int samples, cudaStream_t stream) {
  PairedTiming r;
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  if (cudaEventCreate(&e0) != cudaSuccess || cudaEventCreate(&e1) != cudaSuccess) {
    r.errorMessage = "event creation failed";
    if (e0) cudaEventDestroy(e0);
    return r;
  }
  std::vector<double> tb, tc;
  for (int i = 0; i < samples && r.errorMessage.empty(); ++i)
    for (int which = 0; which < 2; ++which) {
      cudaEventRecord(e0, stream);
      const std::string e = which ? candidate() : baseline();
      cudaEventRecord(e1, stream);
      if (!e.empty() || cudaEventSynchronize(e1) != cudaSuccess) {
        r.errorMessage = e.empty() ? std::string(cudaGetErrorString(cudaGetLastError())) : e;
        break;
      }
      float ms = 0.0f;
      cudaEventElapsedTime(&ms, e0, e1);
      (which ? tc : tb).push_back(ms * 1e3);
    }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (!r.errorMessage.empty()) return r;
  const auto sb = summarizeTimings(tb), sc = summarizeTimings(tc);
  if (!sb || !sc) {
    r.errorMessage = "Benchmark requires at least one sample.";
    return r;
  }
  r.baseline = *sb;
  r.candidate = *sc;
  r.baselineUs = sb->medianUs;
  r.candidateUs = sc->medianUs;
  r.speedup = r.baselineUs / r.candidateUs;
  r.passed = true;
  return r;
}

}  // namespace tensor::planner
