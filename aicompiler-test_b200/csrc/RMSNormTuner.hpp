// RMSNorm tuner: the B200 counterpart of tuneRMSNorm (RMSNormTuner.hpp:14-44,
// RMSNormTuner.cpp:159-309). Candidates are block sizes of the vectorised
// RMSNorm kernel; the baseline is the frozen 256-thread scalar kernel. Every
// launch is validated against an fp64 CPU reference (fp32 storage: atol 1e-5,
// rtol 1e-4; fp16: 2e-3 / 2e-3, RMSNormTuner.cpp:19-20,75-76), then timed in
// two paired rounds of 31 samples after 5 warm-ups; a candidate is admitted
// when both rounds reach 1.05x and ranked by the lower of the two. The
// selection runs once more into a NaN-filled output and is validated again;
// if that fails the baseline is used.
#pragma once

#include <cstddef>
#include <optional>
#include <ostream>
#include <string>
#include <vector>

namespace tensor::planner {

struct RMSNormCandidateReport {
  std::string name;
  int threads = 0;
  std::string outcome;
  std::string reason;
  std::optional<double> medianGpuUs, pairedBaselineUs, speedup;
};

struct RMSNormTuning {
  bool success = false;
  bool usedBaseline = true;
  int selectedThreads = 256;
  RMSNormCandidateReport baseline;
  std::vector<RMSNormCandidateReport> candidates;
  std::vector<float> output;  // the final execution's output, as fp32 values
  double maxAbsoluteError = 0.0;
  std::string errorMessage;
};

// input [rows, width], weight [width]: logical values, stored as fp16 when
// `fp16` (the tuner rounds them) else fp32.
RMSNormTuning tuneRMSNorm(std::size_t rows, std::size_t width, float epsilon, bool fp16,
                          const std::vector<float> &input, const std::vector<float> &weight,
                          const std::vector<int> &candidateThreads, std::ostream &log);

}  // namespace tensor::planner
