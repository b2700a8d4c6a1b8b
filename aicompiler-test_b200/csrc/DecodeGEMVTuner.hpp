// Decode GEMV tuning with an admission gate: the B200 counterpart of the
// reference's tuneDecodeGEMV / DecodeGEMVSelection
// (src/planner/DecodeGEMVTuner.hpp:13-25, DecodeGEMVTuner.cpp:162-304).
//
// The baseline is a generic linear kernel (one CTA per output feature and
// row) in the storage dtype. Decode candidates (batch <= 8) are
// configurations of the decode GEMV (K-split team size 1/2/4/8, with and
// without dynamic row scheduling); the prefill candidate (batch <= 128) is
// the tcgen05 tensor-core GEMM (the reference's tiled-GEMM candidate set,
// DecodeGEMVTuner.cpp:209-213). Both read fp16 weights, so with fp32 storage
// every candidate fails the hardware filter and the baseline is kept. Each
// candidate is validated against an fp64 CPU reference when the shape has at
// most 64M multiply-adds (otherwise against the baseline's output, with 9
// samples instead of 31), then timed in two paired rounds of alternating
// samples; it is admitted when both rounds reach 1.05x, and the fastest
// admitted one is selected.
#pragma once

#include <cstddef>
#include <ostream>
#include <string>
#include <vector>

namespace tensor::planner {

struct DecodeGEMVConfig {
  int ks = 0;               // K-split team size (0: the built-in rule)
  bool dynamic = false;     // pooled dynamic row scheduling
  bool tensorCore = false;  // the tcgen05 GEMM (prefill candidate)
};

struct DecodeGEMVSelection {
  bool success = false;
  bool useBaseline = true;
  DecodeGEMVConfig config;
  double conservativeSpeedup = 1.0;
  std::string errorMessage;
};

// input [batch, inputSize] and weight [outputSize, inputSize] are logical
// values stored as fp16 (fp16Storage) or fp32; batch <= 8 for decode, <= 128
// for prefill; inputSize % 8 == 0.
DecodeGEMVSelection tuneDecodeGEMV(std::size_t batch, std::size_t inputSize, std::size_t outputSize,
                                   const std::vector<float> &input, const std::vector<float> &weight,
                                   std::ostream &log, bool fp16Storage = true, bool prefill = false);

}  // namespace tensor::planner
