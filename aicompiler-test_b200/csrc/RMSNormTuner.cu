// RMSNorm tuner (see RMSNormTuner.hpp).
#include "RMSNormTuner.hpp"

#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstring>
#include <limits>

#include "half_convert.hpp"
#include "paired_timing.hpp"
#include "rmsnorm.cuh"

namespace tensor::planner {
namespace {

constexpr int kWarmup = 5;
constexpr int kSamples = 31;
constexpr double kMinimumSpeedup = 1.05;

struct Buffers {
  void *x = nullptr, *w = nullptr, *y = nullptr;
  ~Buffers() {
    cudaFree(x);
    cudaFree(w);
    cudaFree(y);
  }
};

void reject(RMSNormCandidateReport &r, const std::string &stage, const std::string &reason, std::ostream &log) {
  r.outcome = stage + " FAIL";
  r.reason = reason;
  log << r.name << " | " << r.outcome << ": " << reason << '\n';
}

}  // namespace

RMSNormTuning tuneRMSNorm(std::size_t rows, std::size_t width, float epsilon, bool fp16,
                          const std::vector<float> &input, const std::vector<float> &weight,
                          const std::vector<int> &candidateThreads, std::ostream &log) {
  RMSNormTuning result;
  if (rows == 0 || width == 0 || input.size() != rows * width || weight.size() != width ||
      rows > (std::size_t)std::numeric_limits<int>::max() || width > (std::size_t)std::numeric_limits<int>::max() ||
      !(epsilon > 0.0f)) {
    result.errorMessage = "RMSNorm tuning inputs do not match the shape or epsilon.";
    return result;
  }
  const double atol = fp16 ? 2e-3 : 1e-5, rtol = fp16 ? 2e-3 : 1e-4;
  const std::size_t elem = fp16 ? 2 : 4, count = rows * width;

  // Storage values and the fp64 reference over them (Validator.cpp:40-65).
  std::vector<float> xs(input), ws(weight);
  std::vector<std::uint16_t> xh, wh;
  if (fp16) {
    xh.resize(count);
    wh.resize(width);
    for (std::size_t i = 0; i < count; ++i) xs[i] = tensor::cuda::halfBitsToFloat(xh[i] = tensor::cuda::floatToHalfBits(input[i]));
    for (std::size_t i = 0; i < width; ++i) ws[i] = tensor::cuda::halfBitsToFloat(wh[i] = tensor::cuda::floatToHalfBits(weight[i]));
  }
  std::vector<double> reference(count);
  for (std::size_t r = 0; r < rows; ++r) {
    double ss = 0.0;
    for (std::size_t c = 0; c < width; ++c) ss += (double)xs[r * width + c] * xs[r * width + c];
    const double inv = 1.0 / std::sqrt(ss / (double)width + epsilon);
    for (std::size_t c = 0; c < width; ++c) reference[r * width + c] = (double)xs[r * width + c] * inv * ws[c];
  }

  log << "Enumerate: threads={";
  for (std::size_t i = 0; i < candidateThreads.size(); ++i) log << (i ? ", " : "") << candidateThreads[i];
  log << "}\nCPU correctness baseline: double-accumulation reference\n"
      << "GPU performance baseline: fixed 256-thread scalar RMSNorm\n"
      << "Warmup=" << kWarmup << ", samples=" << kSamples << ", admission requires >= " << kMinimumSpeedup
      << "x in two paired rounds\nMetric: one-dispatch CUDA-event duration\n"
      << "Numerical tolerance: atol=" << atol << ", rtol=" << rtol << '\n';

  Buffers b;
  if (cudaMalloc(&b.x, count * elem) != cudaSuccess || cudaMalloc(&b.w, width * elem) != cudaSuccess ||
      cudaMalloc(&b.y, count * elem) != cudaSuccess) {
    result.errorMessage = "RMSNorm tuning: device allocation failed.";
    return result;
  }
  cudaMemcpy(b.x, fp16 ? (const void *)xh.data() : (const void *)xs.data(), count * elem, cudaMemcpyHostToDevice);
  cudaMemcpy(b.w, fp16 ? (const void *)wh.data() : (const void *)ws.data(), width * elem, cudaMemcpyHostToDevice);
  cudaStream_t s = nullptr;
  if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess) {
    result.errorMessage = "RMSNorm tuning: stream creation failed.";
    return result;
  }

  // threads == 0 selects the baseline.
  auto launch = [&](int threads) -> std::string {
    const cudaError_t e =
        threads == 0 ? tmc::launch_rmsnorm_baseline(b.x, b.w, b.y, (int)rows, (int)width, epsilon, fp16, s)
                     : tmc::launch_rmsnorm(b.x, b.w, b.y, (int)rows, (int)width, epsilon, fp16, threads, s);
    return e == cudaSuccess ? std::string() : std::string(cudaGetErrorString(e));
  };
  // Run once into a NaN-filled output, read back, compare.
  auto runAndValidate = [&](int threads, std::vector<float> *out, double *maxError) -> std::string {
    cudaMemsetAsync(b.y, 0xff, count * elem, s);
    std::string e = launch(threads);
    if (!e.empty()) return "launch: " + e;
    if (cudaStreamSynchronize(s) != cudaSuccess) return std::string("execution: ") + cudaGetErrorString(cudaGetLastError());
    out->assign(count, 0.0f);
    if (fp16) {
      std::vector<std::uint16_t> h(count);
      cudaMemcpy(h.data(), b.y, count * 2, cudaMemcpyDeviceToHost);
      for (std::size_t i = 0; i < count; ++i) (*out)[i] = tensor::cuda::halfBitsToFloat(h[i]);
    } else {
      cudaMemcpy(out->data(), b.y, count * 4, cudaMemcpyDeviceToHost);
    }
    double worst = 0.0;
    for (std::size_t i = 0; i < count; ++i) {
      const double d = std::fabs((double)(*out)[i] - reference[i]);
      if (!(d <= atol + rtol * std::fabs(reference[i])))
        return "numerical: element " + std::to_string(i) + " = " + std::to_string((*out)[i]) + ", expected " +
               std::to_string(reference[i]);
      worst = std::max(worst, d);
    }
    *maxError = worst;
    return {};
  };

  std::vector<float> scratch;
  double err = 0.0;
  result.baseline.name = "baseline";
  result.baseline.threads = 256;
  if (auto e = runAndValidate(0, &scratch, &err); !e.empty()) {
    reject(result.baseline, "Validation", e, log);
    result.errorMessage = "Baseline failed; no valid fallback: " + e;
    cudaStreamDestroy(s);
    return result;
  }
  log << "baseline | Validation: PASS\n";
  for (int i = 0; i < kWarmup; ++i) launch(0);
  log << "baseline | Warmup: PASS\n";
  result.baseline.outcome = "Fallback ready";

  int winner = -1;
  double best = 1.0;
  for (int threads : candidateThreads) {
    RMSNormCandidateReport rep;
    rep.name = "candidate_" + std::to_string(threads);
    rep.threads = threads;
    result.candidates.push_back(rep);
    auto &r = result.candidates.back();
    if (threads < 32 || threads > 1024 || (threads & (threads - 1)) != 0) {
      reject(r, "Hardware Filter", "Thread count is not a power of two in [32, 1024].", log);
      continue;
    }
    if (auto e = runAndValidate(threads, &scratch, &err); !e.empty()) {
      reject(r, "Validation", e, log);
      continue;
    }
    log << r.name << " | Validation: PASS, max absolute error=" << err << '\n';
    for (int i = 0; i < kWarmup; ++i) launch(threads);
    const auto first = measurePair([&] { return launch(0); }, [&] { return launch(threads); }, kSamples, s);
    if (!first.passed) {
      reject(r, "Benchmark", first.errorMessage, log);
      continue;
    }
    r.medianGpuUs = first.candidateUs;
    r.pairedBaselineUs = first.baselineUs;
    r.speedup = first.speedup;
    log << r.name << " | Benchmark: PASS, median(us)=" << first.candidateUs
        << ", paired baseline(us)=" << first.baselineUs << ", speedup=" << first.speedup << "x\n";
    if (first.speedup < kMinimumSpeedup) {
      reject(r, "Compare Baseline", "Speedup is below 1.05x.", log);
      continue;
    }
    const auto second = measurePair([&] { return launch(0); }, [&] { return launch(threads); }, kSamples, s);
    if (!second.passed) {
      reject(r, "Confirmation Benchmark", second.errorMessage, log);
      continue;
    }
    log << r.name << " | Confirmation: median(us)=" << second.candidateUs
        << ", paired baseline(us)=" << second.baselineUs << ", speedup=" << second.speedup << "x\n";
    r.speedup = std::min(first.speedup, second.speedup);
    if (*r.speedup < kMinimumSpeedup) {
      reject(r, "Compare Baseline", "Confirmation did not reach 1.05x.", log);
      continue;
    }
    r.outcome = "Admitted";
    log << r.name << " | Compare Baseline: PASS -> Admit\n";
    if (*r.speedup > best) {
      best = *r.speedup;
      winner = (int)result.candidates.size() - 1;
    }
  }

  // The selection once more, into a fresh NaN-filled output.
  std::string finalError;
  if (winner >= 0) {
    finalError = runAndValidate(result.candidates[winner].threads, &result.output, &result.maxAbsoluteError);
    if (!finalError.empty()) {
      reject(result.candidates[winner], "Final execution", finalError, log);
      log << "Selected candidate failed; executing the retained baseline.\n";
      winner = -1;
    }
  }
  if (winner < 0) finalError = runAndValidate(0, &result.output, &result.maxAbsoluteError);
  cudaStreamDestroy(s);
  if (!finalError.empty()) {
    result.errorMessage = "Final baseline execution/validation failed: " + finalError;
    return result;
  }
  result.usedBaseline = winner < 0;
  result.selectedThreads = winner < 0 ? 256 : result.candidates[winner].threads;
  result.success = true;
  log << "Selected: " << (result.usedBaseline ? std::string("baseline (fallback)") : result.candidates[winner].name)
      << ", threads=" << result.selectedThreads << "\nFinal GPU execution: PASS\nFinal numerical validation: PASS"
      << ", max absolute error=" << result.maxAbsoluteError << '\n';
  return result;
}

}  // namespace tensor::planner
