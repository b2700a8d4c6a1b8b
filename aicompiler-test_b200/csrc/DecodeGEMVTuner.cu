// Decode GEMV tuner (see DecodeGEMVTuner.hpp).
#include "DecodeGEMVTuner.hpp"

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <memory>
#include <sstream>

#include "gemv.cuh"
#include "half_convert.hpp"
#include "paired_timing.hpp"

namespace tensor::planner {
namespace {

constexpr double kMaximumCpuReferenceOperations = 64.0 * 1024 * 1024;
constexpr int kWarmup = 5;
constexpr int kSamples = 31;
constexpr double kMinimumSpeedup = 1.05;

// The generic linear layer: CTA (j, m) computes y[m, j] with a strided K loop
// and a block reduction.
__global__ void linear_baseline(const __half *x, const __half *w, float *y, int k, int n) {
  const int j = blockIdx.x, m = blockIdx.y;
  float s = 0.0f;
  for (int i = threadIdx.x; i < k; i += blockDim.x)
    s += __half2float(x[(size_t)m * k + i]) * __half2float(w[(size_t)j * k + i]);
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  __shared__ float part[32];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.0f;
    for (int i = 0; i < (int)(blockDim.x / 32); ++i) t += part[i];
    y[(size_t)m * n + j] = t;
  }
}

struct DeviceBuffers {
  __half *x = nullptr, *w = nullptr;
  float *y = nullptr;
  unsigned *counters = nullptr;
  ~DeviceBuffers() {
    cudaFree(x);
    cudaFree(w);
    cudaFree(y);
    cudaFree(counters);
  }
};

}  // namespace

DecodeGEMVSelection tuneDecodeGEMV(std::size_t batch, std::size_t k, std::size_t n, const std::vector<float> &input,
                                   const std::vector<float> &weight, std::ostream &log) {
  DecodeGEMVSelection result;
  if (batch < 1 || batch > 8 || k % 8 != 0 || input.size() != batch * k || weight.size() != n * k) {
    result.errorMessage = "Decode GEMV tuning inputs do not match the shape (batch <= 8, K % 8 == 0).";
    return result;
  }
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // fp16 storage of the inputs (what the kernels read).
  std::vector<std::uint16_t> xh(input.size()), wh(weight.size());
  std::vector<float> xr(input.size()), wr(weight.size());
  for (std::size_t i = 0; i < xh.size(); ++i) {
    xh[i] = tensor::cuda::floatToHalfBits(input[i]);
    xr[i] = tensor::cuda::halfBitsToFloat(xh[i]);
  }
  for (std::size_t i = 0; i < wh.size(); ++i) {
    wh[i] = tensor::cuda::floatToHalfBits(weight[i]);
    wr[i] = tensor::cuda::halfBitsToFloat(wh[i]);
  }
  DeviceBuffers b;
  const std::size_t outs = batch * n;
  if (cudaMalloc(&b.x, xh.size() * 2) != cudaSuccess || cudaMalloc(&b.w, wh.size() * 2) != cudaSuccess ||
      cudaMalloc(&b.y, outs * 4) != cudaSuccess ||
      cudaMalloc(&b.counters, tmc::kGemvCounterWords * 4) != cudaSuccess) {
    result.errorMessage = "Decode GEMV tuning: device allocation failed.";
    return result;
  }
  cudaMemcpy(b.x, xh.data(), xh.size() * 2, cudaMemcpyHostToDevice);
  cudaMemcpy(b.w, wh.data(), wh.size() * 2, cudaMemcpyHostToDevice);
  cudaMemset(b.counters, 0, tmc::kGemvCounterWords * 4);
  cudaStream_t s = nullptr;
  cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);

  auto runBaseline = [&]() -> cudaError_t {
    linear_baseline<<<dim3((unsigned)n, (unsigned)batch), 128, 0, s>>>(b.x, b.w, b.y, (int)k, (int)n);
    return cudaGetLastError();
  };
  auto runCandidate = [&](const DecodeGEMVConfig &c) -> cudaError_t {
    tmc::GemvParams p{};
    p.W = b.w;
    p.N = (int)n;
    p.K = (int)k;
    p.M = (int)batch;
    p.prologue = tmc::kProF16;
    p.x = b.x;
    p.x_stride = (long long)k;
    p.epilogue = tmc::kEpiF32;
    p.y_f32 = b.y;
    p.y_stride = (long long)n;
    p.force_ks = c.ks;
    p.work_counter = c.dynamic ? b.counters : nullptr;
    return tmc::launch_gemv(p, s, false, sms);
  };
  auto readOutputs = [&]() {
    std::vector<float> y(outs);
    cudaMemcpy(y.data(), b.y, outs * 4, cudaMemcpyDeviceToHost);
    return y;
  };
  // Reference: fp64 on the CPU for small shapes, else the baseline's output.
  const bool cpuReference = (double)batch * k * n <= kMaximumCpuReferenceOperations;
  std::vector<double> expected(outs);
  if (cpuReference) {
    for (std::size_t m = 0; m < batch; ++m)
      for (std::size_t j = 0; j < n; ++j) {
        double t = 0;
        for (std::size_t i = 0; i < k; ++i) t += (double)xr[m * k + i] * wr[j * k + i];
        expected[m * n + j] = t;
      }
  }
  auto validate = [&](const char *what) -> std::string {
    if (cudaStreamSynchronize(s) != cudaSuccess) return std::string(what) + ": " + cudaGetErrorString(cudaGetLastError());
    const auto y = readOutputs();
    for (std::size_t i = 0; i < outs; ++i)
      if (!(std::fabs(y[i] - expected[i]) <= 1e-3 + 1e-3 * std::fabs(expected[i]))) {
        std::ostringstream m;
        m << what << ": output " << i << " = " << y[i] << ", expected " << expected[i];
        return m.str();
      }
    return {};
  };
  if (runBaseline() != cudaSuccess) {
    result.errorMessage = "Decode GEMV baseline launch failed.";
    cudaStreamDestroy(s);
    return result;
  }
  if (cpuReference) {
    const auto e = validate("baseline");
    if (!e.empty()) {
      result.errorMessage = "Decode GEMV baseline failed: " + e;
      cudaStreamDestroy(s);
      return result;
    }
  } else {
    cudaStreamSynchronize(s);
    const auto y = readOutputs();
    expected.assign(y.begin(), y.end());
    log << "Decode GEMV large-shape validation: baseline GPU reference selected\n";
  }
  for (int i = 0; i < kWarmup; ++i) runBaseline();
  log << "Decode GEMV shape M=" << batch << ", K=" << k << ", N=" << n << ", dtype=fp16, samples=" << kSamples
      << " | baseline validation/warmup: PASS\n";

  auto measure = [&](const DecodeGEMVConfig &c, double *speedup) -> std::string {
    const auto t = measurePair([&] { return runBaseline() == cudaSuccess ? std::string() : "baseline launch failed"; },
                               [&] { return runCandidate(c) == cudaSuccess ? std::string() : "candidate launch failed"; },
                               kSamples, s);
    *speedup = t.speedup;
    return t.errorMessage;
  };
  const std::vector<DecodeGEMVConfig> candidates = {{1, false}, {2, false}, {4, false}, {8, false}, {1, true}};
  double best = 1.0;
  for (const auto &c : candidates) {
    log << "  candidate ks=" << c.ks << ", dynamic=" << (c.dynamic ? "true" : "false");
    cudaMemsetAsync(b.y, 0xff, outs * 4, s);
    if (runCandidate(c) != cudaSuccess) {
      log << " | Launch: FAIL\n";
      cudaGetLastError();
      continue;
    }
    const auto e = validate("candidate");
    if (!e.empty()) {
      log << " | numerical: FAIL: " << e << '\n';
      continue;
    }
    for (int i = 0; i < kWarmup; ++i) runCandidate(c);
    double first = 0, second = 0;
    auto err = measure(c, &first);
    if (!err.empty()) {
      log << " | Benchmark: FAIL: " << err << '\n';
      continue;
    }
    log << " | validation: PASS, speedup=" << first << 'x';
    if (first < kMinimumSpeedup) {
      log << " -> fallback\n";
      continue;
    }
    err = measure(c, &second);
    if (!err.empty()) {
      log << ", confirmation: FAIL: " << err << '\n';
      continue;
    }
    const double conservative = std::min(first, second);
    log << ", confirmation=" << second << 'x';
    if (conservative < kMinimumSpeedup) {
      log << " -> fallback\n";
      continue;
    }
    log << " -> admitted\n";
    if (conservative > best) {
      best = conservative;
      result.useBaseline = false;
      result.config = c;
      result.conservativeSpeedup = conservative;
    }
  }
  cudaStreamDestroy(s);
  result.success = true;
  if (result.useBaseline)
    log << "Decode GEMV selected: generic Linear fallback\n";
  else
    log << "Decode GEMV selected: ks=" << result.config.ks << ", dynamic=" << (result.config.dynamic ? "true" : "false")
        << ", conservative speedup=" << result.conservativeSpeedup << "x\n";
  return result;
}

}  // namespace tensor::planner
