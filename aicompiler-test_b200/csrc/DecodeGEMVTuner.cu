// Decode GEMV tuner (see DecodeGEMVTuner.hpp).
#include "DecodeGEMVTuner.hpp"

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <sstream>

#include "gemm.cuh"
#include "gemv.cuh"
#include "half_convert.hpp"
#include "paired_timing.hpp"

namespace tensor::planner {
namespace {

constexpr double kMaximumCpuReferenceOperations = 64.0 * 1024 * 1024;
constexpr int kWarmup = 5;
constexpr int kSamples = 31;
constexpr int kLargeShapeSamples = 9;  // the reference's count without a CPU reference
constexpr double kMinimumSpeedup = 1.05;

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ float to_f<__half>(__half v) {
  return __half2float(v);
}

// The generic linear layer: CTA (j, m) computes y[m, j] with a strided K loop
// and a block reduction.
template <typename T>
__global__ void linear_baseline(const T *x, const T *w, float *y, int k, int n) {
  const int j = blockIdx.x, m = blockIdx.y;
  float s = 0.0f;
  for (int i = threadIdx.x; i < k; i += blockDim.x) s += to_f(x[(size_t)m * k + i]) * to_f(w[(size_t)j * k + i]);
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
  void *x = nullptr, *w = nullptr, *ws = nullptr;
  float *y = nullptr;
  unsigned *counters = nullptr, *tickets = nullptr;
  ~DeviceBuffers() {
    cudaFree(x);
    cudaFree(w);
    cudaFree(ws);
    cudaFree(y);
    cudaFree(counters);
    cudaFree(tickets);
  }
};

}  // namespace

DecodeGEMVSelection tuneDecodeGEMV(std::size_t batch, std::size_t k, std::size_t n, const std::vector<float> &input,
                                   const std::vector<float> &weight, std::ostream &log, bool fp16Storage,
                                   bool prefill) {
  DecodeGEMVSelection result;
  const std::size_t maxBatch = prefill ? 128 : 8;
  if (batch < 1 || batch > maxBatch || n < 1 || k % 8 != 0 || input.size() != batch * k || weight.size() != n * k) {
    result.errorMessage = "Decode GEMV tuning inputs do not match the shape (batch <= " + std::to_string(maxBatch) +
                          ", K % 8 == 0).";
    return result;
  }
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // Storage values of the inputs (what the kernels read) and their fp32 view.
  const std::size_t elem = fp16Storage ? 2 : 4;
  std::vector<std::uint16_t> xh, wh;
  std::vector<float> xr(input), wr(weight);
  if (fp16Storage) {
    xh.resize(input.size());
    wh.resize(weight.size());
    for (std::size_t i = 0; i < xh.size(); ++i)
      xr[i] = tensor::cuda::halfBitsToFloat(xh[i] = tensor::cuda::floatToHalfBits(input[i]));
    for (std::size_t i = 0; i < wh.size(); ++i)
      wr[i] = tensor::cuda::halfBitsToFloat(wh[i] = tensor::cuda::floatToHalfBits(weight[i]));
  }
  DeviceBuffers b;
  const std::size_t outs = batch * n;
  if (cudaMalloc(&b.x, input.size() * elem) != cudaSuccess || cudaMalloc(&b.w, weight.size() * elem) != cudaSuccess ||
      cudaMalloc(reinterpret_cast<void **>(&b.y), outs * 4) != cudaSuccess ||
      cudaMalloc(reinterpret_cast<void **>(&b.counters), tmc::kGemvCounterWords * 4) != cudaSuccess) {
    result.errorMessage = "Decode GEMV tuning: device allocation failed.";
    return result;
  }
  cudaMemcpy(b.x, fp16Storage ? (const void *)xh.data() : (const void *)xr.data(), input.size() * elem,
             cudaMemcpyHostToDevice);
  cudaMemcpy(b.w, fp16Storage ? (const void *)wh.data() : (const void *)wr.data(), weight.size() * elem,
             cudaMemcpyHostToDevice);
  cudaMemset(b.counters, 0, tmc::kGemvCounterWords * 4);
  cudaStream_t s = nullptr;
  cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);

  // Tensor-core GEMM state (prefill candidate): plan, tensor maps, workspace,
  // zeroed tile counters.
  tmc::GemmPlan plan{};
  CUtensorMap wmap{}, xmap{};
  bool gemmReady = false;
  if (prefill && fp16Storage) {
    plan = tmc::plan_gemm((int)n, (int)k, (int)batch, sms);
    const size_t wsFloats = tmc::gemm_workspace_floats(plan);
    gemmReady = tmc::make_tensor_map_f16(&wmap, b.w, n, k, tmc::kGemmTileRows) == cudaSuccess &&
                tmc::make_tensor_map_f16(&xmap, b.x, batch, k, plan.tn) == cudaSuccess &&
                (wsFloats == 0 || cudaMalloc(&b.ws, wsFloats * 4) == cudaSuccess) &&
                cudaMalloc(reinterpret_cast<void **>(&b.tickets), (size_t)plan.tiles * 8) == cudaSuccess &&
                cudaMemset(b.tickets, 0, (size_t)plan.tiles * 8) == cudaSuccess;
  }

  auto runBaseline = [&]() -> cudaError_t {
    if (fp16Storage)
      linear_baseline<__half><<<dim3((unsigned)n, (unsigned)batch), 128, 0, s>>>(
          static_cast<const __half *>(b.x), static_cast<const __half *>(b.w), b.y, (int)k, (int)n);
    else
      linear_baseline<float><<<dim3((unsigned)n, (unsigned)batch), 128, 0, s>>>(
          static_cast<const float *>(b.x), static_cast<const float *>(b.w), b.y, (int)k, (int)n);
    return cudaGetLastError();
  };
  auto runCandidate = [&](const DecodeGEMVConfig &c) -> cudaError_t {
    tmc::GemvParams p{};
    p.W = static_cast<const __half *>(b.w);
    p.N = (int)n;
    p.K = (int)k;
    p.M = (int)batch;
    p.prologue = tmc::kProF16;
    p.x = b.x;
    p.x_stride = (long long)k;
    p.epilogue = tmc::kEpiF32;
    p.y_f32 = b.y;
    p.y_stride = (long long)n;
    if (c.tensorCore) return tmc::launch_gemm(p, wmap, xmap, plan, static_cast<float *>(b.ws), b.tickets, s, false);
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
  const int samples = cpuReference ? kSamples : kLargeShapeSamples;
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
  log << "Decode GEMV shape M=" << batch << ", K=" << k << ", N=" << n << ", dtype=" << (fp16Storage ? "fp16" : "fp32")
      << ", samples=" << samples << " | baseline validation/warmup: PASS\n";

  auto measure = [&](const DecodeGEMVConfig &c, double *speedup) -> std::string {
    const auto t = measurePair([&] { return runBaseline() == cudaSuccess ? std::string() : "baseline launch failed"; },
                               [&] { return runCandidate(c) == cudaSuccess ? std::string() : "candidate launch failed"; },
                               samples, s);
    *speedup = t.speedup;
    return t.errorMessage;
  };
  std::vector<DecodeGEMVConfig> candidates;
  if (prefill)
    candidates = {{0, false, true}};
  else
    candidates = {{1, false}, {2, false}, {4, false}, {8, false}, {1, true}};
  double best = 1.0;
  for (const auto &c : candidates) {
    if (c.tensorCore)
      log << "  candidate tcgen05 GEMM (tn=" << plan.tn << ", tiles=" << plan.tiles << ", grid=" << plan.grid << ")";
    else
      log << "  candidate ks=" << c.ks << ", dynamic=" << (c.dynamic ? "true" : "false");
    // Hardware filter: the candidates read fp16 weights; the GEMM needs its
    // tensor maps and workspace.
    if (!fp16Storage || (c.tensorCore && !gemmReady)) {
      log << " | Hardware Filter: FAIL\n";
      continue;
    }
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
  else if (result.config.tensorCore)
    log << "Decode GEMV selected: tcgen05 GEMM, conservative speedup=" << result.conservativeSpeedup << "x\n";
  else
    log << "Decode GEMV selected: ks=" << result.config.ks << ", dynamic=" << (result.config.dynamic ? "true" : "false")
        << ", conservative speedup=" << result.conservativeSpeedup << "x\n";
  return result;
}

}  // namespace tensor::planner
