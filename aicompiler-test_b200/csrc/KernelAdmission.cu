// Generated-kernel contracts, admission gate and registry (see KernelAdmission.hpp).
#include "KernelAdmission.hpp"

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <nvrtc.h>

#include <dlfcn.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <filesystem>
#include <optional>
#include <fstream>
#include <mutex>
#include <sstream>
#include <stdexcept>

#include "half_convert.hpp"

namespace tensor::runtime {
namespace {

constexpr std::size_t kMaximumGeneratedGEMVWeightElements = 8u * 1024u * 1024u;
constexpr int kWarmup = 5;
constexpr int kSamples = 31;
constexpr int kBaselineBlock = 64;

// ---- the contract fixtures ---------------------------------------------------
// Deterministic values in [-1, 1) with 1/128 steps (exact in fp16 and bf16), as
// the reference's fixtures are generated (DecoderKernelContracts.cpp:22-27).
std::vector<float> values(std::size_t count, std::size_t seed, float scale = 1.0f) {
  std::vector<float> r(count);
  for (std::size_t i = 0; i < count; ++i) r[i] = float(int((i * 17 + seed * 31) % 257) - 128) / 128 * scale;
  return r;
}
double dot(const std::vector<float> &x, const std::vector<float> &w, std::size_t feature, std::size_t width) {
  double s = 0;
  for (std::size_t i = 0; i < width; ++i) s += double(x[i]) * w[feature * width + i];
  return s;
}
std::pair<std::size_t, std::size_t> gemvShape(const std::string &pattern) {
  const std::string prefix = "decoder_gemv_";
  if (pattern.rfind(prefix, 0) != 0) return {0, 0};
  const auto rest = pattern.substr(prefix.size());
  const auto cut = rest.find('_');
  if (cut == std::string::npos) return {0, 0};
  try {
    std::size_t a = 0, b = 0;
    const auto k = std::stoul(rest.substr(0, cut), &a);
    const auto n = std::stoul(rest.substr(cut + 1), &b);
    if (a != cut || b != rest.size() - cut - 1 || k == 0 || n == 0) return {0, 0};
    return {k, n};
  } catch (const std::exception &) {
    return {0, 0};
  }
}
// Round to fp16 storage (RNE) as a double.
double roundHalf(double v) {
  return cuda::halfBitsToFloat(cuda::floatToHalfBits(static_cast<float>(v)));
}

KernelContract baseContract(const std::string &pattern) {
  KernelContract c;
  c.pattern = pattern;
  c.functionName = "generated_" + pattern;
  c.applicability = "Decoder-only fp32, batch=1, sequence_length=1; no prefill replacement";
  const auto [k, n] = gemvShape(pattern);
  if (k) {
    if (n > kMaximumGeneratedGEMVWeightElements / k)
      throw std::invalid_argument("Generated GEMV contract fixture exceeds 8M weight elements.");
    c.inputNames = {"input", "weight"};
    c.outputNames = {"output"};
    c.workItem = "one output feature per CTA; reduce over K";
    c.semantics = "Bias-free output[j]=sum_i input[i]*weight[j*K+i], row-major weight [N,K], M=1, K=" +
                  std::to_string(k) + ", N=" + std::to_string(n) + ". CTA j owns output[j].";
  } else if (pattern == "decoder_rope") {
    c.groupPerWorkItem = false;
    c.inputNames = {"query", "key", "cosine", "sine", "valid_length"};
    c.outputNames = {"rotated_query", "rotated_key"};
    c.workItem = "one interleaved pair in both Q and K";
    c.applicability += "; hidden=64, heads=4, head_dim=16, cache_capacity=32";
    c.semantics = "Q/K are contiguous [1,1,64]. cosine/sine are position tables [32,8]. valid_length is a "
                  "read-only int [1] including the appended token (1..32). For p<32, c=cosine[(valid_length-1)*8"
                  "+p%8], s=sine[...]; out[2p]=in[2p]*c-in[2p+1]*s; out[2p+1]=in[2p]*s+in[2p+1]*c.";
  } else if (pattern == "decoder_residual_rmsnorm") {
    c.inputNames = {"residual", "update", "weight"};
    c.outputNames = {"sum", "normalized"};
    c.workItem = "one width-64 row per CTA";
    c.applicability += "; hidden=64, rms_epsilon=1e-5";
    c.semantics = "For i<64, sum[i]=residual[i]+update[i]; normalized[i]=sum[i]*rsqrt(mean_j(sum[j]^2)+1e-5)"
                  "*weight[i]. Both outputs [1,64] are required.";
  } else if (pattern == "decoder_gated_mlp") {
    c.inputNames = {"input", "gate_weight", "up_weight"};
    c.outputNames = {"gated"};
    c.workItem = "one intermediate feature per CTA; reduce over hidden=64";
    c.applicability += "; hidden=64, intermediate=128";
    c.semantics = "Input [1,64], gate_weight/up_weight row-major [128,64], no biases. For j<128: gate=sum_i "
                  "input[i]*gate_weight[j*64+i], up=likewise, gated[j]=(gate/(1+exp(-gate)))*up.";
  } else {
    throw std::invalid_argument("Unsupported generated-kernel pattern: " + pattern);
  }
  c.inputTypes.assign(c.inputNames.size(), ContractType::Float32);
  if (pattern == "decoder_rope") c.inputTypes.back() = ContractType::Int32;
  for (std::size_t seed = 1; seed <= 3; ++seed) {
    KernelCase d;
    if (k) {
      d.shape = {1, k, n};
      d.inputs = {values(k, seed), values(k * n, seed + 9, 0.125f)};
      d.references = {std::vector<double>(n)};
      d.workItems = n;
      for (std::size_t j = 0; j < n; ++j) d.references[0][j] = dot(d.inputs[0], d.inputs[1], j, k);
    } else if (pattern == "decoder_rope") {
      const std::size_t length = seed == 1 ? 9 : seed == 2 ? 16 : 32;
      d.shape = {1, 4, 1, 16};
      d.inputs = {values(64, seed), values(64, seed + 1), std::vector<float>(256), std::vector<float>(256),
                  {float(length)}};
      d.references.assign(2, std::vector<double>(64));
      d.workItems = 32;
      for (std::size_t position = 0; position < 32; ++position)
        for (std::size_t pair = 0; pair < 8; ++pair) {
          const auto angle = position * std::pow(10000.0, -double(pair) / 8);
          d.inputs[2][position * 8 + pair] = float(std::cos(angle));
          d.inputs[3][position * 8 + pair] = float(std::sin(angle));
        }
      for (std::size_t out = 0; out < 2; ++out)
        for (std::size_t p = 0; p < 32; ++p) {
          const auto index = (length - 1) * 8 + p % 8;
          const double a = d.inputs[out][2 * p], b = d.inputs[out][2 * p + 1];
          d.references[out][2 * p] = a * d.inputs[2][index] - b * d.inputs[3][index];
          d.references[out][2 * p + 1] = a * d.inputs[3][index] + b * d.inputs[2][index];
        }
    } else if (pattern == "decoder_residual_rmsnorm") {
      d.shape = {1, 64};
      d.inputs = {values(64, seed), values(64, seed + 7, 0.5f), values(64, seed + 4, 0.25f)};
      for (auto &w : d.inputs[2]) w += 1;
      d.references.assign(2, std::vector<double>(64));
      d.workItems = 1;
      double squares = 0;
      for (std::size_t i = 0; i < 64; ++i) {
        const float sum = d.inputs[0][i] + d.inputs[1][i];
        d.references[0][i] = sum;
        squares += double(sum) * sum;
      }
      for (std::size_t i = 0; i < 64; ++i)
        d.references[1][i] = d.references[0][i] / std::sqrt(squares / 64 + 1e-5) * d.inputs[2][i];
    } else {
      d.shape = {1, 64, 128};
      d.inputs = {values(64, seed), values(128 * 64, seed + 3, 0.125f), values(128 * 64, seed + 5, 0.125f)};
      d.references = {std::vector<double>(128)};
      d.workItems = 128;
      for (std::size_t j = 0; j < 128; ++j) {
        const double gate = dot(d.inputs[0], d.inputs[1], j, 64);
        d.references[0][j] = gate / (1 + std::exp(-gate)) * dot(d.inputs[0], d.inputs[2], j, 64);
      }
    }
    c.cases.push_back(std::move(d));
  }
  return c;
}

// ---- template baselines (the kernels a candidate must beat) --------------------
template <typename T>
__device__ __forceinline__ float ld(const T *p, size_t i) {
  return static_cast<float>(p[i]);
}
template <>
__device__ __forceinline__ float ld<__half>(const __half *p, size_t i) {
  return __half2float(p[i]);
}
template <typename T>
__device__ __forceinline__ T st(float v);
template <>
__device__ __forceinline__ float st<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ __half st<__half>(float v) {
  return __float2half_rn(v);
}
template <typename T>
__device__ __forceinline__ float rnd(float v) {
  return static_cast<float>(st<T>(v));
}
template <>
__device__ __forceinline__ float rnd<__half>(float v) {
  return __half2float(__float2half_rn(v));
}

__device__ float block_reduce_sum(float v) {
  __shared__ float part[32];
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = 0.0f;
  if (threadIdx.x < 32) {
    r = threadIdx.x < (blockDim.x + 31) / 32 ? part[threadIdx.x] : 0.0f;
    for (int o = 16; o > 0; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
    if (threadIdx.x == 0) part[0] = r;
  }
  __syncthreads();
  r = part[0];
  __syncthreads();
  return r;
}

template <typename T>
__global__ void template_gemv(const T *x, const T *w, T *y, unsigned k) {
  const unsigned j = blockIdx.x;
  float s = 0.0f;
  for (unsigned i = threadIdx.x; i < k; i += blockDim.x) s += ld(x, i) * ld(w, (size_t)j * k + i);
  s = block_reduce_sum(s);
  if (threadIdx.x == 0) y[j] = st<T>(s);
}
template <typename T>
__global__ void template_rope(const T *q, const T *kin, const float *cosine, const float *sine, const int *valid,
                              T *qo, T *ko) {
  const unsigned p = blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= 32) return;
  const int index = (valid[0] - 1) * 8 + p % 8;
  const float c = cosine[index], s = sine[index];
  const T *in[2] = {q, kin};
  T *out[2] = {qo, ko};
  for (int o = 0; o < 2; ++o) {
    const float a = ld(in[o], 2 * p), b = ld(in[o], 2 * p + 1);
    out[o][2 * p] = st<T>(a * c - b * s);
    out[o][2 * p + 1] = st<T>(a * s + b * c);
  }
}
template <typename T>
__global__ void template_residual_rmsnorm(const T *res, const T *upd, const T *w, T *sum, T *norm) {
  float sq = 0.0f;
  for (unsigned i = threadIdx.x; i < 64; i += blockDim.x) {
    const float v = rnd<T>(ld(res, i) + ld(upd, i));
    sq += v * v;
  }
  sq = block_reduce_sum(sq);
  const float inv = rsqrtf(sq / 64.0f + 1e-5f);
  for (unsigned i = threadIdx.x; i < 64; i += blockDim.x) {
    const float v = rnd<T>(ld(res, i) + ld(upd, i));
    sum[i] = st<T>(v);
    norm[i] = st<T>(v * inv * ld(w, i));
  }
}
template <typename T>
__global__ void template_gated_mlp(const T *x, const T *wg, const T *wu, T *y) {
  const unsigned j = blockIdx.x;
  float g = 0.0f, u = 0.0f;
  for (unsigned i = threadIdx.x; i < 64; i += blockDim.x) {
    g += ld(x, i) * ld(wg, (size_t)j * 64 + i);
    u += ld(x, i) * ld(wu, (size_t)j * 64 + i);
  }
  g = rnd<T>(block_reduce_sum(g));
  u = rnd<T>(block_reduce_sum(u));
  if (threadIdx.x == 0) y[j] = st<T>(rnd<T>(g / (1.0f + expf(-g))) * u);
}

// ---- device buffers of a case ------------------------------------------------
struct DeviceCase {
  std::vector<void *> buffers;  // inputs then outputs
  std::vector<std::size_t> counts;
  std::vector<ContractType> types;
  ~DeviceCase() {
    for (void *b : buffers)
      if (b) cudaFree(b);
  }
};

std::size_t typeBytes(ContractType t) { return t == ContractType::Float16 ? 2 : 4; }

std::string upload(const KernelContract &c, const KernelCase &d, DeviceCase *dc) {
  for (std::size_t i = 0; i < d.inputs.size() + d.references.size(); ++i) {
    const bool in = i < d.inputs.size();
    const ContractType t = in ? c.inputTypes[i] : c.storageType;
    const std::size_t n = in ? d.inputs[i].size() : d.references[i - d.inputs.size()].size();
    void *p = nullptr;
    if (cudaMalloc(&p, std::max<std::size_t>(n, 1) * typeBytes(t)) != cudaSuccess) return "cudaMalloc failed";
    dc->buffers.push_back(p);
    dc->counts.push_back(n);
    dc->types.push_back(t);
    if (!in) {
      cudaMemset(p, 0xff, n * typeBytes(t));  // NaN sentinel: unwritten outputs fail validation
      continue;
    }
    std::vector<unsigned char> host(n * typeBytes(t));
    for (std::size_t e = 0; e < n; ++e) {
      const float v = d.inputs[i][e];
      if (t == ContractType::Float16) {
        const std::uint16_t h = cuda::floatToHalfBits(v);
        std::memcpy(host.data() + 2 * e, &h, 2);
      } else if (t == ContractType::Int32) {
        const std::int32_t iv = static_cast<std::int32_t>(v);
        std::memcpy(host.data() + 4 * e, &iv, 4);
      } else {
        std::memcpy(host.data() + 4 * e, &v, 4);
      }
    }
    if (cudaMemcpy(p, host.data(), host.size(), cudaMemcpyHostToDevice) != cudaSuccess) return "upload failed";
  }
  return {};
}

std::string validate(const KernelContract &c, const KernelCase &d, const DeviceCase &dc) {
  for (std::size_t o = 0; o < d.references.size(); ++o) {
    const std::size_t b = d.inputs.size() + o;
    const std::size_t n = dc.counts[b];
    std::vector<unsigned char> host(n * typeBytes(dc.types[b]));
    if (cudaMemcpy(host.data(), dc.buffers[b], host.size(), cudaMemcpyDeviceToHost) != cudaSuccess)
      return "readback failed";
    for (std::size_t e = 0; e < n; ++e) {
      double v;
      if (dc.types[b] == ContractType::Float16) {
        std::uint16_t h;
        std::memcpy(&h, host.data() + 2 * e, 2);
        v = cuda::halfBitsToFloat(h);
      } else {
        float f;
        std::memcpy(&f, host.data() + 4 * e, 4);
        v = f;
      }
      const double r = d.references[o][e];
      if (!(std::fabs(v - r) <= c.absoluteTolerance + c.relativeTolerance * std::fabs(r))) {
        std::ostringstream m;
        m << c.outputNames[o] << "[" << e << "] = " << v << ", expected " << r;
        return m.str();
      }
    }
  }
  return {};
}

std::string launchBaseline(const KernelContract &c, const KernelCase &d, const DeviceCase &dc, cudaStream_t s) {
  const bool half = c.storageType == ContractType::Float16;
  auto &b = dc.buffers;
  const std::string base = half ? c.pattern.substr(0, c.pattern.size() - 5) : c.pattern;
  if (gemvShape(base).first) {
    const unsigned k = static_cast<unsigned>(d.shape[1]);
    if (half)
      template_gemv<__half><<<(unsigned)d.workItems, kBaselineBlock, 0, s>>>(
          (const __half *)b[0], (const __half *)b[1], (__half *)b[2], k);
    else
      template_gemv<float><<<(unsigned)d.workItems, kBaselineBlock, 0, s>>>((const float *)b[0],
                                                                            (const float *)b[1], (float *)b[2], k);
  } else if (base == "decoder_rope") {
    if (half)
      template_rope<__half><<<1, 32, 0, s>>>((const __half *)b[0], (const __half *)b[1], (const float *)b[2],
                                             (const float *)b[3], (const int *)b[4], (__half *)b[5], (__half *)b[6]);
    else
      template_rope<float><<<1, 32, 0, s>>>((const float *)b[0], (const float *)b[1], (const float *)b[2],
                                            (const float *)b[3], (const int *)b[4], (float *)b[5], (float *)b[6]);
  } else if (base == "decoder_residual_rmsnorm") {
    if (half)
      template_residual_rmsnorm<__half><<<1, kBaselineBlock, 0, s>>>(
          (const __half *)b[0], (const __half *)b[1], (const __half *)b[2], (__half *)b[3], (__half *)b[4]);
    else
      template_residual_rmsnorm<float><<<1, kBaselineBlock, 0, s>>>(
          (const float *)b[0], (const float *)b[1], (const float *)b[2], (float *)b[3], (float *)b[4]);
  } else {
    if (half)
      template_gated_mlp<__half><<<(unsigned)d.workItems, kBaselineBlock, 0, s>>>(
          (const __half *)b[0], (const __half *)b[1], (const __half *)b[2], (__half *)b[3]);
    else
      template_gated_mlp<float><<<(unsigned)d.workItems, kBaselineBlock, 0, s>>>(
          (const float *)b[0], (const float *)b[1], (const float *)b[2], (float *)b[3]);
  }
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? std::string() : std::string("baseline launch: ") + cudaGetErrorString(e);
}

// ---- driver API and NVRTC ------------------------------------------------------
struct Driver {
  decltype(&cuModuleLoadData) moduleLoadData = nullptr;
  decltype(&cuModuleUnload) moduleUnload = nullptr;
  decltype(&cuModuleGetFunction) moduleGetFunction = nullptr;
  decltype(&cuFuncGetParamInfo) funcGetParamInfo = nullptr;
  decltype(&cuLaunchKernel) launchKernel = nullptr;
  std::string error;
};

const Driver &driver() {
  static std::once_flag once;
  static Driver d;
  std::call_once(once, [] {
    auto get = [](const char *name, int version, void **fn) {
      cudaDriverEntryPointQueryResult q;
      return cudaGetDriverEntryPointByVersion(name, fn, version, cudaEnableDefault, &q) == cudaSuccess &&
             q == cudaDriverEntryPointSuccess && *fn != nullptr;
    };
    void *f = nullptr;
    if (get("cuModuleLoadData", 12000, &f)) d.moduleLoadData = reinterpret_cast<decltype(d.moduleLoadData)>(f);
    if (get("cuModuleUnload", 12000, &f)) d.moduleUnload = reinterpret_cast<decltype(d.moduleUnload)>(f);
    if (get("cuModuleGetFunction", 12000, &f))
      d.moduleGetFunction = reinterpret_cast<decltype(d.moduleGetFunction)>(f);
    if (get("cuFuncGetParamInfo", 12040, &f)) d.funcGetParamInfo = reinterpret_cast<decltype(d.funcGetParamInfo)>(f);
    if (get("cuLaunchKernel", 12000, &f)) d.launchKernel = reinterpret_cast<decltype(d.launchKernel)>(f);
    if (!d.moduleLoadData || !d.moduleUnload || !d.moduleGetFunction || !d.funcGetParamInfo || !d.launchKernel)
      d.error = "CUDA driver entry points for module loading are unavailable.";
    (void)cudaGetLastError();
  });
  return d;
}

// NVRTC, loaded on first use (the rest of the library does not need it).
struct Nvrtc {
  decltype(&nvrtcCreateProgram) create = nullptr;
  decltype(&nvrtcCompileProgram) compile = nullptr;
  decltype(&nvrtcGetProgramLogSize) logSize = nullptr;
  decltype(&nvrtcGetProgramLog) log = nullptr;
  decltype(&nvrtcGetCUBINSize) cubinSize = nullptr;
  decltype(&nvrtcGetCUBIN) cubin = nullptr;
  decltype(&nvrtcDestroyProgram) destroy = nullptr;
  decltype(&nvrtcGetErrorString) errorString = nullptr;
  std::string error;
};

const Nvrtc &nvrtc() {
  static std::once_flag once;
  static Nvrtc n;
  std::call_once(once, [] {
    void *h = nullptr;
    for (const char *name : {"libnvrtc.so.12", "libnvrtc.so", "/usr/local/cuda/lib64/libnvrtc.so.12"})
      if ((h = dlopen(name, RTLD_NOW | RTLD_LOCAL)) != nullptr) break;
    if (!h) {
      n.error = "NVRTC (libnvrtc.so.12) is unavailable";
      return;
    }
    n.create = reinterpret_cast<decltype(n.create)>(dlsym(h, "nvrtcCreateProgram"));
    n.compile = reinterpret_cast<decltype(n.compile)>(dlsym(h, "nvrtcCompileProgram"));
    n.logSize = reinterpret_cast<decltype(n.logSize)>(dlsym(h, "nvrtcGetProgramLogSize"));
    n.log = reinterpret_cast<decltype(n.log)>(dlsym(h, "nvrtcGetProgramLog"));
    n.cubinSize = reinterpret_cast<decltype(n.cubinSize)>(dlsym(h, "nvrtcGetCUBINSize"));
    n.cubin = reinterpret_cast<decltype(n.cubin)>(dlsym(h, "nvrtcGetCUBIN"));
    n.destroy = reinterpret_cast<decltype(n.destroy)>(dlsym(h, "nvrtcDestroyProgram"));
    n.errorString = reinterpret_cast<decltype(n.errorString)>(dlsym(h, "nvrtcGetErrorString"));
    if (!n.create || !n.compile || !n.logSize || !n.log || !n.cubinSize || !n.cubin || !n.destroy ||
        !n.errorString)
      n.error = "NVRTC symbols are missing";
  });
  return n;
}

std::string compileCubin(const std::string &source, const std::string &name, std::vector<char> *cubin) {
  const Nvrtc &nv = nvrtc();
  if (!nv.error.empty()) return nv.error;
  nvrtcProgram prog;
  if (nv.create(&prog, source.c_str(), (name + ".cu").c_str(), 0, nullptr, nullptr) != NVRTC_SUCCESS)
    return "nvrtcCreateProgram failed";
  const char *opts[] = {"--gpu-architecture=sm_100a", "-std=c++17", "--include-path=/usr/local/cuda/include"};
  const nvrtcResult r = nv.compile(prog, 3, opts);
  std::string log;
  std::size_t logSize = 0;
  nv.logSize(prog, &logSize);
  if (logSize > 1) {
    log.resize(logSize);
    nv.log(prog, log.data());
  }
  if (r != NVRTC_SUCCESS) {
    nv.destroy(&prog);
    return std::string(nv.errorString(r)) + (log.empty() ? "" : ": " + log);
  }
  std::size_t size = 0;
  nv.cubinSize(prog, &size);
  cubin->resize(size);
  nv.cubin(prog, cubin->data());
  nv.destroy(&prog);
  return {};
}

std::string jsonEscape(const std::string &s) {
  std::string o;
  for (char ch : s) {
    switch (ch) {
      case '"': o += "\\\""; break;
      case '\\': o += "\\\\"; break;
      case '\n': o += "\\n"; break;
      case '\t': o += "\\t"; break;
      case '\r': o += "\\r"; break;
      default:
        if (static_cast<unsigned char>(ch) < 0x20) {
          char buf[8];
          std::snprintf(buf, sizeof(buf), "\\u%04x", ch);
          o += buf;
        } else {
          o += ch;
        }
    }
  }
  return o;
}

// Value of a string or number field in a flat JSON object written by this file.
bool jsonField(const std::string &doc, const std::string &key, std::string *out) {
  const std::string tag = "\"" + key + "\":";
  const auto at = doc.find(tag);
  if (at == std::string::npos) return false;
  std::size_t i = at + tag.size();
  while (i < doc.size() && doc[i] == ' ') ++i;
  if (i >= doc.size()) return false;
  if (doc[i] != '"') {
    const auto end = doc.find_first_of(",}", i);
    *out = doc.substr(i, end - i);
    return true;
  }
  std::string v;
  for (++i; i < doc.size() && doc[i] != '"'; ++i) {
    if (doc[i] != '\\') {
      v += doc[i];
      continue;
    }
    if (++i >= doc.size()) return false;
    switch (doc[i]) {
      case 'n': v += '\n'; break;
      case 't': v += '\t'; break;
      case 'r': v += '\r'; break;
      case 'u': v += static_cast<char>(std::stoi(doc.substr(i + 1, 4), nullptr, 16)); i += 4; break;
      default: v += doc[i];
    }
  }
  *out = v;
  return true;
}

const char *typeName(ContractType t) {
  return t == ContractType::Float16 ? "fp16" : t == ContractType::Int32 ? "int32" : "fp32";
}

std::string writeText(const std::string &path, const std::string &text) {
  if (path.empty()) return {};
  std::ofstream f(path);
  if (!f) return "cannot write " + path;
  f << text;
  return f ? std::string() : "cannot write " + path;
}

std::string feedbackJson(const AdmissionFeedback &f) {
  std::ostringstream o;
  o << "{\"status\":\"" << f.status << "\",\"stage\":\"" << f.stage << "\",\"message\":\"" << jsonEscape(f.message)
    << "\"";
  if (f.speedup > 0)
    o << ",\"baseline_us\":" << f.baselineUs << ",\"candidate_us\":" << f.candidateUs << ",\"speedup\":" << f.speedup;
  o << "}\n";
  return o.str();
}

double median(std::vector<double> v) {
  std::sort(v.begin(), v.end());
  return v[v.size() / 2];
}

}  // namespace

// ---- contracts ---------------------------------------------------------------
KernelContract makeKernelContract(const std::string &pattern) {
  const bool half = pattern.size() > 5 && pattern.compare(pattern.size() - 5, 5, "_fp16") == 0;
  if (!half) return baseContract(pattern);
  const std::string base = pattern.substr(0, pattern.size() - 5);
  KernelContract c = baseContract(base);
  c.pattern = pattern;
  c.functionName = "generated_" + pattern;
  c.storageType = ContractType::Float16;
  c.absoluteTolerance = 2e-2;
  c.relativeTolerance = 2e-2;
  for (std::size_t i = 0; i < c.inputTypes.size(); ++i)
    if (c.inputTypes[i] == ContractType::Float32 && !(base == "decoder_rope" && (i == 2 || i == 3)))
      c.inputTypes[i] = ContractType::Float16;
  // The fixtures are exact in fp16; round the references at the storage boundaries.
  for (auto &d : c.cases) {
    for (std::size_t i = 0; i < d.inputs.size(); ++i)
      if (c.inputTypes[i] == ContractType::Float16)
        for (auto &v : d.inputs[i]) v = static_cast<float>(roundHalf(v));
    if (base == "decoder_residual_rmsnorm") {
      double squares = 0;
      for (std::size_t i = 0; i < d.references[0].size(); ++i) {
        const double v = roundHalf(d.inputs[0][i] + d.inputs[1][i]);
        d.references[0][i] = v;
        squares += v * v;
      }
      const double inverse = 1 / std::sqrt(squares / d.references[0].size() + 1e-5);
      for (std::size_t i = 0; i < d.references[1].size(); ++i)
        d.references[1][i] = roundHalf(d.references[0][i] * inverse * d.inputs[2][i]);
    } else if (base == "decoder_gated_mlp") {
      const auto width = d.inputs[0].size();
      for (std::size_t j = 0; j < d.references[0].size(); ++j) {
        const double gate = roundHalf(dot(d.inputs[0], d.inputs[1], j, width));
        const double up = roundHalf(dot(d.inputs[0], d.inputs[2], j, width));
        d.references[0][j] = roundHalf(roundHalf(gate / (1 + std::exp(-gate))) * up);
      }
    } else {
      for (auto &out : d.references)
        for (auto &v : out) v = roundHalf(v);
    }
  }
  c.applicability = "Decoder-only batch=1, sequence_length=1, storage=fp16; original shape constraints apply.";
  c.semantics += " Storage is fp16; compute in fp32 and round residual sums, Gate/Up projections, SiLU "
                 "results and outputs to fp16. RoPE tables stay fp32.";
  return c;
}

std::string serializeKernelContract(const KernelContract &c) {
  std::ostringstream o;
  o << "{\"pattern\":\"" << c.pattern << "\",\"function_name\":\"" << c.functionName << "\",\"semantics\":\""
    << jsonEscape(c.semantics) << "\",\"work_item\":\"" << jsonEscape(c.workItem) << "\",\"applicability\":\""
    << jsonEscape(c.applicability) << "\",\"group_per_work_item\":" << (c.groupPerWorkItem ? "true" : "false")
    << ",\"storage\":\"" << typeName(c.storageType) << "\",\"inputs\":[";
  for (std::size_t i = 0; i < c.inputNames.size(); ++i)
    o << (i ? "," : "") << "{\"name\":\"" << c.inputNames[i] << "\",\"type\":\"" << typeName(c.inputTypes[i])
      << "\"}";
  o << "],\"outputs\":[";
  for (std::size_t i = 0; i < c.outputNames.size(); ++i)
    o << (i ? "," : "") << "{\"name\":\"" << c.outputNames[i] << "\",\"type\":\"" << typeName(c.storageType)
      << "\"}";
  o << "],\"block_sizes\":[";
  for (std::size_t i = 0; i < c.blockSizes.size(); ++i) o << (i ? "," : "") << c.blockSizes[i];
  o << "],\"absolute_tolerance\":" << c.absoluteTolerance << ",\"relative_tolerance\":" << c.relativeTolerance
    << ",\"minimum_speedup\":" << c.minimumSpeedup << ",\"cases\":[";
  for (std::size_t i = 0; i < c.cases.size(); ++i) {
    o << (i ? "," : "") << "{\"shape\":[";
    for (std::size_t j = 0; j < c.cases[i].shape.size(); ++j) o << (j ? "," : "") << c.cases[i].shape[j];
    o << "],\"work_items\":" << c.cases[i].workItems << "}";
  }
  o << "],\"signature\":\"extern \\\"C\\\" __global__ void " << c.functionName << "(";
  for (std::size_t i = 0; i < c.inputNames.size(); ++i)
    o << (c.inputTypes[i] == ContractType::Int32 ? "const int *"
          : c.inputTypes[i] == ContractType::Float16 ? "const __half *"
                                                      : "const float *")
      << c.inputNames[i] << ", ";
  for (std::size_t i = 0; i < c.outputNames.size(); ++i)
    o << (c.storageType == ContractType::Float16 ? "__half *" : "float *") << c.outputNames[i] << ", ";
  o << "unsigned work_items)\"}";
  return o.str();
}

// ---- compiled kernels --------------------------------------------------------
CompiledKernel::~CompiledKernel() {
  if (module_ && driver().moduleUnload) driver().moduleUnload(static_cast<CUmodule>(module_));
}

std::unique_ptr<CompiledKernel> CompiledKernel::compile(const KernelContract &c, const std::string &source,
                                                        int blockSize, std::string *error) {
  const Driver &d = driver();
  if (!d.error.empty()) {
    *error = d.error;
    return nullptr;
  }
  std::vector<char> cubin;
  *error = compileCubin(source, c.functionName, &cubin);
  if (!error->empty()) return nullptr;
  CUmodule mod = nullptr;
  if (d.moduleLoadData(&mod, cubin.data()) != CUDA_SUCCESS) {
    *error = "cuModuleLoadData failed";
    return nullptr;
  }
  std::unique_ptr<CompiledKernel> k(new CompiledKernel());
  k->module_ = mod;
  CUfunction fn = nullptr;
  if (d.moduleGetFunction(&fn, mod, c.functionName.c_str()) != CUDA_SUCCESS) {
    *error = "kernel " + c.functionName + " not found (extern \"C\" __global__)";
    return nullptr;
  }
  // Interface: one 8-byte pointer per buffer, then the 4-byte work-item count.
  const std::size_t buffers = c.inputNames.size() + c.outputNames.size();
  for (std::size_t i = 0; i <= buffers; ++i) {
    size_t offset = 0, size = 0;
    if (d.funcGetParamInfo(fn, i, &offset, &size) != CUDA_SUCCESS || size != (i < buffers ? 8u : 4u)) {
      *error = "interface: parameter " + std::to_string(i) + " must be " +
               (i < buffers ? "a pointer" : "unsigned work_items");
      return nullptr;
    }
  }
  size_t offset = 0, size = 0;
  if (d.funcGetParamInfo(fn, buffers + 1, &offset, &size) == CUDA_SUCCESS) {
    *error = "interface: more parameters than the contract declares";
    return nullptr;
  }
  k->function_ = fn;
  k->block_ = blockSize;
  k->perWorkItem_ = c.groupPerWorkItem;
  return k;
}

std::string CompiledKernel::launch(const std::vector<void *> &buffers, unsigned workItems, void *stream) const {
  std::vector<void *> ptrs(buffers);
  std::vector<void *> args;
  for (auto &p : ptrs) args.push_back(&p);
  unsigned n = workItems;
  args.push_back(&n);
  const unsigned grid = perWorkItem_ ? workItems : (workItems + block_ - 1) / block_;
  const CUresult r = driver().launchKernel(static_cast<CUfunction>(function_), grid, 1, 1, block_, 1, 1, 0,
                                           static_cast<CUstream>(stream), args.data(), nullptr);
  return r == CUDA_SUCCESS ? std::string() : "candidate launch failed (" + std::to_string((int)r) + ")";
}

// ---- admission -------------------------------------------------------------------
AdmissionFeedback admitGeneratedKernel(const std::string &pattern, const std::string &source, int blockSize,
                                       const std::string &feedbackPath, const std::string &artifactPath,
                                       std::ostream &log) {
  auto finish = [&](AdmissionFeedback f) {
    log << "Generated candidate " << f.stage << ": " << (f.status == "admitted" ? "PASS" : "FAIL") << ": "
        << f.message << '\n'
        << "Generated kernel admission: "
        << (f.status == "admitted" ? "PASS" : f.status == "fatal" ? "FAIL" : "FALLBACK") << '\n'
        << "Selected: " << (f.status == "admitted" ? "generated " : "template ") << pattern << '\n';
    const auto e = writeText(feedbackPath, feedbackJson(f));
    if (!e.empty()) {
      log << "Feedback error: " << e << '\n';
      f.status = "fatal";
    }
    return f;
  };
  KernelContract c;
  try {
    c = makeKernelContract(pattern);
  } catch (const std::exception &e) {
    return finish({"fatal", "contract", e.what()});
  }
  if (std::find(c.blockSizes.begin(), c.blockSizes.end(), blockSize) == c.blockSizes.end())
    return finish({"retry", "hardware_filter", "block size is not legal for this contract"});
  std::string error;
  auto kernel = CompiledKernel::compile(c, source, blockSize, &error);
  if (!kernel) {
    const bool iface = error.rfind("interface", 0) == 0 || error.rfind("kernel ", 0) == 0;
    return finish({"retry", iface ? "interface" : "compile", error});
  }
  log << "Generated candidate compile: PASS\nGenerated candidate interface: PASS, outputs=" << c.outputNames.size()
      << '\n';
  cudaStream_t s = nullptr;
  cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
  std::vector<std::unique_ptr<DeviceCase>> cases;
  auto run = [&](std::size_t i, bool candidate) -> std::string {
    const auto &dc = *cases[i];
    if (candidate) return kernel->launch(dc.buffers, static_cast<unsigned>(c.cases[i].workItems), s);
    return launchBaseline(c, c.cases[i], dc, s);
  };
  auto check = [&](std::size_t i) -> std::string {
    std::string e = run(i, true);
    if (e.empty() && cudaStreamSynchronize(s) != cudaSuccess) e = cudaGetErrorString(cudaGetLastError());
    if (e.empty()) e = validate(c, c.cases[i], *cases[i]);
    return e;
  };
  AdmissionFeedback accepted{"admitted", "admission", "All cases passed correctness and two performance rounds."};
  double worst = 1e30;
  std::optional<AdmissionFeedback> slow;
  AdmissionFeedback result;
  bool done = false;
  for (std::size_t i = 0; i < c.cases.size() && !done; ++i) {
    cases.push_back(std::make_unique<DeviceCase>());
    if (!(error = upload(c, c.cases[i], cases.back().get())).empty()) {
      result = {"fatal", "prepare", error};
      done = true;
      break;
    }
    // The template baseline must itself pass (it defines "correct and faster").
    error = run(i, false);
    if (error.empty() && cudaStreamSynchronize(s) == cudaSuccess) error = validate(c, c.cases[i], *cases[i]);
    if (!error.empty()) {
      result = {"fatal", "baseline", "case " + std::to_string(i) + ": " + error};
      done = true;
      break;
    }
    cudaMemsetAsync(cases[i]->buffers.back(), 0xff, cases[i]->counts.back() * typeBytes(c.storageType), s);
    if (!(error = check(i)).empty()) {
      result = {"retry", "numerical_validation", "case " + std::to_string(i) + ": " + error};
      done = true;
      break;
    }
    log << "Generated candidate case " << i << " all outputs numerical validation: PASS\n";
  }
  for (std::size_t i = 0; i < cases.size() && !done; ++i) {
    for (int w = 0; w < kWarmup; ++w) {
      run(i, false);
      run(i, true);
    }
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    for (int round = 0; round < 2 && !done; ++round) {
      std::vector<double> tb, tc;
      for (int sample = 0; sample < kSamples; ++sample) {
        for (int which = 0; which < 2; ++which) {  // alternating pairs
          cudaEventRecord(e0, s);
          const std::string e = run(i, which == 1);
          cudaEventRecord(e1, s);
          if (!e.empty() || cudaEventSynchronize(e1) != cudaSuccess) {
            result = {"retry", "benchmark", e.empty() ? "event failure" : e};
            done = true;
            break;
          }
          float ms = 0;
          cudaEventElapsedTime(&ms, e0, e1);
          (which ? tc : tb).push_back(ms * 1e3);
        }
        if (done) break;
      }
      if (done) break;
      const double b = median(tb), cu = median(tc), sp = b / cu;
      log << "Generated candidate case " << i << " round " << round + 1 << ": baseline(us)=" << b
          << ", candidate(us)=" << cu << ", speedup=" << sp << "x\n";
      if (sp < worst) {
        worst = sp;
        accepted.baselineUs = b;
        accepted.candidateUs = cu;
        accepted.speedup = sp;
      }
      if (sp < c.minimumSpeedup && (!slow || sp < slow->speedup))
        slow = AdmissionFeedback{"retry", "performance",
                                 "case " + std::to_string(i) + " round " + std::to_string(round + 1) +
                                     " speedup is below " + std::to_string(c.minimumSpeedup) + "x.",
                                 b, cu, sp};
    }
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    if (done) break;
    if (!(error = check(i)).empty()) {
      result = {"retry", "final_validation", error};
      done = true;
    }
  }
  cudaStreamDestroy(s);
  if (done) return finish(result);
  if (slow) return finish(*slow);
  if (!artifactPath.empty()) {
    std::ostringstream a;
    a << "{\"pattern\":\"" << c.pattern << "\",\"function_name\":\"" << c.functionName
      << "\",\"block_size\":" << blockSize << ",\"speedup\":" << accepted.speedup << ",\"baseline_us\":"
      << accepted.baselineUs << ",\"candidate_us\":" << accepted.candidateUs << ",\"source\":\""
      << jsonEscape(source) << "\"}\n";
    const auto e = writeText(artifactPath, a.str());
    if (!e.empty()) return finish({"fatal", "artifact_write", e});
  }
  return finish(accepted);
}

// ---- registry -------------------------------------------------------------------
void KernelRegistry::load(const std::string &directory, std::ostream &log) {
  namespace fs = std::filesystem;
  std::error_code ec;
  if (!fs::is_directory(directory, ec)) {
    log << "Kernel registry: no directory " << directory << '\n';
    return;
  }
  std::vector<fs::path> files;
  for (const auto &e : fs::directory_iterator(directory, ec))
    if (e.path().extension() == ".json") files.push_back(e.path());
  std::sort(files.begin(), files.end());
  for (const auto &path : files) {
    std::ifstream f(path);
    std::stringstream buf;
    buf << f.rdbuf();
    const std::string doc = buf.str();
    std::string pattern, source, block;
    if (!jsonField(doc, "pattern", &pattern) || !jsonField(doc, "source", &source) ||
        !jsonField(doc, "block_size", &block)) {
      log << "Kernel registry: skipped " << path.filename().string() << " (not an admitted artifact)\n";
      continue;
    }
    try {
      const KernelContract c = makeKernelContract(pattern);
      std::string error;
      auto k = CompiledKernel::compile(c, source, std::stoi(block), &error);
      if (!k) {
        log << "Kernel registry: skipped " << pattern << ": " << error << '\n';
        continue;
      }
      entries_[pattern] = std::move(k);
      log << "Kernel registry: loaded " << pattern << " (block " << block << ")\n";
    } catch (const std::exception &e) {
      log << "Kernel registry: skipped " << path.filename().string() << ": " << e.what() << '\n';
    }
  }
}

const CompiledKernel *KernelRegistry::find(const std::string &pattern) const {
  auto it = entries_.find(pattern);
  return it == entries_.end() ? nullptr : it->second.get();
}

std::vector<std::string> KernelRegistry::patterns() const {
  std::vector<std::string> p;
  for (const auto &kv : entries_) p.push_back(kv.first);
  return p;
}

std::size_t KernelRegistry::track(KernelUsage usage) {
  usage_.push_back(std::move(usage));
  return usage_.size() - 1;
}

void KernelRegistry::completed(const std::vector<std::size_t> &uses) {
  for (auto u : uses)
    if (u < usage_.size()) ++usage_[u].completedCalls;
}

void KernelRegistry::report(std::ostream &log) const {
  for (const auto &u : usage_)
    log << "Kernel usage: node=" << u.node << ", pattern=" << u.pattern << ", implementation=" << u.implementation
        << ", dispatches_per_call=" << u.dispatchesPerCall << ", completed_calls=" << u.completedCalls << '\n';
}

}  // namespace tensor::runtime
