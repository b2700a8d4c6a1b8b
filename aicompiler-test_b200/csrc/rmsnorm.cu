// Standalone RMSNorm kernels (see rmsnorm.cuh).
#include "rmsnorm.cuh"

namespace tmc {
namespace {

template <typename T>
__device__ __forceinline__ float load_f(const T *p, size_t i);
template <>
__device__ __forceinline__ float load_f<float>(const float *p, size_t i) {
  return p[i];
}
template <>
__device__ __forceinline__ float load_f<__half>(const __half *p, size_t i) {
  return __half2float(p[i]);
}
__device__ __forceinline__ void store_f(float *p, size_t i, float v) { p[i] = v; }
__device__ __forceinline__ void store_f(__half *p, size_t i, float v) { p[i] = __float2half_rn(v); }

// 16-byte vectors: 4 floats or 8 halves, unpacked to fp32.
template <typename T>
struct Vec;
template <>
struct Vec<float> {
  static constexpr int kN = 4;
  __device__ static void load(const float *p, float *v) {
    const float4 q = *reinterpret_cast<const float4 *>(p);
    v[0] = q.x, v[1] = q.y, v[2] = q.z, v[3] = q.w;
  }
  __device__ static void store(float *p, const float *v) {
    *reinterpret_cast<float4 *>(p) = make_float4(v[0], v[1], v[2], v[3]);
  }
};
template <>
struct Vec<__half> {
  static constexpr int kN = 8;
  __device__ static void load(const __half *p, float *v) {
    const uint4 q = *reinterpret_cast<const uint4 *>(p);
    const __half2 *h = reinterpret_cast<const __half2 *>(&q);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(h[i]);
      v[2 * i] = f.x, v[2 * i + 1] = f.y;
    }
  }
  __device__ static void store(__half *p, const float *v) {
    uint4 q;
    __half2 *h = reinterpret_cast<__half2 *>(&q);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
    *reinterpret_cast<uint4 *>(p) = q;
  }
};

// Block sum through warp shuffles and one shared-memory round.
__device__ __forceinline__ float block_sum(float s, float *scratch) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const int warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
  if ((threadIdx.x & 31) == 0) scratch[warp] = s;
  __syncthreads();
  float t = 0.0f;
  for (int i = 0; i < warps; ++i) t += scratch[i];
  return t;
}

template <typename T, bool VEC>
__global__ void rmsnorm_kernel(const T *__restrict__ x, const T *__restrict__ gamma, T *__restrict__ y, int width,
                               float eps) {
  __shared__ float scratch[32];
  const size_t row = (size_t)blockIdx.x * width;
  float s = 0.0f;
  if constexpr (VEC) {
    constexpr int N = Vec<T>::kN;
    float v[N];
    for (int c = threadIdx.x * N; c < width; c += blockDim.x * N) {
      Vec<T>::load(x + row + c, v);
#pragma unroll
      for (int i = 0; i < N; ++i) s += v[i] * v[i];
    }
    const float inv = rsqrtf(block_sum(s, scratch) / (float)width + eps);
    float g[N];
    for (int c = threadIdx.x * N; c < width; c += blockDim.x * N) {
      Vec<T>::load(x + row + c, v);
      Vec<T>::load(gamma + c, g);
#pragma unroll
      for (int i = 0; i < N; ++i) v[i] = v[i] * inv * g[i];
      Vec<T>::store(y + row + c, v);
    }
  } else {
    for (int c = threadIdx.x; c < width; c += blockDim.x) {
      const float v = load_f(x, row + c);
      s += v * v;
    }
    const float inv = rsqrtf(block_sum(s, scratch) / (float)width + eps);
    for (int c = threadIdx.x; c < width; c += blockDim.x)
      store_f(y, row + c, load_f(x, row + c) * inv * load_f(gamma, (size_t)c));
  }
}

// Baseline: per-thread partial sums folded by a shared-memory halving tree.
template <typename T>
__global__ void __launch_bounds__(256) rmsnorm_baseline_kernel(const T *x, const T *gamma, T *y, int width,
                                                               float eps) {
  __shared__ float partial[256];
  const size_t row = (size_t)blockIdx.x * width;
  float s = 0.0f;
  for (int c = threadIdx.x; c < width; c += 256) {
    const float v = load_f(x, row + c);
    s += v * v;
  }
  partial[threadIdx.x] = s;
  __syncthreads();
  for (int stride = 128; stride > 0; stride >>= 1) {
    if ((int)threadIdx.x < stride) partial[threadIdx.x] += partial[threadIdx.x + stride];
    __syncthreads();
  }
  const float inv = rsqrtf(partial[0] / (float)width + eps);
  for (int c = threadIdx.x; c < width; c += 256)
    store_f(y, row + c, load_f(x, row + c) * inv * load_f(gamma, (size_t)c));
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

cudaError_t launch_rmsnorm(const void *x, const void *gamma, void *y, int rows, int width, float eps, bool fp16,
                           int threads, cudaStream_t stream) {
  if (rows <= 0 || width <= 0 || threads < 32 || threads > 1024 || (threads & (threads - 1)) != 0)
    return cudaErrorInvalidValue;
  const int vec = fp16 ? 8 : 4;
  const bool v = width % vec == 0 && aligned16(x) && aligned16(gamma) && aligned16(y);
  if (fp16) {
    auto *xs = static_cast<const __half *>(x);
    auto *gs = static_cast<const __half *>(gamma);
    auto *ys = static_cast<__half *>(y);
    if (v)
      rmsnorm_kernel<__half, true><<<rows, threads, 0, stream>>>(xs, gs, ys, width, eps);
    else
      rmsnorm_kernel<__half, false><<<rows, threads, 0, stream>>>(xs, gs, ys, width, eps);
  } else {
    auto *xs = static_cast<const float *>(x);
    auto *gs = static_cast<const float *>(gamma);
    auto *ys = static_cast<float *>(y);
    if (v)
      rmsnorm_kernel<float, true><<<rows, threads, 0, stream>>>(xs, gs, ys, width, eps);
    else
      rmsnorm_kernel<float, false><<<rows, threads, 0, stream>>>(xs, gs, ys, width, eps);
  }
  return cudaGetLastError();
}

cudaError_t launch_rmsnorm_baseline(const void *x, const void *gamma, void *y, int rows, int width, float eps,
                                    bool fp16, cudaStream_t stream) {
  if (rows <= 0 || width <= 0) return cudaErrorInvalidValue;
  if (fp16)
    rmsnorm_baseline_kernel<__half><<<rows, 256, 0, stream>>>(
        static_cast<const __half *>(x), static_cast<const __half *>(gamma), static_cast<__half *>(y), width, eps);
  else
    rmsnorm_baseline_kernel<float><<<rows, 256, 0, stream>>>(
        static_cast<const float *>(x), static_cast<const float *>(gamma), static_cast<float *>(y), width, eps);
  return cudaGetLastError();
}

}  // namespace tmc
