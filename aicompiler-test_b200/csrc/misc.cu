// Small device utilities: synthetic weight fill, argmax finalisation for the
// vocab-parallel LM head, and scalar helpers used by the executors.
#include "misc.cuh"

#include <cmath>

namespace tmc {
namespace {

__device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
  x += 0x9e3779b97f4a7c15ull;
  x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ull;
  x = (x ^ (x >> 27)) * 0x94d049bb133111ebull;
  return x ^ (x >> 31);
}

// Box-Muller on two 24-bit uniforms in (0, 1].
__global__ void fill_normal_kernel(__half *dst, size_t count, uint64_t seed, float mean,
                                   float stddev) {
  const size_t pairs = (count + 1) / 2;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < pairs;
       i += (size_t)gridDim.x * blockDim.x) {
    const uint64_t h = splitmix64(seed ^ splitmix64(i));
    const float u1 = (static_cast<float>((h >> 40) & 0xffffffu) + 1.0f) * (1.0f / 16777216.0f);
    const float u2 = static_cast<float>((h >> 8) & 0xffffffu) * (1.0f / 16777216.0f);
    const float r = sqrtf(-2.0f * logf(u1));
    float s, c;
    sincospif(2.0f * u2, &s, &c);
    const size_t j = 2 * i;
    dst[j] = __float2half_rn(mean + stddev * r * c);
    if (j + 1 < count) dst[j + 1] = __float2half_rn(mean + stddev * r * s);
  }
}

__global__ void fill_uniform_f32_kernel(float *dst, size_t count, uint64_t seed, float lo,
                                        float hi) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < count;
       i += (size_t)gridDim.x * blockDim.x) {
    const uint64_t h = splitmix64(seed ^ splitmix64(i));
    const float u = static_cast<float>((h >> 40) & 0xffffffu) * (1.0f / 16777216.0f);
    dst[i] = lo + (hi - lo) * u;
  }
}

// Resolve packed argmax keys (after a cross-rank max) into token ids and reset.
__global__ void argmax_finalize_kernel(unsigned long long *keys, int rows, int *next_tokens,
                                       int *feed_tokens, int *feed_positions) {
  pdl_wait();
  const int m = threadIdx.x;
  if (m < rows) {
    const unsigned long long key = keys[m];
    keys[m] = 0ull;
    const int tok = argmax_key_index(key);
    next_tokens[m] = tok;
    if (feed_tokens != nullptr) feed_tokens[m] = tok;
    if (feed_positions != nullptr) feed_positions[m] += 1;
  }
}

__global__ void add_residual_f32_kernel(__half *h, const float *partial, int n) {
  pdl_wait();
  pdl_launch_dependents();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    h[i] = __float2half_rn(__fadd_rn(__half2float(h[i]), round_half(partial[i])));
  }
}

}  // namespace

cudaError_t launch_fill_normal_f16(__half *dst, size_t count, uint64_t seed, float mean,
                                   float stddev, cudaStream_t stream) {
  if (count == 0) return cudaSuccess;
  const size_t pairs = (count + 1) / 2;
  int blocks = static_cast<int>((pairs + 255) / 256);
  if (blocks > 148 * 32) blocks = 148 * 32;
  fill_normal_kernel<<<blocks, 256, 0, stream>>>(dst, count, seed, mean, stddev);
  return cudaGetLastError();
}

cudaError_t launch_fill_uniform_f32(float *dst, size_t count, uint64_t seed, float lo, float hi,
                                    cudaStream_t stream) {
  if (count == 0) return cudaSuccess;
  int blocks = static_cast<int>((count + 255) / 256);
  if (blocks > 148 * 32) blocks = 148 * 32;
  fill_uniform_f32_kernel<<<blocks, 256, 0, stream>>>(dst, count, seed, lo, hi);
  return cudaGetLastError();
}

cudaError_t launch_argmax_finalize(unsigned long long *keys, int rows, int *next_tokens,
                                   int *feed_tokens, int *feed_positions, cudaStream_t stream,
                                   bool pdl) {
  if (rows <= 0 || rows > 1024) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(((rows + 31) / 32) * 32);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, argmax_finalize_kernel, keys, rows, next_tokens, feed_tokens,
                            feed_positions);
}

cudaError_t launch_add_residual_f32(__half *h, const float *partial, int n, cudaStream_t stream,
                                    bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((n + 255) / 256 < 148 ? (n + 255) / 256 : 148);
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, add_residual_f32_kernel, h, partial, n);
}

}  // namespace tmc
