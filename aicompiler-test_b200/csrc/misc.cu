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

// dst[r * dst_stride + c] = N(mean, std) drawn for the LOGICAL element
// (logical_row0 + r) * logical_cols + logical_col0 + c, so a tensor-parallel
// shard or an interleaved/fused layout receives exactly the values of the
// unsharded tensor.
__global__ void fill_normal_2d_kernel(__half *dst, int rows, int cols, long long dst_stride,
                                      uint64_t seed, long long logical_row0, long long logical_cols,
                                      long long logical_col0, float mean, float stddev) {
  const long long total = (long long)rows * cols;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / cols, c = i % cols;
    const unsigned long long li =
        (unsigned long long)((logical_row0 + r) * logical_cols + logical_col0 + c);
    const uint64_t h = splitmix64(seed ^ splitmix64(li >> 1));
    const float u1 = (static_cast<float>((h >> 40) & 0xffffffu) + 1.0f) * (1.0f / 16777216.0f);
    const float u2 = static_cast<float>((h >> 8) & 0xffffffu) * (1.0f / 16777216.0f);
    const float rr = sqrtf(-2.0f * logf(u1));
    float sn, cs;
    sincospif(2.0f * u2, &sn, &cs);
    dst[r * dst_stride + c] = __float2half_rn(mean + stddev * rr * ((li & 1) ? sn : cs));
  }
}

__global__ void fill_value_f16_kernel(__half *dst, size_t count, float value) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < count;
       i += (size_t)gridDim.x * blockDim.x)
    dst[i] = __float2half_rn(value);
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
                                       int *feed_tokens, int *feed_positions, int *history,
                                       unsigned int *history_counter) {
  pdl_wait();
  const int m = threadIdx.x;
  const unsigned int step = history != nullptr ? *history_counter : 0u;
  if (m < rows) {
    const unsigned long long key = keys[m];
    keys[m] = 0ull;
    const int tok = argmax_key_index(key);
    next_tokens[m] = tok;
    if (feed_tokens != nullptr) feed_tokens[m] = tok;
    if (feed_positions != nullptr) feed_positions[m] += 1;
    if (history != nullptr) history[(size_t)step * rows + m] = tok;
  }
  __syncthreads();
  if (m == 0 && history != nullptr) *history_counter = step + 1;
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

cudaError_t launch_fill_normal_2d(__half *dst, int rows, int cols, long long dst_stride,
                                  uint64_t seed, long long logical_row0, long long logical_cols,
                                  long long logical_col0, float mean, float stddev,
                                  cudaStream_t stream) {
  const long long total = (long long)rows * cols;
  if (total <= 0) return cudaSuccess;
  long long blocks = (total + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  fill_normal_2d_kernel<<<static_cast<int>(blocks), 256, 0, stream>>>(
      dst, rows, cols, dst_stride, seed, logical_row0, logical_cols, logical_col0, mean, stddev);
  return cudaGetLastError();
}

cudaError_t launch_fill_value_f16(__half *dst, size_t count, float value, cudaStream_t stream) {
  if (count == 0) return cudaSuccess;
  int blocks = static_cast<int>((count + 255) / 256);
  if (blocks > 148 * 32) blocks = 148 * 32;
  fill_value_f16_kernel<<<blocks, 256, 0, stream>>>(dst, count, value);
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
                                   int *feed_tokens, int *feed_positions, int *history,
                                   unsigned int *history_counter, cudaStream_t stream, bool pdl) {
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
                            feed_positions, history, history_counter);
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

namespace {
__global__ void page_copy_kernel(__half *const *pools, const int *pages, int npages, size_t page_elems,
                                 __half *packed, bool to_packed) {
  const int i = blockIdx.x, lk = blockIdx.y;  // page index, layer * 2 + kv
  uint4 *pool = reinterpret_cast<uint4 *>(pools[lk] + (size_t)pages[i] * page_elems);
  uint4 *pack = reinterpret_cast<uint4 *>(packed + ((size_t)lk * npages + i) * page_elems);
  const size_t n = page_elems / 8;
  for (size_t j = threadIdx.x; j < n; j += blockDim.x) {
    if (to_packed)
      pack[j] = pool[j];
    else
      pool[j] = pack[j];
  }
}
}  // namespace

cudaError_t launch_page_copy(__half *const *pools, const int *pages, int npages, int layers, size_t page_elems,
                             __half *packed, bool to_packed, cudaStream_t stream) {
  if (npages <= 0 || layers <= 0 || page_elems % 8 != 0 || layers * 2 > 65535) return cudaErrorInvalidValue;
  page_copy_kernel<<<dim3(npages, layers * 2), 256, 0, stream>>>(pools, pages, npages, page_elems, packed, to_packed);
  return cudaGetLastError();
}

}  // namespace tmc
