// Fused graph regions (see fusion.cuh).
#include "fusion.cuh"

namespace tmc {
namespace {

template <typename T>
__device__ __forceinline__ float ld(const T *p, size_t i);
template <>
__device__ __forceinline__ float ld<float>(const float *p, size_t i) {
  return p[i];
}
template <>
__device__ __forceinline__ float ld<__half>(const __half *p, size_t i) {
  return __half2float(p[i]);
}
// Round an fp32 value to the storage type and back.
template <typename T>
__device__ __forceinline__ float rnd(float v);
template <>
__device__ __forceinline__ float rnd<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ float rnd<__half>(float v) {
  return __half2float(__float2half_rn(v));
}
__device__ __forceinline__ void st(float *p, size_t i, float v) { p[i] = v; }
__device__ __forceinline__ void st(__half *p, size_t i, float v) { p[i] = __float2half_rn(v); }

constexpr int kNormThreads = 256;

// One CTA per row: v = T(x + b); statistics in fp32; y = T((v - mean) * inv * w [+ c]).
template <typename T, bool LN>
__global__ void __launch_bounds__(kNormThreads) add_norm_kernel(const T *__restrict__ x, const T *__restrict__ b,
                                                                 const T *__restrict__ w, const T *__restrict__ c,
                                                                 T *__restrict__ y, int width, int b_rows,
                                                                 float eps) {
  __shared__ float red[2][kNormThreads / 32];
  const size_t row = blockIdx.x, base = row * width, bbase = b_rows == 1 ? 0 : base;
  float sum = 0.0f, squares = 0.0f;
  for (int i = threadIdx.x; i < width; i += kNormThreads) {
    const float v = rnd<T>(ld(x, base + i) + ld(b, bbase + i));
    sum += v;
    squares += v * v;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    sum += __shfl_xor_sync(0xffffffffu, sum, o);
    squares += __shfl_xor_sync(0xffffffffu, squares, o);
  }
  if ((threadIdx.x & 31) == 0) {
    red[0][threadIdx.x >> 5] = sum;
    red[1][threadIdx.x >> 5] = squares;
  }
  __syncthreads();
  sum = 0.0f;
  squares = 0.0f;
#pragma unroll
  for (int i = 0; i < kNormThreads / 32; ++i) {
    sum += red[0][i];
    squares += red[1][i];
  }
  float mean = 0.0f, inv;
  if (LN) {
    mean = sum / (float)width;
    inv = rsqrtf(fmaxf(squares / (float)width - mean * mean, 0.0f) + eps);
  } else {
    inv = rsqrtf(squares / (float)width + eps);
  }
  for (int i = threadIdx.x; i < width; i += kNormThreads) {
    const float v = rnd<T>(ld(x, base + i) + ld(b, bbase + i));
    float out = (v - mean) * inv * ld(w, (size_t)i);
    if (LN) out += ld(c, (size_t)i);
    st(y, base + i, out);
  }
}

// y = T(T(silu(x)) * b), silu evaluated on the side of zero that keeps exp's
// argument non-positive.
template <typename T>
__global__ void silu_mul_kernel(const T *__restrict__ x, const T *__restrict__ b, T *__restrict__ y, size_t count,
                                int width, int b_rows) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += (size_t)gridDim.x * blockDim.x) {
    const float v = ld(x, i);
    const float e = expf(v >= 0.0f ? -v : v);
    const float act = rnd<T>(v >= 0.0f ? v / (1.0f + e) : v * e / (1.0f + e));
    const size_t bi = b_rows == 1 ? i % (size_t)width : i;
    st(y, i, act * ld(b, bi));
  }
}

// y[m, n] = T(max(T(T(sum_k a[m, k] w[k, n]) + bias[n]), 0)): 16 x 16 output
// tiles, K in 16-wide slabs through shared memory, sums in K order.
constexpr int kTile = 16;
template <typename T>
__global__ void linear_relu_kernel(const T *__restrict__ a, const T *__restrict__ w, const T *__restrict__ bias,
                                   T *__restrict__ y, int m, int k, int n) {
  __shared__ float sa[kTile][kTile + 1], sw[kTile][kTile + 1];
  const int row = blockIdx.y * kTile + threadIdx.y, col = blockIdx.x * kTile + threadIdx.x;
  float sum = 0.0f;
  for (int k0 = 0; k0 < k; k0 += kTile) {
    const int ka = k0 + threadIdx.x, kw = k0 + threadIdx.y;
    sa[threadIdx.y][threadIdx.x] = row < m && ka < k ? ld(a, (size_t)row * k + ka) : 0.0f;
    sw[threadIdx.y][threadIdx.x] = kw < k && col < n ? ld(w, (size_t)kw * n + col) : 0.0f;
    __syncthreads();
    const int kk = min(kTile, k - k0);
    for (int i = 0; i < kk; ++i) sum += sa[threadIdx.y][i] * sw[i][threadIdx.x];
    __syncthreads();
  }
  if (row < m && col < n) {
    const float linear = rnd<T>(sum);
    const float biased = rnd<T>(linear + ld(bias, (size_t)col));
    st(y, (size_t)row * n + col, fmaxf(biased, 0.0f));
  }
}

}  // namespace

cudaError_t launch_fused_add_norm(const void *x, const void *b, const void *w, const void *c, void *y, int rows,
                                  int width, int b_rows, float eps, bool layer_norm, bool fp16, cudaStream_t stream) {
  if (rows <= 0 || width <= 0 || (b_rows != 1 && b_rows != rows) || (layer_norm && c == nullptr))
    return cudaErrorInvalidValue;
#define TMC_ADD_NORM(T, LN)                                                                                   \
  add_norm_kernel<T, LN><<<rows, kNormThreads, 0, stream>>>(                                                  \
      static_cast<const T *>(x), static_cast<const T *>(b), static_cast<const T *>(w), static_cast<const T *>(c), \
      static_cast<T *>(y), width, b_rows, eps)
  if (fp16) {
    if (layer_norm)
      TMC_ADD_NORM(__half, true);
    else
      TMC_ADD_NORM(__half, false);
  } else {
    if (layer_norm)
      TMC_ADD_NORM(float, true);
    else
      TMC_ADD_NORM(float, false);
  }
#undef TMC_ADD_NORM
  return cudaGetLastError();
}

cudaError_t launch_fused_silu_mul(const void *x, const void *b, void *y, int rows, int width, int b_rows, bool fp16,
                                  cudaStream_t stream) {
  if (rows <= 0 || width <= 0 || (b_rows != 1 && b_rows != rows)) return cudaErrorInvalidValue;
  const size_t count = (size_t)rows * width;
  const int grid = (int)((count + 255) / 256 < 4096 ? (count + 255) / 256 : 4096);
  if (fp16)
    silu_mul_kernel<__half><<<grid, 256, 0, stream>>>(static_cast<const __half *>(x), static_cast<const __half *>(b),
                                                      static_cast<__half *>(y), count, width, b_rows);
  else
    silu_mul_kernel<float><<<grid, 256, 0, stream>>>(static_cast<const float *>(x), static_cast<const float *>(b),
                                                     static_cast<float *>(y), count, width, b_rows);
  return cudaGetLastError();
}

cudaError_t launch_fused_linear_relu(const void *a, const void *w, const void *bias, void *y, int m, int k, int n,
                                     bool fp16, cudaStream_t stream) {
  if (m <= 0 || k <= 0 || n <= 0 || m > 65535 * kTile) return cudaErrorInvalidValue;
  const dim3 grid((n + kTile - 1) / kTile, (m + kTile - 1) / kTile), block(kTile, kTile);
  if (fp16)
    linear_relu_kernel<__half><<<grid, block, 0, stream>>>(static_cast<const __half *>(a),
                                                           static_cast<const __half *>(w),
                                                           static_cast<const __half *>(bias), static_cast<__half *>(y),
                                                           m, k, n);
  else
    linear_relu_kernel<float><<<grid, block, 0, stream>>>(static_cast<const float *>(a), static_cast<const float *>(w),
                                                          static_cast<const float *>(bias), static_cast<float *>(y), m,
                                                          k, n);
  return cudaGetLastError();
}

}  // namespace tmc
