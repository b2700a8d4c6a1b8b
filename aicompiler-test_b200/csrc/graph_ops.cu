// Generic graph-path kernels for nodes no fused region covers (see
// graph_ops.cuh): binary Add / Mul with row broadcast, ReLU / SiLU, and a tiled
// MatMul. Every result is computed in fp32 and rounded once to the storage
// type, as the reference's evaluateGraph stores each node's value
// (src/validation/GraphReference.cpp:82-87).
#include "graph_ops.cuh"

namespace tmc {
namespace {

template <typename T>
__device__ __forceinline__ float ldv(const T *p, size_t i);
template <>
__device__ __forceinline__ float ldv<float>(const float *p, size_t i) {
  return p[i];
}
template <>
__device__ __forceinline__ float ldv<__half>(const __half *p, size_t i) {
  return __half2float(p[i]);
}
__device__ __forceinline__ void stv(float *p, size_t i, float v) { p[i] = v; }
__device__ __forceinline__ void stv(__half *p, size_t i, float v) { p[i] = __float2half_rn(v); }

// y[i] = T(x[i] op b[j]), j = i (b_rows == rows) or i mod width (b_rows == 1).
template <typename T, bool MUL>
__global__ void binary_kernel(const T *__restrict__ x, const T *__restrict__ b, T *__restrict__ y, size_t count,
                              int width, int b_rows) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += (size_t)gridDim.x * blockDim.x) {
    const float a = ldv(x, i);
    const float c = ldv(b, b_rows == 1 ? i % (size_t)width : i);
    stv(y, i, MUL ? __fmul_rn(a, c) : __fadd_rn(a, c));
  }
}

// ReLU, or SiLU with exp's argument kept non-positive (the fused region's form).
template <typename T, bool SILU>
__global__ void unary_kernel(const T *__restrict__ x, T *__restrict__ y, size_t count) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += (size_t)gridDim.x * blockDim.x) {
    const float v = ldv(x, i);
    float r;
    if (SILU) {
      const float e = expf(v >= 0.0f ? -v : v);
      r = v >= 0.0f ? v / (1.0f + e) : v * e / (1.0f + e);
    } else {
      r = fmaxf(v, 0.0f);
    }
    stv(y, i, r);
  }
}

// y[m, n] = T(sum_k a[m, k] w(k, n)), w(k, n) = w[k * n_total + n] or, for a
// Transpose view of a [N, K] matrix, w[n * K + k]: 16 x 16 output tiles, K in
// 16-wide slabs through shared memory, sums in K order.
constexpr int kTile = 16;
template <typename TA, typename TW>
__global__ void matmul_kernel(const TA *__restrict__ a, const TW *__restrict__ w, TA *__restrict__ y, int m, int k,
                              int n, int w_transposed) {
  __shared__ float sa[kTile][kTile + 1], sw[kTile][kTile + 1];
  const int row = blockIdx.y * kTile + threadIdx.y, col = blockIdx.x * kTile + threadIdx.x;
  float sum = 0.0f;
  for (int k0 = 0; k0 < k; k0 += kTile) {
    const int ka = k0 + threadIdx.x, kw = k0 + threadIdx.y;
    sa[threadIdx.y][threadIdx.x] = row < m && ka < k ? ldv(a, (size_t)row * k + ka) : 0.0f;
    float wv = 0.0f;
    if (kw < k && col < n) wv = w_transposed ? ldv(w, (size_t)col * k + kw) : ldv(w, (size_t)kw * n + col);
    sw[threadIdx.y][threadIdx.x] = wv;
    __syncthreads();
    const int kk = min(kTile, k - k0);
    for (int i = 0; i < kk; ++i) sum = fmaf(sa[threadIdx.y][i], sw[i][threadIdx.x], sum);
    __syncthreads();
  }
  if (row < m && col < n) stv(y, (size_t)row * n + col, sum);
}

int grid_for(size_t count) {
  const size_t blocks = (count + 255) / 256;
  return (int)(blocks < 4096 ? (blocks > 0 ? blocks : 1) : 4096);
}

}  // namespace

cudaError_t launch_graph_binary(const void *x, const void *b, void *y, int rows, int width, int b_rows, bool mul,
                                bool fp16, cudaStream_t stream) {
  if (rows <= 0 || width <= 0 || (b_rows != 1 && b_rows != rows)) return cudaErrorInvalidValue;
  const size_t count = (size_t)rows * width;
  const int grid = grid_for(count);
#define TMC_BIN(T, MUL)                                                                                     \
  binary_kernel<T, MUL><<<grid, 256, 0, stream>>>(static_cast<const T *>(x), static_cast<const T *>(b), \
                                                  static_cast<T *>(y), count, width, b_rows)
  if (fp16) {
    if (mul) TMC_BIN(__half, true); else TMC_BIN(__half, false);
  } else {
    if (mul) TMC_BIN(float, true); else TMC_BIN(float, false);
  }
#undef TMC_BIN
  return cudaGetLastError();
}

cudaError_t launch_graph_unary(const void *x, void *y, size_t count, bool silu, bool fp16, cudaStream_t stream) {
  if (count == 0) return cudaErrorInvalidValue;
  const int grid = grid_for(count);
  if (fp16) {
    if (silu)
      unary_kernel<__half, true><<<grid, 256, 0, stream>>>(static_cast<const __half *>(x), static_cast<__half *>(y), count);
    else
      unary_kernel<__half, false><<<grid, 256, 0, stream>>>(static_cast<const __half *>(x), static_cast<__half *>(y), count);
  } else {
    if (silu)
      unary_kernel<float, true><<<grid, 256, 0, stream>>>(static_cast<const float *>(x), static_cast<float *>(y), count);
    else
      unary_kernel<float, false><<<grid, 256, 0, stream>>>(static_cast<const float *>(x), static_cast<float *>(y), count);
  }
  return cudaGetLastError();
}

cudaError_t launch_graph_matmul(const void *a, const void *w, void *y, int m, int k, int n, bool w_transposed,
                                bool a_fp16, bool w_fp16, cudaStream_t stream) {
  if (m <= 0 || k <= 0 || n <= 0 || m > 65535 * kTile || (a_fp16 && !w_fp16)) return cudaErrorInvalidValue;
  const dim3 grid((n + kTile - 1) / kTile, (m + kTile - 1) / kTile), block(kTile, kTile);
  const int wt = w_transposed ? 1 : 0;
  if (a_fp16)
    matmul_kernel<__half, __half><<<grid, block, 0, stream>>>(static_cast<const __half *>(a),
                                                              static_cast<const __half *>(w), static_cast<__half *>(y),
                                                              m, k, n, wt);
  else if (w_fp16)
    matmul_kernel<float, __half><<<grid, block, 0, stream>>>(static_cast<const float *>(a),
                                                             static_cast<const __half *>(w), static_cast<float *>(y),
                                                             m, k, n, wt);
  else
    matmul_kernel<float, float><<<grid, block, 0, stream>>>(static_cast<const float *>(a), static_cast<const float *>(w),
                                                            static_cast<float *>(y), m, k, n, wt);
  return cudaGetLastError();
}

}  // namespace tmc
