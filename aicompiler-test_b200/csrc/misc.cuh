#pragma once

#include "common.cuh"

namespace tmc {

cudaError_t launch_fill_normal_f16(__half *dst, size_t count, uint64_t seed, float mean,
                                   float stddev, cudaStream_t stream);
// Logical-index N(mean, std) fill of a [rows, cols] window (see misc.cu).
cudaError_t launch_fill_normal_2d(__half *dst, int rows, int cols, long long dst_stride,
                                  uint64_t seed, long long logical_row0, long long logical_cols,
                                  long long logical_col0, float mean, float stddev,
                                  cudaStream_t stream);
cudaError_t launch_fill_value_f16(__half *dst, size_t count, float value, cudaStream_t stream);
cudaError_t launch_fill_uniform_f32(float *dst, size_t count, uint64_t seed, float lo, float hi,
                                    cudaStream_t stream);
// Tokens from packed argmax keys (see argmax_key in common.cuh); resets keys.
cudaError_t launch_argmax_finalize(unsigned long long *keys, int rows, int *next_tokens,
                                   int *feed_tokens, int *feed_positions, int *history,
                                   unsigned int *history_counter, cudaStream_t stream, bool pdl);
// h = half(h + half(partial)) for a reduced row-parallel projection.
cudaError_t launch_add_residual_f32(__half *h, const float *partial, int n, cudaStream_t stream,
                                    bool pdl);

// Page images between the per-layer K/V pools and a packed buffer:
// packed[((l * 2 + kv) * npages + i) * page_elems ..] <-> pools[l * 2 + kv][pages[i] * page_elems ..]
// (pools: a device array of 2 * layers pool pointers, K then V per layer).
// to_packed gathers (spill), otherwise scatters (restore). page_elems % 8 == 0.
cudaError_t launch_page_copy(__half *const *pools, const int *pages, int npages, int layers, size_t page_elems,
                             __half *packed, bool to_packed, cudaStream_t stream);

}  // namespace tmc
