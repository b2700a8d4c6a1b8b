// Fused graph regions of the TensorGraph path: the bodies formRegions
// (PatternAnalyzer.cpp:32-132) groups and emitFusion (FusionMetalEmitter.cpp:81-214)
// emits -- Add -> RMSNorm, residual Add -> LayerNorm, SiLU -> Mul and
// MatMul -> Add(bias) -> ReLU -- with the same arithmetic: fp32, every
// intermediate node rounded to the storage type (fp32 or fp16) before the next
// reads it, the LayerNorm variance as max(E[v^2] - mean^2, 0).
//
// x [rows, width] row-major; an Add / Mul operand b is [b_rows, width] with
// b_rows 1 (broadcast over rows) or rows; norm weight / bias [width]. The
// linear layer is y = relu(a . w + bias) with a [m, k], w [k, n] (row-major
// K x N, the MatMul operand order of the graph), bias [n].
#pragma once

#include "common.cuh"

namespace tmc {

cudaError_t launch_fused_add_norm(const void *x, const void *b, const void *w, const void *c, void *y, int rows,
                                  int width, int b_rows, float eps, bool layer_norm, bool fp16, cudaStream_t stream);
cudaError_t launch_fused_silu_mul(const void *x, const void *b, void *y, int rows, int width, int b_rows, bool fp16,
                                  cudaStream_t stream);
cudaError_t launch_fused_linear_relu(const void *a, const void *w, const void *bias, void *y, int m, int k, int n,
                                     bool fp16, cudaStream_t stream);

}  // namespace tmc
