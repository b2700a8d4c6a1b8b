// Graph-path kernels for the nodes of a compiled tensor graph that no fused
// region or decode kernel covers: the reference's per-node kernels emitted by
// emitKernel (src/backend/metal/GraphMetalEmitter.cpp:122-346) for Add / Mul
// (with the row broadcast the fused regions also accept), ReLU, SiLU and
// MatMul. Storage is all fp32 or all fp16, except that a MatMul's right-hand
// operand may be fp16 under an fp32 left-hand side (weights kept in fp16).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace tmc {

// y = x + b or x * b; x, y [rows, width], b [b_rows, width] with b_rows 1 or rows.
cudaError_t launch_graph_binary(const void *x, const void *b, void *y, int rows, int width, int b_rows, bool mul,
                                bool fp16, cudaStream_t stream);
// y = relu(x) or silu(x) over `count` elements.
cudaError_t launch_graph_unary(const void *x, void *y, size_t count, bool silu, bool fp16, cudaStream_t stream);
// y [m, n] = a [m, k] . W, with W either row-major [k, n] or (w_transposed) a
// Transpose view of a row-major [n, k] matrix.
cudaError_t launch_graph_matmul(const void *a, const void *w, void *y, int m, int k, int n, bool w_transposed,
                                bool a_fp16, bool w_fp16, cudaStream_t stream);

}  // namespace tmc
