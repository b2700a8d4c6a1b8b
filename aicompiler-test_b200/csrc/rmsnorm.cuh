// Standalone RMSNorm over rows: y[r, c] = x[r, c] * rsqrt(mean_c(x[r, :]^2) + eps) * gamma[c],
// fp32 accumulation, x / gamma / y all fp32 or all fp16 (RMSNormOp,
// TensorIR.hpp:98-104; emitRMSNorm, MetalEmitter.cpp:12-76). The decoder never
// launches this: its RMSNorms are fused into the GEMV / GEMM prologues. It is
// the graph-level operator and the subject of the RMSNorm tuner.
#pragma once

#include "common.cuh"

namespace tmc {

// One CTA per row, `threads` in {32, 64, ..., 1024}; 16-byte vector loads when
// the width and every pointer allow, else scalar loads.
cudaError_t launch_rmsnorm(const void *x, const void *gamma, void *y, int rows, int width, float eps, bool fp16,
                           int threads, cudaStream_t stream);
// The frozen baseline: 256 threads, scalar loads, shared-memory tree reduction.
cudaError_t launch_rmsnorm_baseline(const void *x, const void *gamma, void *y, int rows, int width, float eps,
                                    bool fp16, cudaStream_t stream);

}  // namespace tmc
