// Single-token decode of one layer boundary as one persistent kernel: the
// O projection of layer l (+ residual), gate/up (+ RMSNorm prologue, SwiGLU),
// down (+ residual), then the QKV projection of layer l + 1 (+ RMSNorm, RoPE,
// KV append) or, after the last layer, the LM head (+ final RMSNorm, argmax).
//
// Why: at one token per step every projection is a weight stream (about 1
// flop per byte), and the step's time goes to the gaps between them -- each
// kernel boundary costs a dependency hand-off of a few microseconds and each
// small GEMV a ramp-up and a tail. Here one CTA per SM runs all four phases,
// separated by bounded grid barriers, and every warp streams its weight rows
// into a shared-memory ring with 1-D bulk copies (cp.async.bulk) issued ahead
// of its consumption: the copies for the next phase are in flight while the
// warp waits at the barrier for the activations the phase needs, so HBM keeps
// streaming through the dependency. Per step: 1 QKV GEMV, then per layer one
// attention kernel and one of these (65 launches for 32 layers instead of 161).
//
// Arithmetic: every output row is computed exactly as the decode GEMV computes
// it for one token (gemv.cu): the same RMSNorm prologue (256 threads, same
// sum order and block reduction), the lane of a warp accumulating the 16-byte
// chunks lane, lane + 32, ... of the row in order, the same butterfly
// reduction and the same epilogue functions -- so the two paths give
// bit-identical results and either may serve any step.
#pragma once

#include "gemv.cuh"

namespace tmc {

constexpr int kStreamPhases = 4;
constexpr int kStreamSyncWords = 2 * 32;  // grid-barrier counter line, exit counter line

struct StreamParams {
  // phase[0] O projection (kProF16 x = attention context, kEpiResidual),
  // phase[1] gate/up (kProF16Norm, kEpiSwiGLU), phase[2] down (kProF16,
  // kEpiResidual), phase[3] next layer's QKV (kProF16Norm, kEpiQKV) or the LM
  // head (kProF16Norm, kEpiArgmax). M = 1 in every phase.
  GemvParams phase[kStreamPhases];
  unsigned int *sync;  // kStreamSyncWords words, zero before the launch; left zero
};

// False when the phases' shapes do not fit the kernel (largest K staged in
// shared memory next to a ring of at least two stages per warp).
bool layer_stream_fits(const StreamParams &p);
cudaError_t launch_layer_stream(const StreamParams &p, cudaStream_t stream, bool pdl, int num_sms);

}  // namespace tmc
