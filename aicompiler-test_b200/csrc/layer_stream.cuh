// Single-token decode of one layer boundary as one persistent kernel: the
// O projection of layer l (+ residual), gate/up (+ RMSNorm prologue, SwiGLU),
// down (+ residual), then the QKV projection of layer l + 1 (+ RMSNorm, RoPE,
// KV append) or, after the last layer, the LM head (+ final RMSNorm, argmax).
//
// Why: at one token per step every projection is a weight stream (about 1
// flop per byte), and a separate kernel per projection pays a launch and a
// dependency hand-off at every boundary. Here one grid (two CTAs of 8 warps
// per SM, every CTA resident) runs the four phases of the decode GEMV's own
// loop (gemv.cu) back to back, separated by bounded grid barriers: before a
// phase's inputs exist, each warp already holds its first batch of weights in
// registers and has bulk-prefetched its share into L2 -- what the GEMV does
// before its programmatic-dependency wait -- so the barrier replaces a kernel
// boundary. Per step: 1 QKV GEMV, then per layer one attention kernel and one
// of these (65 launches for 32 layers instead of 161). At the end of a launch
// the next layer's O weights are prefetched into L2 while attention runs.
//
// Arithmetic: each phase is the GEMV's code for one row (prologue, lane chunk
// order, reductions, epilogue functions), so the two paths give bit-identical
// results and either may serve any step.
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
  // The next launch's first weights (the next layer's O projection, [rows,
  // k] fp16), pulled into L2 once this launch has issued all of its own
  // loads, so they stream from HBM while the attention kernel in between
  // runs; null after the last layer.
  const __half *next_w;
  int next_rows, next_k;
};

// False when the phases do not fit the kernel (one row, no peer exchange, the
// O / gate-up / down / QKV-or-LM-head epilogues, staged activations within
// the GEMV's shared-memory budget).
bool layer_stream_fits(const StreamParams &p);
cudaError_t launch_layer_stream(const StreamParams &p, cudaStream_t stream, bool pdl, int num_sms);

}  // namespace tmc
