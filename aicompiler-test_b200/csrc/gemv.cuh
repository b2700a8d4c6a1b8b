// Decode GEMV family: y[m, n] = sum_k x[m, k] * W[n, k] with fp16 W (row-major
// [N, K]), fp32 accumulation, an optional fused prologue on x (RMSNorm,
// embedding gather) and a fused epilogue (store, residual add, RoPE + KV-cache
// append, SwiGLU, LM-head argmax).
//
// This replaces the reference's Metal emitters for the decode linear layers:
// emitDecodeGEMV / emitLinearBaseline (DecodeGEMVMetalEmitter.cpp:18-132),
// emitDecoderQKVFusion (DecoderLLMMetalEmitter.cpp:538-602),
// emitDecoderGatedMLP (:479-536), emitLinearResidual (:604-621),
// emitLMHeadPartialArgmax/FinalArgmax (:700-753) and the RMSNorm prologue of
// emitDecoderRMSNorm (:63-108).
#pragma once

#include "common.cuh"

namespace tmc {

enum GemvPrologue : int {
  kProF32 = 0,        // xs = x (fp32 input)
  kProF32Norm = 1,    // xs = x * rsqrt(mean(x^2)+eps) * gamma, all fp32 (C1 graph)
  kProF16 = 2,        // xs = x (fp16 input)
  kProF16Norm = 3,    // xs = half(x * inv * gamma)   (decoder RMSNorm, fp16 storage)
  kProEmbedNorm = 4,  // x = embedding[token[m]]; CTA 0 stores x to h_out; then kProF16Norm
  kProResidualNorm = 5,  // x = half(h[m] + half(partial[m])) (reduced row-parallel output,
                         // or the rank-ordered sum of the peer-exchange slots);
                         // CTA 0 stores x to h_out; then kProF16Norm
};

enum GemvEpilogue : int {
  kEpiF32 = 0,       // y_f32[m, n] = acc
  kEpiF16 = 1,       // y_f16[m, n] = half(acc)
  kEpiResidual = 2,  // y_f16[m, n] = half(residual[m, n] + half(acc))   (in place allowed)
  kEpiQKV = 3,       // rows = [q | k | v]; RoPE on q,k; q -> y_f16; k,v -> paged cache
  kEpiSwiGLU = 4,    // rows interleaved (gate_i, up_i) -> y_f16[m, i] = half(half(silu(g)) * u)
  kEpiArgmax = 5,    // LM head: logits (fp16-rounded) -> y_f32 (optional) + argmax token
  kEpiF32Partial = 6 // y_f32[m, n] = acc (row-parallel partial sum, reduced across ranks),
                     // or stored into every rank's exchange slot (xchg.world > 0)
};

// ---- one-shot peer exchange over NVLink (tensor parallelism) ------------------
// Each rank owns an exchange window in its HBM that every other rank maps
// (CUDA IPC). A row-parallel GEMV (O, down) stores its fp32 partial outputs
// straight into slot [parity][own rank] of EVERY rank's window as it produces
// them, and its last CTA then raises flag [parity][own rank] in every window;
// the next kernel's prologue waits (bounded) for all ranks' flags in its own
// window and sums the slots in rank order -- the same values in the same order
// on every rank, so the replicated residual stream stays bit-identical. The
// LM head exchanges its packed argmax keys the same way and its last CTA
// finalises the token. Flag values grow monotonically (epoch * phases + phase
// + 1 for partial sums, epoch + 1 for argmax keys), so a wait is "flag >=
// value"; a slot parity is reused only after every rank has consumed it (a
// rank writes phase q + 2 only after it waited for every rank's phase q + 1,
// which each rank produces only after consuming phase q).
constexpr int kMaxPeers = 8;
constexpr int kPeerFlagStride = 32;  // uints: one 128-byte line per (set, source rank)
constexpr int kPeerFlagSets = 4;     // partial-sum parity 0/1, argmax parity 0/1
constexpr size_t kPeerFlagBytes = (size_t)kPeerFlagSets * kMaxPeers * kPeerFlagStride * 4;

__host__ __device__ inline size_t peer_key_offset() { return kPeerFlagBytes; }
__host__ __device__ inline size_t peer_slot_offset(int slot_rows) {
  return kPeerFlagBytes + ((size_t)2 * kMaxPeers * slot_rows * 8 + 255) / 256 * 256;
}
__host__ __device__ inline size_t peer_window_bytes(int slot_rows, int width) {
  return peer_slot_offset(slot_rows) + (size_t)2 * kMaxPeers * slot_rows * width * 4;
}

struct PeerExchange {
  int world;             // ranks exchanging; 0 = this launch exchanges nothing
  int rank;
  int wait;              // consumers wait for the flags (0 only for isolated timing runs)
  int signal;            // producers raise the flags (0 on all but the last row-split launch)
  int slot_rows;         // rows per slot (the decoder's max rows)
  int width;             // features per slot row (hidden size)
  int row0;              // first slot row of this launch (row-split launches)
  unsigned int phase;    // partial-sum phase produced or consumed by this launch
  unsigned int phases;   // partial-sum phases per step
  char *window[kMaxPeers];  // every rank's window, mapped into this process
  unsigned int *epoch;   // steps completed on this rank (the LM head's last CTA advances it)
  unsigned int *done;    // CTA-completion counter of this launch site (zero between launches)
};

struct GemvParams {
  const __half *W;  // [N, K]
  int N, K, M;
  // ---- prologue ----
  int prologue;
  const void *x;       // [M, x_stride] (fp32 or fp16 per prologue)
  long long x_stride;  // elements
  const void *gamma;   // [K] fp32 (kProF32Norm) or fp16 (kProF16Norm/kProEmbedNorm)
  float eps;
  const __half *embedding;  // [vocab, K]
  const int *tokens;        // [M]
  int vocab;
  __half *h_out;            // [M, K] residual-stream write-back (embedding / residual prologue)
  const float *partial;     // [M, K] reduced fp32 projection (kProResidualNorm)
  // ---- epilogue ----
  int epilogue;
  float *y_f32;
  __half *y_f16;
  long long y_stride;      // elements between output rows
  const __half *residual;  // [M, y_stride] (kEpiResidual)
  // QKV / cache append
  int q_rows;            // Hq_local * D
  int kv_rows;           // Hkv_local * D
  int head_dim;
  const float *rope_cos;  // [capacity, D/2]
  const float *rope_sin;
  const int *positions;   // [M] position of the row's token
  const int *table_rows;  // [M] block-table row of the row's sequence
  const int *block_table; // [rows, table_stride]
  int table_stride;       // max logical pages per sequence
  int page_size;
  int pool_pages;
  int capacity;           // max position + 1
  __half *k_pool;         // [pages, Hkv_local, page_size, D]
  __half *v_pool;
  // argmax
  unsigned long long *argmax_keys;  // [M] (zero before launch; the last CTA resets)
  unsigned int *argmax_counter;     // [1]
  int *next_tokens;                 // [M]
  int *feed_tokens;                 // [M] optional: next step's input tokens
  int *feed_positions;              // [M] optional: positions += 1 (greedy loop)
  int *history;                     // optional [steps, M] generated tokens
  unsigned int *history_counter;    // [1] steps recorded so far
  int vocab_offset;                 // global index of local row 0 (vocab-parallel head)
  TmcDeviceStatus *status;
  TraceSink trace;                  // optional timeline (records == nullptr: off)
  // Optional dynamic row-group scheduling: kGemvPools ticket counters, each on
  // its own 128-byte line (stride kGemvPoolStride uints), then a CTA exit
  // ticket; all zero before the launch and reset by the last CTA. Null: the
  // static interleaved assignment.
  unsigned int *work_counter;
  // Bytes of W this launch may bulk-prefetch into L2 before its inputs are
  // ready (0: none).
  long long l2_prefetch_bytes;
  // Budgets of this launch's bounded waits, in ns of global time (0: the
  // defaults): peer_wait_ns for another rank's exchange flags (10 s),
  // local_wait_ns for the GEMM's mbarrier and split-tile waits (1 s).
  unsigned long long peer_wait_ns;
  unsigned long long local_wait_ns;
  // K-split team size chosen by the decode GEMV tuner (1, 2, 4 or 8); 0: the
  // built-in rule.
  int force_ks;
  // Nonzero when the residual rows (kEpiResidual) were final before the
  // preceding kernel started, i.e. written two or more kernels back in a chain
  // where every kernel releases its dependents only after its own dependency
  // wait. Single-row launches then read their first row group's residuals
  // before their own wait instead of in the epilogue.
  int early_epilogue_inputs;
  // Tensor parallelism over peer memory (kEpiF32Partial producers,
  // kProResidualNorm consumers, kEpiArgmax key exchange); world 0: off.
  PeerExchange xchg;
};

// One 16-byte chunk (8 fp16 weights) of a row against 8 staged activations,
// accumulated in element order with fused multiply-adds. Every kernel that
// computes decode-GEMV rows uses this, so their per-row sums agree bit for bit.
__device__ __forceinline__ float gemv_dot8(const uint4 w, const float (&x)[8], float acc) {
  float2 a = half2_bits_to_float2(w.x);
  acc = fmaf(a.x, x[0], acc); acc = fmaf(a.y, x[1], acc);
  a = half2_bits_to_float2(w.y);
  acc = fmaf(a.x, x[2], acc); acc = fmaf(a.y, x[3], acc);
  a = half2_bits_to_float2(w.z);
  acc = fmaf(a.x, x[4], acc); acc = fmaf(a.y, x[5], acc);
  a = half2_bits_to_float2(w.w);
  acc = fmaf(a.x, x[6], acc); acc = fmaf(a.y, x[7], acc);
  return acc;
}

constexpr int kGemvPools = 8;
constexpr int kGemvPoolStride = 32;
constexpr int kGemvCounterWords = (kGemvPools + 1) * kGemvPoolStride;

// Host-side launcher; returns a cudaError_t. Chooses the template instance
// from (M, K) and the grid from the device occupancy.
cudaError_t launch_gemv(const GemvParams &p, cudaStream_t stream, bool pdl,
                        int num_sms);

// The prologue alone, for the batched tensor-core GEMM: xn[m, :] = fp16 row m
// after p.prologue (fp16 prologues only; M any positive count), one CTA per
// row; h_out and the exchange waits behave as in the GEMV.
cudaError_t launch_row_prologue(const GemvParams &p, __half *xn, cudaStream_t stream, bool pdl);

}  // namespace tmc
