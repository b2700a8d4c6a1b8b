// Decoder-only LLM executor for B200: single-token (and chunked) decode of a
// pre-norm RMSNorm / interleaved-RoPE / GQA / SwiGLU model with fp16 storage
// and fp32 accumulation, whole steps captured as CUDA graphs.
//
// Mirrors tensor::runtime::CompiledDecoderLLM (reference
// src/runtime/DecoderLLMExecutor.hpp:46-102) and its compile options
// (DecoderLLMCompileOptions, :19-29):
//   prefill / decode / currentLength / readKeyPrefix / readValuePrefix /
//   kvBlockTable / stageKVLength / commitKVLength / rollbackKVLength /
//   snapshotKVCache / restoreKVCache / releaseKVCache / storage accounting.
// Extensions over the reference (which is MHA-only with theta 1e4 and one
// request per executor): grouped-query attention (kvHeads), rope theta, up to
// maxSlots sequences with their own KV state sharing one page pool, a
// device-resident greedy loop (generate), and tensor parallelism across ranks.
//
// One decode step over R rows (each row = one token of one sequence) is, per
// layer, 5 kernels (all launched with programmatic dependent launch):
//   1. QKV GEMV   prologue RMSNorm(h) [layer 0: embedding gather]
//                 epilogue RoPE(q, k) + paged KV append (k, v)
//   2. attention  block-table GQA split-K decode attention
//   3. O GEMV     epilogue h = half(h + half(o))          [TP: fp32 partial + allreduce]
//   4. gate/up    prologue RMSNorm(h), epilogue SwiGLU  [TP: prologue adds the reduced o]
//   5. down GEMV  epilogue h = half(h + half(down))       [TP: fp32 partial + allreduce]
// then the LM head GEMV (prologue final RMSNorm, epilogue fp16 logits + argmax).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <map>
#include <tuple>
#include <memory>
#include <string>
#include <utility>
#include <vector>

#include "CudaRuntime.hpp"
#include "KVCacheState.hpp"
#include "common.cuh"
#include "gemm.cuh"
#include "gemv.cuh"

namespace tensor::runtime {

struct DecoderConfig {
  int hidden = 0;
  int heads = 0;
  int kvHeads = 0;       // == heads for the reference's MHA models
  int headDim = 0;
  int intermediate = 0;
  int vocab = 0;
  int layers = 0;
  int capacity = 0;      // max positions per sequence (RoPE table rows)
  float epsilon = 1e-5f;
  double ropeTheta = 10000.0;
  int maxRows = 8;       // rows per step (tokens across all sequences)
  int maxSlots = 1;      // sequences with KV state
  int pageSize = 0;      // 0 = contiguous per sequence (page = capacity)
  int poolPages = 0;     // 0 = maxSlots * pages per full sequence
  int tpRank = 0;
  int tpSize = 1;
  bool useGraphs = true;
  bool usePDL = true;
  // Budgets of the kernels' bounded waits in ns (0: the kernel defaults, 10 s
  // for another rank's exchange flags and 1 s for a GEMM's mbarrier and
  // split-tile waits). A wait that runs out is reported through the device
  // status block and the call returns a "device status" error.
  std::uint64_t peerWaitNs = 0;
  std::uint64_t localWaitNs = 0;
};

// Cross-rank sum/max used by tensor parallelism (implemented over NCCL).
class Collective {
 public:
  virtual ~Collective() = default;
  virtual cudaError_t allReduceSumF32(float *buf, std::size_t count, cudaStream_t s) = 0;
  virtual cudaError_t allReduceMaxU64(unsigned long long *buf, std::size_t count, cudaStream_t s) = 0;
  virtual std::string lastError() const = 0;
};

struct StepTiming {
  double gpuUs = 0.0;
  double cpuUs = 0.0;
};

class DecoderExecutor {
 public:
  // Kernel kinds of one decode step, in launch order per layer.
  enum KernelKind : int {
    kKernelQKV = 0,
    kKernelAttention = 1,
    kKernelO = 2,
    kKernelGateUp = 3,
    kKernelDown = 4,
    kKernelLMHead = 5,
  };
  static std::unique_ptr<DecoderExecutor> create(cuda::CudaRuntime &runtime, const DecoderConfig &config,
                                                 std::string *error);
  ~DecoderExecutor();
  DecoderExecutor(const DecoderExecutor &) = delete;
  DecoderExecutor &operator=(const DecoderExecutor &) = delete;

  const DecoderConfig &config() const { return cfg_; }
  int localHeads() const { return hqL_; }
  int localKVHeads() const { return hkvL_; }
  int localIntermediate() const { return iL_; }
  int localVocab() const { return vL_; }
  int vocabOffset() const { return cfg_.tpRank * vL_; }

  // ---- weights (logical, unsharded names of the reference manifest:
  // export_decoder_llm.py:531-547) ----
  std::string loadWeight(const std::string &name, const float *values, std::size_t count);
  std::string loadWeightF16(const std::string &name, const std::uint16_t *bits, std::size_t count);
  // Logical weight readback (rank-local shard for sharded tensors) as fp32.
  std::string readWeight(const std::string &name, std::vector<float> *out) const;
  // Every matrix ~N(0, stddev) from a counter-based generator indexed by the
  // logical element (identical across tensor-parallel layouts); norms = 1.
  std::string initRandom(std::uint64_t seed, float stddev);
  // RoPE tables [capacity, headDim/2] (the manifest's rope.cosine/rope.sine).
  std::string setRope(const float *cosine, const float *sine, std::size_t rows);
  std::string setCollective(std::shared_ptr<Collective> collective);
  // ---- tensor parallelism over peer memory (no reference counterpart: the
  // reference has no multi-GPU code) ----
  // CUDA IPC handle (cudaIpcMemHandle_t bytes) of this rank's exchange window.
  std::string exchangeHandle(void *out, std::size_t size);
  // Map every rank's window (rank r's exchangeHandle at handles + r * size)
  // and switch the row-parallel reductions and the LM-head argmax from the
  // collective to the one-shot peer exchange fused into the GEMV kernels.
  std::string attachPeers(const void *handles, std::size_t size, int world, int rank);
  // The same over ranks driven by this process (ranks[r] = rank r's
  // executor, on any device with peer access to this one): their windows are
  // used directly, without IPC.
  std::string attachLocalPeers(const std::vector<DecoderExecutor *> &ranks, int rank);
  bool peersAttached() const { return peersAttached_; }
  // Replace the bounded-wait budgets (DecoderConfig::peerWaitNs/localWaitNs).
  std::string setWaitBudgets(std::uint64_t peerNs, std::uint64_t localNs);

  // ---- execution (CompiledDecoderLLM API) ----
  // Prefill `count` tokens of one sequence in chunks of maxRows rows.
  // logits (optional): [count, localVocab]; nextToken: greedy token after the last.
  std::string prefill(int slot, const std::int32_t *tokens, int count, float *logits,
                      std::int32_t *nextToken, StepTiming *timing = nullptr);
  // One token for each of `rows` sequences (distinct slots).
  std::string decode(const std::int32_t *slots, const std::int32_t *tokens, int rows, float *logits,
                     std::int32_t *nextTokens, StepTiming *timing = nullptr);
  // Greedy loop on the device: `steps` graph replays, each feeding its argmax
  // back as the next input. tokensOut: [steps, rows].
  std::string generate(const std::int32_t *slots, const std::int32_t *tokens, int rows, int steps,
                       std::int32_t *tokensOut, StepTiming *timing = nullptr);

  // Time one kernel kind in isolation: a CUDA graph of `rounds` passes over
  // every layer's launch of that kernel (its real weights and parameters),
  // replayed on the executor stream between CUDA events. Reports the mean
  // duration of one launch and the algorithmic HBM bytes one launch moves.
  // Uses the step inputs of the last decode/generate call; the QKV kind
  // rewrites the KV entries at those positions with the same values.
  std::string profileKernel(int kind, int rows, int rounds, double *avgUs, double *bytesPerLaunch,
                            int *launchesPerStep);

  // ---- tracing ----
  // capacity > 0: every kernel of later steps appends per-CTA timeline records
  // (tmc::TraceRecord; tag = ((layer << 8) | kind) << 32 | CTA); 0 turns it off.
  // Step graphs are recaptured either way.
  std::string setTrace(std::size_t capacity);
  // Copy out and clear the records collected so far.
  std::string readTrace(std::vector<tmc::TraceRecord> *out);

  // ---- KV state ----
  std::size_t currentLength(int slot) const;
  std::string stageLength(int slot, std::size_t length);
  std::string commitLength(int slot, std::size_t length);
  std::string rollbackLength(int slot, std::size_t length);
  std::string releaseSlot(int slot);
  std::vector<std::int32_t> blockTable(int slot) const;
  // [localKVHeads, length, headDim] logical values (reference readKeyPrefix).
  std::string readKV(int layer, int slot, std::vector<float> *key, std::vector<float> *value) const;
  // Write a [localKVHeads, length, headDim] prefix into a freshly staged slot
  // (reference restoreKVCache, DecoderLLMExecutor.cpp:1138-1162).
  std::string restoreKV(int slot, std::size_t length, const std::vector<std::vector<float>> &keys,
                        const std::vector<std::vector<float>> &values);
  KVPagePool &pagePool() { return *pool_; }
  // Spill / restore of a whole sequence as raw fp16 page images (every layer,
  // K and V): one gather kernel and one device-to-host copy out, one copy and
  // one scatter kernel back into freshly staged pages -- the preemption path
  // of the serving scheduler (reference preempt / resume, ServingRuntime.cpp:
  // 469-490, which rewrites per-head rows instead).
  using Timing = StepTiming;  // the per-step timing the prefill / decode calls report
  struct KVPageSnapshot {
    std::size_t length = 0;
    std::vector<std::uint16_t> pages;  // [layers][K, V][pages][page elements]
  };
  std::string snapshotPages(int slot, KVPageSnapshot *out);
  std::string restorePages(int slot, const KVPageSnapshot &snap);

 private:
  std::string ensureSpill(std::size_t bytes, int npages);

 public:

  // ---- accounting (DecoderLLMExecutor.cpp:205-229) ----
  std::size_t modelStorageBytes() const { return modelBytes_; }
  std::size_t kvStorageBytes() const { return kvBytes_; }
  std::size_t activationStorageBytes() const { return activationBytes_; }
  // Kernel launches in one R-row step graph.
  int kernelsPerStep(int rows) const;
  // Bytes of weights + KV a single R-row step must read (roofline numerator).
  double stepAlgorithmicBytes(int rows, const std::vector<int> &contextLengths) const;

  cudaStream_t stream() const { return rt_.stream(); }
  cuda::CudaRuntime &runtime() { return rt_; }

 private:
  DecoderExecutor(cuda::CudaRuntime &runtime, const DecoderConfig &config);
  std::string allocate();
  // `distinct`: every row belongs to a different sequence (decode); prefill
  // chunks put several rows of one sequence in a step.
  // head: the LM head runs (a prefill chunk whose logits and token nobody
  // reads skips it).
  std::string enqueueStep(int rows, bool feed, bool distinct, bool head = true);
  std::string enqueueKernel(int kind, int layer, int rows, bool feed, bool distinct);
  // The GEMV / GEMM parameters of one projection (kinds QKV, O, gate/up,
  // down, LM head) of layer `layer` for `rows` rows.
  tmc::GemvParams projection(int kind, int layer, int rows, bool feed) const;
  std::string launchStep(int rows, bool feed, bool distinct, bool head = true);
  // Step graphs differ by rows, feed-back, distinct rows and the attention
  // split cap the step's contexts need.
  int graphKey(int rows, bool feed, bool distinct, bool head = true) const {
    return attnSplitCap_ * 8192 + rows * 8 + (head ? 4 : 0) + (feed ? 2 : 0) + (distinct ? 1 : 0);
  }
  // Uploads a step's tokens, positions and table rows and sets the attention
  // split cap for contexts up to max(position) + steps.
  std::string uploadStepInputs(int rows, const std::int32_t *tokens, const std::int32_t *positions,
                               const std::int32_t *tableRows, int steps = 1, std::int32_t *stage = nullptr);
  std::string writeBlockRow(int slot, const std::vector<std::int32_t> &row);
  void computeRope();

  struct Layer {
    cuda::BufferHandle inputNorm, qkv, o, postNorm, gateUp, down;
    cuda::BufferHandle kPool, vPool;
  };

  cuda::CudaRuntime &rt_;
  DecoderConfig cfg_;
  int hqL_ = 0, hkvL_ = 0, iL_ = 0, vL_ = 0;
  int qkvRows_ = 0;
  int maxPagesPerSeq_ = 0;
  int poolPages_ = 0;
  int pageSize_ = 0;
  int attnMaxSplits_ = 1;
  int attnMinChunk_ = 64;
  int numSms_ = 148;

  cuda::BufferHandle embedding_, finalNorm_, lmHead_, ropeCos_, ropeSin_;
  std::vector<Layer> layers_;
  // activations / step state
  cuda::BufferHandle h_, hB_, q_, ctx_, act_, logits_, partialF32_;
  cuda::BufferHandle stepIO_;       // int32 [3, maxRows]: tokens, positions, table rows
  cuda::BufferHandle blockTable_;   // int32 [maxSlots, maxPagesPerSeq]
  cuda::BufferHandle nextTokens_, argmaxKeys_, argmaxCounter_, history_, historyCounter_;
  cuda::BufferHandle attnWorkspace_, attnCounters_;
  cuda::BufferHandle workCounters_;  // per launch site: tmc::kGemvCounterWords uints
  unsigned int *workCounter(int layer, int kind) const;
  // Host staging: [3 * maxRows] step inputs, [maxRows] next tokens, then one
  // [3 * maxRows] block per prefill chunk (a whole prompt's chunks are queued
  // without waiting, so each keeps its own staging until its copy runs).
  std::int32_t *pinnedIO_ = nullptr;
  std::int32_t *prefillStage_ = nullptr;
  std::size_t prefillChunks_ = 0;
  // Page spill / restore: device array of the 2 * layers pool pointers, page-id
  // list, packed device staging and pinned host staging (grown on demand).
  cuda::BufferHandle poolPtrs_, spillPages_;
  void *spillDevice_ = nullptr, *spillHost_ = nullptr;
  std::size_t spillBytes_ = 0;
  int historyCapacity_ = 0;
  std::vector<int> lastPositions_;  // positions of the last staged step (profiling)
  cuda::BufferHandle traceRecords_, traceCount_;
  // Peer exchange (TP): this rank's window, per-phase CTA-done counters, the
  // step epoch; every rank's window as mapped here.
  cuda::BufferHandle xchgWindow_, xchgDone_, xchgEpoch_;
  char *peerWindows_[8] = {};
  std::vector<void *> peerMappings_;
  bool peersAttached_ = false;
  bool profiling_ = false;  // isolated kernel timing: consumers do not wait for peers
  void dropGraphs();
  tmc::PeerExchange exchange(int phase) const;
  // Batched (> 8 rows) projections on the tensor cores.
  static constexpr int kGemvMaxRows = 8;
  cuda::BufferHandle xn_, gemmWs_, gemmTickets_;
  std::map<std::tuple<const void *, int, int, int>, CUtensorMap> tensorMaps_;
  const CUtensorMap *tensorMap(const void *base, int rows, int cols, int boxRows, std::string *err);
  std::string launchProjection(const tmc::GemvParams &p, const char *what);
  std::size_t traceCapacity_ = 0;
  tmc::TraceSink traceSink(int layer, int kind) const;
  bool ropeSet_ = false;

  std::shared_ptr<KVPagePool> pool_;
  std::vector<std::unique_ptr<KVCacheState>> slots_;
  std::shared_ptr<Collective> collective_;

  struct Graph {
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
  };
  std::map<int, Graph> graphs_;
  // Attention split slots of the next step's launch: the splits its longest
  // context can use under this decoder's chunk policy, in whole 16-CTA
  // clusters (idle clusters would still be launched and scheduled).
  int attnSplitCap_ = 64;

  std::size_t modelBytes_ = 0, kvBytes_ = 0, activationBytes_ = 0;
};

}  // namespace tensor::runtime
