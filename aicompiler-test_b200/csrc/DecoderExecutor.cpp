// DecoderExecutor implementation (see DecoderExecutor.hpp).
#include "DecoderExecutor.hpp"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <sstream>
#include <stdexcept>

#include "attention.cuh"
#include "gemm.cuh"
#include "gemv.cuh"
#include "half_convert.hpp"
#include "misc.cuh"

namespace tensor::runtime {

using cuda::BufferHandle;
using cuda::ElementType;

namespace {

// Weight bytes one GEMV launch may pull into L2 while its predecessor drains.
// Measured over a whole bs1 step: 16 MB 3.61 ms, 32 MB 3.67, 64 MB 3.65,
// none 3.70 -- larger budgets evict more of the next kernels' lines.
constexpr long long kL2PrefetchBytes = 16ll << 20;

std::string cudaText(const char *what, cudaError_t e) {
  std::ostringstream s;
  s << what << ": " << cudaGetErrorName(e) << " (" << cudaGetErrorString(e) << ")";
  return s.str();
}

#define TMC_TRY(expr)                               \
  do {                                              \
    cudaError_t tmc_e_ = (expr);                    \
    if (tmc_e_ != cudaSuccess) {                    \
      cudaGetLastError();                           \
      return cudaText(#expr, tmc_e_);               \
    }                                               \
  } while (0)

__half *hp(const BufferHandle &b) { return b ? static_cast<__half *>(b->data()) : nullptr; }
float *fp(const BufferHandle &b) { return b ? static_cast<float *>(b->data()) : nullptr; }

std::uint64_t mix64(std::uint64_t x) {
  x += 0x9e3779b97f4a7c15ull;
  x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ull;
  x = (x ^ (x >> 27)) * 0x94d049bb133111ebull;
  return x ^ (x >> 31);
}

// Parse "layer{i}.{kind}.weight".
bool parseLayerName(const std::string &name, int *layer, std::string *kind) {
  if (name.rfind("layer", 0) != 0) return false;
  const auto dot = name.find('.');
  if (dot == std::string::npos) return false;
  try {
    *layer = std::stoi(name.substr(5, dot - 5));
  } catch (...) {
    return false;
  }
  const auto rest = name.substr(dot + 1);
  const std::string suffix = ".weight";
  if (rest.size() <= suffix.size() || rest.compare(rest.size() - suffix.size(), suffix.size(), suffix) != 0)
    return false;
  *kind = rest.substr(0, rest.size() - suffix.size());
  return true;
}

}  // namespace

DecoderExecutor::DecoderExecutor(cuda::CudaRuntime &runtime, const DecoderConfig &config)
    : rt_(runtime), cfg_(config) {}

DecoderExecutor::~DecoderExecutor() {
  for (auto &kv : graphs_) {
    if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
    if (kv.second.graph) cudaGraphDestroy(kv.second.graph);
  }
  slots_.clear();
  if (pinnedIO_) cudaFreeHost(pinnedIO_);
  if (spillHost_) cudaFreeHost(spillHost_);
  if (spillDevice_) cudaFree(spillDevice_);
  if (!peerMappings_.empty()) {
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(rt_.device());
    cudaStreamSynchronize(rt_.stream());
    for (void *ptr : peerMappings_) cudaIpcCloseMemHandle(ptr);
    cudaSetDevice(prev);
  }
}

void DecoderExecutor::dropGraphs() {
  for (auto &kv : graphs_) {
    if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
    if (kv.second.graph) cudaGraphDestroy(kv.second.graph);
  }
  graphs_.clear();
}

std::unique_ptr<DecoderExecutor> DecoderExecutor::create(cuda::CudaRuntime &runtime,
                                                         const DecoderConfig &config,
                                                         std::string *error) {
  const auto &c = config;
  std::string why;
  if (!runtime.isAvailable()) why = runtime.initializationError();
  else if (c.hidden <= 0 || c.heads <= 0 || c.kvHeads <= 0 || c.headDim <= 0 || c.intermediate <= 0 ||
           c.vocab <= 0 || c.layers <= 0 || c.capacity <= 0)
    why = "Decoder dimensions must be positive.";
  else if (c.heads % c.kvHeads != 0) why = "heads must be a multiple of kvHeads.";
  else if (c.headDim % 2 != 0) why = "The RoPE head dimension must be even.";
  else if (c.hidden % 8 != 0 || c.intermediate % 8 != 0 || (c.heads * c.headDim) % 8 != 0)
    why = "hidden, intermediate and heads*headDim must be multiples of 8 (16-byte rows).";
  else if (c.tpSize < 1 || c.tpRank < 0 || c.tpRank >= c.tpSize) why = "Invalid tensor-parallel rank.";
  else if (c.heads % c.tpSize || c.kvHeads % c.tpSize || c.intermediate % c.tpSize || c.vocab % c.tpSize)
    why = "heads, kvHeads, intermediate and vocab must divide by the tensor-parallel size.";
  else if ((c.intermediate / c.tpSize) % 8 != 0 || ((c.heads / c.tpSize) * c.headDim) % 8 != 0)
    why = "Per-rank intermediate and head widths must be multiples of 8.";
  else if (c.maxRows < 1 || c.maxRows > 256)
    why = "maxRows must be in [1, 256] (up to 8: GEMV; more: tensor-core projections).";
  else if (c.maxSlots < 1) why = "maxSlots must be positive.";
  else if (c.pageSize < 0 || c.pageSize > c.capacity) why = "pageSize must be in [0, capacity].";
  else if (!(c.epsilon > 0.0f) || !std::isfinite(c.epsilon)) why = "epsilon must be finite and positive.";
  else if (!(c.ropeTheta > 0.0)) why = "rope theta must be positive.";
  if (!why.empty()) {
    if (error) *error = why;
    return nullptr;
  }
  std::unique_ptr<DecoderExecutor> ex(new DecoderExecutor(runtime, config));
  why = ex->allocate();
  if (!why.empty()) {
    if (error) *error = why;
    return nullptr;
  }
  return ex;
}

std::string DecoderExecutor::allocate() {
  const int tp = cfg_.tpSize;
  hqL_ = cfg_.heads / tp;
  hkvL_ = cfg_.kvHeads / tp;
  iL_ = cfg_.intermediate / tp;
  vL_ = cfg_.vocab / tp;
  const int H = cfg_.hidden, D = cfg_.headDim;
  qkvRows_ = (hqL_ + 2 * hkvL_) * D;
  pageSize_ = cfg_.pageSize == 0 ? cfg_.capacity : cfg_.pageSize;
  maxPagesPerSeq_ = (cfg_.capacity + pageSize_ - 1) / pageSize_;
  poolPages_ = cfg_.poolPages > 0 ? cfg_.poolPages : cfg_.maxSlots * maxPagesPerSeq_;
  numSms_ = rt_.hardwareInfo().multiprocessorCount > 0 ? rt_.hardwareInfo().multiprocessorCount : 148;

  auto make = [&](std::size_t count, ElementType t, BufferHandle *out, std::size_t *bytes) -> std::string {
    auto r = rt_.createBuffer(count, nullptr, t);
    if (!r.buffer) return r.errorMessage;
    *out = r.buffer;
    if (bytes) *bytes += r.buffer->byteCount();
    return {};
  };
  std::string e;
  auto F16 = ElementType::Float16, F32 = ElementType::Float32, I32 = ElementType::Int32;
  if (!(e = make((size_t)cfg_.vocab * H, F16, &embedding_, &modelBytes_)).empty()) return e;
  if (!(e = make(H, F16, &finalNorm_, &modelBytes_)).empty()) return e;
  if (!(e = make((size_t)vL_ * H, F16, &lmHead_, &modelBytes_)).empty()) return e;
  if (!(e = make((size_t)cfg_.capacity * (D / 2), F32, &ropeCos_, &modelBytes_)).empty()) return e;
  if (!(e = make((size_t)cfg_.capacity * (D / 2), F32, &ropeSin_, &modelBytes_)).empty()) return e;
  layers_.resize(cfg_.layers);
  const size_t poolElems = (size_t)poolPages_ * hkvL_ * pageSize_ * D;
  for (auto &L : layers_) {
    if (!(e = make(H, F16, &L.inputNorm, &modelBytes_)).empty()) return e;
    if (!(e = make((size_t)qkvRows_ * H, F16, &L.qkv, &modelBytes_)).empty()) return e;
    if (!(e = make((size_t)H * hqL_ * D, F16, &L.o, &modelBytes_)).empty()) return e;
    if (!(e = make(H, F16, &L.postNorm, &modelBytes_)).empty()) return e;
    if (!(e = make((size_t)2 * iL_ * H, F16, &L.gateUp, &modelBytes_)).empty()) return e;
    if (!(e = make((size_t)H * iL_, F16, &L.down, &modelBytes_)).empty()) return e;
    if (!(e = make(poolElems, F16, &L.kPool, &kvBytes_)).empty()) return e;
    if (!(e = make(poolElems, F16, &L.vPool, &kvBytes_)).empty()) return e;
  }
  const int R = cfg_.maxRows;
  if (!(e = make((size_t)R * H, F16, &h_, &activationBytes_)).empty()) return e;
  if (!(e = make((size_t)R * H, F16, &hB_, &activationBytes_)).empty()) return e;  // second residual buffer (TP)
  if (cfg_.tpSize > 1 && !(e = make((size_t)R * H, F32, &partialF32_, &activationBytes_)).empty()) return e;
  if (R > kGemvMaxRows) {
    // Batched steps: prologue rows for the tensor-core projections, the
    // partial-tile workspace (the largest any projection's plan needs) and
    // tile tickets.
    if (!(e = make((size_t)R * H, F16, &xn_, &activationBytes_)).empty()) return e;
    const int dims[5][2] = {{qkvRows_, H}, {H, hqL_ * D}, {2 * iL_, H}, {H, iL_}, {vL_, H}};
    size_t wsFloats = 1, tiles = 1;
    for (const auto &d : dims) {
      const tmc::GemmPlan plan = tmc::plan_gemm(d[0], d[1], R, numSms_);
      wsFloats = std::max(wsFloats, tmc::gemm_workspace_floats(plan));
      tiles = std::max(tiles, (size_t)plan.tiles);
    }
    if (!(e = make(wsFloats, F32, &gemmWs_, &activationBytes_)).empty()) return e;
    if (!(e = make(2 * tiles, I32, &gemmTickets_, &activationBytes_)).empty()) return e;
  }
  if (cfg_.tpSize > 1) {
    // Exchange window (zeroed int32 words), CTA-done counters per partial-sum
    // phase (one 128-byte line each) and the step epoch.
    const size_t words = (tmc::peer_window_bytes(R, H) + 3) / 4;
    if (!(e = make(words, I32, &xchgWindow_, &activationBytes_)).empty()) return e;
    if (!(e = make((size_t)cfg_.layers * 2 * 32, I32, &xchgDone_, &activationBytes_)).empty()) return e;
    if (!(e = make(32, I32, &xchgEpoch_, &activationBytes_)).empty()) return e;
  }
  if (!(e = make((size_t)R * hqL_ * D, F16, &q_, &activationBytes_)).empty()) return e;
  if (!(e = make((size_t)R * hqL_ * D, F16, &ctx_, &activationBytes_)).empty()) return e;
  if (!(e = make((size_t)R * iL_, F16, &act_, &activationBytes_)).empty()) return e;
  if (!(e = make((size_t)R * vL_, F32, &logits_, &activationBytes_)).empty()) return e;
  if (!(e = make((size_t)3 * R, I32, &stepIO_, &activationBytes_)).empty()) return e;
  if (!(e = make((size_t)cfg_.maxSlots * maxPagesPerSeq_, I32, &blockTable_, &activationBytes_)).empty()) return e;
  if (!(e = make(R, I32, &nextTokens_, &activationBytes_)).empty()) return e;
  if (!(e = make((size_t)2 * R, I32, &argmaxKeys_, &activationBytes_)).empty()) return e;  // u64 [R]
  if (!(e = make(4, I32, &argmaxCounter_, &activationBytes_)).empty()) return e;
  historyCapacity_ = cfg_.capacity * R;
  lastPositions_.assign(R, 0);
  if (!(e = make((size_t)historyCapacity_, I32, &history_, &activationBytes_)).empty()) return e;
  if (!(e = make(4, I32, &historyCounter_, &activationBytes_)).empty()) return e;
  const int maxSplits = 64;
  const size_t wsBytes = std::max(tmc::attention_workspace_bytes(R, hqL_, hkvL_, D, maxSplits),
                                  tmc::attention_group_workspace_bytes(D));
  if (!(e = make(wsBytes / 4 + 1, F32, &attnWorkspace_, &activationBytes_)).empty()) return e;
  if (!(e = make((size_t)R * hkvL_, I32, &attnCounters_, &activationBytes_)).empty()) return e;
  if (!(e = make((size_t)cfg_.layers * 6 * tmc::kGemvCounterWords, I32, &workCounters_, &activationBytes_)).empty())
    return e;
  // Zero the state the kernels expect zero (int32 buffers were zero-filled by
  // createBuffer); residual-stream buffers start at zero too.
  cudaStream_t s0 = rt_.stream();
  TMC_TRY(cudaMemsetAsync(argmaxKeys_->data(), 0, argmaxKeys_->byteCount(), s0));
  TMC_TRY(cudaMemsetAsync(h_->data(), 0, h_->byteCount(), s0));
  TMC_TRY(cudaMemsetAsync(hB_->data(), 0, hB_->byteCount(), s0));
  // Block table: -1 = unmapped.
  TMC_TRY(cudaMemsetAsync(blockTable_->data(), 0xff, blockTable_->byteCount(), s0));
  prefillChunks_ = (std::size_t)(cfg_.capacity + R - 1) / R;
  TMC_TRY(cudaMallocHost(&pinnedIO_, sizeof(std::int32_t) * (4 * R + 3 * R * prefillChunks_)));
  prefillStage_ = pinnedIO_ + 4 * R;
  // Norm weights default to 1 (nn.Parameter(torch.ones), decoder_llm.py:11).
  for (auto &L : layers_) {
    TMC_TRY(tmc::launch_fill_value_f16(hp(L.inputNorm), H, 1.0f, rt_.stream()));
    TMC_TRY(tmc::launch_fill_value_f16(hp(L.postNorm), H, 1.0f, rt_.stream()));
  }
  TMC_TRY(tmc::launch_fill_value_f16(hp(finalNorm_), H, 1.0f, rt_.stream()));
  computeRope();

  pool_ = std::make_shared<KVPagePool>(pageSize_, poolPages_);
  slots_.resize(cfg_.maxSlots);
  for (int s = 0; s < cfg_.maxSlots; ++s) {
    slots_[s] = std::make_unique<KVCacheState>(
        pool_, cfg_.capacity, s,
        [this](int slot, const std::vector<std::int32_t> &row) { return writeBlockRow(slot, row); });
  }
  return rt_.synchronize();
}

void DecoderExecutor::computeRope() {
  // The reference's tables (decoder_llm.py:48-55, export_decoder_llm.py:420-431):
  // freq_i = exp(2i * (-ln(theta) / D)), angle = position * freq, fp32.
  const int D = cfg_.headDim, half = D / 2;
  std::vector<float> c((size_t)cfg_.capacity * half), s((size_t)cfg_.capacity * half);
  const float scale = static_cast<float>(-std::log(cfg_.ropeTheta) / D);
  for (int i = 0; i < half; ++i) {
    const float f = static_cast<float>(std::exp(static_cast<double>(static_cast<float>(2 * i) * scale)));
    for (int p = 0; p < cfg_.capacity; ++p) {
      const float angle = static_cast<float>(p) * f;
      c[(size_t)p * half + i] = static_cast<float>(std::cos(static_cast<double>(angle)));
      s[(size_t)p * half + i] = static_cast<float>(std::sin(static_cast<double>(angle)));
    }
  }
  (void)rt_.writeBuffer(ropeCos_, c.data(), c.size());
  (void)rt_.writeBuffer(ropeSin_, s.data(), s.size());
}

std::string DecoderExecutor::setRope(const float *cosine, const float *sine, std::size_t rows) {
  const size_t half = cfg_.headDim / 2;
  if (rows < static_cast<size_t>(cfg_.capacity)) return "RoPE tables must cover the cache capacity.";
  auto e = rt_.writeBuffer(ropeCos_, cosine, (size_t)cfg_.capacity * half);
  if (e.empty()) e = rt_.writeBuffer(ropeSin_, sine, (size_t)cfg_.capacity * half);
  if (e.empty()) ropeSet_ = true;
  return e;
}

std::string DecoderExecutor::setCollective(std::shared_ptr<Collective> collective) {
  if (cfg_.tpSize > 1 && !collective) return "tensor parallelism needs a collective.";
  collective_ = std::move(collective);
  dropGraphs();
  return {};
}

std::string DecoderExecutor::exchangeHandle(void *out, std::size_t size) {
  if (cfg_.tpSize <= 1 || !xchgWindow_) return "peer exchange needs tensor parallelism (tp_size > 1).";
  if (out == nullptr || size != sizeof(cudaIpcMemHandle_t))
    return "exchange handle: buffer must hold " + std::to_string(sizeof(cudaIpcMemHandle_t)) + " bytes.";
  auto e = rt_.synchronize();  // the window's zero fill has landed before any peer can write
  if (!e.empty()) return e;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(rt_.device());
  cudaIpcMemHandle_t h;
  const cudaError_t ce = cudaIpcGetMemHandle(&h, xchgWindow_->data());
  cudaSetDevice(prev);
  if (ce != cudaSuccess) return cudaText("cudaIpcGetMemHandle", ce);
  std::memcpy(out, &h, sizeof(h));
  return {};
}

std::string DecoderExecutor::attachPeers(const void *handles, std::size_t size, int world, int rank) {
  if (cfg_.tpSize <= 1 || !xchgWindow_) return "peer exchange needs tensor parallelism (tp_size > 1).";
  if (world != cfg_.tpSize || rank != cfg_.tpRank)
    return "peer exchange: world size and rank must equal the decoder's tp_size and tp_rank.";
  if (world > tmc::kMaxPeers) return "peer exchange: at most 8 ranks.";
  if (handles == nullptr || size != sizeof(cudaIpcMemHandle_t))
    return "peer exchange: handles must be " + std::to_string(sizeof(cudaIpcMemHandle_t)) + " bytes each.";
  if (peersAttached_) return "peer exchange already attached.";
  auto e = rt_.synchronize();
  if (!e.empty()) return e;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(rt_.device());
  const auto *bytes = static_cast<const unsigned char *>(handles);
  std::string err;
  for (int r = 0; r < world && err.empty(); ++r) {
    if (r == rank) {
      peerWindows_[r] = static_cast<char *>(xchgWindow_->data());
      continue;
    }
    cudaIpcMemHandle_t h;
    std::memcpy(&h, bytes + (size_t)r * size, sizeof(h));
    void *ptr = nullptr;
    const cudaError_t ce = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (ce != cudaSuccess) {
      cudaGetLastError();
      err = "cudaIpcOpenMemHandle (rank " + std::to_string(r) + "): " + cudaGetErrorString(ce);
      break;
    }
    peerMappings_.push_back(ptr);
    peerWindows_[r] = static_cast<char *>(ptr);
  }
  if (!err.empty()) {
    for (void *ptr : peerMappings_) cudaIpcCloseMemHandle(ptr);
    peerMappings_.clear();
    for (auto &w : peerWindows_) w = nullptr;
  }
  cudaSetDevice(prev);
  if (!err.empty()) return err;
  peersAttached_ = true;
  dropGraphs();
  return {};
}

std::string DecoderExecutor::attachLocalPeers(const std::vector<DecoderExecutor *> &ranks, int rank) {
  if (cfg_.tpSize <= 1 || !xchgWindow_) return "peer exchange needs tensor parallelism (tp_size > 1).";
  const int world = static_cast<int>(ranks.size());
  if (world != cfg_.tpSize || rank != cfg_.tpRank)
    return "peer exchange: world size and rank must equal the decoder's tp_size and tp_rank.";
  if (world > tmc::kMaxPeers) return "peer exchange: at most 8 ranks.";
  if (ranks[rank] != this) return "peer exchange: ranks[rank] must be this decoder.";
  if (peersAttached_) return "peer exchange already attached.";
  for (int r = 0; r < world; ++r) {
    const DecoderExecutor *o = ranks[r];
    if (o == nullptr || !o->xchgWindow_) return "peer exchange: rank " + std::to_string(r) + " has no window.";
    if (o->cfg_.tpSize != world || o->cfg_.tpRank != r || o->cfg_.hidden != cfg_.hidden ||
        o->cfg_.maxRows != cfg_.maxRows || o->cfg_.layers != cfg_.layers)
      return "peer exchange: rank " + std::to_string(r) + " is not a shard of the same model.";
    auto e = o->rt_.synchronize();  // its window's zero fill has landed
    if (!e.empty()) return e;
  }
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(rt_.device());
  std::string err;
  for (int r = 0; r < world && err.empty(); ++r) {
    const int dev = ranks[r]->rt_.device();
    if (dev != rt_.device()) {
      const cudaError_t ce = cudaDeviceEnablePeerAccess(dev, 0);
      if (ce != cudaSuccess && ce != cudaErrorPeerAccessAlreadyEnabled)
        err = "cudaDeviceEnablePeerAccess (rank " + std::to_string(r) + "): " + cudaGetErrorString(ce);
      cudaGetLastError();
    }
    peerWindows_[r] = static_cast<char *>(ranks[r]->xchgWindow_->data());
  }
  cudaSetDevice(prev);
  if (!err.empty()) {
    for (auto &w : peerWindows_) w = nullptr;
    return err;
  }
  peersAttached_ = true;
  dropGraphs();
  return {};
}

std::string DecoderExecutor::setWaitBudgets(std::uint64_t peerNs, std::uint64_t localNs) {
  cfg_.peerWaitNs = peerNs;
  cfg_.localWaitNs = localNs;
  dropGraphs();  // the budgets are baked into the captured launches
  return {};
}

tmc::PeerExchange DecoderExecutor::exchange(int phase) const {
  tmc::PeerExchange x{};
  if (!peersAttached_) return x;
  x.world = cfg_.tpSize;
  x.rank = cfg_.tpRank;
  x.wait = profiling_ ? 0 : 1;
  x.signal = 1;
  x.slot_rows = cfg_.maxRows;
  x.width = cfg_.hidden;
  x.row0 = 0;
  x.phase = static_cast<unsigned int>(phase);
  x.phases = static_cast<unsigned int>(2 * cfg_.layers);
  for (int r = 0; r < cfg_.tpSize; ++r) x.window[r] = peerWindows_[r];
  x.epoch = static_cast<unsigned int *>(xchgEpoch_->data());
  x.done = static_cast<unsigned int *>(xchgDone_->data()) + (size_t)phase * 32;
  return x;
}

// ---- weights ----------------------------------------------------------------

namespace {
struct Window {
  BufferHandle buffer;
  size_t dstOffset = 0;     // elements
  size_t dstPitch = 0;      // elements between destination rows
  size_t rows = 0, cols = 0;
  size_t srcRow0 = 0, srcCol0 = 0, srcCols = 0;  // logical source layout
  size_t logicalCount = 0;
};
}  // namespace

// Locate the rank-local window of a logical tensor.
static std::string locate(const DecoderExecutor &ex, const std::string &name,
                          const std::function<BufferHandle(int, const std::string &)> &layerBuf,
                          const BufferHandle &emb, const BufferHandle &finalNorm, const BufferHandle &lm,
                          Window *w) {
  const auto &c = ex.config();
  const size_t H = c.hidden, D = c.headDim, rank = c.tpRank;
  const size_t hq = ex.localHeads(), hkv = ex.localKVHeads(), il = ex.localIntermediate(), vl = ex.localVocab();
  if (name == "embedding.weight") {
    *w = {emb, 0, H, (size_t)c.vocab, H, 0, 0, H, (size_t)c.vocab * H};
    return {};
  }
  if (name == "final_norm.weight") {
    *w = {finalNorm, 0, H, 1, H, 0, 0, H, H};
    return {};
  }
  if (name == "lm_head.weight") {
    *w = {lm, 0, H, vl, H, rank * vl, 0, H, (size_t)c.vocab * H};
    return {};
  }
  int layer = -1;
  std::string kind;
  if (!parseLayerName(name, &layer, &kind) || layer < 0 || layer >= c.layers)
    return "Unknown decoder weight: " + name;
  const auto buf = layerBuf(layer, kind);
  if (kind == "input_norm" || kind == "post_norm") {
    *w = {buf, 0, H, 1, H, 0, 0, H, H};
  } else if (kind == "q") {
    *w = {buf, 0, H, hq * D, H, rank * hq * D, 0, H, (size_t)c.heads * D * H};
  } else if (kind == "k") {
    *w = {buf, hq * D * H, H, hkv * D, H, rank * hkv * D, 0, H, (size_t)c.kvHeads * D * H};
  } else if (kind == "v") {
    *w = {buf, (hq + hkv) * D * H, H, hkv * D, H, rank * hkv * D, 0, H, (size_t)c.kvHeads * D * H};
  } else if (kind == "o") {
    *w = {buf, 0, hq * D, H, hq * D, 0, rank * hq * D, (size_t)c.heads * D, H * (size_t)c.heads * D};
  } else if (kind == "gate") {
    *w = {buf, 0, 2 * H, il, H, rank * il, 0, H, (size_t)c.intermediate * H};
  } else if (kind == "up") {
    *w = {buf, H, 2 * H, il, H, rank * il, 0, H, (size_t)c.intermediate * H};
  } else if (kind == "down") {
    *w = {buf, 0, il, H, il, 0, rank * il, (size_t)c.intermediate, H * (size_t)c.intermediate};
  } else {
    return "Unknown decoder weight: " + name;
  }
  return {};
}

std::string DecoderExecutor::loadWeightF16(const std::string &name, const std::uint16_t *bits,
                                           std::size_t count) {
  if (name == "rope.cosine" || name == "rope.sine") {
    std::vector<float> f(count);
    for (size_t i = 0; i < count; ++i) f[i] = cuda::halfBitsToFloat(bits[i]);
    return loadWeight(name, f.data(), count);
  }
  Window w;
  auto layerBuf = [this](int l, const std::string &k) -> BufferHandle {
    auto &L = layers_[l];
    if (k == "input_norm") return L.inputNorm;
    if (k == "post_norm") return L.postNorm;
    if (k == "q" || k == "k" || k == "v") return L.qkv;
    if (k == "o") return L.o;
    if (k == "gate" || k == "up") return L.gateUp;
    if (k == "down") return L.down;
    return {};
  };
  auto e = locate(*this, name, layerBuf, embedding_, finalNorm_, lmHead_, &w);
  if (!e.empty()) return e;
  if (count != w.logicalCount) {
    std::ostringstream s;
    s << "Weight " << name << " has " << count << " values; expected " << w.logicalCount << ".";
    return s.str();
  }
  const auto *src = bits + w.srcRow0 * w.srcCols + w.srcCol0;
  TMC_TRY(cudaMemcpy2DAsync(static_cast<std::uint16_t *>(w.buffer->data()) + w.dstOffset, w.dstPitch * 2, src,
                            w.srcCols * 2, w.cols * 2, w.rows, cudaMemcpyHostToDevice, rt_.stream()));
  TMC_TRY(cudaStreamSynchronize(rt_.stream()));
  return {};
}

std::string DecoderExecutor::loadWeight(const std::string &name, const float *values, std::size_t count) {
  if (name == "rope.cosine" || name == "rope.sine") {
    const size_t half = cfg_.headDim / 2;
    if (count % half != 0 || count / half < static_cast<size_t>(cfg_.capacity))
      return "RoPE tables must be [>= capacity, headDim/2].";
    return rt_.writeBuffer(name == "rope.cosine" ? ropeCos_ : ropeSin_, values, (size_t)cfg_.capacity * half);
  }
  std::vector<std::uint16_t> bits(count);
  for (size_t i = 0; i < count; ++i) bits[i] = cuda::floatToHalfBits(values[i]);
  return loadWeightF16(name, bits.data(), count);
}

std::string DecoderExecutor::readWeight(const std::string &name, std::vector<float> *out) const {
  if (name == "rope.cosine" || name == "rope.sine") {
    *out = (name == "rope.cosine" ? ropeCos_ : ropeSin_)->read();
    return {};
  }
  Window w;
  auto layerBuf = [this](int l, const std::string &k) -> BufferHandle {
    const auto &L = layers_[l];
    if (k == "input_norm") return L.inputNorm;
    if (k == "post_norm") return L.postNorm;
    if (k == "q" || k == "k" || k == "v") return L.qkv;
    if (k == "o") return L.o;
    if (k == "gate" || k == "up") return L.gateUp;
    if (k == "down") return L.down;
    return {};
  };
  auto e = locate(*this, name, layerBuf, embedding_, finalNorm_, lmHead_, &w);
  if (!e.empty()) return e;
  std::vector<std::uint16_t> bits(w.rows * w.cols);
  TMC_TRY(cudaStreamSynchronize(rt_.stream()));
  TMC_TRY(cudaMemcpy2D(bits.data(), w.cols * 2, static_cast<const std::uint16_t *>(w.buffer->data()) + w.dstOffset,
                       w.dstPitch * 2, w.cols * 2, w.rows, cudaMemcpyDeviceToHost));
  out->resize(bits.size());
  for (size_t i = 0; i < bits.size(); ++i) (*out)[i] = cuda::halfBitsToFloat(bits[i]);
  return {};
}

std::string DecoderExecutor::initRandom(std::uint64_t seed, float stddev) {
  const int H = cfg_.hidden, D = cfg_.headDim, rank = cfg_.tpRank;
  cudaStream_t s = rt_.stream();
  auto tseed = [&](std::uint64_t id) { return mix64(seed ^ mix64(id + 0x1234567ull)); };
  // embedding (id 1), lm_head (id 2), layer tensors (id 16 + layer*16 + kind)
  TMC_TRY(tmc::launch_fill_normal_2d(hp(embedding_), cfg_.vocab, H, H, tseed(1), 0, H, 0, 0.0f, stddev, s));
  TMC_TRY(tmc::launch_fill_normal_2d(hp(lmHead_), vL_, H, H, tseed(2), (long long)rank * vL_, H, 0, 0.0f, stddev, s));
  for (int l = 0; l < cfg_.layers; ++l) {
    auto &L = layers_[l];
    const std::uint64_t b = 16 + (std::uint64_t)l * 16;
    __half *qkv = hp(L.qkv);
    TMC_TRY(tmc::launch_fill_normal_2d(qkv, hqL_ * D, H, H, tseed(b + 0), (long long)rank * hqL_ * D, H, 0, 0.0f, stddev, s));
    TMC_TRY(tmc::launch_fill_normal_2d(qkv + (size_t)hqL_ * D * H, hkvL_ * D, H, H, tseed(b + 1),
                                       (long long)rank * hkvL_ * D, H, 0, 0.0f, stddev, s));
    TMC_TRY(tmc::launch_fill_normal_2d(qkv + (size_t)(hqL_ + hkvL_) * D * H, hkvL_ * D, H, H, tseed(b + 2),
                                       (long long)rank * hkvL_ * D, H, 0, 0.0f, stddev, s));
    TMC_TRY(tmc::launch_fill_normal_2d(hp(L.o), H, hqL_ * D, (long long)hqL_ * D, tseed(b + 3), 0,
                                       (long long)cfg_.heads * D, (long long)rank * hqL_ * D, 0.0f, stddev, s));
    TMC_TRY(tmc::launch_fill_normal_2d(hp(L.gateUp), iL_, H, 2LL * H, tseed(b + 4), (long long)rank * iL_, H, 0,
                                       0.0f, stddev, s));
    TMC_TRY(tmc::launch_fill_normal_2d(hp(L.gateUp) + H, iL_, H, 2LL * H, tseed(b + 5), (long long)rank * iL_, H, 0,
                                       0.0f, stddev, s));
    TMC_TRY(tmc::launch_fill_normal_2d(hp(L.down), H, iL_, iL_, tseed(b + 6), 0, cfg_.intermediate,
                                       (long long)rank * iL_, 0.0f, stddev, s));
  }
  return rt_.synchronize();
}

// ---- KV state ----------------------------------------------------------------

std::string DecoderExecutor::writeBlockRow(int slot, const std::vector<std::int32_t> &row) {
  if (row.size() != static_cast<size_t>(maxPagesPerSeq_)) return "block table row size mismatch";
  TMC_TRY(cudaMemcpyAsync(static_cast<std::int32_t *>(blockTable_->data()) + (size_t)slot * maxPagesPerSeq_,
                          row.data(), row.size() * 4, cudaMemcpyHostToDevice, rt_.stream()));
  // `row` is host memory owned by the caller; finish the copy before returning.
  TMC_TRY(cudaStreamSynchronize(rt_.stream()));
  return {};
}

std::size_t DecoderExecutor::currentLength(int slot) const {
  if (slot < 0 || slot >= cfg_.maxSlots) return 0;
  return slots_[slot]->currentLength();
}

std::string DecoderExecutor::stageLength(int slot, std::size_t length) {
  if (slot < 0 || slot >= cfg_.maxSlots) return "slot out of range";
  return slots_[slot]->stageLength(length);
}

std::string DecoderExecutor::commitLength(int slot, std::size_t length) {
  if (slot < 0 || slot >= cfg_.maxSlots) return "slot out of range";
  try {
    slots_[slot]->commitLength(length);
  } catch (const std::exception &e) {
    return e.what();
  }
  return {};
}

std::string DecoderExecutor::rollbackLength(int slot, std::size_t length) {
  if (slot < 0 || slot >= cfg_.maxSlots) return "slot out of range";
  return slots_[slot]->rollbackLength(length);
}

std::string DecoderExecutor::releaseSlot(int slot) {
  if (slot < 0 || slot >= cfg_.maxSlots) return "slot out of range";
  return slots_[slot]->reset();
}

std::vector<std::int32_t> DecoderExecutor::blockTable(int slot) const {
  if (slot < 0 || slot >= cfg_.maxSlots) return {};
  return slots_[slot]->pageTable();
}

std::string DecoderExecutor::readKV(int layer, int slot, std::vector<float> *key,
                                    std::vector<float> *value) const {
  if (layer < 0 || layer >= cfg_.layers || slot < 0 || slot >= cfg_.maxSlots) return "layer or slot out of range";
  const auto &st = *slots_[slot];
  const size_t len = st.currentLength(), D = cfg_.headDim, P = pageSize_;
  const auto &row = st.blockTableRow();
  key->assign((size_t)hkvL_ * len * D, 0.0f);
  value->assign((size_t)hkvL_ * len * D, 0.0f);
  TMC_TRY(cudaStreamSynchronize(rt_.stream()));
  const size_t pageElems = (size_t)hkvL_ * P * D;
  std::vector<std::uint16_t> kb(pageElems), vb(pageElems);
  for (size_t lp = 0; lp * P < len; ++lp) {
    const int page = row[lp];
    if (page < 0) return "KV page missing for a committed position";
    TMC_TRY(cudaMemcpy(kb.data(), static_cast<const std::uint16_t *>(layers_[layer].kPool->data()) + page * pageElems,
                       pageElems * 2, cudaMemcpyDeviceToHost));
    TMC_TRY(cudaMemcpy(vb.data(), static_cast<const std::uint16_t *>(layers_[layer].vPool->data()) + page * pageElems,
                       pageElems * 2, cudaMemcpyDeviceToHost));
    for (size_t h = 0; h < (size_t)hkvL_; ++h)
      for (size_t off = 0; off < P && lp * P + off < len; ++off)
        for (size_t d = 0; d < D; ++d) {
          const size_t src = (h * P + off) * D + d;
          const size_t dst = (h * len + lp * P + off) * D + d;
          (*key)[dst] = cuda::halfBitsToFloat(kb[src]);
          (*value)[dst] = cuda::halfBitsToFloat(vb[src]);
        }
  }
  return {};
}

std::string DecoderExecutor::snapshotPages(int slot, KVPageSnapshot *out) {
  if (slot < 0 || slot >= cfg_.maxSlots || out == nullptr) return "slot out of range";
  const auto &st = *slots_[slot];
  const size_t len = st.currentLength(), P = pageSize_;
  out->length = len;
  out->pages.clear();
  if (len == 0) return {};
  const int npages = (int)((len + P - 1) / P);
  const auto &row = st.blockTableRow();
  std::vector<std::int32_t> ids(row.begin(), row.begin() + npages);
  for (int id : ids)
    if (id < 0) return "KV page missing for a committed position";
  const size_t pageElems = (size_t)hkvL_ * P * cfg_.headDim;
  const size_t bytes = (size_t)cfg_.layers * 2 * npages * pageElems * 2;
  auto e = ensureSpill(bytes, npages);
  if (!e.empty()) return e;
  cudaStream_t s = rt_.stream();
  TMC_TRY(cudaMemcpyAsync(spillPages_->data(), ids.data(), ids.size() * 4, cudaMemcpyHostToDevice, s));
  TMC_TRY(tmc::launch_page_copy(static_cast<__half *const *>(poolPtrs_->data()),
                                static_cast<const int *>(spillPages_->data()), npages, cfg_.layers, pageElems,
                                static_cast<__half *>(spillDevice_), true, s));
  TMC_TRY(cudaMemcpyAsync(spillHost_, spillDevice_, bytes, cudaMemcpyDeviceToHost, s));
  TMC_TRY(cudaStreamSynchronize(s));
  out->pages.resize(bytes / 2);
  std::memcpy(out->pages.data(), spillHost_, bytes);
  return {};
}

std::string DecoderExecutor::restorePages(int slot, const KVPageSnapshot &snap) {
  if (slot < 0 || slot >= cfg_.maxSlots) return "slot out of range";
  auto &st = *slots_[slot];
  if (st.currentLength() != 0) return "KV cache restore requires an empty request state.";
  const size_t len = snap.length, P = pageSize_;
  if (len == 0 || len > (size_t)cfg_.capacity) return "KV cache restore snapshot shape is invalid.";
  const int npages = (int)((len + P - 1) / P);
  const size_t pageElems = (size_t)hkvL_ * P * cfg_.headDim;
  const size_t bytes = (size_t)cfg_.layers * 2 * npages * pageElems * 2;
  if (snap.pages.size() * 2 != bytes) return "KV cache restore snapshot shape is invalid.";
  auto e = ensureSpill(bytes, npages);
  if (!e.empty()) return e;
  e = st.stageLength(len);
  if (!e.empty()) return e;
  const auto &row = st.blockTableRow();
  std::vector<std::int32_t> ids(row.begin(), row.begin() + npages);
  cudaStream_t s = rt_.stream();
  std::memcpy(spillHost_, snap.pages.data(), bytes);
  cudaError_t ce = cudaMemcpyAsync(spillPages_->data(), ids.data(), ids.size() * 4, cudaMemcpyHostToDevice, s);
  if (ce == cudaSuccess) ce = cudaMemcpyAsync(spillDevice_, spillHost_, bytes, cudaMemcpyHostToDevice, s);
  if (ce == cudaSuccess)
    ce = tmc::launch_page_copy(static_cast<__half *const *>(poolPtrs_->data()),
                               static_cast<const int *>(spillPages_->data()), npages, cfg_.layers, pageElems,
                               static_cast<__half *>(spillDevice_), false, s);
  if (ce == cudaSuccess) ce = cudaStreamSynchronize(s);
  if (ce != cudaSuccess) {
    (void)st.rollbackLength(0);
    return cudaText("page restore", ce);
  }
  st.commitLength(len);
  return {};
}

std::string DecoderExecutor::ensureSpill(std::size_t bytes, int npages) {
  if (!poolPtrs_) {
    std::vector<void *> ptrs;
    for (const auto &L : layers_) {
      ptrs.push_back(L.kPool->data());
      ptrs.push_back(L.vPool->data());
    }
    auto r = rt_.createBuffer(ptrs.size() * 2, nullptr, ElementType::Int32);  // 8-byte pointers as int32 pairs
    if (!r.buffer) return r.errorMessage;
    poolPtrs_ = r.buffer;
    TMC_TRY(cudaMemcpy(poolPtrs_->data(), ptrs.data(), ptrs.size() * sizeof(void *), cudaMemcpyHostToDevice));
    auto q = rt_.createBuffer((size_t)maxPagesPerSeq_, nullptr, ElementType::Int32);
    if (!q.buffer) return q.errorMessage;
    spillPages_ = q.buffer;
  }
  if (npages > maxPagesPerSeq_) return "KV snapshot has more pages than a sequence can hold";
  if (bytes > spillBytes_) {
    if (spillDevice_) cudaFree(spillDevice_);
    if (spillHost_) cudaFreeHost(spillHost_);
    spillDevice_ = spillHost_ = nullptr;
    spillBytes_ = 0;
    TMC_TRY(cudaMalloc(&spillDevice_, bytes));
    TMC_TRY(cudaMallocHost(&spillHost_, bytes));
    spillBytes_ = bytes;
  }
  return {};
}

std::string DecoderExecutor::restoreKV(int slot, std::size_t length,
                                       const std::vector<std::vector<float>> &keys,
                                       const std::vector<std::vector<float>> &values) {
  if (slot < 0 || slot >= cfg_.maxSlots) return "slot out of range";
  auto &st = *slots_[slot];
  if (st.currentLength() != 0) return "KV cache restore requires an empty request state.";
  const size_t D = cfg_.headDim, P = pageSize_;
  if (length == 0 || length > (size_t)cfg_.capacity || keys.size() != (size_t)cfg_.layers ||
      values.size() != (size_t)cfg_.layers)
    return "KV cache restore snapshot shape is invalid.";
  for (int l = 0; l < cfg_.layers; ++l)
    if (keys[l].size() != (size_t)hkvL_ * length * D || values[l].size() != (size_t)hkvL_ * length * D)
      return "KV cache restore snapshot shape is invalid.";
  auto e = st.stageLength(length);
  if (!e.empty()) return e;
  const auto &row = st.blockTableRow();
  const size_t pageElems = (size_t)hkvL_ * P * D;
  std::vector<std::uint16_t> kb(pageElems), vb(pageElems);
  for (int l = 0; l < cfg_.layers; ++l) {
    for (size_t lp = 0; lp * P < length; ++lp) {
      const int page = row[lp];
      std::fill(kb.begin(), kb.end(), 0);
      std::fill(vb.begin(), vb.end(), 0);
      for (size_t h = 0; h < (size_t)hkvL_; ++h)
        for (size_t off = 0; off < P && lp * P + off < length; ++off)
          for (size_t d = 0; d < D; ++d) {
            const size_t dst = (h * P + off) * D + d;
            const size_t src = (h * length + lp * P + off) * D + d;
            kb[dst] = cuda::floatToHalfBits(keys[l][src]);
            vb[dst] = cuda::floatToHalfBits(values[l][src]);
          }
      cudaError_t ce = cudaMemcpyAsync(static_cast<std::uint16_t *>(layers_[l].kPool->data()) + page * pageElems,
                                       kb.data(), pageElems * 2, cudaMemcpyHostToDevice, rt_.stream());
      if (ce == cudaSuccess)
        ce = cudaMemcpyAsync(static_cast<std::uint16_t *>(layers_[l].vPool->data()) + page * pageElems, vb.data(),
                             pageElems * 2, cudaMemcpyHostToDevice, rt_.stream());
      if (ce == cudaSuccess) ce = cudaStreamSynchronize(rt_.stream());
      if (ce != cudaSuccess) {
        (void)st.rollbackLength(0);
        return cudaText("restore copy", ce);
      }
    }
  }
  st.commitLength(length);
  return {};
}

// ---- step --------------------------------------------------------------------

int DecoderExecutor::kernelsPerStep(int rows) const {
  const bool tp = cfg_.tpSize > 1;
  // Batched steps add a prologue kernel before the QKV, gate/up and LM-head projections.
  const int perLayer = rows > kGemvMaxRows ? 7 : 5;
  const int head = rows > kGemvMaxRows ? 2 : 1;
  return cfg_.layers * perLayer + head + (tp && !peersAttached_ ? 1 : 0);  // + argmax finalize after the collective
}

double DecoderExecutor::stepAlgorithmicBytes(int rows, const std::vector<int> &ctx) const {
  const double H = cfg_.hidden, D = cfg_.headDim;
  double w = 0.0;
  w += (double)qkvRows_ * H + H * hqL_ * D + 2.0 * iL_ * H + H * iL_ + 2.0 * H;  // per layer
  w *= cfg_.layers;
  w += (double)vL_ * H + H;  // LM head + final norm
  double bytes = 2.0 * w + 2.0 * rows * H;  // weights + embedding rows
  for (int c : ctx) bytes += 2.0 * 2.0 * hkvL_ * D * c * cfg_.layers;  // K and V reads
  bytes += 2.0 * 2.0 * hkvL_ * D * rows * cfg_.layers;                // K and V appends
  return bytes;
}

const CUtensorMap *DecoderExecutor::tensorMap(const void *base, int rows, int cols, int boxRows, std::string *err) {
  const auto key = std::make_tuple(base, rows, cols, boxRows);
  auto it = tensorMaps_.find(key);
  if (it != tensorMaps_.end()) return &it->second;
  CUtensorMap map;
  const cudaError_t e = tmc::make_tensor_map_f16(&map, base, rows, cols, boxRows);
  if (e != cudaSuccess) {
    *err = cudaText("tensor map", e);
    return nullptr;
  }
  return &tensorMaps_.emplace(key, map).first->second;
}

// One projection: the GEMV for up to 8 rows; for more, the prologue kernel
// (when there is one) and the tensor-core GEMM over the same parameters.
std::string DecoderExecutor::launchProjection(const tmc::GemvParams &p, const char *what) {
  cudaStream_t s = rt_.stream();
  const bool pdl = cfg_.usePDL;
  cudaError_t e;
  if (p.M <= kGemvMaxRows) {
    if ((e = tmc::launch_gemv(p, s, pdl, numSms_)) != cudaSuccess) return cudaText(what, e);
    return {};
  }
  const void *x = p.x;
  if (p.prologue != tmc::kProF16) {
    if ((e = tmc::launch_row_prologue(p, hp(xn_), s, pdl)) != cudaSuccess) return cudaText(what, e);
    x = xn_->data();
  } else if (p.x_stride != p.K) {
    return std::string(what) + ": batched projection needs contiguous activation rows.";
  }
  const tmc::GemmPlan plan = tmc::plan_gemm(p.N, p.K, p.M, numSms_);
  std::string err;
  const CUtensorMap *wm = tensorMap(p.W, p.N, p.K, tmc::kGemmTileRows, &err);
  const CUtensorMap *xm = wm ? tensorMap(x, cfg_.maxRows, p.K, plan.tn, &err) : nullptr;
  if (!xm) return std::string(what) + ": " + err;
  if ((e = tmc::launch_gemm(p, *wm, *xm, plan, fp(gemmWs_), static_cast<unsigned int *>(gemmTickets_->data()), s,
                            pdl)) != cudaSuccess)
    return cudaText(what, e);
  return {};
}

tmc::GemvParams DecoderExecutor::projection(int kind, int l, int R, bool feed) const {
  const bool tp = cfg_.tpSize > 1;
  const int H = cfg_.hidden, D = cfg_.headDim;
  auto *io = static_cast<int *>(stepIO_->data());
  int *tokens = io, *positions = io + cfg_.maxRows, *tableRows = io + 2 * cfg_.maxRows;
  // Residual stream buffers: TP ping-pongs between hA and hB because the
  // consumer kernel that folds the reduced projection into h also reads h.
  __half *hA = hp(h_), *hB = hp(hB_);
  auto *status = rt_.deviceStatus();
  float *partialF32 = fp(partialF32_);  // [R, H] row-parallel sums (TP with a collective)
  // TP over peer memory: partial-sum phase 2l = O of layer l, 2l + 1 = down.
  const bool xchg = tp && peersAttached_;
  const Layer &L = layers_[kind == kKernelLMHead ? 0 : l];
  tmc::GemvParams p{};
  p.M = R;
  p.status = status;
  p.trace = traceSink(kind == kKernelLMHead ? 0 : l, kind);
  p.work_counter = workCounter(kind == kKernelLMHead ? 0 : l, kind);
  p.l2_prefetch_bytes = kL2PrefetchBytes;
  p.peer_wait_ns = cfg_.peerWaitNs;
  p.local_wait_ns = cfg_.localWaitNs;
  switch (kind) {
    case kKernelQKV:
      p.W = hp(L.qkv);
      p.N = qkvRows_;
      p.K = H;
      if (l == 0) {
        p.prologue = tmc::kProEmbedNorm;
        p.embedding = hp(embedding_);
        p.tokens = tokens;
        p.vocab = cfg_.vocab;
        p.h_out = hA;
      } else if (tp) {
        p.prologue = tmc::kProResidualNorm;
        p.x = hB;
        p.partial = partialF32;
        p.h_out = hA;
        if (xchg) p.xchg = exchange(2 * (l - 1) + 1);
      } else {
        p.prologue = tmc::kProF16Norm;
        p.x = hA;
      }
      p.x_stride = H;
      p.gamma = hp(L.inputNorm);
      p.eps = cfg_.epsilon;
      p.epilogue = tmc::kEpiQKV;
      p.y_f16 = hp(q_);
      p.y_stride = (long long)hqL_ * D;
      p.q_rows = hqL_ * D;
      p.kv_rows = hkvL_ * D;
      p.head_dim = D;
      p.rope_cos = fp(ropeCos_);
      p.rope_sin = fp(ropeSin_);
      p.positions = positions;
      p.table_rows = tableRows;
      p.block_table = static_cast<const int *>(blockTable_->data());
      p.table_stride = maxPagesPerSeq_;
      p.page_size = pageSize_;
      p.pool_pages = poolPages_;
      p.capacity = cfg_.capacity;
      p.k_pool = hp(L.kPool);
      p.v_pool = hp(L.vPool);
      break;
    case kKernelO:
      p.W = hp(L.o);
      p.N = H;
      p.K = hqL_ * D;
      p.prologue = tmc::kProF16;
      p.x = hp(ctx_);
      p.x_stride = (long long)hqL_ * D;
      p.y_stride = H;
      if (tp) {
        p.epilogue = tmc::kEpiF32Partial;
        p.y_f32 = partialF32;
        if (xchg) p.xchg = exchange(2 * l);
      } else {
        p.epilogue = tmc::kEpiResidual;
        p.y_f16 = hA;
        p.residual = hA;
      }
      break;
    case kKernelGateUp:
      p.W = hp(L.gateUp);
      p.N = 2 * iL_;
      p.K = H;
      if (tp) {
        p.prologue = tmc::kProResidualNorm;
        p.x = hA;
        p.partial = partialF32;
        p.h_out = hB;
        if (xchg) p.xchg = exchange(2 * l);
      } else {
        p.prologue = tmc::kProF16Norm;
        p.x = hA;
      }
      p.x_stride = H;
      p.gamma = hp(L.postNorm);
      p.eps = cfg_.epsilon;
      p.epilogue = tmc::kEpiSwiGLU;
      p.y_f16 = hp(act_);
      p.y_stride = iL_;
      break;
    case kKernelDown:
      p.W = hp(L.down);
      p.N = H;
      p.K = iL_;
      p.prologue = tmc::kProF16;
      p.x = hp(act_);
      p.x_stride = iL_;
      p.y_stride = H;
      if (tp) {
        p.epilogue = tmc::kEpiF32Partial;
        p.y_f32 = partialF32;
        if (xchg) p.xchg = exchange(2 * l + 1);
      } else {
        p.epilogue = tmc::kEpiResidual;
        p.y_f16 = hA;
        p.residual = hA;
      }
      break;
    case kKernelLMHead:
      p.W = hp(lmHead_);
      p.N = vL_;
      p.K = H;
      if (tp) {
        p.prologue = tmc::kProResidualNorm;
        p.x = hB;
        p.partial = partialF32;
        p.h_out = hA;
        if (xchg) p.xchg = exchange(2 * (cfg_.layers - 1) + 1);  // also carries the argmax keys
      } else {
        p.prologue = tmc::kProF16Norm;
        p.x = hA;
      }
      p.x_stride = H;
      p.gamma = hp(finalNorm_);
      p.eps = cfg_.epsilon;
      p.epilogue = tmc::kEpiArgmax;
      p.y_f32 = fp(logits_);  // this rank's vocabulary slice
      p.y_stride = vL_;
      p.argmax_keys = static_cast<unsigned long long *>(argmaxKeys_->data());
      p.argmax_counter = static_cast<unsigned int *>(argmaxCounter_->data());
      p.vocab_offset = cfg_.tpRank * vL_;
      if (!tp || xchg) {
        p.next_tokens = static_cast<int *>(nextTokens_->data());
        if (feed) {
          p.feed_tokens = tokens;
          p.feed_positions = positions;
          p.history = static_cast<int *>(history_->data());
          p.history_counter = static_cast<unsigned int *>(historyCounter_->data());
        }
      }
      break;
    default:
      break;
  }
  // Every kernel of a step releases its dependents only after its own
  // dependency wait, so what was written two or more kernels back is final
  // when a kernel starts: the residual rows that O and down add to (written by
  // the previous layer's down, three kernels back, and by O, two back).
  // Single-row GEMVs read them before their own wait. (Reading the QKV
  // epilogue's positions, pages and RoPE rows early gained nothing.)
  p.early_epilogue_inputs = !tp && (kind == kKernelO || kind == kKernelDown);
  return p;
}

std::string DecoderExecutor::enqueueKernel(int kind, int l, int R, bool feed, bool distinct) {
  cudaStream_t s = rt_.stream();
  const bool pdl = cfg_.usePDL;
  const bool tp = cfg_.tpSize > 1;
  const int H = cfg_.hidden, D = cfg_.headDim;
  auto *io = static_cast<int *>(stepIO_->data());
  int *tokens = io, *positions = io + cfg_.maxRows, *tableRows = io + 2 * cfg_.maxRows;
  auto *status = rt_.deviceStatus();
  // Attention splits per (row, KV head): few pairs -> enough splits to cover
  // the SMs twice; many pairs (batched decode) -> a power of two that gives
  // about 8 CTAs per SM (bs64: 2 splits of ~576 positions; 4 splits, ~16 per
  // SM, cost 86.6 us against 80.7 per layer), so the last partial wave is short.
  int splits = std::max(1, std::min(64, (2 * numSms_ + R * hkvL_ - 1) / (R * hkvL_)));
  if (R * hkvL_ < numSms_) splits = std::min(splits, attnSplitCap_);
  if (R * hkvL_ >= numSms_) {
    splits = 1;
    while (splits < 16 && 2 * splits * R * hkvL_ <= 8 * numSms_) splits *= 2;
  }
  float *partialF32 = fp(partialF32_);
  const bool xchg = tp && peersAttached_;
  cudaError_t e;
  Layer &L = layers_[kind == kKernelLMHead ? 0 : l];
  switch (kind) {
    case kKernelQKV:
      return launchProjection(projection(kind, l, R, feed), "qkv projection");
    case kKernelAttention: {

      tmc::AttentionParams a{};
      a.q = hp(q_);
      a.q_stride = (long long)hqL_ * D;
      a.out = hp(ctx_);
      a.out_stride = (long long)hqL_ * D;
      a.k_pool = hp(L.kPool);
      a.v_pool = hp(L.vPool);
      a.block_table = static_cast<const int *>(blockTable_->data());
      a.table_stride = maxPagesPerSeq_;
      a.table_rows = tableRows;
      a.positions = positions;
      a.rows = R;
      a.hq = hqL_;
      a.hkv = hkvL_;
      a.head_dim = D;
      a.page_size = pageSize_;
      a.pool_pages = poolPages_;
      a.capacity = cfg_.capacity;
      a.scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(D)));
      a.max_splits = splits;
      a.min_chunk = 64;
      a.max_chunk = 128;
      // One row per sequence: only each row's newest K/V comes from the QKV
      // kernel still running, older rows can be gathered before its completion.
      a.early_mode = distinct ? 1 : 0;
      // A prefill chunk's rows are consecutive positions of one sequence: the
      // streaming schedule serves them in groups that share each K/V tile.
      a.row_group = (!distinct && R > 1) ? 16 / (hqL_ / hkvL_) : 1;
      a.ws_acc = fp(attnWorkspace_);
      a.ws_ml = fp(attnWorkspace_) + (size_t)R * hqL_ * splits * D;
      a.ws_floats = attnWorkspace_->elementCount();
      a.counters = static_cast<unsigned int *>(attnCounters_->data());
      a.status = status;
      a.trace = traceSink(l, kind);
      if ((D == 64 || D == 128) && pageSize_ % 16 == 0) {
        // 16-position page boxes through tensor maps over the pools.
        std::string err;
        a.k_map = tensorMap(L.kPool->data(), poolPages_ * hkvL_ * pageSize_, D, 16, &err);
        a.v_map = a.k_map ? tensorMap(L.vPool->data(), poolPages_ * hkvL_ * pageSize_, D, 16, &err) : nullptr;
        if (!a.v_map) return "attention: " + err;
      }
      if ((e = tmc::launch_attention(a, s, pdl)) != cudaSuccess) return cudaText("attention", e);
      (void)H;
      return {};
    }
    case kKernelO:
    case kKernelDown: {
      if (auto pe = launchProjection(projection(kind, l, R, feed), kind == kKernelO ? "o projection" : "down projection");
          !pe.empty())
        return pe;
      if (tp && !xchg && (e = collective_->allReduceSumF32(partialF32, (size_t)R * H, s)) != cudaSuccess)
        return std::string(kind == kKernelO ? "allreduce (o): " : "allreduce (down): ") + collective_->lastError();
      return {};
    }
    case kKernelGateUp:
      return launchProjection(projection(kind, l, R, feed), "gate/up projection");
    case kKernelLMHead: {
      const tmc::GemvParams p = projection(kind, 0, R, feed);
      if (auto pe = launchProjection(p, "lm head projection"); !pe.empty()) return pe;
      if (tp && !xchg) {
        if ((e = collective_->allReduceMaxU64(p.argmax_keys, R, s)) != cudaSuccess)
          return "allreduce (argmax): " + collective_->lastError();
        if ((e = tmc::launch_argmax_finalize(p.argmax_keys, R, static_cast<int *>(nextTokens_->data()),
                                             feed ? tokens : nullptr, feed ? positions : nullptr,
                                             feed ? static_cast<int *>(history_->data()) : nullptr,
                                             feed ? static_cast<unsigned int *>(historyCounter_->data()) : nullptr,
                                             s, false)) != cudaSuccess)
          return cudaText("argmax finalize", e);
      }
      return {};
    }
    default:
      return "unknown kernel kind";
  }
}

std::string DecoderExecutor::enqueueStep(int R, bool feed, bool distinct, bool head) {
  const bool tp = cfg_.tpSize > 1;
  if (tp && !collective_ && !peersAttached_)
    return "tensor parallelism needs a collective (setCollective) or attached peers (attachPeers).";
  for (int l = 0; l < cfg_.layers; ++l)
    for (int kind = kKernelQKV; kind <= kKernelDown; ++kind) {
      auto e = enqueueKernel(kind, l, R, feed, distinct);
      if (!e.empty()) return e;
    }
  return head ? enqueueKernel(kKernelLMHead, 0, R, feed, distinct) : std::string();
}

unsigned int *DecoderExecutor::workCounter(int layer, int kind) const {
  return static_cast<unsigned int *>(workCounters_->data()) + (size_t)(layer * 6 + kind) * tmc::kGemvCounterWords;
}

tmc::TraceSink DecoderExecutor::traceSink(int layer, int kind) const {
  tmc::TraceSink t{};
  if (traceCapacity_ == 0) return t;
  t.records = static_cast<tmc::TraceRecord *>(traceRecords_->data());
  t.count = static_cast<unsigned int *>(traceCount_->data());
  t.capacity = static_cast<unsigned int>(traceCapacity_);
  t.tag = (static_cast<unsigned int>(layer) << 8) | static_cast<unsigned int>(kind);
  return t;
}

std::string DecoderExecutor::setTrace(std::size_t capacity) {
  auto e = rt_.synchronize();
  if (!e.empty()) return e;
  for (auto &kv : graphs_) {
    if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
    if (kv.second.graph) cudaGraphDestroy(kv.second.graph);
  }
  graphs_.clear();
  traceCapacity_ = 0;
  traceRecords_.reset();
  traceCount_.reset();
  if (capacity == 0) return {};
  auto r = rt_.createBuffer(capacity * sizeof(tmc::TraceRecord) / 4, nullptr, ElementType::Int32);
  if (!r.buffer) return r.errorMessage;
  auto c = rt_.createBuffer(4, nullptr, ElementType::Int32);
  if (!c.buffer) return c.errorMessage;
  traceRecords_ = r.buffer;
  traceCount_ = c.buffer;
  traceCapacity_ = capacity;
  return rt_.synchronize();
}

std::string DecoderExecutor::readTrace(std::vector<tmc::TraceRecord> *out) {
  out->clear();
  if (traceCapacity_ == 0) return "tracing is off";
  auto e = rt_.synchronize();
  if (!e.empty()) return e;
  unsigned int n = 0;
  TMC_TRY(cudaMemcpy(&n, traceCount_->data(), 4, cudaMemcpyDeviceToHost));
  n = std::min<unsigned int>(n, static_cast<unsigned int>(traceCapacity_));
  out->resize(n);
  if (n) TMC_TRY(cudaMemcpy(out->data(), traceRecords_->data(), n * sizeof(tmc::TraceRecord), cudaMemcpyDeviceToHost));
  TMC_TRY(cudaMemsetAsync(traceCount_->data(), 0, 4, rt_.stream()));
  return rt_.synchronize();
}

std::string DecoderExecutor::profileKernel(int kind, int R, int rounds, double *avgUs,
                                           double *bytesPerLaunch, int *launchesPerStep) {
  if (kind < kKernelQKV || kind > kKernelLMHead) return "unknown kernel kind";
  if (R < 1 || R > cfg_.maxRows || rounds < 1) return "profileKernel: bad rows or rounds";
  if (cfg_.tpSize > 1 && (kind == kKernelO || kind == kKernelDown))
    return "profileKernel: row-parallel kernels include a collective under TP";
  const double H = cfg_.hidden, D = cfg_.headDim;
  double bytes = 0.0;
  switch (kind) {
    case kKernelQKV:
      bytes = 2.0 * qkvRows_ * H + 2.0 * R * H + 2.0 * H + 2.0 * R * qkvRows_;
      break;
    case kKernelAttention: {
      double ctx = 0.0;
      for (int r = 0; r < R; ++r) ctx += lastPositions_[r] + 1.0;
      bytes = 2.0 * 2.0 * hkvL_ * D * ctx + 2.0 * 2.0 * R * hqL_ * D;
      break;
    }
    case kKernelO:
      bytes = 2.0 * H * hqL_ * D + 2.0 * R * hqL_ * D + 2.0 * 2.0 * R * H;
      break;
    case kKernelGateUp:
      bytes = 2.0 * 2.0 * iL_ * H + 2.0 * R * H + 2.0 * H + 2.0 * R * iL_;
      break;
    case kKernelDown:
      bytes = 2.0 * H * iL_ + 2.0 * R * iL_ + 2.0 * 2.0 * R * H;
      break;
    case kKernelLMHead:
      bytes = 2.0 * vL_ * H + 2.0 * R * H + 2.0 * H + 4.0 * R * vL_;
      break;
  }
  const int perRound = kind == kKernelLMHead ? 1 : cfg_.layers;
  cudaStream_t s = rt_.stream();
  auto sync = rt_.synchronize();
  if (!sync.empty()) return sync;
  TMC_TRY(cudaStreamBeginCapture(s, cudaStreamCaptureModeRelaxed));
  std::string err;
  profiling_ = true;  // partial-sum consumers read whatever the slots hold
  for (int r = 0; r < rounds && err.empty(); ++r)
    for (int l = 0; l < perRound && err.empty(); ++l) err = enqueueKernel(kind, l, R, false, true);
  profiling_ = false;
  cudaGraph_t graph = nullptr;
  const cudaError_t ce = cudaStreamEndCapture(s, &graph);
  if (!err.empty() || ce != cudaSuccess) {
    if (graph) cudaGraphDestroy(graph);
    cudaGetLastError();
    return !err.empty() ? err : cudaText("cudaStreamEndCapture", ce);
  }
  cudaGraphExec_t exec = nullptr;
  cudaError_t ie = cudaGraphInstantiate(&exec, graph, 0);
  if (ie != cudaSuccess) {
    cudaGraphDestroy(graph);
    return cudaText("cudaGraphInstantiate", ie);
  }
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  cudaGraphLaunch(exec, s);  // warm-up
  cudaEventRecord(e0, s);
  cudaGraphLaunch(exec, s);
  cudaEventRecord(e1, s);
  err = rt_.synchronize();
  float ms = 0.0f;
  if (err.empty()) cudaEventElapsedTime(&ms, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  cudaGraphExecDestroy(exec);
  cudaGraphDestroy(graph);
  if (!err.empty()) return err;
  if (avgUs) *avgUs = ms * 1000.0 / (double)(rounds * perRound);
  if (bytesPerLaunch) *bytesPerLaunch = bytes;
  if (launchesPerStep) *launchesPerStep = perRound;
  return {};
}

std::string DecoderExecutor::launchStep(int R, bool feed, bool distinct, bool head) {
  if (!cfg_.useGraphs) return enqueueStep(R, feed, distinct, head);
  const int key = graphKey(R, feed, distinct, head);
  auto it = graphs_.find(key);
  if (it == graphs_.end()) {
    cudaStream_t s = rt_.stream();
    TMC_TRY(cudaStreamBeginCapture(s, cudaStreamCaptureModeRelaxed));
    const std::string err = enqueueStep(R, feed, distinct, head);
    cudaGraph_t graph = nullptr;
    const cudaError_t ce = cudaStreamEndCapture(s, &graph);
    if (!err.empty() || ce != cudaSuccess) {
      if (graph) cudaGraphDestroy(graph);
      cudaGetLastError();
      return !err.empty() ? "capture: " + err : cudaText("cudaStreamEndCapture", ce);
    }
    Graph g;
    g.graph = graph;
    const cudaError_t ie = cudaGraphInstantiate(&g.exec, graph, 0);
    if (ie != cudaSuccess) {
      cudaGraphDestroy(graph);
      cudaGetLastError();
      return cudaText("cudaGraphInstantiate", ie);
    }
    it = graphs_.emplace(key, g).first;
  }
  TMC_TRY(cudaGraphLaunch(it->second.exec, rt_.stream()));
  return {};
}

std::string DecoderExecutor::uploadStepInputs(int R, const std::int32_t *tokens, const std::int32_t *positions,
                                              const std::int32_t *tableRows, int steps, std::int32_t *stage) {
  const int M = cfg_.maxRows;
  std::int32_t *io = stage ? stage : pinnedIO_;
  // The attention chunk policy below (min_chunk 64, max_chunk 128, one
  // 16-CTA cluster filled before a second): splits for the longest context.
  int maxLen = 1;
  for (int r = 0; r < R; ++r) maxLen = std::max(maxLen, positions[r] + steps);
  int need = (maxLen + 63) / 64;
  if (need > 16) need = std::max((maxLen + 127) / 128, 16);
  attnSplitCap_ = (need + 15) / 16 * 16;
  for (int i = 0; i < 3 * M; ++i) io[i] = 0;
  for (int r = 0; r < M; ++r) lastPositions_[r] = r < R ? positions[r] : 0;
  for (int r = 0; r < R; ++r) {
    io[r] = tokens[r];
    io[M + r] = positions[r];
    io[2 * M + r] = tableRows[r];
  }
  TMC_TRY(cudaMemcpyAsync(stepIO_->data(), io, sizeof(std::int32_t) * 3 * M, cudaMemcpyHostToDevice,
                          rt_.stream()));
  return {};
}

std::string DecoderExecutor::decode(const std::int32_t *slots, const std::int32_t *tokens, int rows,
                                    float *logits, std::int32_t *nextTokens, StepTiming *timing) {
  if (rows < 1 || rows > cfg_.maxRows) return "decode: rows must be in [1, maxRows].";
  std::vector<std::int32_t> positions(rows), tableRows(rows);
  for (int r = 0; r < rows; ++r) {
    const int slot = slots[r];
    if (slot < 0 || slot >= cfg_.maxSlots) return "decode: slot out of range.";
    for (int q = 0; q < r; ++q)
      if (slots[q] == slot) return "decode: slots must be distinct within a step.";
    if (tokens[r] < 0 || tokens[r] >= cfg_.vocab) return "decode: token id out of vocabulary range.";
  }
  int staged = 0;
  std::string err;
  for (; staged < rows; ++staged) {
    auto &st = *slots_[slots[staged]];
    positions[staged] = static_cast<std::int32_t>(st.currentLength());
    tableRows[staged] = slots[staged];
    err = st.stageLength(st.currentLength() + 1);
    if (!err.empty()) break;
  }
  auto unwind = [&](int n) {
    for (int r = 0; r < n; ++r) (void)slots_[slots[r]]->rollbackLength(slots_[slots[r]]->currentLength());
  };
  if (!err.empty()) {
    unwind(staged);
    return err;
  }
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  if (timing) {
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
  }
  const auto c0 = std::chrono::steady_clock::now();
  err = uploadStepInputs(rows, tokens, positions.data(), tableRows.data());
  if (timing) cudaEventRecord(e0, rt_.stream());
  if (err.empty()) err = launchStep(rows, false, true);
  if (timing) cudaEventRecord(e1, rt_.stream());
  if (err.empty()) {
    cudaError_t ce = cudaMemcpyAsync(pinnedIO_ + 3 * cfg_.maxRows, nextTokens_->data(), sizeof(std::int32_t) * rows,
                                     cudaMemcpyDeviceToHost, rt_.stream());
    if (ce == cudaSuccess && logits)
      ce = cudaMemcpyAsync(logits, logits_->data(), sizeof(float) * rows * vL_, cudaMemcpyDeviceToHost, rt_.stream());
    if (ce != cudaSuccess) err = cudaText("decode readback", ce);
  }
  const std::string sync = rt_.synchronize();
  if (err.empty()) err = sync;
  if (timing) {
    float ms = 0.0f;
    if (err.empty() && cudaEventElapsedTime(&ms, e0, e1) == cudaSuccess) timing->gpuUs = ms * 1000.0;
    timing->cpuUs = std::chrono::duration<double, std::micro>(std::chrono::steady_clock::now() - c0).count();
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
  }
  if (!err.empty()) {
    unwind(rows);
    return err;
  }
  for (int r = 0; r < rows; ++r) {
    auto &st = *slots_[slots[r]];
    st.commitLength(st.currentLength() + 1);
    if (nextTokens) nextTokens[r] = pinnedIO_[3 * cfg_.maxRows + r];
  }
  return {};
}

std::string DecoderExecutor::prefill(int slot, const std::int32_t *tokens, int count, float *logits,
                                     std::int32_t *nextToken, StepTiming *timing) {
  if (slot < 0 || slot >= cfg_.maxSlots) return "prefill: slot out of range.";
  if (count < 1) return "prefill: token count must be positive.";
  for (int i = 0; i < count; ++i)
    if (tokens[i] < 0 || tokens[i] >= cfg_.vocab) return "prefill: token id out of vocabulary range.";
  auto &st = *slots_[slot];
  const size_t start = st.currentLength();
  auto err = st.stageLength(start + count);
  if (!err.empty()) return err;
  // Chunks of maxRows rows (the reference's prefillChunked,
  // DecoderLLMExecutor.cpp:982-1034), queued back to back: each chunk's inputs
  // come from its own pinned staging block, so the host never waits between
  // chunks; one synchronisation at the end (per chunk only when logits are
  // copied to pageable host memory).
  const int M = cfg_.maxRows;
  std::vector<std::int32_t> pos(M), trow(M, slot);
  double gpuUs = 0.0;
  const auto c0 = std::chrono::steady_clock::now();
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  if (timing) {
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    cudaEventRecord(e0, rt_.stream());
  }
  int last = 0;
  for (int done = 0, chunk = 0; done < count && err.empty(); ++chunk) {
    const int R = std::min(M, count - done);
    if ((std::size_t)chunk >= prefillChunks_) {
      err = "prefill: more chunks than the staging holds.";
      break;
    }
    for (int r = 0; r < R; ++r) pos[r] = static_cast<std::int32_t>(start + done + r);
    err = uploadStepInputs(R, tokens + done, pos.data(), trow.data(), 1, prefillStage_ + (std::size_t)chunk * 3 * M);
    // Only the last chunk's LM head is read unless logits are asked for (the
    // peer exchange's step epoch advances in the head, so it always runs then).
    const bool head = logits != nullptr || done + R == count || (cfg_.tpSize > 1 && peersAttached_);
    if (err.empty()) err = launchStep(R, false, R == 1, head);
    if (err.empty() && logits) {
      cudaError_t ce = cudaMemcpyAsync(logits + (size_t)done * vL_, logits_->data(), sizeof(float) * R * vL_,
                                       cudaMemcpyDeviceToHost, rt_.stream());
      if (ce != cudaSuccess) err = cudaText("prefill logits readback", ce);
    }
    if (err.empty() && done + R == count) {
      cudaError_t ce = cudaMemcpyAsync(pinnedIO_ + 3 * M, nextTokens_->data(), sizeof(std::int32_t) * R,
                                       cudaMemcpyDeviceToHost, rt_.stream());
      if (ce != cudaSuccess) err = cudaText("prefill token readback", ce);
    }
    last = R;
    done += R;
  }
  if (timing) cudaEventRecord(e1, rt_.stream());
  const std::string sync = rt_.synchronize();
  if (err.empty()) err = sync;
  if (timing) {
    float ms = 0.0f;
    if (err.empty() && cudaEventElapsedTime(&ms, e0, e1) == cudaSuccess) gpuUs = ms * 1000.0;
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
  }
  if (err.empty() && nextToken) *nextToken = pinnedIO_[3 * M + last - 1];
  if (timing) {
    timing->gpuUs = gpuUs;
    timing->cpuUs = std::chrono::duration<double, std::micro>(std::chrono::steady_clock::now() - c0).count();
  }
  if (!err.empty()) {
    (void)st.rollbackLength(start);
    return err;
  }
  st.commitLength(start + count);
  return {};
}

std::string DecoderExecutor::generate(const std::int32_t *slots, const std::int32_t *tokens, int rows, int steps,
                                      std::int32_t *tokensOut, StepTiming *timing) {
  if (rows < 1 || rows > cfg_.maxRows) return "generate: rows must be in [1, maxRows].";
  if (steps < 1) return "generate: steps must be positive.";
  if ((size_t)steps * rows > (size_t)historyCapacity_) return "generate: too many steps for the history buffer.";
  std::vector<std::int32_t> positions(rows), tableRows(rows);
  for (int r = 0; r < rows; ++r) {
    if (slots[r] < 0 || slots[r] >= cfg_.maxSlots) return "generate: slot out of range.";
    for (int q = 0; q < r; ++q)
      if (slots[q] == slots[r]) return "generate: slots must be distinct.";
    if (tokens[r] < 0 || tokens[r] >= cfg_.vocab) return "generate: token id out of vocabulary range.";
  }
  int staged = 0;
  std::string err;
  for (; staged < rows; ++staged) {
    auto &st = *slots_[slots[staged]];
    positions[staged] = static_cast<std::int32_t>(st.currentLength());
    tableRows[staged] = slots[staged];
    err = st.stageLength(st.currentLength() + steps);
    if (!err.empty()) break;
  }
  auto unwind = [&](int n) {
    for (int r = 0; r < n; ++r) (void)slots_[slots[r]]->rollbackLength(slots_[slots[r]]->currentLength());
  };
  if (!err.empty()) {
    unwind(staged);
    return err;
  }
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  const auto c0 = std::chrono::steady_clock::now();
  err = uploadStepInputs(rows, tokens, positions.data(), tableRows.data(), steps);
  if (err.empty()) {
    cudaError_t ce = cudaMemsetAsync(historyCounter_->data(), 0, 4, rt_.stream());
    if (ce != cudaSuccess) err = cudaText("history reset", ce);
  }
  // Build the graph before timing so capture cost is not counted.
  if (err.empty() && cfg_.useGraphs && !graphs_.count(graphKey(rows, true, true))) {
    err = rt_.synchronize();
    if (err.empty()) {
      cudaStream_t s = rt_.stream();
      cudaError_t ce = cudaStreamBeginCapture(s, cudaStreamCaptureModeRelaxed);
      if (ce != cudaSuccess) err = cudaText("capture", ce);
      std::string ee = err.empty() ? enqueueStep(rows, true, true) : err;
      cudaGraph_t graph = nullptr;
      ce = cudaStreamEndCapture(s, &graph);
      if (!ee.empty() || ce != cudaSuccess) {
        if (graph) cudaGraphDestroy(graph);
        cudaGetLastError();
        err = !ee.empty() ? ee : cudaText("cudaStreamEndCapture", ce);
      } else {
        Graph g;
        g.graph = graph;
        ce = cudaGraphInstantiate(&g.exec, graph, 0);
        if (ce != cudaSuccess) {
          cudaGraphDestroy(graph);
          err = cudaText("cudaGraphInstantiate", ce);
        } else {
          graphs_.emplace(graphKey(rows, true, true), g);
        }
      }
    }
  }
  cudaEventRecord(e0, rt_.stream());
  for (int i = 0; i < steps && err.empty(); ++i) err = launchStep(rows, true, true);
  cudaEventRecord(e1, rt_.stream());
  if (err.empty()) {
    cudaError_t ce = cudaMemcpyAsync(tokensOut, history_->data(), sizeof(std::int32_t) * steps * rows,
                                     cudaMemcpyDeviceToHost, rt_.stream());
    if (ce != cudaSuccess) err = cudaText("generate readback", ce);
  }
  const std::string sync = rt_.synchronize();
  if (err.empty()) err = sync;
  float ms = 0.0f;
  if (timing) {
    if (err.empty() && cudaEventElapsedTime(&ms, e0, e1) == cudaSuccess) timing->gpuUs = ms * 1000.0;
    timing->cpuUs = std::chrono::duration<double, std::micro>(std::chrono::steady_clock::now() - c0).count();
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (!err.empty()) {
    unwind(rows);
    return err;
  }
  for (int r = 0; r < rows; ++r) {
    auto &st = *slots_[slots[r]];
    st.commitLength(st.currentLength() + steps);
  }
  return {};
}

}  // namespace tensor::runtime
