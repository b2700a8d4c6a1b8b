// extern "C" boundary of the decoder executor (declarations and reference
// citations in include/tmc_cuda.h).
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <memory>
#include <sstream>
#include <string>
#include <vector>

#include <nccl.h>

#include "CudaRuntime.hpp"
#include "DecoderExecutor.hpp"
#include "DecoderManifest.hpp"
#include "NcclCollective.hpp"
#include "ServingRuntime.hpp"
#include "api_util.hpp"
#include "tmc_cuda.h"

using tensor::runtime::DecoderConfig;
using tensor::runtime::DecoderExecutor;
using namespace tmc_api;

struct tmc_decoder {
  std::unique_ptr<DecoderExecutor> ex;
  int device = 0;
  tensor::runtime::StepTiming lastPrefill;  // the last tmc_decoder_prefill call
};

struct tmc_manifest {
  tensor::importer::DecoderManifest m;
};

namespace {

int status_of(const std::string &e) {
  if (e.rfind("device status", 0) == 0) return TMC_ERR_DEVICE_STATUS;
  if (e.find("exhausted") != std::string::npos) return TMC_ERR_OUT_OF_MEMORY;
  if (e.find("cuda") != std::string::npos || e.find("Cuda") != std::string::npos) return TMC_ERR_CUDA;
  return TMC_ERR_INVALID;
}

int done(const std::string &e) { return e.empty() ? ok() : fail(status_of(e), e); }

bool bind(tmc_decoder *d) {
  if (d == nullptr || !d->ex) return false;
  int cur = -1;
  if (cudaGetDevice(&cur) == cudaSuccess && cur != d->device) cudaSetDevice(d->device);
  return true;
}

}  // namespace

extern "C" {

int tmc_decoder_create(tmc_runtime *rt, const tmc_decoder_config *c, tmc_decoder **out) {
  if (rt == nullptr || c == nullptr || out == nullptr) return fail(TMC_ERR_INVALID, "null argument");
  *out = nullptr;
  cudaSetDevice(rt->rt->device());
  DecoderConfig cfg;
  cfg.hidden = c->hidden_size;
  cfg.heads = c->heads;
  cfg.kvHeads = c->kv_heads > 0 ? c->kv_heads : c->heads;
  cfg.headDim = c->head_dim > 0 ? c->head_dim : (c->heads > 0 ? c->hidden_size / c->heads : 0);
  cfg.intermediate = c->intermediate_size;
  cfg.vocab = c->vocab_size;
  cfg.layers = c->layers;
  cfg.capacity = c->capacity;
  cfg.epsilon = c->epsilon;
  cfg.ropeTheta = c->rope_theta > 0.0 ? c->rope_theta : 10000.0;
  cfg.maxRows = c->max_rows > 0 ? c->max_rows : 8;
  cfg.maxSlots = c->max_slots > 0 ? c->max_slots : 1;
  cfg.pageSize = c->page_size;
  cfg.poolPages = c->pool_pages;
  cfg.tpRank = c->tp_rank;
  cfg.tpSize = c->tp_size > 0 ? c->tp_size : 1;
  cfg.useGraphs = c->use_graphs != 0;
  cfg.usePDL = c->use_pdl != 0;
  std::string err;
  auto ex = DecoderExecutor::create(*rt->rt, cfg, &err);
  if (!ex) return fail(err.find("cudaMalloc") != std::string::npos ? TMC_ERR_OUT_OF_MEMORY : TMC_ERR_INVALID, err);
  *out = new tmc_decoder{std::move(ex), rt->rt->device()};
  return ok();
}

void tmc_decoder_destroy(tmc_decoder *dec) {
  if (dec) {
    bind(dec);
    delete dec;
  }
}

int tmc_decoder_load_weight(tmc_decoder *dec, const char *name, const float *values, size_t count) {
  if (!bind(dec) || name == nullptr || values == nullptr) return fail(TMC_ERR_INVALID, "null argument");
  return done(dec->ex->loadWeight(name, values, count));
}

int tmc_decoder_load_weight_f16(tmc_decoder *dec, const char *name, const uint16_t *bits, size_t count) {
  if (!bind(dec) || name == nullptr || bits == nullptr) return fail(TMC_ERR_INVALID, "null argument");
  return done(dec->ex->loadWeightF16(name, bits, count));
}

int tmc_manifest_open(const char *path, tmc_manifest **out) {
  if (path == nullptr || out == nullptr) return fail(TMC_ERR_INVALID, "null argument");
  auto h = std::make_unique<tmc_manifest>();
  const auto e = tensor::importer::importDecoderManifest(path, &h->m);
  if (!e.empty()) return fail(TMC_ERR_INVALID, e);
  *out = h.release();
  return ok();
}

void tmc_manifest_close(tmc_manifest *m) { delete m; }

int tmc_manifest_get_info(const tmc_manifest *m, tmc_manifest_info *info) {
  if (m == nullptr || info == nullptr) return fail(TMC_ERR_INVALID, "null argument");
  const auto &d = m->m;
  tmc_manifest_info r{};
  r.version = d.version;
  r.batch = (int)d.batch;
  r.hidden_size = (int)d.hidden;
  r.heads = (int)d.heads;
  r.head_dim = (int)(d.hidden / d.heads);
  r.intermediate_size = (int)d.intermediate;
  r.vocab_size = (int)d.vocab;
  r.layers = (int)d.layers;
  r.capacity = (int)d.capacity;
  r.prefill_length = (int)d.prefillLength;
  r.decode_count = (int)d.decodeCount;
  r.epsilon = d.epsilon;
  std::snprintf(r.requested_dtype, sizeof r.requested_dtype, "%s", d.requestedDtype.c_str());
  std::snprintf(r.effective_dtype, sizeof r.effective_dtype, "%s", d.effectiveDtype.c_str());
  r.kv_heads = (int)d.kvHeads;
  r.rope_theta = d.ropeTheta;
  *info = r;
  return ok();
}

int tmc_manifest_tensor(const tmc_manifest *m, const char *name, const float **values, size_t *count) {
  if (m == nullptr || name == nullptr || values == nullptr || count == nullptr)
    return fail(TMC_ERR_INVALID, "null argument");
  *values = m->m.tensor(name, count);
  if (*values == nullptr) return fail(TMC_ERR_INVALID, std::string("manifest has no tensor '") + name + "'");
  return ok();
}

int tmc_decoder_load_manifest(tmc_decoder *dec, const tmc_manifest *m) {
  if (!bind(dec) || m == nullptr) return fail(TMC_ERR_INVALID, "null argument");
  const auto &c = dec->ex->config();
  const auto &d = m->m;
  const std::pair<const char *, std::pair<std::size_t, std::size_t>> dims[] = {
      {"hidden size", {(std::size_t)c.hidden, d.hidden}},
      {"head count", {(std::size_t)c.heads, d.heads}},
      {"KV head count", {(std::size_t)c.kvHeads, d.kvHeads}},
      {"head dimension", {(std::size_t)c.headDim, d.hidden / d.heads}},
      {"intermediate size", {(std::size_t)c.intermediate, d.intermediate}},
      {"vocabulary size", {(std::size_t)c.vocab, d.vocab}},
      {"layer count", {(std::size_t)c.layers, d.layers}}};
  for (const auto &x : dims)
    if (x.second.first != x.second.second)
      return fail(TMC_ERR_INVALID, std::string("decoder ") + x.first + " " + std::to_string(x.second.first) +
                                       " does not match the manifest's " + std::to_string(x.second.second));
  // The reference resolves fp32, fp16 or bf16 storage (DecoderLLMExecutor.cpp:1218-1240);
  // this backend's decoder stores and computes in fp16 only, so a manifest
  // exported for another storage type is refused rather than silently converted.
  if (d.dtypeLine && d.effectiveDtype != "F16")
    return fail(TMC_ERR_UNSUPPORTED, "decoder storage dtype is fp16 on this backend; the manifest asks for " +
                                         d.effectiveDtype + " (requested " + d.requestedDtype +
                                         "): re-export it with DTYPE F16");
  for (const auto &name : tensor::importer::decoderWeightNames(m->m.layers)) {
    size_t count = 0;
    const float *v = m->m.tensor(name, &count);
    if (v == nullptr) return fail(TMC_ERR_INVALID, "manifest has no tensor '" + name + "'");
    const std::string e = dec->ex->loadWeight(name, v, count);
    if (!e.empty()) return done("manifest tensor '" + name + "': " + e);
  }
  return ok();
}

int tmc_decoder_read_weight(tmc_decoder *dec, const char *name, float *out, size_t count) {
  if (!bind(dec) || name == nullptr || out == nullptr) return fail(TMC_ERR_INVALID, "null argument");
  std::vector<float> v;
  auto e = dec->ex->readWeight(name, &v);
  if (!e.empty()) return done(e);
  if (v.size() != count) return fail(TMC_ERR_INVALID, "count does not match the rank-local weight size " + std::to_string(v.size()));
  std::memcpy(out, v.data(), count * sizeof(float));
  return ok();
}

int tmc_decoder_init_random(tmc_decoder *dec, uint64_t seed, float stddev) {
  if (!bind(dec)) return fail(TMC_ERR_INVALID, "null decoder");
  return done(dec->ex->initRandom(seed, stddev));
}

int tmc_decoder_prefill(tmc_decoder *dec, int slot, const int32_t *tokens, int count, float *logits,
                        int32_t *next_token) {
  if (!bind(dec) || tokens == nullptr) return fail(TMC_ERR_INVALID, "null argument");
  dec->lastPrefill = {};
  return done(dec->ex->prefill(slot, tokens, count, logits, next_token, &dec->lastPrefill));
}

int tmc_decoder_prefill_timing(tmc_decoder *dec, double *gpu_us, double *cpu_us) {
  if (!bind(dec)) return fail(TMC_ERR_INVALID, "null decoder");
  if (gpu_us) *gpu_us = dec->lastPrefill.gpuUs;
  if (cpu_us) *cpu_us = dec->lastPrefill.cpuUs;
  return ok();
}

int tmc_decoder_decode(tmc_decoder *dec, const int32_t *slots, const int32_t *tokens, int rows, float *logits,
                       int32_t *next_tokens) {
  if (!bind(dec) || slots == nullptr || tokens == nullptr) return fail(TMC_ERR_INVALID, "null argument");
  return done(dec->ex->decode(slots, tokens, rows, logits, next_tokens));
}

int tmc_decoder_generate(tmc_decoder *dec, const int32_t *slots, const int32_t *tokens, int rows, int steps,
                         int32_t *tokens_out, double *gpu_us) {
  if (!bind(dec) || slots == nullptr || tokens == nullptr || tokens_out == nullptr)
    return fail(TMC_ERR_INVALID, "null argument");
  tensor::runtime::StepTiming t;
  auto e = dec->ex->generate(slots, tokens, rows, steps, tokens_out, &t);
  if (gpu_us) *gpu_us = t.gpuUs;
  return done(e);
}

size_t tmc_decoder_current_length(tmc_decoder *dec, int slot) {
  if (!bind(dec)) return 0;
  return dec->ex->currentLength(slot);
}

int tmc_decoder_read_kv(tmc_decoder *dec, int layer, int slot, float *key, float *value, size_t count) {
  if (!bind(dec) || key == nullptr || value == nullptr) return fail(TMC_ERR_INVALID, "null argument");
  std::vector<float> k, v;
  auto e = dec->ex->readKV(layer, slot, &k, &v);
  if (!e.empty()) return done(e);
  if (k.size() != count) return fail(TMC_ERR_INVALID, "count must be local_kv_heads*length*head_dim = " + std::to_string(k.size()));
  std::memcpy(key, k.data(), count * sizeof(float));
  std::memcpy(value, v.data(), count * sizeof(float));
  return ok();
}

int tmc_decoder_restore_kv(tmc_decoder *dec, int slot, size_t length, const float *keys, const float *values) {
  if (!bind(dec) || keys == nullptr || values == nullptr) return fail(TMC_ERR_INVALID, "null argument");
  const auto &c = dec->ex->config();
  const size_t per = (size_t)dec->ex->localKVHeads() * length * c.headDim;
  std::vector<std::vector<float>> k(c.layers), v(c.layers);
  for (int l = 0; l < c.layers; ++l) {
    k[l].assign(keys + l * per, keys + (l + 1) * per);
    v[l].assign(values + l * per, values + (l + 1) * per);
  }
  return done(dec->ex->restoreKV(slot, length, k, v));
}

int tmc_decoder_block_table(tmc_decoder *dec, int slot, int32_t *out, size_t capacity, size_t *count) {
  if (!bind(dec) || count == nullptr) return fail(TMC_ERR_INVALID, "null argument");
  const auto t = dec->ex->blockTable(slot);
  *count = t.size();
  if (out != nullptr) std::memcpy(out, t.data(), std::min(capacity, t.size()) * sizeof(int32_t));
  return ok();
}

int tmc_decoder_stage_length(tmc_decoder *dec, int slot, size_t length) {
  if (!bind(dec)) return fail(TMC_ERR_INVALID, "null decoder");
  return done(dec->ex->stageLength(slot, length));
}

int tmc_decoder_commit_length(tmc_decoder *dec, int slot, size_t length) {
  if (!bind(dec)) return fail(TMC_ERR_INVALID, "null decoder");
  return done(dec->ex->commitLength(slot, length));
}

int tmc_decoder_rollback_length(tmc_decoder *dec, int slot, size_t length) {
  if (!bind(dec)) return fail(TMC_ERR_INVALID, "null decoder");
  return done(dec->ex->rollbackLength(slot, length));
}

int tmc_decoder_release(tmc_decoder *dec, int slot) {
  if (!bind(dec)) return fail(TMC_ERR_INVALID, "null decoder");
  return done(dec->ex->releaseSlot(slot));
}

int tmc_decoder_storage(tmc_decoder *dec, size_t *model_bytes, size_t *kv_bytes, size_t *activation_bytes) {
  if (!bind(dec)) return fail(TMC_ERR_INVALID, "null decoder");
  if (model_bytes) *model_bytes = dec->ex->modelStorageBytes();
  if (kv_bytes) *kv_bytes = dec->ex->kvStorageBytes();
  if (activation_bytes) *activation_bytes = dec->ex->activationStorageBytes();
  return ok();
}

int tmc_decoder_local_dims(tmc_decoder *dec, int *heads, int *kv_heads, int *intermediate, int *vocab,
                           int *vocab_offset) {
  if (!bind(dec)) return fail(TMC_ERR_INVALID, "null decoder");
  if (heads) *heads = dec->ex->localHeads();
  if (kv_heads) *kv_heads = dec->ex->localKVHeads();
  if (intermediate) *intermediate = dec->ex->localIntermediate();
  if (vocab) *vocab = dec->ex->localVocab();
  if (vocab_offset) *vocab_offset = dec->ex->vocabOffset();
  return ok();
}

int tmc_decoder_pool_stats(tmc_decoder *dec, size_t *capacity, size_t *used, size_t *peak, size_t *allocations,
                           size_t *releases) {
  if (!bind(dec)) return fail(TMC_ERR_INVALID, "null decoder");
  auto &p = dec->ex->pagePool();
  if (capacity) *capacity = p.capacityPages();
  if (used) *used = p.usedPages();
  if (peak) *peak = p.peakUsedPages();
  if (allocations) *allocations = p.allocationCount();
  if (releases) *releases = p.releaseCount();
  return ok();
}

int tmc_decoder_inject_page_failures(tmc_decoder *dec, size_t n) {
  if (!bind(dec)) return fail(TMC_ERR_INVALID, "null decoder");
  dec->ex->pagePool().failNextAllocations(n);
  return ok();
}

int tmc_decoder_kernels_per_step(tmc_decoder *dec, int rows) {
  if (!bind(dec)) return -1;
  return dec->ex->kernelsPerStep(rows);
}

double tmc_decoder_step_bytes(tmc_decoder *dec, int rows, const int32_t *context_lengths) {
  if (!bind(dec) || context_lengths == nullptr) return 0.0;
  std::vector<int> ctx(context_lengths, context_lengths + rows);
  return dec->ex->stepAlgorithmicBytes(rows, ctx);
}

int tmc_decoder_profile_kernel(tmc_decoder *dec, int kind, int rows, int rounds, double *avg_us,
                               double *bytes_per_launch, int *launches_per_step) {
  if (!bind(dec)) return fail(TMC_ERR_INVALID, "null decoder");
  return done(dec->ex->profileKernel(kind, rows, rounds, avg_us, bytes_per_launch, launches_per_step));
}

int tmc_decoder_set_trace(tmc_decoder *dec, size_t capacity) {
  if (!bind(dec)) return fail(TMC_ERR_INVALID, "null decoder");
  return done(dec->ex->setTrace(capacity));
}

int tmc_decoder_read_trace(tmc_decoder *dec, uint64_t *out, size_t capacity, size_t *count) {
  if (!bind(dec) || count == nullptr) return fail(TMC_ERR_INVALID, "null argument");
  std::vector<tmc::TraceRecord> recs;
  auto e = dec->ex->readTrace(&recs);
  if (!e.empty()) return done(e);
  *count = recs.size();
  if (out != nullptr) std::memcpy(out, recs.data(), std::min(capacity, recs.size()) * sizeof(tmc::TraceRecord));
  return ok();
}

int tmc_nccl_unique_id(uint8_t *id, size_t nbytes) {
  if (id == nullptr || nbytes < NCCL_UNIQUE_ID_BYTES) return fail(TMC_ERR_INVALID, "id buffer too small");
  auto e = tensor::runtime::ncclUniqueIdBytes(id);
  return e.empty() ? ok() : fail(TMC_ERR_UNAVAILABLE, e);
}

int tmc_decoder_attach_nccl(tmc_decoder *dec, const uint8_t *id, size_t nbytes, int world, int rank) {
  if (!bind(dec) || id == nullptr || nbytes < NCCL_UNIQUE_ID_BYTES) return fail(TMC_ERR_INVALID, "bad argument");
  const auto &c = dec->ex->config();
  if (world != c.tpSize || rank != c.tpRank) return fail(TMC_ERR_INVALID, "world/rank must match the decoder's tensor-parallel config");
  std::string err;
  auto coll = tensor::runtime::NcclCollective::create(id, world, rank, &err);
  if (!coll) return fail(TMC_ERR_UNAVAILABLE, err);
  return done(dec->ex->setCollective(coll));
}

int tmc_serving_run(tmc_decoder *dec, int count, const int32_t *prompt_offsets, const int32_t *prompt_tokens,
                    const int32_t *decode_counts, const int32_t *arrival_ticks, int32_t *generated, double *ttft_us,
                    double *finish_us, float *prefill_logits, float *decode_logits, tmc_serving_metrics *metrics,
                    char *log, size_t log_size) {
  if (!bind(dec) || count <= 0 || !prompt_offsets || !prompt_tokens || !decode_counts || !arrival_ticks ||
      !generated)
    return fail(TMC_ERR_INVALID, "bad argument");
  std::vector<tensor::runtime::ServingRequestSpec> specs(count);
  for (int i = 0; i < count; ++i) {
    if (prompt_offsets[i + 1] < prompt_offsets[i] || decode_counts[i] < 0 || arrival_ticks[i] < 0)
      return fail(TMC_ERR_INVALID, "request " + std::to_string(i) + ": bad offsets, decode count or arrival");
    specs[i].id = "req" + std::to_string(i);
    specs[i].promptTokenIds.assign(prompt_tokens + prompt_offsets[i], prompt_tokens + prompt_offsets[i + 1]);
    specs[i].decodeTokenCount = static_cast<size_t>(decode_counts[i]);
    specs[i].arrivalStep = static_cast<size_t>(arrival_ticks[i]);
  }
  tensor::runtime::ServingConfig config;
  config.recordLogits = prefill_logits != nullptr || decode_logits != nullptr;
  std::ostringstream text;
  auto r = tensor::runtime::runContinuousBatch(*dec->ex, specs, config, text);
  if (log != nullptr && log_size > 0) {
    const std::string t = text.str();
    const size_t n = std::min(log_size - 1, t.size());
    std::memcpy(log, t.data(), n);
    log[n] = '\0';
  }
  if (!r.passed) return done(r.errorMessage.empty() ? "serving failed" : r.errorMessage);
  const size_t vL = static_cast<size_t>(dec->ex->localVocab());
  size_t g = 0, pl = 0, dl = 0;
  for (int i = 0; i < count; ++i) {
    const auto &o = r.requests[i];
    std::copy(o.generatedTokenIds.begin(), o.generatedTokenIds.end(), generated + g);
    g += o.generatedTokenIds.size();
    if (ttft_us) ttft_us[i] = o.timeToFirstTokenUs;
    if (finish_us) finish_us[i] = o.finishUs;
    if (prefill_logits) std::copy(o.prefillLogits.begin(), o.prefillLogits.end(), prefill_logits + pl * vL);
    pl += specs[i].promptTokenIds.size();
    if (decode_logits)
      for (const auto &step : o.decodeLogits) {
        std::copy(step.begin(), step.end(), decode_logits + dl * vL);
        ++dl;
      }
  }
  if (metrics) {
    const auto &m = r.metrics;
    *metrics = tmc_serving_metrics{m.totalTimeUs, m.tokensPerSecond, m.prefillGpuUs, m.decodeGpuUs,
                                   m.schedulerOverheadUs, m.kvManagementOverheadUs, m.preemptionOverheadUs,
                                   m.averageActiveBatchSize, m.maximumActiveBatchSize, m.preemptionCount,
                                   m.resumeCount, m.peakPages, m.pageAllocationCount, m.pageReleaseCount,
                                   m.decodeCommandSubmissions, m.decodedTokens, m.prefillTokens, m.ticks,
                                   m.modelStorageBytes, m.kvPoolStorageBytes, m.activationStorageBytes};
  }
  return ok();
}

static_assert(sizeof(cudaIpcMemHandle_t) == TMC_EXCHANGE_HANDLE_BYTES, "IPC handle size");

int tmc_decoder_exchange_handle(tmc_decoder *dec, uint8_t *handle, size_t nbytes) {
  if (!bind(dec) || handle == nullptr) return fail(TMC_ERR_INVALID, "bad argument");
  if (nbytes != TMC_EXCHANGE_HANDLE_BYTES) return fail(TMC_ERR_INVALID, "handle buffer must be TMC_EXCHANGE_HANDLE_BYTES");
  return done(dec->ex->exchangeHandle(handle, nbytes));
}

int tmc_decoder_attach_local_peers(tmc_decoder *dec, tmc_decoder *const *ranks, int world, int rank) {
  if (!bind(dec) || ranks == nullptr || world < 1) return fail(TMC_ERR_INVALID, "bad argument");
  std::vector<DecoderExecutor *> ex(world);
  for (int r = 0; r < world; ++r) {
    if (ranks[r] == nullptr || !ranks[r]->ex) return fail(TMC_ERR_INVALID, "null rank decoder");
    ex[r] = ranks[r]->ex.get();
  }
  return done(dec->ex->attachLocalPeers(ex, rank));
}

int tmc_decoder_set_wait_budgets(tmc_decoder *dec, uint64_t peer_wait_ns, uint64_t local_wait_ns) {
  if (!bind(dec)) return fail(TMC_ERR_INVALID, "null decoder");
  return done(dec->ex->setWaitBudgets(peer_wait_ns, local_wait_ns));
}

int tmc_decoder_attach_peers(tmc_decoder *dec, const uint8_t *handles, size_t nbytes_each, int world,
                             int rank) {
  if (!bind(dec) || handles == nullptr) return fail(TMC_ERR_INVALID, "bad argument");
  if (nbytes_each != TMC_EXCHANGE_HANDLE_BYTES) return fail(TMC_ERR_INVALID, "handles must be TMC_EXCHANGE_HANDLE_BYTES each");
  return done(dec->ex->attachPeers(handles, nbytes_each, world, rank));
}

}  // extern "C"
