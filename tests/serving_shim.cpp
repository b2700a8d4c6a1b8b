// Test-only host executor for the continuous-batching scheduler
// (aicompiler-test_b200/csrc/ServingScheduler.hpp), compiled with g++ by
// tests/test_serving_scheduler.py. It keeps the real page pool and per-slot
// cache states (KVCacheState.cpp) but replaces the model with a hash: a
// sequence's "KV contents" are its token history, and the next token is
// next_token(history). So a request's tokens depend only on its own history,
// whatever the batching, preemption or resume order, and the test can compare
// them with a sequential chain computed in Python.
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <memory>
#include <sstream>
#include <string>
#include <vector>

#include "KVCacheState.hpp"
#include "ServingScheduler.hpp"

using namespace tensor::runtime;

namespace {
std::string g_error, g_log;

// FNV-1a over the history's tokens, folded into the vocabulary.
std::int32_t next_token(const std::vector<std::int32_t> &h, int vocab) {
  std::uint64_t x = 1469598103934665603ull;
  for (auto t : h) {
    x ^= static_cast<std::uint32_t>(t);
    x *= 1099511628211ull;
  }
  return static_cast<std::int32_t>(x % static_cast<std::uint64_t>(vocab));
}

struct FakeExecutor {
  struct Config {
    int maxSlots, capacity, maxRows;
  };
  struct KVPageSnapshot {
    std::size_t length = 0;
    std::vector<std::int32_t> history;
  };
  struct Timing {
    double gpuUs = 0.0;
  };

  Config cfg;
  int vocab;
  std::shared_ptr<KVPagePool> pool;
  std::vector<std::unique_ptr<KVCacheState>> states;
  std::vector<std::vector<std::int32_t>> history;
  std::size_t maxRowsSeen = 0, decodeCalls = 0, snapshots = 0, restores = 0;

  FakeExecutor(Config c, int v, std::size_t pageSize, std::size_t pages)
      : cfg(c), vocab(v), pool(std::make_shared<KVPagePool>(pageSize, pages)), history(c.maxSlots) {
    for (int s = 0; s < c.maxSlots; ++s)
      states.push_back(std::make_unique<KVCacheState>(pool, (std::size_t)c.capacity, s, nullptr));
  }

  const Config &config() const { return cfg; }
  KVPagePool &pagePool() { return *pool; }
  int localVocab() const { return vocab; }
  std::size_t modelStorageBytes() const { return 0; }
  std::size_t kvStorageBytes() const { return 0; }
  std::size_t activationStorageBytes() const { return 0; }
  std::size_t currentLength(int slot) const { return states.at(slot)->currentLength(); }
  std::vector<std::int32_t> blockTable(int slot) const { return states.at(slot)->pageTable(); }

  std::string releaseSlot(int slot) {
    history.at(slot).clear();
    return states.at(slot)->reset();
  }

  std::string prefill(int slot, const std::int32_t *tokens, int count, float *logits, std::int32_t *next,
                      Timing *) {
    auto &st = *states.at(slot);
    if (st.currentLength() != 0) return "prefill into a busy slot";
    auto e = st.stageLength((std::size_t)count);
    if (!e.empty()) return e;
    history[slot].assign(tokens, tokens + count);
    st.commitLength((std::size_t)count);
    *next = next_token(history[slot], vocab);
    if (logits) std::fill(logits, logits + (std::size_t)count * vocab, 0.0f);
    return {};
  }

  std::string decode(const std::int32_t *slots, const std::int32_t *tokens, int rows, float *logits,
                     std::int32_t *next, Timing *) {
    ++decodeCalls;
    maxRowsSeen = std::max(maxRowsSeen, (std::size_t)rows);
    if (rows > cfg.maxRows) return "more rows than maxRows";
    for (int j = 0; j < rows; ++j) {
      auto &st = *states.at(slots[j]);
      const auto len = st.currentLength();
      if (len == 0) return "decode of an empty slot";
      // The scheduler must have made room: a failed stage here is its bug.
      auto e = st.stageLength(len + 1);
      if (!e.empty()) return "decode could not stage a row: " + e;
      history[slots[j]].push_back(tokens[j]);
      st.commitLength(len + 1);
      next[j] = next_token(history[slots[j]], vocab);
    }
    if (logits) std::fill(logits, logits + (std::size_t)rows * vocab, 0.0f);
    return {};
  }

  std::string snapshotPages(int slot, KVPageSnapshot *out) {
    ++snapshots;
    out->length = states.at(slot)->currentLength();
    out->history = history.at(slot);
    return {};
  }

  std::string restorePages(int slot, const KVPageSnapshot &snap) {
    ++restores;
    auto &st = *states.at(slot);
    if (st.currentLength() != 0) return "restore into a busy slot";
    auto e = st.stageLength(snap.length);
    if (!e.empty()) return e;
    history[slot] = snap.history;
    st.commitLength(snap.length);
    return {};
  }
};
}  // namespace

extern "C" {

const char *serving_last_error() { return g_error.c_str(); }
const char *serving_log() { return g_log.c_str(); }

// Requests: n prompts concatenated (prompt_lens each), decode counts and
// arrival ticks. tokens_out: per request 1 + decode_count tokens, concatenated.
// stats_out[12]: preemptions, resumes, peak pages, page allocations, page
// releases, decode submissions, decoded tokens, prefill tokens, ticks, maximum
// active batch, largest rows per decode call, pages in use at the end.
// Returns 0, or -1 with serving_last_error() set.
int serving_run(int n, const int *prompt_lens, const std::int32_t *prompts, const int *decode_counts,
                const int *arrivals, int max_slots, int capacity, int max_rows, int page_size, int pool_pages,
                int vocab, std::int32_t *tokens_out, std::size_t *stats_out) {
  try {
    FakeExecutor ex({max_slots, capacity, max_rows}, vocab, (std::size_t)page_size, (std::size_t)pool_pages);
    std::vector<ServingRequestSpec> specs(n);
    std::size_t off = 0;
    for (int i = 0; i < n; ++i) {
      specs[i].id = "r" + std::to_string(i);
      specs[i].promptTokenIds.assign(prompts + off, prompts + off + prompt_lens[i]);
      off += prompt_lens[i];
      specs[i].decodeTokenCount = (std::size_t)decode_counts[i];
      specs[i].arrivalStep = (std::size_t)arrivals[i];
    }
    ServingConfig config;
    config.maxTicks = 100000;
    std::ostringstream log;
    const auto r = runServingScheduler(ex, specs, config, log);
    g_log = log.str();
    if (!r.passed) {
      g_error = r.errorMessage;
      return -1;
    }
    std::size_t o = 0;
    for (const auto &req : r.requests)
      for (auto t : req.generatedTokenIds) tokens_out[o++] = t;
    const auto &m = r.metrics;
    const std::size_t stats[12] = {m.preemptionCount, m.resumeCount,    m.peakPages,
                                   m.pageAllocationCount, m.pageReleaseCount, m.decodeCommandSubmissions,
                                   m.decodedTokens,   m.prefillTokens,  m.ticks,
                                   m.maximumActiveBatchSize, ex.maxRowsSeen, ex.pool->usedPages()};
    std::memcpy(stats_out, stats, sizeof stats);
    return 0;
  } catch (const std::exception &e) {
    g_error = e.what();
    return -1;
  }
}
}
