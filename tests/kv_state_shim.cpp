// Test-only C wrapper around the host KV page pool and per-sequence cache state
// (aicompiler-test_b200/csrc/KVCacheState.{hpp,cpp}), compiled with g++ by
// tests/test_kv_state.py so the host logic is checked without a GPU. A block
// table sink records every row it receives and can be told to fail.
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "KVCacheState.hpp"

using tensor::runtime::KVCacheState;
using tensor::runtime::KVPagePool;

namespace {
std::string g_error;

int fail(const std::string &e) {
  g_error = e;
  return -1;
}

struct Sink {
  std::vector<std::vector<std::int32_t>> rows;
  int failures = 0;  // the next `failures` deliveries fail
};

struct State {
  std::shared_ptr<Sink> sink;
  std::unique_ptr<KVCacheState> state;
};
}  // namespace

extern "C" {

const char *kv_last_error() { return g_error.c_str(); }

void *kv_pool_new(std::size_t page_size, std::size_t pages) {
  try {
    return new std::shared_ptr<KVPagePool>(std::make_shared<KVPagePool>(page_size, pages));
  } catch (const std::exception &e) {
    g_error = e.what();
    return nullptr;
  }
}
void kv_pool_free(void *p) { delete static_cast<std::shared_ptr<KVPagePool> *>(p); }

// stats: capacity, used, available, peak, allocations, releases
void kv_pool_stats(void *p, std::size_t *out) {
  const auto &pool = **static_cast<std::shared_ptr<KVPagePool> *>(p);
  out[0] = pool.capacityPages();
  out[1] = pool.usedPages();
  out[2] = pool.availablePages();
  out[3] = pool.peakUsedPages();
  out[4] = pool.allocationCount();
  out[5] = pool.releaseCount();
}
int kv_pool_allocate(void *p) { return (*static_cast<std::shared_ptr<KVPagePool> *>(p))->allocatePage(); }
int kv_pool_release(void *p, int page) {
  try {
    (*static_cast<std::shared_ptr<KVPagePool> *>(p))->releasePage(page);
    return 0;
  } catch (const std::exception &e) {
    return fail(e.what());
  }
}
int kv_pool_is_allocated(void *p, int page) {
  return (*static_cast<std::shared_ptr<KVPagePool> *>(p))->isAllocated(page) ? 1 : 0;
}
void kv_pool_fail_next(void *p, std::size_t n) { (*static_cast<std::shared_ptr<KVPagePool> *>(p))->failNextAllocations(n); }

void *kv_state_new(void *p, std::size_t capacity, int slot, int with_sink) {
  try {
    auto s = std::make_unique<State>();
    tensor::runtime::BlockTableSink sink;
    if (with_sink) {
      s->sink = std::make_shared<Sink>();
      auto rec = s->sink;
      sink = [rec](int, const std::vector<std::int32_t> &row) -> std::string {
        rec->rows.push_back(row);
        if (rec->failures > 0) {
          --rec->failures;
          return "block table upload failed";
        }
        return {};
      };
    }
    s->state = std::make_unique<KVCacheState>(*static_cast<std::shared_ptr<KVPagePool> *>(p), capacity, slot,
                                              std::move(sink));
    return s.release();
  } catch (const std::exception &e) {
    g_error = e.what();
    return nullptr;
  }
}
void kv_state_free(void *s) { delete static_cast<State *>(s); }

static int status(const std::string &e) { return e.empty() ? 0 : fail(e); }
int kv_state_stage(void *s, std::size_t length) { return status(static_cast<State *>(s)->state->stageLength(length)); }
int kv_state_rollback(void *s, std::size_t length) {
  return status(static_cast<State *>(s)->state->rollbackLength(length));
}
int kv_state_reset(void *s) { return status(static_cast<State *>(s)->state->reset()); }
int kv_state_commit(void *s, std::size_t length) {
  try {
    static_cast<State *>(s)->state->commitLength(length);
    return 0;
  } catch (const std::exception &e) {
    return fail(e.what());
  }
}
std::size_t kv_state_length(void *s) { return static_cast<State *>(s)->state->currentLength(); }
std::size_t kv_state_max_pages(void *s) { return static_cast<State *>(s)->state->maxPages(); }

// The allocated page ids (pageTable) into out; returns their count.
std::size_t kv_state_pages(void *s, int *out, std::size_t cap) {
  const auto t = static_cast<State *>(s)->state->pageTable();
  std::memcpy(out, t.data(), std::min(cap, t.size()) * sizeof(int));
  return t.size();
}
// The whole block-table row (-1 for unallocated logical pages).
std::size_t kv_state_row(void *s, int *out, std::size_t cap) {
  const auto &r = static_cast<State *>(s)->state->blockTableRow();
  std::memcpy(out, r.data(), std::min(cap, r.size()) * sizeof(int));
  return r.size();
}

void kv_sink_fail_next(void *s, int n) { static_cast<State *>(s)->sink->failures = n; }
std::size_t kv_sink_count(void *s) { return static_cast<State *>(s)->sink->rows.size(); }
// Row `i` the sink received; returns its length.
std::size_t kv_sink_row(void *s, std::size_t i, int *out, std::size_t cap) {
  const auto &r = static_cast<State *>(s)->sink->rows.at(i);
  std::memcpy(out, r.data(), std::min(cap, r.size()) * sizeof(int));
  return r.size();
}
}
