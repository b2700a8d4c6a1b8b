// The continuous-batching scheduler, written against any executor that offers
// the decoder's slot interface (DecoderExecutor in the product; a host-only
// fake in the CPU tests). The B200 counterpart of the reference's
// runContinuousBatch (src/runtime/ServingRuntime.cpp:513-930).
//
// One scheduler tick, as in the reference:
//   1. resume preempted requests whose KV snapshot fits the free pages;
//   2. admit arrived requests (arrival tick <= tick) whose prompt fits the free
//      pages and a free sequence slot: chunked prefill, first token;
//   3. while the next decode token of every active request does not fit,
//      preempt the active request holding the most pages (KV snapshot, pages
//      and slot released);
//   4. one batched decode step over all active requests (more active rows than
//      the executor's maxRows are decoded in several steps), outputs appended,
//      finished requests released;
//   5. audit that no two active requests own the same physical page.
//
// Executor requirements: config() with maxSlots, capacity, maxRows;
// pagePool() (a KVPagePool); currentLength, releaseSlot, blockTable, prefill,
// decode, snapshotPages, restorePages with DecoderExecutor's signatures;
// localVocab and the three storage-byte queries; member types KVPageSnapshot
// (with `length`) and Timing (with `gpuUs`).
#pragma once

#include <algorithm>
#include <chrono>
#include <cstddef>
#include <cstdint>
#include <optional>
#include <ostream>
#include <set>
#include <stdexcept>
#include <string>
#include <vector>

namespace tensor::runtime {

struct ServingRequestSpec {
  std::string id;
  std::vector<std::int32_t> promptTokenIds;
  std::size_t decodeTokenCount = 0;
  std::size_t arrivalStep = 0;  // scheduler tick at which the request arrives
};

struct ServingConfig {
  bool recordLogits = false;    // keep prefill and decode logits per request
  std::size_t maxTicks = 1000000;  // progress limit (the reference uses 10000)
};

struct ServingRequestOutput {
  std::string id;
  std::vector<float> prefillLogits;                // [prompt, localVocab] when recorded
  std::vector<std::vector<float>> decodeLogits;    // per decode step, [localVocab]
  std::vector<std::int32_t> generatedTokenIds;     // 1 (prefill) + decodeTokenCount
  double timeToFirstTokenUs = 0.0;                 // arrival -> first token
  double finishUs = 0.0;                           // arrival -> last token
};

struct ServingMetrics {
  double totalTimeUs = 0.0;
  double tokensPerSecond = 0.0;      // decoded tokens / total time
  double prefillGpuUs = 0.0;         // sums over all prefill / decode steps
  double decodeGpuUs = 0.0;
  double schedulerOverheadUs = 0.0;
  double kvManagementOverheadUs = 0.0;
  double preemptionOverheadUs = 0.0;
  double averageActiveBatchSize = 0.0;
  std::size_t maximumActiveBatchSize = 0;
  std::size_t preemptionCount = 0;
  std::size_t resumeCount = 0;
  std::size_t peakPages = 0;
  std::size_t pageAllocationCount = 0;
  std::size_t pageReleaseCount = 0;
  std::size_t decodeCommandSubmissions = 0;
  std::size_t decodedTokens = 0;
  std::size_t prefillTokens = 0;
  std::size_t ticks = 0;
  std::size_t modelStorageBytes = 0;
  std::size_t kvPoolStorageBytes = 0;
  std::size_t activationStorageBytes = 0;
};

struct ServingExecutionResult {
  bool passed = false;
  std::vector<ServingRequestOutput> requests;
  ServingMetrics metrics;
  std::string errorMessage;
};

namespace serving_detail {

using Clock = std::chrono::steady_clock;

inline double elapsedUs(Clock::time_point a, Clock::time_point b) {
  return std::chrono::duration<double, std::micro>(b - a).count();
}

inline std::size_t pagesFor(std::size_t length, std::size_t pageSize) { return (length + pageSize - 1) / pageSize; }

enum class RequestState { Waiting, Decode, Preempted, Finished };

template <class Snapshot>
struct Request {
  ServingRequestSpec spec;
  RequestState state = RequestState::Waiting;
  int slot = -1;
  std::int32_t nextToken = 0;
  std::size_t decoded = 0;
  std::optional<Snapshot> snapshot;  // a preempted request's KV state
  std::optional<Clock::time_point> arrival;
  ServingRequestOutput output;
};

}  // namespace serving_detail

// Serve `specs` on `dec` (a multi-slot executor; its weights loaded). Every
// scheduling decision depends only on ticks and page counts, so tensor-parallel
// ranks that call this with the same requests take the same steps.
template <class Executor>
ServingExecutionResult runServingScheduler(Executor &dec, const std::vector<ServingRequestSpec> &specs,
                                           const ServingConfig &config, std::ostream &log) {
  using namespace serving_detail;
  using KVSnapshot = typename Executor::KVPageSnapshot;
  using Timing = typename Executor::Timing;
  using Request = serving_detail::Request<KVSnapshot>;

  ServingExecutionResult result;
  auto &m = result.metrics;
  try {
    const auto &cfg = dec.config();
    auto &pool = dec.pagePool();
    const std::size_t pageSize = pool.pageSize();
    if (specs.empty()) throw std::invalid_argument("Serving configuration and requests must be nonempty.");
    std::size_t largest = 0;
    for (const auto &s : specs) {
      if (s.id.empty() || s.promptTokenIds.empty() || s.promptTokenIds.size() >= (std::size_t)cfg.capacity ||
          s.decodeTokenCount > (std::size_t)cfg.capacity - s.promptTokenIds.size())
        throw std::invalid_argument("Serving request dimensions are invalid.");
      largest = std::max(largest, pagesFor(s.promptTokenIds.size() + s.decodeTokenCount, pageSize));
    }
    if (pool.capacityPages() < largest) throw std::invalid_argument("Shared KV pool cannot hold the largest configured request.");
    for (int s = 0; s < cfg.maxSlots; ++s)
      if (dec.currentLength(s) != 0) throw std::invalid_argument("Serving needs every sequence slot empty.");

    const std::size_t vL = static_cast<std::size_t>(dec.localVocab());
    std::vector<Request> reqs(specs.size());
    for (std::size_t i = 0; i < specs.size(); ++i) {
      reqs[i].spec = specs[i];
      reqs[i].output.id = specs[i].id;
    }
    std::vector<int> freeSlots;
    for (int s = cfg.maxSlots - 1; s >= 0; --s) freeSlots.push_back(s);
    m.modelStorageBytes = dec.modelStorageBytes();
    m.kvPoolStorageBytes = dec.kvStorageBytes();
    m.activationStorageBytes = dec.activationStorageBytes();
    const std::size_t alloc0 = pool.allocationCount(), release0 = pool.releaseCount();

    std::size_t completed = 0, tick = 0, batchSamples = 0, batchSum = 0;
    const auto runStart = Clock::now();
    auto releaseRequest = [&](Request &r) {
      const auto k0 = Clock::now();
      const auto e = dec.releaseSlot(r.slot);
      if (!e.empty()) throw std::runtime_error("Request " + r.spec.id + " release failed: " + e);
      freeSlots.push_back(r.slot);
      r.slot = -1;
      m.kvManagementOverheadUs += elapsedUs(k0, Clock::now());
    };

    while (completed < reqs.size()) {
      if (tick > config.maxTicks) throw std::runtime_error("Serving scheduler exceeded its progress limit.");
      bool progress = false;

      // 1. resume preempted requests that fit
      for (auto &r : reqs) {
        const auto s0 = Clock::now();
        const bool fits = r.state == RequestState::Preempted && r.snapshot && !freeSlots.empty() &&
                          pool.availablePages() >= pagesFor(r.snapshot->length, pageSize);
        m.schedulerOverheadUs += elapsedUs(s0, Clock::now());
        if (!fits) continue;
        const auto p0 = Clock::now();
        r.slot = freeSlots.back();
        freeSlots.pop_back();
        const auto e = dec.restorePages(r.slot, *r.snapshot);
        m.preemptionOverheadUs += elapsedUs(p0, Clock::now());
        if (!e.empty()) throw std::runtime_error("Request " + r.spec.id + " resume failed: " + e);
        r.snapshot.reset();
        r.state = RequestState::Decode;
        ++m.resumeCount;
        log << "Serving request " << r.spec.id << ": resumed at length=" << dec.currentLength(r.slot) << '\n';
        progress = true;
      }

      // 2. admit arrived requests whose prompt fits
      for (auto &r : reqs) {
        const auto s0 = Clock::now();
        const bool eligible = r.state == RequestState::Waiting && r.spec.arrivalStep <= tick;
        if (eligible && !r.arrival) r.arrival = Clock::now();
        const bool fits = eligible && !freeSlots.empty() &&
                          pool.availablePages() >= pagesFor(r.spec.promptTokenIds.size(), pageSize);
        m.schedulerOverheadUs += elapsedUs(s0, Clock::now());
        if (!fits) continue;
        r.slot = freeSlots.back();
        freeSlots.pop_back();
        const int n = static_cast<int>(r.spec.promptTokenIds.size());
        if (config.recordLogits) r.output.prefillLogits.assign((std::size_t)n * vL, 0.0f);
        Timing timing;
        std::int32_t next = 0;
        const auto e = dec.prefill(r.slot, r.spec.promptTokenIds.data(), n,
                                   config.recordLogits ? r.output.prefillLogits.data() : nullptr, &next, &timing);
        if (!e.empty()) throw std::runtime_error("Request " + r.spec.id + " prefill failed: " + e);
        m.prefillGpuUs += timing.gpuUs;
        m.prefillTokens += (std::size_t)n;
        r.nextToken = next;
        r.output.generatedTokenIds.push_back(next);
        r.output.timeToFirstTokenUs = elapsedUs(*r.arrival, Clock::now());
        r.state = RequestState::Decode;
        log << "Serving request " << r.spec.id << ": prefill complete, pages=" << dec.blockTable(r.slot).size()
            << ", ttft(us)=" << r.output.timeToFirstTokenUs << '\n';
        progress = true;
        if (r.spec.decodeTokenCount == 0) {
          releaseRequest(r);
          r.output.finishUs = r.output.timeToFirstTokenUs;
          r.state = RequestState::Finished;
          ++completed;
        }
      }

      // 3. preempt until the next token of every active request fits
      auto activeSet = [&] {
        std::vector<std::size_t> a;
        for (std::size_t i = 0; i < reqs.size(); ++i)
          if (reqs[i].state == RequestState::Decode) a.push_back(i);
        return a;
      };
      auto required = [&](const std::vector<std::size_t> &a) {
        std::size_t need = 0;
        for (auto i : a) {
          const auto len = dec.currentLength(reqs[i].slot);
          need += pagesFor(len + 1, pageSize) - pagesFor(len, pageSize);
        }
        return need;
      };
      const auto s0 = Clock::now();
      auto active = activeSet();
      auto need = required(active);
      m.schedulerOverheadUs += elapsedUs(s0, Clock::now());
      while (!active.empty() && pool.availablePages() < need) {
        std::size_t victim = active.front(), victimPages = 0;
        for (auto i : active) {
          const auto pages = dec.blockTable(reqs[i].slot).size();
          if (pages > victimPages) {
            victim = i;
            victimPages = pages;
          }
        }
        auto &r = reqs[victim];
        const auto p0 = Clock::now();
        KVSnapshot snap;
        const auto e = dec.snapshotPages(r.slot, &snap);
        if (!e.empty()) throw std::runtime_error("Request " + r.spec.id + " snapshot failed: " + e);
        r.snapshot = std::move(snap);
        m.preemptionOverheadUs += elapsedUs(p0, Clock::now());
        releaseRequest(r);
        r.state = RequestState::Preempted;
        ++m.preemptionCount;
        log << "Serving request " << r.spec.id << ": preempted for page pressure\n";
        progress = true;
        active = activeSet();
        need = required(active);
      }

      // 4. one batched decode step over the active requests
      if (!active.empty()) {
        const std::size_t R = static_cast<std::size_t>(cfg.maxRows);
        for (std::size_t b0 = 0; b0 < active.size(); b0 += R) {
          const std::size_t rows = std::min(R, active.size() - b0);
          std::vector<std::int32_t> slots(rows), tokens(rows), next(rows);
          for (std::size_t j = 0; j < rows; ++j) {
            slots[j] = reqs[active[b0 + j]].slot;
            tokens[j] = reqs[active[b0 + j]].nextToken;
          }
          std::vector<float> logits(config.recordLogits ? rows * vL : 0);
          Timing timing;
          const auto e = dec.decode(slots.data(), tokens.data(), static_cast<int>(rows),
                                    config.recordLogits ? logits.data() : nullptr, next.data(), &timing);
          if (!e.empty()) throw std::runtime_error("Batched decode failed: " + e);
          m.decodeGpuUs += timing.gpuUs;
          ++m.decodeCommandSubmissions;
          for (std::size_t j = 0; j < rows; ++j) {
            auto &r = reqs[active[b0 + j]];
            if (config.recordLogits)
              r.output.decodeLogits.emplace_back(logits.begin() + (std::ptrdiff_t)(j * vL),
                                                 logits.begin() + (std::ptrdiff_t)((j + 1) * vL));
            r.nextToken = next[j];
            r.output.generatedTokenIds.push_back(next[j]);
            ++r.decoded;
            ++m.decodedTokens;
            if (r.decoded == r.spec.decodeTokenCount) {
              releaseRequest(r);
              r.output.finishUs = elapsedUs(*r.arrival, Clock::now());
              r.state = RequestState::Finished;
              ++completed;
              log << "Serving request " << r.spec.id << ": finished\n";
            }
          }
        }
        progress = true;
        ++batchSamples;
        batchSum += active.size();
        m.maximumActiveBatchSize = std::max(m.maximumActiveBatchSize, active.size());
      }

      // 5. no physical page may belong to two live sequences
      std::set<std::int32_t> owners;
      for (const auto &r : reqs) {
        if (r.state != RequestState::Decode) continue;
        for (auto page : dec.blockTable(r.slot))
          if (!owners.insert(page).second)
            throw std::runtime_error("Two active requests own the same physical KV page.");
      }
      if (!progress) {
        const bool future = std::any_of(reqs.begin(), reqs.end(), [&](const Request &r) {
          return r.state == RequestState::Waiting && r.spec.arrivalStep > tick;
        });
        if (!future) throw std::runtime_error("Serving scheduler made no progress.");
      }
      ++tick;
    }

    m.totalTimeUs = elapsedUs(runStart, Clock::now());
    m.ticks = tick;
    if (m.totalTimeUs > 0.0) m.tokensPerSecond = (double)m.decodedTokens * 1e6 / m.totalTimeUs;
    if (batchSamples) m.averageActiveBatchSize = (double)batchSum / (double)batchSamples;
    m.peakPages = pool.peakUsedPages();
    m.pageAllocationCount = pool.allocationCount() - alloc0;
    m.pageReleaseCount = pool.releaseCount() - release0;
    if (pool.usedPages() != 0) throw std::runtime_error("Serving completed with unreleased KV pages.");
    for (auto &r : reqs) result.requests.push_back(std::move(r.output));
    result.passed = true;
  } catch (const std::exception &error) {
    result.errorMessage = error.what();
  }
  return result;
}

}  // namespace tensor::runtime
