// Continuous batching over the paged KV cache: the B200 counterpart of the
// reference's ServingRuntime (src/runtime/ServingRuntime.hpp:15-75,
// ServingRuntime.cpp:513-930).
//
// One scheduler tick, as in the reference:
//   1. resume preempted requests whose KV snapshot fits the free pages;
//   2. admit arrived requests (arrival tick <= tick) whose prompt fits the free
//      pages and a free sequence slot: chunked prefill, first token;
//   3. while the next decode token of every active request does not fit,
//      preempt the active request holding the most pages (KV snapshot to the
//      host, pages and slot released);
//   4. one batched decode step over all active requests (the executor stages,
//      decodes and commits each row; more active rows than the executor's
//      max_rows are decoded in several steps), outputs appended, finished
//      requests released;
//   5. audit that no two active requests own the same physical page.
// Differences by design: one shared KV pool serves every layer (all layers of
// a sequence use the same page ids), sequence slots are reused across
// requests, and the decode steps are the executor's CUDA-graph steps with the
// GEMV (<= 8 rows) or tensor-core (more rows) projections.
#pragma once

#include <cstddef>
#include <cstdint>
#include <ostream>
#include <string>
#include <vector>

#include "DecoderExecutor.hpp"
#include "ServingScheduler.hpp"

namespace tensor::runtime {

// Serve `requests` on `decoder` (a multi-slot executor; its weights loaded).
// All tensor-parallel ranks must call this with the same requests: every
// scheduling decision depends only on ticks and page counts.
[[nodiscard]] ServingExecutionResult runContinuousBatch(DecoderExecutor &decoder,
                                                        const std::vector<ServingRequestSpec> &requests,
                                                        const ServingConfig &config, std::ostream &log);

}  // namespace tensor::runtime
