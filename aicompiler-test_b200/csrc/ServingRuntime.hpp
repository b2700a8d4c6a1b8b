// Continuous batching over the paged KV cache on the B200 decoder executor: the
// counterpart of the reference's ServingRuntime (src/runtime/ServingRuntime.hpp:15-75,
// ServingRuntime.cpp:513-930). The tick loop (resume, admit, preempt by page
// pressure, one batched decode, page-ownership audit) is runServingScheduler in
// ServingScheduler.hpp; this file runs it on DecoderExecutor.
// Differences by design: one shared KV pool serves every layer (all layers of
// a sequence use the same page ids), sequence slots are reused across
// requests, a preempted sequence is kept as raw fp16 page images in host
// memory, and the decode steps are the executor's CUDA-graph steps with the
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
