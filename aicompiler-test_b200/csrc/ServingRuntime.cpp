// Continuous-batching scheduler on the decoder executor (see ServingRuntime.hpp;
// the tick loop itself is runServingScheduler in ServingScheduler.hpp).
#include "ServingRuntime.hpp"

namespace tensor::runtime {

ServingExecutionResult runContinuousBatch(DecoderExecutor &decoder, const std::vector<ServingRequestSpec> &requests,
                                          const ServingConfig &config, std::ostream &log) {
  return runServingScheduler(decoder, requests, config, log);
}

}  // namespace tensor::runtime
