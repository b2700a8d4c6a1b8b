// C ABI of the generated-kernel contracts, admission gate and registry
// (declarations and citations in include/tmc_cuda.h).
#include <cstring>
#include <sstream>
#include <string>
#include <vector>

#include <algorithm>

#include "DecodeGEMVTuner.hpp"
#include "KernelAdmission.hpp"
#include "RMSNormTuner.hpp"
#include "api_util.hpp"
#include "tmc_cuda.h"

using namespace tmc_api;

struct tmc_registry {
  tensor::runtime::KernelRegistry reg;
};

namespace {
void copy_text(const std::string &text, char *out, size_t size) {
  if (out == nullptr || size == 0) return;
  const size_t n = std::min(size - 1, text.size());
  std::memcpy(out, text.data(), n);
  out[n] = '\0';
}
}  // namespace

extern "C" {

int tmc_kernel_contract_json(const char *pattern, char *out, size_t size, size_t *needed) {
  if (pattern == nullptr) return fail(TMC_ERR_INVALID, "null pattern");
  try {
    const std::string json = tensor::runtime::serializeKernelContract(tensor::runtime::makeKernelContract(pattern));
    if (needed) *needed = json.size() + 1;
    copy_text(json, out, size);
    return ok();
  } catch (const std::exception &e) {
    return fail(TMC_ERR_UNSUPPORTED, e.what());
  }
}

int tmc_admit_generated_kernel(const char *pattern, const char *source, int block_size, const char *feedback_path,
                               const char *artifact_path, int *admitted, double *speedup, char *log,
                               size_t log_size) {
  if (pattern == nullptr || source == nullptr) return fail(TMC_ERR_INVALID, "null pattern or source");
  std::ostringstream text;
  const auto f = tensor::runtime::admitGeneratedKernel(pattern, source, block_size,
                                                       feedback_path ? feedback_path : "",
                                                       artifact_path ? artifact_path : "", text);
  copy_text(text.str(), log, log_size);
  if (admitted) *admitted = f.status == "admitted" ? 1 : 0;
  if (speedup) *speedup = f.speedup;
  if (f.status == "fatal") return fail(TMC_ERR_CUDA, f.stage + ": " + f.message);
  return ok();
}

int tmc_tune_decode_gemv(int rows, int k, int n, const float *input, const float *weight, int fp16_storage,
                         int prefill, tmc_gemv_selection *out, char *log, size_t log_size) {
  if (input == nullptr || weight == nullptr || out == nullptr || rows <= 0 || k <= 0 || n <= 0)
    return fail(TMC_ERR_INVALID, "bad argument");
  std::ostringstream text;
  const auto sel = tensor::planner::tuneDecodeGEMV(
      rows, k, n, std::vector<float>(input, input + (size_t)rows * k),
      std::vector<float>(weight, weight + (size_t)n * k), text, fp16_storage != 0, prefill != 0);
  copy_text(text.str(), log, log_size);
  *out = tmc_gemv_selection{sel.success ? 1 : 0, sel.useBaseline ? 1 : 0, sel.config.ks, sel.config.dynamic ? 1 : 0,
                            sel.config.tensorCore ? 1 : 0, sel.conservativeSpeedup};
  return sel.success ? ok() : fail(TMC_ERR_INVALID, sel.errorMessage);
}

int tmc_tune_rmsnorm(int rows, int width, float eps, int fp16, const float *input, const float *weight,
                     const int *candidate_threads, int candidates, tmc_rmsnorm_selection *out, float *output,
                     char *log, size_t log_size) {
  if (input == nullptr || weight == nullptr || out == nullptr || rows <= 0 || width <= 0 || candidates < 0 ||
      (candidates > 0 && candidate_threads == nullptr))
    return fail(TMC_ERR_INVALID, "bad argument");
  std::ostringstream text;
  const auto t = tensor::planner::tuneRMSNorm(
      rows, width, eps, fp16 != 0, std::vector<float>(input, input + (size_t)rows * width),
      std::vector<float>(weight, weight + width), std::vector<int>(candidate_threads, candidate_threads + candidates),
      text);
  copy_text(text.str(), log, log_size);
  double speedup = 1.0;
  for (const auto &c : t.candidates)
    if (!t.usedBaseline && c.threads == t.selectedThreads && c.speedup) speedup = *c.speedup;
  *out = tmc_rmsnorm_selection{t.success ? 1 : 0, t.usedBaseline ? 1 : 0, t.selectedThreads, speedup,
                               t.maxAbsoluteError};
  if (t.success && output != nullptr) std::copy(t.output.begin(), t.output.end(), output);
  return t.success ? ok() : fail(TMC_ERR_INVALID, t.errorMessage);
}

int tmc_registry_create(tmc_registry **out) {
  if (out == nullptr) return fail(TMC_ERR_INVALID, "null output");
  *out = new tmc_registry();
  return ok();
}

void tmc_registry_destroy(tmc_registry *reg) { delete reg; }

int tmc_registry_load(tmc_registry *reg, const char *directory, int *loaded, char *log, size_t log_size) {
  if (reg == nullptr || directory == nullptr) return fail(TMC_ERR_INVALID, "null argument");
  std::ostringstream text;
  reg->reg.load(directory, text);
  copy_text(text.str(), log, log_size);
  if (loaded) *loaded = static_cast<int>(reg->reg.patterns().size());
  return ok();
}

int tmc_registry_launch(tmc_registry *reg, const char *pattern, void *const *buffers, int count, unsigned work_items,
                        void *stream) {
  if (reg == nullptr || pattern == nullptr || (count > 0 && buffers == nullptr))
    return fail(TMC_ERR_INVALID, "null argument");
  const auto *k = reg->reg.find(pattern);
  if (k == nullptr) return fail(TMC_ERR_UNAVAILABLE, std::string("no admitted kernel for ") + pattern);
  const auto e = k->launch(std::vector<void *>(buffers, buffers + count), work_items, stream);
  return e.empty() ? ok() : fail(TMC_ERR_CUDA, e);
}

}  // extern "C"
