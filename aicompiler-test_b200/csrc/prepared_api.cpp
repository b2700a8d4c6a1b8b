// extern "C" prepared-execution surface: built-in kernels by name, prepared
// launches with retained buffers, and sequences replayed as CUDA graphs
// (declarations and reference citations in include/tmc_cuda.h).
#include <memory>
#include <string>
#include <vector>

#include "KernelCatalog.hpp"
#include "api_util.hpp"
#include "tmc_cuda.h"

using tensor::cuda::BufferHandle;
using tensor::cuda::DispatchSize;
using tensor::cuda::ExecutionResult;
using tensor::cuda::KernelEntry;
using tensor::cuda::PreparedExecution;
using tensor::cuda::PreparedSequence;

struct tmc_kernel {
  const KernelEntry *entry;
};
struct tmc_prepared {
  std::shared_ptr<PreparedExecution> exec;
  std::size_t firstOutputCount = 0;
};
struct tmc_sequence {
  std::vector<std::shared_ptr<PreparedExecution>> steps;  // keep the graph's buffers alive
  std::unique_ptr<PreparedSequence> seq;
  tensor::cuda::CudaRuntime *rt = nullptr;
};

using namespace tmc_api;

namespace {

const std::vector<tmc_kernel> &handles() {
  static const std::vector<tmc_kernel> all = [] {
    std::vector<tmc_kernel> v;
    for (const auto &k : tensor::cuda::kernelCatalog()) v.push_back({&k});
    return v;
  }();
  return all;
}

int report(const ExecutionResult &r, double *gpu_us, double *cpu_us) {
  if (gpu_us) *gpu_us = r.gpuExecutionTimeUs ? *r.gpuExecutionTimeUs : 0.0;
  if (cpu_us) *cpu_us = r.cpuSubmitToCompletionTimeUs;
  if (!r.executionPassed) {
    const bool device = r.errorMessage.rfind("device status", 0) == 0;
    return fail(device ? TMC_ERR_DEVICE_STATUS : TMC_ERR_CUDA, r.errorMessage);
  }
  return ok();
}

}  // namespace

extern "C" {

int tmc_kernel_count(void) { return static_cast<int>(handles().size()); }

int tmc_kernel_at(int index, const tmc_kernel **out) {
  if (out == nullptr) return fail(TMC_ERR_INVALID, "out is null");
  if (index < 0 || index >= tmc_kernel_count()) return fail(TMC_ERR_INVALID, "kernel index out of range");
  *out = &handles()[index];
  return ok();
}

int tmc_kernel_lookup(const char *name, const tmc_kernel **out) {
  if (name == nullptr || out == nullptr) return fail(TMC_ERR_INVALID, "null name or out");
  for (const auto &h : handles())
    if (std::string(name) == h.entry->name) {
      *out = &h;
      return ok();
    }
  *out = nullptr;
  return fail(TMC_ERR_UNSUPPORTED, std::string("no built-in kernel named '") + name + "'");
}

int tmc_kernel_describe(const tmc_kernel *kernel, const char **name, int *inputs, int *outputs, int *constants,
                        const char **signature) {
  if (kernel == nullptr) return fail(TMC_ERR_INVALID, "kernel is null");
  if (name) *name = kernel->entry->name;
  if (inputs) *inputs = kernel->entry->inputs;
  if (outputs) *outputs = kernel->entry->outputs;
  if (constants) *constants = kernel->entry->constants;
  if (signature) *signature = kernel->entry->signature;
  return ok();
}

int tmc_prepare(tmc_runtime *rt, const tmc_kernel *kernel, tmc_buffer *const *inputs, int n_inputs,
                tmc_buffer *const *outputs, int n_outputs, size_t groups, size_t threads, const uint32_t *constants,
                int n_constants, tmc_prepared **out) {
  if (rt == nullptr || kernel == nullptr || out == nullptr) return fail(TMC_ERR_INVALID, "null runtime, kernel or out");
  *out = nullptr;
  if (n_inputs < 0 || n_outputs < 0 || n_constants < 0 || (n_inputs > 0 && !inputs) ||
      (n_outputs > 0 && !outputs) || (n_constants > 0 && !constants))
    return fail(TMC_ERR_INVALID, "null binding array");
  std::vector<BufferHandle> in, outb;
  for (int i = 0; i < n_inputs; ++i) {
    if (inputs[i] == nullptr || inputs[i]->rt != rt->rt.get())
      return fail(TMC_ERR_INVALID, "Input is missing, on another device, or aliases an output.");
    in.push_back(inputs[i]->buf);
  }
  for (int i = 0; i < n_outputs; ++i) {
    if (outputs[i] == nullptr || outputs[i]->rt != rt->rt.get())
      return fail(TMC_ERR_INVALID, "Outputs must be distinct buffers on the current device.");
    outb.push_back(outputs[i]->buf);
  }
  const std::size_t firstCount = outb.empty() ? 0 : outb.front()->elementCount();
  std::vector<std::uint32_t> c(constants, constants + n_constants);
  auto r = tensor::cuda::prepareKernel(*rt->rt, *kernel->entry, std::move(in), std::move(outb),
                                       DispatchSize{groups, threads}, std::move(c));
  if (!r.execution) return fail(TMC_ERR_INVALID, r.errorMessage);
  *out = new tmc_prepared{std::shared_ptr<PreparedExecution>(std::move(r.execution)), firstCount};
  return ok();
}

void tmc_prepared_destroy(tmc_prepared *prepared) { delete prepared; }

int tmc_prepared_run(tmc_prepared *prepared, float *output, size_t count, double *gpu_us, double *cpu_us) {
  if (prepared == nullptr) return fail(TMC_ERR_INVALID, "prepared is null");
  if (output != nullptr && count != prepared->firstOutputCount)
    return fail(TMC_ERR_INVALID, "output count must equal the first output buffer's element count (" +
                                     std::to_string(prepared->firstOutputCount) + ")");
  const ExecutionResult r = prepared->exec->run();
  const int code = report(r, gpu_us, cpu_us);
  if (code == TMC_OK && output != nullptr) std::copy(r.output.begin(), r.output.end(), output);
  return code;
}

int tmc_prepared_execute(tmc_prepared *prepared, double *gpu_us, double *cpu_us) {
  if (prepared == nullptr) return fail(TMC_ERR_INVALID, "prepared is null");
  return report(prepared->exec->execute(), gpu_us, cpu_us);
}

int tmc_sequence_create(tmc_runtime *rt, tmc_prepared *const *steps, int n, tmc_sequence **out) {
  if (rt == nullptr || out == nullptr || (n > 0 && steps == nullptr)) return fail(TMC_ERR_INVALID, "null argument");
  *out = nullptr;
  auto s = std::make_unique<tmc_sequence>();
  std::vector<const PreparedExecution *> raw;
  for (int i = 0; i < n; ++i) {
    if (steps[i] == nullptr) return fail(TMC_ERR_INVALID, "null step");
    s->steps.push_back(steps[i]->exec);
    raw.push_back(steps[i]->exec.get());
  }
  auto r = rt->rt->prepareSequence(raw);
  if (!r.execution) return fail(TMC_ERR_INVALID, r.errorMessage);
  s->seq = std::move(r.execution);
  s->rt = rt->rt.get();
  *out = s.release();
  return ok();
}

void tmc_sequence_destroy(tmc_sequence *sequence) { delete sequence; }

int tmc_sequence_execute(tmc_sequence *sequence, double *gpu_us, double *cpu_us) {
  if (sequence == nullptr) return fail(TMC_ERR_INVALID, "sequence is null");
  return report(sequence->seq->execute(), gpu_us, cpu_us);
}

int tmc_sequence_launch(tmc_sequence *sequence, int replays) {
  if (sequence == nullptr || replays < 0) return fail(TMC_ERR_INVALID, "null sequence or negative replays");
  cudaSetDevice(sequence->rt->device());
  for (int i = 0; i < replays; ++i) {
    const cudaError_t e = cudaGraphLaunch(sequence->seq->graph(), sequence->rt->stream());
    if (e != cudaSuccess) return cuda_fail(e, "cudaGraphLaunch");
  }
  return ok();
}

}  // extern "C"
