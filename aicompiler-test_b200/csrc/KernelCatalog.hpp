// Built-in kernels by name for the prepared-execution surface.
//
// The reference compiles an emitted Metal source into "the current pipeline"
// (MetalRuntime::createComputePipeline, MetalRuntime.hpp:176-178) and then
// binds buffers and packed uint32 constants to it with prepareBuffers
// (MetalRuntime.hpp:199-206, MetalRuntime.mm:594-648). Here every kernel is a
// precompiled sm_100a function of this library, so a kernel is looked up by
// name instead of compiled; each catalog entry states its buffer interface
// (inputs, then outputs, in binding order), its constants, and binds them to
// the kernel's own launcher. Generated kernels (NVRTC) have their own registry
// (KernelAdmission.hpp).
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include "CudaRuntime.hpp"

namespace tensor::cuda {

struct KernelBinding {
  std::vector<BufferHandle> inputs;
  std::vector<BufferHandle> outputs;
  std::vector<std::uint32_t> constants;
  DispatchSize dispatch;
  BufferHandle workspace;  // allocated by bind() when the kernel needs one
  BufferHandle counters;   // zeroed tickets (attention)
  tmc::TmcDeviceStatus *status = nullptr;
  int numSms = 148;
};

struct KernelEntry {
  const char *name;
  int inputs;
  int outputs;
  int constants;
  // Interface in words: buffers in binding order with element types and
  // sizes, then the constants.
  const char *signature;
  // Checks element types, sizes and the dispatch against the constants;
  // allocates a workspace when the kernel needs one. "" on success.
  std::string (*bind)(CudaRuntime &runtime, KernelBinding &binding);
  cudaError_t (*launch)(const KernelBinding &binding, cudaStream_t stream);
  // Launch with programmatic dependent launch (null when the kernel does not
  // wait on its predecessor before reading its inputs), and the inputs it
  // reads before that wait (a bit per input index: its weights).
  cudaError_t (*launchOverlapped)(const KernelBinding &binding, cudaStream_t stream) = nullptr;
  unsigned earlyInputs = 0;
};

[[nodiscard]] const std::vector<KernelEntry> &kernelCatalog();
[[nodiscard]] const KernelEntry *findKernel(const std::string &name);

// prepareBuffers for a catalog kernel: the reference's binding-count,
// dispatch-limit and alias rules, then the kernel's own interface check.
[[nodiscard]] PreparationResult prepareKernel(CudaRuntime &runtime, const KernelEntry &kernel,
                                              std::vector<BufferHandle> inputs,
                                              std::vector<BufferHandle> outputs, DispatchSize dispatch,
                                              std::vector<std::uint32_t> constants);

}  // namespace tensor::cuda
