// CudaRuntime: the device runtime beneath the decode backend.
//
// Mirrors the C++ surface of tensor::metal::MetalRuntime
// (reference src/backend/metal/MetalRuntime.hpp:12-208) so that tuners,
// executors and the admission gate keep their call shapes:
//   * HardwareInfo / deviceName / isAvailable         (MetalRuntime.hpp:14-19,170-173)
//   * typed buffers created from logical host floats,
//     NaN-initialised floating outputs, read() back to
//     logical floats                                  (MetalRuntime.hpp:55-80,190-196)
//   * ExecutionResult with GPU time                   (MetalRuntime.hpp:91-99)
//   * PreparedExecution (one launch, retained buffers) and PreparedSequence
//     (a dependency-ordered chain), here a CUDA graph (MetalRuntime.hpp:101-147)
// Kernels are precompiled sm_100a functions; a PreparedExecution wraps a
// launch closure instead of a Metal pipeline state.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <functional>
#include <memory>
#include <optional>
#include <string>
#include <vector>

#include "common.cuh"

namespace tensor::cuda {

enum class ElementType { Float16, Float32, BFloat16, Int32 };

[[nodiscard]] std::size_t elementBytes(ElementType type);
[[nodiscard]] const char *elementName(ElementType type);

struct HardwareInfo {
  std::size_t maxThreadsPerThreadgroup = 0;     // maxThreadsPerBlock
  std::size_t maxThreadgroupMemoryLength = 0;   // opt-in shared memory per block
  std::size_t maxBufferLength = 0;              // total global memory
  bool supportsBFloat16 = false;
  int multiprocessorCount = 0;
  std::size_t l2CacheBytes = 0;
  int computeMajor = 0;
  int computeMinor = 0;
  std::string name;
};

// Device storage owned by a shared handle. read() requires completed work.
class CudaBuffer {
 public:
  ~CudaBuffer();
  CudaBuffer(const CudaBuffer &) = delete;
  CudaBuffer &operator=(const CudaBuffer &) = delete;
  [[nodiscard]] std::size_t elementCount() const { return count_; }
  [[nodiscard]] ElementType elementType() const { return type_; }
  [[nodiscard]] std::size_t byteCount() const { return count_ * elementBytes(type_); }
  [[nodiscard]] void *data() const { return ptr_; }
  // Logical float values (fp16/bf16/int32 converted on the host).
  [[nodiscard]] std::vector<float> read() const;

 private:
  friend class CudaRuntime;
  CudaBuffer(void *ptr, std::size_t count, ElementType type, int device)
      : ptr_(ptr), count_(count), type_(type), device_(device) {}
  void *ptr_ = nullptr;
  std::size_t count_ = 0;
  ElementType type_ = ElementType::Float32;
  int device_ = 0;
};

using BufferHandle = std::shared_ptr<CudaBuffer>;
struct BufferResult {
  BufferHandle buffer;
  std::string errorMessage;
};

struct DispatchSize {
  std::size_t threadgroupCount = 0;
  std::size_t threadsPerThreadgroup = 0;
};

struct ExecutionResult {
  bool executionPassed = false;
  std::vector<float> output;
  std::optional<double> gpuExecutionTimeUs;
  double cpuSubmitToCompletionTimeUs = 0.0;
  std::string errorMessage;
};

class CudaRuntime;

// A launch closure with its retained buffers (reference PreparedExecution,
// MetalRuntime.hpp:101-121). run() resets floating outputs to NaN sentinels
// first (MetalRuntime.mm:201-214); execute() only launches.
class PreparedExecution {
 public:
  using Launch = std::function<cudaError_t(cudaStream_t)>;
  PreparedExecution(CudaRuntime *runtime, Launch launch, std::vector<BufferHandle> inputs,
                    std::vector<BufferHandle> outputs, std::string name);
  [[nodiscard]] ExecutionResult run() const;
  [[nodiscard]] ExecutionResult execute() const;
  [[nodiscard]] std::vector<std::vector<float>> readOutputs() const;
  [[nodiscard]] const std::string &name() const { return name_; }
  [[nodiscard]] cudaError_t enqueue(cudaStream_t stream) const { return launch_(stream); }
  // Programmatic dependent launch inside a sequence: `overlapped` starts the
  // kernel while its predecessor drains; it waits (griddepcontrol.wait)
  // before reading anything an earlier launch wrote, except `earlyReads`
  // (weights), which it may read before that wait.
  void allowOverlap(Launch overlapped, std::vector<BufferHandle> earlyReads) {
    overlap_ = std::move(overlapped);
    earlyReads_ = std::move(earlyReads);
  }
  // True when this execution may overlap the end of its predecessor in a
  // sequence whose earlier steps are `earlier`: it has an overlapped launch
  // and no buffer it reads early is written by an earlier step.
  [[nodiscard]] bool canOverlapAfter(const std::vector<const PreparedExecution *> &earlier) const;
  [[nodiscard]] cudaError_t enqueueOverlapped(cudaStream_t stream) const { return overlap_(stream); }
  [[nodiscard]] const std::vector<BufferHandle> &outputs() const { return outputs_; }

 private:
  CudaRuntime *runtime_;
  Launch launch_;
  Launch overlap_;
  std::vector<BufferHandle> earlyReads_;
  std::vector<BufferHandle> inputs_;
  std::vector<BufferHandle> outputs_;
  std::string name_;
};

struct PreparationResult {
  std::unique_ptr<PreparedExecution> execution;
  std::string errorMessage;
};

// A dependency-ordered chain captured once as a CUDA graph and replayed
// (reference PreparedSequence: one Metal command buffer, MetalRuntime.mm:292-341).
// Steps that allow it (PreparedExecution::canOverlapAfter) are captured with
// programmatic dependent launch, so their weight loads overlap the previous
// kernel's tail.
class PreparedSequence {
 public:
  ~PreparedSequence();
  PreparedSequence(const PreparedSequence &) = delete;
  PreparedSequence &operator=(const PreparedSequence &) = delete;
  [[nodiscard]] ExecutionResult execute() const;
  [[nodiscard]] cudaGraphExec_t graph() const { return exec_; }

 private:
  friend class CudaRuntime;
  PreparedSequence(CudaRuntime *runtime, cudaGraph_t graph, cudaGraphExec_t exec)
      : runtime_(runtime), graph_(graph), exec_(exec) {}
  CudaRuntime *runtime_;
  cudaGraph_t graph_ = nullptr;
  cudaGraphExec_t exec_ = nullptr;
};

struct SequencePreparationResult {
  std::unique_ptr<PreparedSequence> execution;
  std::string errorMessage;
};

class CudaRuntime {
 public:
  explicit CudaRuntime(int device = 0);
  ~CudaRuntime();
  CudaRuntime(const CudaRuntime &) = delete;
  CudaRuntime &operator=(const CudaRuntime &) = delete;

  [[nodiscard]] bool isAvailable() const noexcept { return error_.empty(); }
  [[nodiscard]] std::string deviceName() const { return info_.name; }
  [[nodiscard]] std::string initializationError() const { return error_; }
  [[nodiscard]] HardwareInfo hardwareInfo() const { return info_; }
  [[nodiscard]] int device() const { return device_; }
  [[nodiscard]] cudaStream_t stream() const { return stream_; }

  [[nodiscard]] BufferResult createBuffer(std::size_t elementCount,
                                          const float *initialData = nullptr,
                                          ElementType type = ElementType::Float32) const;
  [[nodiscard]] std::string writeBuffer(const BufferHandle &buffer, const float *data,
                                        std::size_t elementCount,
                                        std::size_t elementOffset = 0) const;
  // Raw byte copy into device storage (large weight uploads, fp16 bit patterns).
  [[nodiscard]] std::string writeBufferBytes(const BufferHandle &buffer, const void *bytes,
                                             std::size_t byteCount,
                                             std::size_t byteOffset = 0) const;
  // Fill floating buffers with NaN sentinels (integers with zero).
  [[nodiscard]] std::string fillSentinel(const BufferHandle &buffer) const;

  [[nodiscard]] PreparationResult prepare(PreparedExecution::Launch launch,
                                          std::vector<BufferHandle> inputs,
                                          std::vector<BufferHandle> outputs,
                                          std::string name) ;
  [[nodiscard]] SequencePreparationResult
  prepareSequence(const std::vector<const PreparedExecution *> &steps);

  // Device-side status block shared by this runtime's kernels.
  [[nodiscard]] tmc::TmcDeviceStatus *deviceStatus() const { return status_; }
  // Read and clear the status block; returns "" when no kernel reported.
  [[nodiscard]] std::string consumeDeviceStatus() const;

  // Synchronise the runtime stream and translate any failure to a message.
  [[nodiscard]] std::string synchronize() const;

 private:
  int device_ = 0;
  std::string error_;
  HardwareInfo info_;
  cudaStream_t stream_ = nullptr;
  tmc::TmcDeviceStatus *status_ = nullptr;
};

// Human-readable name of a device status code.
[[nodiscard]] std::string describeDeviceStatus(const tmc::TmcDeviceStatus &status);

}  // namespace tensor::cuda
