// CudaRuntime implementation (see CudaRuntime.hpp).
#include "CudaRuntime.hpp"

#include <algorithm>
#include <chrono>
#include <cstring>
#include <cmath>
#include <limits>
#include <sstream>

#include "half_convert.hpp"

namespace tensor::cuda {

std::size_t elementBytes(ElementType type) {
  switch (type) {
    case ElementType::Float16:
    case ElementType::BFloat16:
      return 2;
    case ElementType::Float32:
    case ElementType::Int32:
      return 4;
  }
  return 4;
}

const char *elementName(ElementType type) {
  switch (type) {
    case ElementType::Float16: return "fp16";
    case ElementType::Float32: return "fp32";
    case ElementType::BFloat16: return "bf16";
    case ElementType::Int32: return "int32";
  }
  return "?";
}

namespace {

std::string cudaMessage(const char *what, cudaError_t e) {
  std::ostringstream s;
  s << what << ": " << cudaGetErrorName(e) << " (" << cudaGetErrorString(e) << ")";
  return s.str();
}

// Logical floats -> storage bytes (RNE for fp16/bf16; truncation for int32 as
// the reference's storeValue does, GraphReference.cpp:82-87).
void encode(const float *src, std::size_t n, ElementType type, void *dst) {
  switch (type) {
    case ElementType::Float32:
      std::memcpy(dst, src, n * 4);
      break;
    case ElementType::Float16: {
      auto *d = static_cast<std::uint16_t *>(dst);
      for (std::size_t i = 0; i < n; ++i) d[i] = floatToHalfBits(src[i]);
      break;
    }
    case ElementType::BFloat16: {
      auto *d = static_cast<std::uint16_t *>(dst);
      for (std::size_t i = 0; i < n; ++i) d[i] = floatToBFloat16Bits(src[i]);
      break;
    }
    case ElementType::Int32: {
      auto *d = static_cast<std::int32_t *>(dst);
      for (std::size_t i = 0; i < n; ++i) d[i] = static_cast<std::int32_t>(src[i]);
      break;
    }
  }
}

void decode(const void *src, std::size_t n, ElementType type, float *dst) {
  switch (type) {
    case ElementType::Float32:
      std::memcpy(dst, src, n * 4);
      break;
    case ElementType::Float16: {
      const auto *s = static_cast<const std::uint16_t *>(src);
      for (std::size_t i = 0; i < n; ++i) dst[i] = halfBitsToFloat(s[i]);
      break;
    }
    case ElementType::BFloat16: {
      const auto *s = static_cast<const std::uint16_t *>(src);
      for (std::size_t i = 0; i < n; ++i) dst[i] = bfloat16BitsToFloat(s[i]);
      break;
    }
    case ElementType::Int32: {
      const auto *s = static_cast<const std::int32_t *>(src);
      for (std::size_t i = 0; i < n; ++i) dst[i] = static_cast<float>(s[i]);
      break;
    }
  }
}

class DeviceGuard {
 public:
  explicit DeviceGuard(int device) {
    cudaGetDevice(&previous_);
    if (previous_ != device) cudaSetDevice(device);
    restore_ = previous_ != device;
  }
  ~DeviceGuard() {
    if (restore_) cudaSetDevice(previous_);
  }

 private:
  int previous_ = 0;
  bool restore_ = false;
};

}  // namespace

CudaBuffer::~CudaBuffer() {
  if (ptr_ != nullptr) {
    DeviceGuard guard(device_);
    cudaFree(ptr_);
  }
}

std::vector<float> CudaBuffer::read() const {
  DeviceGuard guard(device_);
  std::vector<unsigned char> raw(byteCount());
  std::vector<float> out(count_);
  if (count_ == 0) return out;
  if (cudaMemcpy(raw.data(), ptr_, raw.size(), cudaMemcpyDeviceToHost) != cudaSuccess) {
    std::fill(out.begin(), out.end(), std::numeric_limits<float>::quiet_NaN());
    return out;
  }
  decode(raw.data(), count_, type_, out.data());
  return out;
}

CudaRuntime::CudaRuntime(int device) : device_(device) {
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess || count == 0) {
    error_ = e != cudaSuccess ? cudaMessage("cudaGetDeviceCount", e) : "No CUDA device is visible.";
    return;
  }
  if (device < 0 || device >= count) {
    error_ = "CUDA device index out of range.";
    return;
  }
  DeviceGuard guard(device);
  cudaDeviceProp prop;
  e = cudaGetDeviceProperties(&prop, device);
  if (e != cudaSuccess) {
    error_ = cudaMessage("cudaGetDeviceProperties", e);
    return;
  }
  info_.name = prop.name;
  info_.maxThreadsPerThreadgroup = prop.maxThreadsPerBlock;
  info_.maxThreadgroupMemoryLength = prop.sharedMemPerBlockOptin;
  info_.maxBufferLength = prop.totalGlobalMem;
  info_.supportsBFloat16 = prop.major >= 8;
  info_.multiprocessorCount = prop.multiProcessorCount;
  info_.l2CacheBytes = prop.l2CacheSize;
  info_.computeMajor = prop.major;
  info_.computeMinor = prop.minor;
  if (prop.major != 10 || prop.minor != 0) {
    std::ostringstream s;
    s << "This build targets sm_100a (B200); device " << prop.name << " is sm_" << prop.major
      << prop.minor << ".";
    error_ = s.str();
    return;
  }
  e = cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking);
  if (e != cudaSuccess) {
    error_ = cudaMessage("cudaStreamCreate", e);
    return;
  }
  e = cudaMalloc(&status_, sizeof(tmc::TmcDeviceStatus));
  if (e == cudaSuccess) e = cudaMemsetAsync(status_, 0, sizeof(tmc::TmcDeviceStatus), stream_);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream_);
  if (e != cudaSuccess) error_ = cudaMessage("status block", e);
}

CudaRuntime::~CudaRuntime() {
  DeviceGuard guard(device_);
  if (stream_ != nullptr) cudaStreamDestroy(stream_);
  if (status_ != nullptr) cudaFree(status_);
}

BufferResult CudaRuntime::createBuffer(std::size_t elementCount, const float *initialData,
                                       ElementType type) const {
  BufferResult result;
  if (!isAvailable()) {
    result.errorMessage = error_;
    return result;
  }
  if (elementCount == 0) {
    result.errorMessage = "Buffer element count must be positive.";
    return result;
  }
  DeviceGuard guard(device_);
  void *ptr = nullptr;
  const std::size_t bytes = elementCount * elementBytes(type);
  cudaError_t e = cudaMalloc(&ptr, bytes);
  if (e != cudaSuccess) {
    cudaGetLastError();
    result.errorMessage = cudaMessage("cudaMalloc", e);
    return result;
  }
  result.buffer = BufferHandle(new CudaBuffer(ptr, elementCount, type, device_));
  if (initialData != nullptr) {
    result.errorMessage = writeBuffer(result.buffer, initialData, elementCount, 0);
  } else {
    result.errorMessage = fillSentinel(result.buffer);
  }
  if (!result.errorMessage.empty()) result.buffer.reset();
  return result;
}

std::string CudaRuntime::writeBuffer(const BufferHandle &buffer, const float *data,
                                     std::size_t elementCount, std::size_t elementOffset) const {
  if (!buffer) return "writeBuffer: null buffer.";
  if (data == nullptr && elementCount != 0) return "writeBuffer: null host data.";
  if (elementOffset > buffer->elementCount() ||
      elementCount > buffer->elementCount() - elementOffset) {
    return "writeBuffer: write exceeds the buffer.";
  }
  if (elementCount == 0) return {};
  std::vector<unsigned char> raw(elementCount * elementBytes(buffer->elementType()));
  encode(data, elementCount, buffer->elementType(), raw.data());
  return writeBufferBytes(buffer, raw.data(), raw.size(),
                          elementOffset * elementBytes(buffer->elementType()));
}

std::string CudaRuntime::writeBufferBytes(const BufferHandle &buffer, const void *bytes,
                                          std::size_t byteCount, std::size_t byteOffset) const {
  if (!buffer) return "writeBufferBytes: null buffer.";
  if (byteOffset > buffer->byteCount() || byteCount > buffer->byteCount() - byteOffset)
    return "writeBufferBytes: write exceeds the buffer.";
  if (byteCount == 0) return {};
  DeviceGuard guard(device_);
  // Ordered on the runtime stream (kernels run there; the legacy default
  // stream does not synchronise with a non-blocking stream), then completed
  // before returning because `bytes` is caller-owned pageable memory.
  cudaError_t e = cudaMemcpyAsync(static_cast<char *>(buffer->data()) + byteOffset, bytes, byteCount,
                                  cudaMemcpyHostToDevice, stream_);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream_);
  return e == cudaSuccess ? std::string() : cudaMessage("cudaMemcpy H2D", e);
}

std::string CudaRuntime::fillSentinel(const BufferHandle &buffer) const {
  if (!buffer) return "fillSentinel: null buffer.";
  DeviceGuard guard(device_);
  // Integers 0; floating types all-ones bits, a NaN for fp32, fp16 and bf16.
  const int pattern = buffer->elementType() == ElementType::Int32 ? 0 : 0xff;
  cudaError_t e = cudaMemsetAsync(buffer->data(), pattern, buffer->byteCount(), stream_);
  return e == cudaSuccess ? std::string() : cudaMessage("cudaMemset", e);
}

PreparationResult CudaRuntime::prepare(PreparedExecution::Launch launch,
                                       std::vector<BufferHandle> inputs,
                                       std::vector<BufferHandle> outputs, std::string name) {
  PreparationResult result;
  if (!isAvailable()) {
    result.errorMessage = error_;
    return result;
  }
  // Alias rules of prepareBuffers (MetalRuntime.mm:594-648): outputs are
  // distinct and no input aliases an output.
  for (std::size_t i = 0; i < outputs.size(); ++i) {
    if (!outputs[i]) {
      result.errorMessage = "prepare: null output buffer.";
      return result;
    }
    for (std::size_t j = i + 1; j < outputs.size(); ++j)
      if (outputs[i] == outputs[j]) {
        result.errorMessage = "prepare: output buffers must be distinct.";
        return result;
      }
    for (const auto &in : inputs)
      if (in == outputs[i]) {
        result.errorMessage = "prepare: an input aliases an output.";
        return result;
      }
  }
  result.execution = std::make_unique<PreparedExecution>(this, std::move(launch), std::move(inputs),
                                                         std::move(outputs), std::move(name));
  return result;
}

SequencePreparationResult CudaRuntime::prepareSequence(
    const std::vector<const PreparedExecution *> &steps) {
  SequencePreparationResult result;
  if (!isAvailable()) {
    result.errorMessage = error_;
    return result;
  }
  if (steps.empty()) {
    result.errorMessage = "prepareSequence: empty sequence.";
    return result;
  }
  DeviceGuard guard(device_);
  cudaGraph_t graph = nullptr;
  cudaError_t e = cudaStreamBeginCapture(stream_, cudaStreamCaptureModeRelaxed);
  if (e != cudaSuccess) {
    result.errorMessage = cudaMessage("cudaStreamBeginCapture", e);
    return result;
  }
  cudaError_t launchError = cudaSuccess;
  std::vector<const PreparedExecution *> earlier;
  for (const auto *step : steps) {
    if (step == nullptr) {
      launchError = cudaErrorInvalidValue;
      break;
    }
    launchError = !earlier.empty() && step->canOverlapAfter(earlier) ? step->enqueueOverlapped(stream_)
                                                                    : step->enqueue(stream_);
    if (launchError != cudaSuccess) break;
    earlier.push_back(step);
  }
  e = cudaStreamEndCapture(stream_, &graph);
  if (launchError != cudaSuccess || e != cudaSuccess) {
    if (graph) cudaGraphDestroy(graph);
    cudaGetLastError();
    result.errorMessage = cudaMessage("sequence capture", launchError != cudaSuccess ? launchError : e);
    return result;
  }
  cudaGraphExec_t exec = nullptr;
  e = cudaGraphInstantiate(&exec, graph, 0);
  if (e != cudaSuccess) {
    cudaGraphDestroy(graph);
    result.errorMessage = cudaMessage("cudaGraphInstantiate", e);
    return result;
  }
  result.execution.reset(new PreparedSequence(this, graph, exec));
  return result;
}

std::string describeDeviceStatus(const tmc::TmcDeviceStatus &s) {
  if (s.code == tmc::kStatusOk) return {};
  std::ostringstream out;
  out << "device status: ";
  switch (s.code) {
    case tmc::kStatusTokenRange: out << "token id " << s.info0 << " out of vocabulary range (row " << s.info1 << ")"; break;
    case tmc::kStatusLengthRange: out << "position " << s.info0 << " outside the cache capacity (row " << s.info1 << ")"; break;
    case tmc::kStatusPageMissing: out << "logical page " << s.info0 << " has no physical page (row " << s.info1 << ")"; break;
    case tmc::kStatusPageRange: out << "physical page " << s.info0 << " outside the page pool (row " << s.info1 << ")"; break;
    case tmc::kStatusWaitTimeout:
      if (s.where == tmc::kWhereExchange)
        out << "bounded wait timed out for rank " << s.info0 << "'s exchange flag (phase " << s.info1 << ")";
      else
        out << "bounded wait timed out (tile " << s.info0 << ", row " << s.info1 << ")";
      break;
    case tmc::kStatusShape: out << "shape mismatch (" << s.info0 << ", " << s.info1 << ")"; break;
    default: out << "code " << s.code;
  }
  static const char *const kSites[] = {"", "gemv", "attention", "embedding", "lm head", "cache append", "misc",
                                       "gemm", "peer exchange"};
  if (s.where > 0 && s.where < (int)(sizeof(kSites) / sizeof(kSites[0])))
    out << " [" << kSites[s.where] << "]";
  else
    out << " [kernel " << s.where << "]";
  return out.str();
}

std::string CudaRuntime::consumeDeviceStatus() const {
  if (status_ == nullptr) return {};
  DeviceGuard guard(device_);
  tmc::TmcDeviceStatus host{};
  cudaError_t e = cudaMemcpy(&host, status_, sizeof(host), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cudaMessage("status readback", e);
  if (host.code == 0) return {};
  cudaMemsetAsync(status_, 0, sizeof(host), stream_);  // ordered before later kernels
  return describeDeviceStatus(host);
}

std::string CudaRuntime::synchronize() const {
  DeviceGuard guard(device_);
  cudaError_t e = cudaStreamSynchronize(stream_);
  if (e != cudaSuccess) return cudaMessage("cudaStreamSynchronize", e);
  return consumeDeviceStatus();
}

PreparedExecution::PreparedExecution(CudaRuntime *runtime, Launch launch,
                                     std::vector<BufferHandle> inputs,
                                     std::vector<BufferHandle> outputs, std::string name)
    : runtime_(runtime),
      launch_(std::move(launch)),
      inputs_(std::move(inputs)),
      outputs_(std::move(outputs)),
      name_(std::move(name)) {}

bool PreparedExecution::canOverlapAfter(const std::vector<const PreparedExecution *> &earlier) const {
  if (!overlap_) return false;
  for (const auto *prev : earlier)
    for (const auto &written : prev->outputs())
      for (const auto &read : earlyReads_)
        if (written == read) return false;
  return true;
}

ExecutionResult PreparedExecution::execute() const {
  ExecutionResult result;
  DeviceGuard guard(runtime_->device());
  cudaEvent_t start = nullptr, stop = nullptr;
  cudaEventCreate(&start);
  cudaEventCreate(&stop);
  const auto cpuStart = std::chrono::steady_clock::now();
  cudaEventRecord(start, runtime_->stream());
  cudaError_t e = launch_(runtime_->stream());
  cudaEventRecord(stop, runtime_->stream());
  if (e != cudaSuccess) {
    cudaGetLastError();
    result.errorMessage = cudaMessage(name_.c_str(), e);
  }
  const std::string sync = runtime_->synchronize();
  const auto cpuStop = std::chrono::steady_clock::now();
  result.cpuSubmitToCompletionTimeUs =
      std::chrono::duration<double, std::micro>(cpuStop - cpuStart).count();
  if (result.errorMessage.empty()) result.errorMessage = sync;
  float ms = 0.0f;
  if (result.errorMessage.empty() && cudaEventElapsedTime(&ms, start, stop) == cudaSuccess)
    result.gpuExecutionTimeUs = static_cast<double>(ms) * 1000.0;
  cudaEventDestroy(start);
  cudaEventDestroy(stop);
  result.executionPassed = result.errorMessage.empty();
  return result;
}

ExecutionResult PreparedExecution::run() const {
  for (const auto &out : outputs_) {
    const std::string e = runtime_->fillSentinel(out);
    if (!e.empty()) {
      ExecutionResult r;
      r.errorMessage = e;
      return r;
    }
  }
  auto result = execute();
  if (result.executionPassed && !outputs_.empty()) result.output = outputs_.front()->read();
  return result;
}

std::vector<std::vector<float>> PreparedExecution::readOutputs() const {
  std::vector<std::vector<float>> all;
  for (const auto &out : outputs_) all.push_back(out->read());
  return all;
}

PreparedSequence::~PreparedSequence() {
  if (exec_) cudaGraphExecDestroy(exec_);
  if (graph_) cudaGraphDestroy(graph_);
}

ExecutionResult PreparedSequence::execute() const {
  ExecutionResult result;
  DeviceGuard guard(runtime_->device());
  cudaEvent_t start = nullptr, stop = nullptr;
  cudaEventCreate(&start);
  cudaEventCreate(&stop);
  const auto cpuStart = std::chrono::steady_clock::now();
  cudaEventRecord(start, runtime_->stream());
  cudaError_t e = cudaGraphLaunch(exec_, runtime_->stream());
  cudaEventRecord(stop, runtime_->stream());
  if (e != cudaSuccess) result.errorMessage = cudaMessage("cudaGraphLaunch", e);
  const std::string sync = runtime_->synchronize();
  const auto cpuStop = std::chrono::steady_clock::now();
  result.cpuSubmitToCompletionTimeUs =
      std::chrono::duration<double, std::micro>(cpuStop - cpuStart).count();
  if (result.errorMessage.empty()) result.errorMessage = sync;
  float ms = 0.0f;
  if (result.errorMessage.empty() && cudaEventElapsedTime(&ms, start, stop) == cudaSuccess)
    result.gpuExecutionTimeUs = static_cast<double>(ms) * 1000.0;
  cudaEventDestroy(start);
  cudaEventDestroy(stop);
  result.executionPassed = result.errorMessage.empty();
  return result;
}

}  // namespace tensor::cuda
