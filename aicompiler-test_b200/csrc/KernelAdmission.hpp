// Generated-kernel contracts, the validate-then-benchmark admission gate and
// the registry of admitted kernels: the B200 counterparts of the reference's
// KernelContract / makeKernelContract (src/llm/KernelContract.hpp:10-65,
// KernelContract.cpp:35-100, DecoderKernelContracts.cpp:129-245),
// admitGeneratedKernel (src/runtime/GeneratedKernelAdmission.cpp:204-318) and
// KernelRegistry / writeAdmittedKernel (src/runtime/KernelRegistry.hpp).
//
// A contract is owned by the compiler: the pattern's semantics, buffer
// interface, launch geometry, three seeded cases with fp64 references,
// tolerances and the minimum speedup. A candidate supplies only CUDA C++
// source and a block size. Admission: NVRTC compiles it for sm_100a (in
// memory), the driver loads it, the parameter layout is checked against the
// contract (cuFuncGetParamInfo), every case is validated, then two paired
// timing rounds against the template baseline must each reach the minimum
// speedup, and the cases are validated again. Only then is the artifact
// written; the registry reloads (recompiles) admitted artifacts.
//
// Candidate kernel signature (one pointer per input, then per output, then
// the work-item count):
//   extern "C" __global__ void generated_<pattern>(const T *in0, ..., T *out0, ..., unsigned work_items)
// with T = float (fp32 storage) or __half (the `_fp16` patterns; the RoPE
// tables stay float and `valid_length` is int). Launch geometry: one CTA of
// the candidate's block size per work item when the contract says so
// (groupPerWorkItem), else ceil(work_items / block) CTAs.
#pragma once

#include <cstddef>
#include <cstdint>
#include <map>
#include <memory>
#include <ostream>
#include <string>
#include <vector>

namespace tensor::runtime {

enum class ContractType { Float32, Float16, Int32 };

struct KernelCase {
  std::vector<std::size_t> shape;
  std::vector<std::vector<float>> inputs;       // logical values (already storage-rounded)
  std::vector<std::vector<double>> references;  // one per output
  std::size_t workItems = 0;
};

struct KernelContract {
  std::string pattern;
  std::string functionName;
  std::string semantics;
  std::string workItem;
  std::string applicability;
  std::vector<std::string> inputNames, outputNames;
  std::vector<ContractType> inputTypes;
  ContractType storageType = ContractType::Float32;
  bool groupPerWorkItem = true;
  std::vector<int> blockSizes{32, 64, 128};
  double absoluteTolerance = 2e-4;
  double relativeTolerance = 2e-3;
  double minimumSpeedup = 1.05;
  std::vector<KernelCase> cases;
};

// Patterns: decoder_gemv_<K>_<N> (K * N <= 8M), decoder_rope,
// decoder_residual_rmsnorm, decoder_gated_mlp, each optionally with `_fp16`.
// Throws std::invalid_argument for an unknown pattern.
KernelContract makeKernelContract(const std::string &pattern);
// The contract as JSON (what a generator is given).
std::string serializeKernelContract(const KernelContract &contract);

struct AdmissionFeedback {
  std::string status;  // "admitted", "retry" or "fatal"
  std::string stage;   // compile, interface, numerical_validation, performance, ...
  std::string message;
  double baselineUs = 0.0, candidateUs = 0.0, speedup = 0.0;  // worst round
};

// Admit `source` for `pattern` with `blockSize`. Writes the feedback JSON to
// feedbackPath (if not empty) and, when admitted, the artifact JSON to
// artifactPath (if not empty). `log` receives a step-by-step report.
AdmissionFeedback admitGeneratedKernel(const std::string &pattern, const std::string &source, int blockSize,
                                       const std::string &feedbackPath, const std::string &artifactPath,
                                       std::ostream &log);

// A compiled candidate or admitted kernel: launch with device pointers in
// contract order (inputs, then outputs) and the work-item count.
class CompiledKernel {
 public:
  ~CompiledKernel();
  CompiledKernel(const CompiledKernel &) = delete;
  CompiledKernel &operator=(const CompiledKernel &) = delete;
  static std::unique_ptr<CompiledKernel> compile(const KernelContract &contract, const std::string &source,
                                                 int blockSize, std::string *error);
  std::string launch(const std::vector<void *> &buffers, unsigned workItems, void *stream) const;
  int blockSize() const { return block_; }

 private:
  CompiledKernel() = default;
  void *module_ = nullptr;
  void *function_ = nullptr;
  int block_ = 0;
  bool perWorkItem_ = true;
};

struct KernelUsage {
  std::string node, pattern, implementation;
  std::size_t dispatchesPerCall = 0, completedCalls = 0;
};

// Admitted kernels by pattern, loaded from a directory of artifacts.
class KernelRegistry {
 public:
  // Loads every *.json artifact in `directory` whose contract pattern is
  // known, recompiling its source; invalid artifacts are reported and skipped.
  void load(const std::string &directory, std::ostream &log);
  const CompiledKernel *find(const std::string &pattern) const;
  std::vector<std::string> patterns() const;
  std::size_t track(KernelUsage usage);
  void completed(const std::vector<std::size_t> &uses);
  void report(std::ostream &log) const;

 private:
  std::map<std::string, std::unique_ptr<CompiledKernel>> entries_;
  std::vector<KernelUsage> usage_;
};

}  // namespace tensor::runtime
