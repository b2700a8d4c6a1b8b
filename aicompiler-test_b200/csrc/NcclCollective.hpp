// NCCL-backed Collective for tensor parallelism over NVLink / NVSwitch.
// NCCL is resolved at run time (dlopen "libnccl.so.2"), so single-GPU use
// never needs it; inside a PyTorch process the already-loaded NCCL is reused.
#pragma once

#include <nccl.h>

#include <memory>
#include <string>

#include "DecoderExecutor.hpp"

namespace tensor::runtime {

// Fill `id` (NCCL_UNIQUE_ID_BYTES) on the root rank; "" on success.
std::string ncclUniqueIdBytes(unsigned char *id);

class NcclCollective : public Collective {
 public:
  // Collective over `world` ranks; `id` from ncclUniqueIdBytes on rank 0.
  static std::shared_ptr<NcclCollective> create(const unsigned char *id, int world, int rank,
                                                std::string *error);
  ~NcclCollective() override;
  cudaError_t allReduceSumF32(float *buf, std::size_t count, cudaStream_t s) override;
  cudaError_t allReduceMaxU64(unsigned long long *buf, std::size_t count, cudaStream_t s) override;
  std::string lastError() const override { return error_; }
  // Abort in-flight work (failure path; the communicator is unusable afterwards).
  void abort();

 private:
  NcclCollective() = default;
  ncclComm_t comm_ = nullptr;
  std::string error_;
};

}  // namespace tensor::runtime
