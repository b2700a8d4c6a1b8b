// Shared error plumbing of the extern "C" layer.
#pragma once

#include <cuda_runtime.h>

#include <string>

#include <memory>

#include "CudaRuntime.hpp"

// Opaque handle types of include/tmc_cuda.h.
struct tmc_runtime {
  std::unique_ptr<tensor::cuda::CudaRuntime> rt;
};
struct tmc_buffer {
  tensor::cuda::BufferHandle buf;
  tensor::cuda::CudaRuntime *rt;
};

namespace tmc_api {

// Record `message` as the calling thread's last error and return `code`.
int fail(int code, const std::string &message);
// Map a CUDA error to TMC_ERR_CUDA / TMC_ERR_OUT_OF_MEMORY with its message.
int cuda_fail(cudaError_t e, const char *what);
// Clear the last error and return TMC_OK.
int ok();
// Multiprocessor count of the current device (cached per thread).
int num_sms();
bool to_element_type(int dtype, tensor::cuda::ElementType *out);

}  // namespace tmc_api
