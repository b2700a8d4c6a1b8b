// extern "C" boundary: runtime, buffers and kernel entry points
// (declarations and reference citations in include/tmc_cuda.h).
#include <cstdio>
#include <cstring>
#include <memory>
#include <string>

#include "CudaRuntime.hpp"
#include "api_util.hpp"
#include "attention.cuh"
#include "gemm.cuh"
#include "gemv.cuh"
#include "misc.cuh"
#include "fusion.cuh"
#include "rmsnorm.cuh"
#include "tmc_cuda.h"

using tensor::cuda::BufferHandle;
using tensor::cuda::CudaRuntime;
using tensor::cuda::ElementType;


namespace tmc_api {

thread_local std::string g_last_error;

int fail(int code, const std::string &message) {
  g_last_error = message;
  return code;
}

int cuda_fail(cudaError_t e, const char *what) {
  cudaGetLastError();
  return fail(e == cudaErrorMemoryAllocation ? TMC_ERR_OUT_OF_MEMORY : TMC_ERR_CUDA,
              std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")");
}

int ok() {
  g_last_error.clear();
  return TMC_OK;
}

int num_sms() {
  static thread_local int cached_dev = -1;
  static thread_local int cached_sms = 148;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev != cached_dev) {
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && sms > 0)
      cached_sms = sms;
    cached_dev = dev;
  }
  return cached_sms;
}

bool to_element_type(int dtype, ElementType *out) {
  switch (dtype) {
    case TMC_F16: *out = ElementType::Float16; return true;
    case TMC_F32: *out = ElementType::Float32; return true;
    case TMC_BF16: *out = ElementType::BFloat16; return true;
    case TMC_I32: *out = ElementType::Int32; return true;
    default: return false;
  }
}

}  // namespace tmc_api

using namespace tmc_api;

extern "C" {

const char *tmc_cuda_last_error(void) { return g_last_error.c_str(); }

int tmc_cuda_abi_version(void) { return 2; }

int tmc_cuda_device_count(int *count) {
  if (count == nullptr) return fail(TMC_ERR_INVALID, "count is null");
  cudaError_t e = cudaGetDeviceCount(count);
  if (e != cudaSuccess) {
    *count = 0;
    cudaGetLastError();
    return fail(TMC_ERR_UNAVAILABLE, std::string("cudaGetDeviceCount: ") + cudaGetErrorString(e));
  }
  return ok();
}

int tmc_cuda_device_info(int device, tmc_device_info *out) {
  if (out == nullptr) return fail(TMC_ERR_INVALID, "out is null");
  cudaDeviceProp prop;
  cudaError_t e = cudaGetDeviceProperties(&prop, device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceProperties");
  std::memset(out, 0, sizeof(*out));
  std::snprintf(out->name, sizeof(out->name), "%s", prop.name);
  out->compute_major = prop.major;
  out->compute_minor = prop.minor;
  out->multiprocessor_count = prop.multiProcessorCount;
  out->max_threads_per_block = prop.maxThreadsPerBlock;
  out->max_shared_per_block = prop.sharedMemPerBlockOptin;
  out->total_global_mem = prop.totalGlobalMem;
  out->l2_cache_bytes = prop.l2CacheSize;
  out->supports_bf16 = prop.major >= 8 ? 1 : 0;
  return ok();
}

int tmc_runtime_create(int device, tmc_runtime **out) {
  if (out == nullptr) return fail(TMC_ERR_INVALID, "out is null");
  *out = nullptr;
  auto rt = std::make_unique<CudaRuntime>(device);
  if (!rt->isAvailable()) return fail(TMC_ERR_UNAVAILABLE, rt->initializationError());
  // One runtime per device and thread: kernels launch on the current device.
  cudaSetDevice(device);
  *out = new tmc_runtime{std::move(rt)};
  return ok();
}

void tmc_runtime_destroy(tmc_runtime *rt) { delete rt; }

void *tmc_runtime_stream(tmc_runtime *rt) { return rt ? static_cast<void *>(rt->rt->stream()) : nullptr; }

int tmc_runtime_synchronize(tmc_runtime *rt) {
  if (rt == nullptr) return fail(TMC_ERR_INVALID, "runtime is null");
  const std::string e = rt->rt->synchronize();
  if (!e.empty()) return fail(e.rfind("device status", 0) == 0 ? TMC_ERR_DEVICE_STATUS : TMC_ERR_CUDA, e);
  return ok();
}

void *tmc_runtime_status_ptr(tmc_runtime *rt) { return rt ? static_cast<void *>(rt->rt->deviceStatus()) : nullptr; }

int tmc_buffer_create(tmc_runtime *rt, size_t count, int dtype, const float *init, tmc_buffer **out) {
  if (rt == nullptr || out == nullptr) return fail(TMC_ERR_INVALID, "null runtime or out");
  *out = nullptr;
  ElementType type;
  if (!to_element_type(dtype, &type)) return fail(TMC_ERR_INVALID, "unknown dtype");
  auto created = rt->rt->createBuffer(count, init, type);
  if (!created.buffer) return fail(TMC_ERR_OUT_OF_MEMORY, created.errorMessage);
  *out = new tmc_buffer{created.buffer, rt->rt.get()};
  return ok();
}

void tmc_buffer_destroy(tmc_buffer *buf) { delete buf; }

int tmc_buffer_write(tmc_buffer *buf, const float *values, size_t count, size_t offset) {
  if (buf == nullptr) return fail(TMC_ERR_INVALID, "buffer is null");
  const std::string e = buf->rt->writeBuffer(buf->buf, values, count, offset);
  return e.empty() ? ok() : fail(TMC_ERR_INVALID, e);
}

int tmc_buffer_read(const tmc_buffer *buf, float *out, size_t count) {
  if (buf == nullptr || out == nullptr) return fail(TMC_ERR_INVALID, "null buffer or out");
  if (count > buf->buf->elementCount()) return fail(TMC_ERR_INVALID, "read exceeds the buffer");
  const std::string s = buf->rt->synchronize();
  if (!s.empty()) return fail(TMC_ERR_CUDA, s);
  auto values = buf->buf->read();
  std::memcpy(out, values.data(), count * sizeof(float));
  return ok();
}

int tmc_buffer_write_bytes(tmc_buffer *buf, const void *bytes, size_t nbytes, size_t offset) {
  if (buf == nullptr) return fail(TMC_ERR_INVALID, "buffer is null");
  const std::string e = buf->rt->writeBufferBytes(buf->buf, bytes, nbytes, offset);
  return e.empty() ? ok() : fail(TMC_ERR_INVALID, e);
}

int tmc_buffer_read_bytes(const tmc_buffer *buf, void *out, size_t nbytes, size_t offset) {
  if (buf == nullptr || out == nullptr) return fail(TMC_ERR_INVALID, "null buffer or out");
  if (offset > buf->buf->byteCount() || nbytes > buf->buf->byteCount() - offset)
    return fail(TMC_ERR_INVALID, "read exceeds the buffer");
  const std::string s = buf->rt->synchronize();
  if (!s.empty()) return fail(TMC_ERR_CUDA, s);
  cudaError_t e = cudaMemcpy(out, static_cast<char *>(buf->buf->data()) + offset, nbytes,
                             cudaMemcpyDeviceToHost);
  return e == cudaSuccess ? ok() : cuda_fail(e, "cudaMemcpy D2H");
}

void *tmc_buffer_device_ptr(tmc_buffer *buf) { return buf ? buf->buf->data() : nullptr; }
size_t tmc_buffer_count(const tmc_buffer *buf) { return buf ? buf->buf->elementCount() : 0; }
int tmc_buffer_dtype(const tmc_buffer *buf) {
  if (buf == nullptr) return -1;
  switch (buf->buf->elementType()) {
    case ElementType::Float16: return TMC_F16;
    case ElementType::Float32: return TMC_F32;
    case ElementType::BFloat16: return TMC_BF16;
    case ElementType::Int32: return TMC_I32;
  }
  return -1;
}

int tmc_k_rmsnorm(const void *x, const void *gamma, void *y, int rows, int width, float eps, int fp16,
                  int threads, void *stream) {
  if (!x || !gamma || !y) return fail(TMC_ERR_INVALID, "null pointer");
  if (rows < 1 || width < 1) return fail(TMC_ERR_INVALID, "rmsnorm: need rows >= 1, width >= 1");
  if (!(eps > 0.0f)) return fail(TMC_ERR_INVALID, "eps must be positive");
  if (threads != 0 && (threads < 32 || threads > 1024 || (threads & (threads - 1)) != 0))
    return fail(TMC_ERR_UNSUPPORTED, "rmsnorm: threads must be 0 or a power of two in [32, 1024]");
  auto st = static_cast<cudaStream_t>(stream);
  const cudaError_t e = threads == 0 ? tmc::launch_rmsnorm_baseline(x, gamma, y, rows, width, eps, fp16 != 0, st)
                                     : tmc::launch_rmsnorm(x, gamma, y, rows, width, eps, fp16 != 0, threads, st);
  return e == cudaSuccess ? ok() : cuda_fail(e, "rmsnorm launch");
}

int tmc_k_fused_add_norm(const void *x, const void *b, const void *w, const void *c, void *y, int rows, int width,
                         int b_rows, float eps, int layer_norm, int fp16, void *stream) {
  if (!x || !b || !w || !y || (layer_norm && !c)) return fail(TMC_ERR_INVALID, "null pointer");
  if (rows < 1 || width < 1 || (b_rows != 1 && b_rows != rows))
    return fail(TMC_ERR_INVALID, "fused add-norm: rows, width >= 1 and b_rows 1 or rows");
  if (!(eps > 0.0f)) return fail(TMC_ERR_INVALID, "eps must be positive");
  const cudaError_t e = tmc::launch_fused_add_norm(x, b, w, c, y, rows, width, b_rows, eps, layer_norm != 0, fp16 != 0,
                                                   static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? ok() : cuda_fail(e, "fused add-norm launch");
}

int tmc_k_fused_silu_mul(const void *x, const void *b, void *y, int rows, int width, int b_rows, int fp16,
                         void *stream) {
  if (!x || !b || !y) return fail(TMC_ERR_INVALID, "null pointer");
  if (rows < 1 || width < 1 || (b_rows != 1 && b_rows != rows))
    return fail(TMC_ERR_INVALID, "fused silu-mul: rows, width >= 1 and b_rows 1 or rows");
  const cudaError_t e =
      tmc::launch_fused_silu_mul(x, b, y, rows, width, b_rows, fp16 != 0, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? ok() : cuda_fail(e, "fused silu-mul launch");
}

int tmc_k_fused_linear_relu(const void *a, const void *w, const void *bias, void *y, int m, int k, int n, int fp16,
                            void *stream) {
  if (!a || !w || !bias || !y) return fail(TMC_ERR_INVALID, "null pointer");
  if (m < 1 || k < 1 || n < 1) return fail(TMC_ERR_INVALID, "fused linear-relu: m, k, n >= 1");
  const cudaError_t e =
      tmc::launch_fused_linear_relu(a, w, bias, y, m, k, n, fp16 != 0, static_cast<cudaStream_t>(stream));
  if (e == cudaErrorInvalidValue) return fail(TMC_ERR_UNSUPPORTED, "fused linear-relu: unsupported shape");
  return e == cudaSuccess ? ok() : cuda_fail(e, "fused linear-relu launch");
}

int tmc_k_rmsnorm_gemv_f32(const float *x, const float *gamma, const void *w_f16, float *y,
                           int rows, int k, int n, float eps, void *stream) {
  if (!x || !gamma || !w_f16 || !y) return fail(TMC_ERR_INVALID, "null pointer");
  if (rows < 1 || rows > 4 || k < 8 || (k % 8) != 0 || n < 1)
    return fail(TMC_ERR_UNSUPPORTED, "rmsnorm_gemv: need 1<=rows<=4, k%8==0, n>=1");
  if (!(eps > 0.0f)) return fail(TMC_ERR_INVALID, "eps must be positive");
  tmc::GemvParams p{};
  p.W = static_cast<const __half *>(w_f16);
  p.N = n;
  p.K = k;
  p.M = rows;
  p.prologue = tmc::kProF32Norm;
  p.x = x;
  p.x_stride = k;
  p.gamma = gamma;
  p.eps = eps;
  p.epilogue = tmc::kEpiF32;
  p.y_f32 = y;
  p.y_stride = n;
  cudaError_t e = tmc::launch_gemv(p, static_cast<cudaStream_t>(stream), false, num_sms());
  return e == cudaSuccess ? ok() : cuda_fail(e, "rmsnorm_gemv launch");
}

static int gemv_f16_common(const void *x, const void *w, void *y_f16, float *y_f32, int rows, int k,
                           int n, void *stream) {
  if (!x || !w || (!y_f16 && !y_f32)) return fail(TMC_ERR_INVALID, "null pointer");
  if (rows < 1 || rows > 8 || k < 8 || (k % 8) != 0 || n < 1)
    return fail(TMC_ERR_UNSUPPORTED, "gemv: need 1<=rows<=8, k%8==0, n>=1");
  tmc::GemvParams p{};
  p.W = static_cast<const __half *>(w);
  p.N = n;
  p.K = k;
  p.M = rows;
  p.prologue = tmc::kProF16;
  p.x = x;
  p.x_stride = k;
  p.epilogue = y_f16 ? tmc::kEpiF16 : tmc::kEpiF32;
  p.y_f16 = static_cast<__half *>(y_f16);
  p.y_f32 = y_f32;
  p.y_stride = n;
  cudaError_t e = tmc::launch_gemv(p, static_cast<cudaStream_t>(stream), false, num_sms());
  return e == cudaSuccess ? ok() : cuda_fail(e, "gemv launch");
}

int tmc_k_gemv_f16(const void *x_f16, const void *w_f16, void *y_f16, int rows, int k, int n,
                   void *stream) {
  return gemv_f16_common(x_f16, w_f16, y_f16, nullptr, rows, k, n, stream);
}

int tmc_k_gemv_f16_f32out(const void *x_f16, const void *w_f16, float *y, int rows, int k, int n,
                          void *stream) {
  return gemv_f16_common(x_f16, w_f16, nullptr, y, rows, k, n, stream);
}

namespace {
int sm_count() {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}
}  // namespace

size_t tmc_k_batched_gemm_workspace_bytes(int n, int k, int rows) {
  if (n <= 0 || k <= 0 || rows <= 0 || rows > 256) return 0;
  const tmc::GemmPlan plan = tmc::plan_gemm(n, k, rows, sm_count());
  const size_t partial = (tmc::gemm_workspace_floats(plan) * 4 + 255) / 256 * 256;
  return partial + (size_t)plan.tiles * 8;
}

int tmc_k_batched_gemm_f16_f32out(const void *x_f16, const void *w_f16, float *y, int rows, int k, int n,
                                  void *workspace, void *status, void *stream) {
  if (!x_f16 || !w_f16 || !y || !workspace) return fail(TMC_ERR_INVALID, "null pointer");
  if (rows <= 0 || rows > 256 || n <= 0 || k <= 0 || k % 8 != 0)
    return fail(TMC_ERR_UNSUPPORTED, "batched gemm: rows in [1, 128], k % 8 == 0");
  const tmc::GemmPlan plan = tmc::plan_gemm(n, k, rows, sm_count());
  const size_t partial = (tmc::gemm_workspace_floats(plan) * 4 + 255) / 256 * 256;
  auto *ws = static_cast<unsigned char *>(workspace);
  auto *tickets = reinterpret_cast<unsigned int *>(ws + partial);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(tickets, 0, (size_t)plan.tiles * 8, s);
  if (e != cudaSuccess) return cuda_fail(e, "clearing gemm tickets");
  CUtensorMap wm, xm;
  if ((e = tmc::make_tensor_map_f16(&wm, w_f16, n, k, tmc::kGemmTileRows)) != cudaSuccess)
    return cuda_fail(e, "weight tensor map");
  if ((e = tmc::make_tensor_map_f16(&xm, x_f16, rows, k, plan.tn)) != cudaSuccess)
    return cuda_fail(e, "activation tensor map");
  tmc::GemvParams p{};
  p.W = static_cast<const __half *>(w_f16);
  p.N = n;
  p.K = k;
  p.M = rows;
  p.prologue = tmc::kProF16;
  p.x = x_f16;
  p.x_stride = k;
  p.epilogue = tmc::kEpiF32;
  p.y_f32 = y;
  p.y_stride = n;
  p.status = static_cast<tmc::TmcDeviceStatus *>(status);
  e = tmc::launch_gemm(p, wm, xm, plan, reinterpret_cast<float *>(ws), tickets, s, false);
  if (e == cudaErrorInvalidValue) return fail(TMC_ERR_UNSUPPORTED, "batched gemm: unsupported shape");
  return e == cudaSuccess ? ok() : cuda_fail(e, "batched gemm launch");
}

size_t tmc_k_attention_workspace_bytes(int rows, int hq, int hkv, int d, int max_splits) {
  return tmc::attention_workspace_bytes(rows, hq, hkv, d, max_splits);
}

int tmc_k_paged_attention_f16(const void *q, void *out, const void *k_pool, const void *v_pool,
                              const int32_t *block_table, int table_stride,
                              const int32_t *table_rows, const int32_t *positions, int rows, int hq,
                              int hkv, int d, int page_size, int pool_pages, int capacity,
                              int max_splits, int min_chunk, void *workspace, uint32_t *counters,
                              void *status, void *stream) {
  return tmc_k_paged_attention_f16_ex(q, out, k_pool, v_pool, block_table, table_stride, table_rows, positions,
                                      rows, hq, hkv, d, page_size, pool_pages, capacity, max_splits, min_chunk,
                                      workspace, counters, 0, 1, status, stream);
}

int tmc_k_paged_attention_f16_ex(const void *q, void *out, const void *k_pool, const void *v_pool,
                                 const int32_t *block_table, int table_stride, const int32_t *table_rows,
                                 const int32_t *positions, int rows, int hq, int hkv, int d, int page_size,
                                 int pool_pages, int capacity, int max_splits, int min_chunk, void *workspace,
                                 uint32_t *counters, int schedule, int row_group, void *status, void *stream) {
  if (!q || !out || !k_pool || !v_pool || !block_table || !table_rows || !positions || !counters)
    return fail(TMC_ERR_INVALID, "null pointer");
  if (schedule < 0 || schedule > 2) return fail(TMC_ERR_INVALID, "schedule must be 0, 1 or 2");
  if (row_group != 0 && row_group != 1 && row_group != 2)
    return fail(TMC_ERR_INVALID, "row_group must be 1 (rows one by one) or 2 (prefill row groups)");
  if (max_splits > 1 && workspace == nullptr) return fail(TMC_ERR_INVALID, "workspace is null");
  tmc::AttentionParams p{};
  p.q = static_cast<const __half *>(q);
  p.q_stride = static_cast<long long>(hq) * d;
  p.out = static_cast<__half *>(out);
  p.out_stride = static_cast<long long>(hq) * d;
  p.k_pool = static_cast<const __half *>(k_pool);
  p.v_pool = static_cast<const __half *>(v_pool);
  p.block_table = block_table;
  p.table_stride = table_stride;
  p.table_rows = table_rows;
  p.positions = positions;
  p.rows = rows;
  p.hq = hq;
  p.hkv = hkv;
  p.head_dim = d;
  p.page_size = page_size;
  p.pool_pages = pool_pages;
  p.capacity = capacity;
  p.scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(d)));
  p.max_splits = max_splits;
  p.min_chunk = min_chunk;
  p.early_mode = 2;  // standalone call: no kernel produces K/V concurrently
  const size_t acc_bytes = (size_t)rows * hq * max_splits * d * 4;
  p.ws_acc = static_cast<float *>(workspace);
  p.ws_ml = reinterpret_cast<float *>(static_cast<char *>(workspace) + acc_bytes);
  p.ws_floats = workspace ? tmc::attention_workspace_bytes(rows, hq, hkv, d, max_splits) / 4 : 0;
  p.schedule = schedule;
  p.row_group = row_group == 2 ? 2 : 1;
  p.counters = counters;
  p.status = static_cast<tmc::TmcDeviceStatus *>(status);
  CUtensorMap km, vm;
  if ((d == 64 || d == 128) && page_size % 16 == 0 &&
      (reinterpret_cast<uintptr_t>(k_pool) & 15) == 0 && (reinterpret_cast<uintptr_t>(v_pool) & 15) == 0) {
    const uint64_t rows = (uint64_t)pool_pages * hkv * page_size;
    if (tmc::make_tensor_map_f16(&km, k_pool, rows, d, 16) == cudaSuccess &&
        tmc::make_tensor_map_f16(&vm, v_pool, rows, d, 16) == cudaSuccess) {
      p.k_map = &km;
      p.v_map = &vm;
    }
  }
  cudaError_t e = tmc::launch_attention(p, static_cast<cudaStream_t>(stream), false);
  if (e == cudaErrorInvalidValue) return fail(TMC_ERR_UNSUPPORTED, "attention: unsupported shape");
  return e == cudaSuccess ? ok() : cuda_fail(e, "attention launch");
}

int tmc_k_fill_normal_f16(void *dst, size_t count, uint64_t seed, float mean, float stddev,
                          void *stream) {
  if (!dst) return fail(TMC_ERR_INVALID, "null pointer");
  cudaError_t e = tmc::launch_fill_normal_f16(static_cast<__half *>(dst), count, seed, mean, stddev,
                                              static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? ok() : cuda_fail(e, "fill_normal launch");
}

}  // extern "C"
