/*
 * tmc_cuda.h -- C ABI of the B200 (sm_100a) decode backend.
 *
 * The reference (AICompiler-test) runs its decode path through the C++ class
 * tensor::metal::MetalRuntime and the executors built on it; it has no foreign
 * function interface of its own. This header is the flat, plain-pointer
 * boundary that replaces MetalRuntime and exposes the executors, so a C++ host
 * (or a ctypes / cffi binding) can drive the CUDA path without any torch or
 * CUDA types in the signatures. Each declaration names the reference interface
 * it replaces (path within the reference project, file:line).
 *
 * Conventions
 *   - Every function returns an int status: TMC_OK (0) on success. On failure
 *     tmc_cuda_last_error() returns a message for the calling thread. The
 *     reference reports errors as strings in result structs
 *     (MetalRuntime.hpp:91-99, DecoderLLMExecutor.hpp:38-45); the message text
 *     here is that string.
 *   - Host arrays are plain pointers with explicit element counts. Logical host
 *     values are float32 and are rounded to the storage type on the host with
 *     IEEE round-to-nearest-even (MetalRuntime.mm:42-104 does the same).
 *   - "stream" arguments are cudaStream_t values passed as void*; NULL is the
 *     legacy default stream.
 *   - Kernel entry points (tmc_k_*) take DEVICE pointers and only enqueue work;
 *     they never allocate. Executor entry points (tmc_decoder_*, tmc_serving_*)
 *     take HOST pointers and synchronise before returning.
 */
#ifndef TMC_CUDA_H
#define TMC_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes -------------------------------------------------------- */
enum {
  TMC_OK = 0,
  TMC_ERR_INVALID = 1,        /* bad argument, shape or state */
  TMC_ERR_CUDA = 2,           /* a CUDA runtime call failed */
  TMC_ERR_OUT_OF_MEMORY = 3,  /* device allocation or KV page pool exhausted */
  TMC_ERR_DEVICE_STATUS = 4,  /* a kernel reported a range/page/timeout error */
  TMC_ERR_UNSUPPORTED = 5,    /* shape or dtype outside the kernel family */
  TMC_ERR_UNAVAILABLE = 6     /* no sm_100 device, or a library is missing */
};

/* Storage element types: tensor::metal::ElementType (MetalRuntime.hpp:12). */
enum { TMC_F16 = 0, TMC_F32 = 1, TMC_BF16 = 2, TMC_I32 = 3 };

/* Message for the calling thread's last failing call ("" if none). */
const char *tmc_cuda_last_error(void);
/* ABI version of this header (bumped on any signature change). */
int tmc_cuda_abi_version(void);

/* ---- device --------------------------------------------------------------
 * Replaces MetalRuntime::isAvailable / deviceName / hardwareInfo
 * (MetalRuntime.hpp:14-19, 170-173; MetalRuntime.mm:384-395). */
typedef struct {
  char name[256];
  int compute_major, compute_minor;  /* 10.0 for B200 */
  int multiprocessor_count;
  size_t max_threads_per_block;      /* HardwareInfo::maxThreadsPerThreadgroup */
  size_t max_shared_per_block;       /* HardwareInfo::maxThreadgroupMemoryLength (opt-in) */
  size_t total_global_mem;           /* HardwareInfo::maxBufferLength */
  size_t l2_cache_bytes;
  int supports_bf16;                 /* HardwareInfo::supportsBFloat16 */
} tmc_device_info;

int tmc_cuda_device_count(int *count);
int tmc_cuda_device_info(int device, tmc_device_info *out);

/* ---- runtime + buffers ---------------------------------------------------
 * tmc_runtime replaces one MetalRuntime instance (one device, one queue):
 * MetalRuntime::MetalRuntime (MetalRuntime.hpp:165).
 * tmc_buffer replaces MetalBuffer / BufferHandle (MetalRuntime.hpp:55-78):
 * createBuffer (MetalRuntime.hpp:190-192, MetalRuntime.mm:515-561: uninitialised
 * floating buffers hold NaN, integers 0), writeBuffer (MetalRuntime.hpp:193-196),
 * MetalBuffer::read (MetalRuntime.hpp:62). */
typedef struct tmc_runtime tmc_runtime;
typedef struct tmc_buffer tmc_buffer;

int tmc_runtime_create(int device, tmc_runtime **out);
void tmc_runtime_destroy(tmc_runtime *rt);
/* The runtime's own stream (cudaStream_t as void*). */
void *tmc_runtime_stream(tmc_runtime *rt);
int tmc_runtime_synchronize(tmc_runtime *rt);
/* Device status block (int[4]: code, kernel, info0, info1) kernels write on
 * range/page/timeout errors; pass it to tmc_k_* calls. */
void *tmc_runtime_status_ptr(tmc_runtime *rt);

int tmc_buffer_create(tmc_runtime *rt, size_t count, int dtype, const float *init,
                      tmc_buffer **out);
void tmc_buffer_destroy(tmc_buffer *buf);
int tmc_buffer_write(tmc_buffer *buf, const float *values, size_t count, size_t offset);
int tmc_buffer_read(const tmc_buffer *buf, float *out, size_t count);
int tmc_buffer_write_bytes(tmc_buffer *buf, const void *bytes, size_t nbytes, size_t offset);
int tmc_buffer_read_bytes(const tmc_buffer *buf, void *out, size_t nbytes, size_t offset);
void *tmc_buffer_device_ptr(tmc_buffer *buf);
size_t tmc_buffer_count(const tmc_buffer *buf);
int tmc_buffer_dtype(const tmc_buffer *buf);

/* ---- kernels (device pointers; enqueue only) ------------------------------ */

/* Fused RMSNorm -> GEMV, fp32 activations, fp16 weights, fp32 accumulate:
 *   y[m, n] = sum_k (x[m,k] * rsqrt(mean_k x[m,:]^2 + eps) * gamma[k]) * W[n, k]
 * Replaces the pair emitRMSNorm (MetalEmitter.cpp:12-76) -> emitDecodeGEMV
 * (DecodeGEMVMetalEmitter.cpp:68-132) that compileGraph dispatches for the
 * graph RMSNorm -> Transpose(W) -> MatMul (GraphExecutor.cpp:346-431).
 * x [rows, k] f32, gamma [k] f32, W [n, k] f16 row-major, y [rows, n] f32;
 * rows <= 4, k % 8 == 0. */
int tmc_k_rmsnorm_gemv_f32(const float *x, const float *gamma, const void *w_f16, float *y,
                           int rows, int k, int n, float eps, void *stream);

/* Decode GEMV y = x W^T with fp16 x, W and y, fp32 accumulation: replaces
 * emitDecodeGEMV / emitLinearBaseline (DecodeGEMVMetalEmitter.cpp:18-132).
 * x [rows, k], W [n, k], y [rows, n]; rows <= 8, k % 8 == 0. */
int tmc_k_gemv_f16(const void *x_f16, const void *w_f16, void *y_f16, int rows, int k, int n,
                   void *stream);

/* Same with fp32 output (no storage rounding). */
int tmc_k_gemv_f16_f32out(const void *x_f16, const void *w_f16, float *y, int rows, int k,
                          int n, void *stream);

/* Block-table GQA decode attention over a paged fp16 KV pool, split-K:
 * replaces emitServingPagedKVAttention (KVCacheMetalEmitter.cpp:312-406).
 *   q        [rows, hq, d] f16         out [rows, hq, d] f16
 *   k_pool,
 *   v_pool   [pool_pages, hkv, page_size, d] f16
 *   block_table [table_rows_total, table_stride] int32 (physical page per logical page)
 *   table_rows  [rows] int32 (block-table row of each query row)
 *   positions   [rows] int32 (keys 0..position are attended; position < capacity)
 * d in {16, 32, 64, 128}; hq % hkv == 0 and hq / hkv in {1, 2, 4, 8}.
 * workspace: tmc_k_attention_workspace_bytes(...) bytes of device memory, plus
 * counters: rows*hkv uint32 that must be zero before the first call (each call
 * leaves them zero). status: tmc_runtime_status_ptr() or NULL. */
size_t tmc_k_attention_workspace_bytes(int rows, int hq, int hkv, int d, int max_splits);
int tmc_k_paged_attention_f16(const void *q, void *out, const void *k_pool, const void *v_pool,
                              const int32_t *block_table, int table_stride,
                              const int32_t *table_rows, const int32_t *positions, int rows,
                              int hq, int hkv, int d, int page_size, int pool_pages,
                              int capacity, int max_splits, int min_chunk, void *workspace,
                              uint32_t *counters, void *status, void *stream);

/* Deterministic N(0, std^2) fp16 fill from a counter-based hash generator
 * (synthetic random-init weights without a host round trip). */
int tmc_k_fill_normal_f16(void *dst, size_t count, uint64_t seed, float mean, float stddev,
                          void *stream);

#ifdef __cplusplus
}
#endif

#endif /* TMC_CUDA_H */
