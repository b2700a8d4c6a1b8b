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

/* ---- prepared executions and sequences -----------------------------------
 * The reference compiles an emitted source into the runtime's current pipeline
 * (MetalRuntime::createComputePipeline, MetalRuntime.hpp:176-178), binds
 * buffers and packed uint32 constants to it (prepareBuffers,
 * MetalRuntime.hpp:199-206, MetalRuntime.mm:594-648), runs it (PreparedExecution
 * run / execute, MetalRuntime.hpp:101-121, MetalRuntime.mm:197-277) and chains
 * launches into one submission (prepareSequence, MetalRuntime.mm:751-781).
 * Here the kernels are this library's precompiled sm_100a functions, looked up
 * by name (tmc_kernel_lookup; tmc_kernel_describe gives each one's buffer
 * interface and constants), and a sequence is one CUDA graph.
 *
 * tmc_prepare binds inputs, then outputs, then constants, with the reference's
 * checks: at least one input and one output, at most 31 bindings and 1024
 * constants, groups and threads non-zero and within the device limits
 * ("Kernel dispatch exceeds device or pipeline limits."), outputs distinct
 * and on this runtime, no input aliasing an output; then the kernel's own
 * interface (element types, sizes against the constants). Floating constants
 * (eps) are passed as their float bit patterns. Kernels whose launcher sizes
 * its own grid (the GEMV, GEMM and attention families) take the dispatch only
 * for the limit check; rmsnorm takes its threads per CTA from it. A prepared
 * execution retains its buffers (and any workspace it needed) until destroyed.
 *
 * tmc_prepared_run fills every output with NaN sentinels (integers with 0),
 * executes, synchronises and, when `output` is not NULL, copies the first
 * output as logical floats (count = its element count); tmc_prepared_execute
 * only executes and synchronises. gpu_us / cpu_us (optional) receive the
 * CUDA-event time and the host submit-to-completion time.
 * tmc_sequence_create captures the executions in order into one CUDA graph
 * (retaining them); tmc_sequence_execute replays it once synchronously;
 * tmc_sequence_launch enqueues `replays` replays on the runtime stream and
 * returns (tmc_runtime_synchronize waits). */
typedef struct tmc_kernel tmc_kernel;
typedef struct tmc_prepared tmc_prepared;
typedef struct tmc_sequence tmc_sequence;
int tmc_kernel_count(void);
int tmc_kernel_at(int index, const tmc_kernel **out);
int tmc_kernel_lookup(const char *name, const tmc_kernel **out);
int tmc_kernel_describe(const tmc_kernel *kernel, const char **name, int *inputs, int *outputs, int *constants,
                        const char **signature);
int tmc_prepare(tmc_runtime *rt, const tmc_kernel *kernel, tmc_buffer *const *inputs, int n_inputs,
                tmc_buffer *const *outputs, int n_outputs, size_t groups, size_t threads, const uint32_t *constants,
                int n_constants, tmc_prepared **out);
void tmc_prepared_destroy(tmc_prepared *prepared);
int tmc_prepared_run(tmc_prepared *prepared, float *output, size_t count, double *gpu_us, double *cpu_us);
int tmc_prepared_execute(tmc_prepared *prepared, double *gpu_us, double *cpu_us);
int tmc_sequence_create(tmc_runtime *rt, tmc_prepared *const *steps, int n, tmc_sequence **out);
void tmc_sequence_destroy(tmc_sequence *sequence);
int tmc_sequence_execute(tmc_sequence *sequence, double *gpu_us, double *cpu_us);
int tmc_sequence_launch(tmc_sequence *sequence, int replays);

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

/* Standalone RMSNorm, one CTA of `threads` per row (RMSNormOp, TensorIR.hpp:98-104;
 * emitRMSNorm, MetalEmitter.cpp:12-76; the frozen 256-thread baseline,
 * RMSNormBaseline.cpp:13-73, with threads == 0):
 *   y[r, c] = x[r, c] * rsqrt(mean_c x[r, :]^2 + eps) * gamma[c], fp32 accumulation.
 * x, gamma, y all fp32 (fp16 == 0) or all fp16 (fp16 != 0); x/y [rows, width]. */
int tmc_k_rmsnorm(const void *x, const void *gamma, void *y, int rows, int width, float eps, int fp16,
                  int threads, void *stream);

/* Fused graph regions of the TensorGraph path (formRegions,
 * PatternAnalyzer.cpp:32-132; emitFusion, FusionMetalEmitter.cpp:81-214), same
 * arithmetic: fp32, each intermediate node rounded to the storage type (all
 * buffers fp32 when fp16 == 0, fp16 otherwise).
 *   add_norm:    y = norm(T(x + b)) * w (+ c): RMSNorm (layer_norm == 0) or
 *                LayerNorm with variance max(E[v^2] - mean^2, 0) (c required);
 *                x, y [rows, width]; b [b_rows, width], b_rows 1 or rows;
 *                w, c [width].
 *   silu_mul:    y = T(T(silu(x)) * b), x, y [rows, width], b as above.
 *   linear_relu: y = T(max(T(T(a . w) + bias), 0)), a [m, k], w [k, n]
 *                (row-major K x N), bias [n], y [m, n]. */
int tmc_k_fused_add_norm(const void *x, const void *b, const void *w, const void *c, void *y, int rows, int width,
                         int b_rows, float eps, int layer_norm, int fp16, void *stream);
int tmc_k_fused_silu_mul(const void *x, const void *b, void *y, int rows, int width, int b_rows, int fp16,
                         void *stream);
int tmc_k_fused_linear_relu(const void *a, const void *w, const void *bias, void *y, int m, int k, int n, int fp16,
                            void *stream);

/* Decode GEMV y = x W^T with fp16 x, W and y, fp32 accumulation: replaces
 * emitDecodeGEMV / emitLinearBaseline (DecodeGEMVMetalEmitter.cpp:18-132).
 * x [rows, k], W [n, k], y [rows, n]; rows <= 8, k % 8 == 0. */
int tmc_k_gemv_f16(const void *x_f16, const void *w_f16, void *y_f16, int rows, int k, int n,
                   void *stream);

/* Same with fp32 output (no storage rounding). */
int tmc_k_gemv_f16_f32out(const void *x_f16, const void *w_f16, float *y, int rows, int k,
                          int n, void *stream);

/* Batched projection on tcgen05 tensor cores, y = x W^T with fp16 x [rows, k]
 * and W [n, k], fp32 accumulation in tensor memory, fp32 y [rows, n]:
 * replaces emitTiledGEMM (DecodeGEMVMetalEmitter.cpp:134-169), the
 * reference's batched linear layer. rows <= 256, k % 8 == 0, x and W 16-byte
 * aligned. `workspace` holds tmc_k_batched_gemm_workspace_bytes(n, k, rows)
 * bytes (split-K partials and tile tickets; the call clears the tickets). */
size_t tmc_k_batched_gemm_workspace_bytes(int n, int k, int rows);
int tmc_k_batched_gemm_f16_f32out(const void *x_f16, const void *w_f16, float *y, int rows, int k,
                                  int n, void *workspace, void *status, void *stream);

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
/* The same with the schedule chosen (tmc_k_paged_attention_f16 passes 0):
 * 0 automatic; 1 split-K over (splits, kv head, row) CTAs merged through
 * thread-block clusters (the latency schedule, few (row, kv head) pairs);
 * 2 streaming: one wave of persistent CTAs streams the 64-position tiles of
 * all pairs with a producer warp, pairs cut between CTAs merged through the
 * workspace (the throughput schedule; needs d 64 or 128, page_size % 16 == 0,
 * rows <= 1024 and a workspace of at least 2 * G * (d + 2) floats per
 * resident CTA, else TMC_ERR_UNSUPPORTED). Automatic picks 2 when it applies
 * and rows * hkv >= half the SM count. row_group 2: the rows are prefill rows of
 * one sequence at consecutive positions sharing one block-table row (the
 * decoder's prefill chunks); the streaming schedule then serves them in
 * groups of 16 / (hq / hkv) rows, reading each K/V tile once per group
 * (workspace: also 640 * 2 * 16 * (d + 2) floats); 1: rows one by one. */
int tmc_k_paged_attention_f16_ex(const void *q, void *out, const void *k_pool, const void *v_pool,
                                 const int32_t *block_table, int table_stride, const int32_t *table_rows,
                                 const int32_t *positions, int rows, int hq, int hkv, int d, int page_size,
                                 int pool_pages, int capacity, int max_splits, int min_chunk, void *workspace,
                                 uint32_t *counters, int schedule, int row_group, void *status, void *stream);

/* Allocation-free variant of tmc_k_paged_attention_f16, for callers that cannot
 * allocate device memory at call time (a host that hands all device memory to
 * its own pool up front, a runtime whose memory plan forbids allocation after
 * start-up, or a latency-critical path that cannot afford cudaMalloc's implicit
 * device synchronisation). This entry point has no counterpart in the
 * reference. Same arguments and results as tmc_k_paged_attention_f16 minus the
 * workspace and counters: the split partials and tickets live in one fixed
 * 8 MiB device array that the library reserves on every GPU that loads it,
 * until process exit. It calls no allocator.
 * Limit: with s = min(max_splits, 64) (the kernel never cuts a row into more
 * than 64 splits), rows*hq*s*(d+2)*4 bytes, rounded up to 256, plus rows*hkv*4
 * bytes must fit in 8 MiB (8388608); larger requests fail with
 * TMC_ERR_UNSUPPORTED before anything is launched (max_splits = 1 needs only
 * the tickets). The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress) with that device current; make that first call before
 * any stream capture. The address is kept for the life of the process: do not
 * call this entry point after cudaDeviceReset in the same process. All calls
 * share the array and it keeps the previous call's contents; the tickets are
 * cleared on `stream` before each launch, so calls that overlap on the GPU
 * (e.g. on different streams) race and must be serialised by the caller. */
int tmc_k_paged_attention_f16_noalloc(const void *q, void *out, const void *k_pool,
                                      const void *v_pool, const int32_t *block_table,
                                      int table_stride, const int32_t *table_rows,
                                      const int32_t *positions, int rows, int hq, int hkv, int d,
                                      int page_size, int pool_pages, int capacity, int max_splits,
                                      int min_chunk, void *status, void *stream);

/* Deterministic N(0, std^2) fp16 fill from a counter-based hash generator
 * (synthetic random-init weights without a host round trip). */
int tmc_k_fill_normal_f16(void *dst, size_t count, uint64_t seed, float mean, float stddev,
                          void *stream);


/* ---- decoder executor ----------------------------------------------------
 * tmc_decoder replaces tensor::runtime::CompiledDecoderLLM and
 * compileDecoderLLM (DecoderLLMExecutor.hpp:46-101) for fp16 storage. One
 * executor holds up to max_slots sequences (the reference holds one request per
 * executor and shares KV pools between executors, ServingRuntime.cpp:569-618).
 * Config fields follow DecoderLLMPlan / KVCachePlan (DecoderLLMPlan.hpp:9-22,
 * KVCachePlan.hpp:9-22) and DecoderLLMCompileOptions (DecoderLLMExecutor.hpp:19-29),
 * extended with kv_heads (grouped-query attention) and rope_theta. */
typedef struct {
  int hidden_size, heads, kv_heads, head_dim, intermediate_size, vocab_size, layers;
  int capacity;      /* KVCachePlan::capacity: positions per sequence */
  float epsilon;     /* DecoderLLMPlan::rmsNormEpsilon */
  double rope_theta;
  int max_rows;      /* tokens per step, 1..256 (> 8: tensor-core projections) */
  int max_slots;     /* sequences with KV state */
  int page_size;     /* DecoderLLMCompileOptions::kvPageSize; 0 = contiguous */
  int pool_pages;    /* 0 = max_slots * ceil(capacity / page_size) */
  int tp_rank, tp_size;
  int use_graphs, use_pdl;
} tmc_decoder_config;

typedef struct tmc_decoder tmc_decoder;

/* Decoder-only model manifests in the reference's export format
 * ("TMC_DECODER_LLM 1|2" text header + float32 payload beside it), read as
 * importDecoderLLMWorkload does (DecoderLLMImporter.cpp:154-281, written by
 * export_decoder_llm.py:554-595), with the same checks. tmc_manifest_tensor
 * gives a view of any named tensor (weights, RoPE tables, the exporter's
 * reference tokens / logits / KV caches) valid until tmc_manifest_close;
 * tmc_decoder_load_manifest loads every weight and the RoPE tables into a
 * decoder created with the manifest's dimensions (head_dim = hidden / heads) and
 * rejects a decoder whose dimensions differ. An optional header line
 * "ATTENTION <kv_heads> <rope_theta>" after CONFIG (this backend's extension for
 * grouped-query models) sets kv_heads and rope_theta; without it kv_heads =
 * heads and rope_theta = 10000, so the reference's manifests import unchanged.
 * Dtype tokens: "F32", "F16" or "BF16". */
typedef struct tmc_manifest tmc_manifest;
typedef struct {
  int version, batch, hidden_size, heads, head_dim, intermediate_size, vocab_size, layers, capacity;
  int prefill_length, decode_count;
  float epsilon;
  char requested_dtype[8], effective_dtype[8];
  int kv_heads;
  double rope_theta;
} tmc_manifest_info;
int tmc_manifest_open(const char *path, tmc_manifest **out);
void tmc_manifest_close(tmc_manifest *m);
int tmc_manifest_get_info(const tmc_manifest *m, tmc_manifest_info *info);
int tmc_manifest_tensor(const tmc_manifest *m, const char *name, const float **values, size_t *count);

/* formRegions (PatternAnalyzer.cpp:32-132) with analyze()'s topological order
 * (GraphAnalyzer.cpp:278-364), for a graph whose value types are already known:
 * which nodes run as one fused kernel (Add+RMSNorm, residual Add+LayerNorm,
 * SiLU*Mul, MatMul+Add+ReLU -> tmc_k_fused_add_norm / tmc_k_fused_silu_mul /
 * tmc_k_fused_linear_relu). Values 0..input_count-1 are the graph inputs; the
 * nodes are encoded as {op, operand count, operands...} (op numbered as the
 * reference's tensor::OpType), node i defining value input_count + i, in an
 * array of nodes_len ints; contiguous[v] != 0 when value v's storage is
 * contiguous (a Transpose view is not). Writes order[node_count] and the regions
 * as {kind (0 unfused, 1 Add+RMSNorm, 2 Add+LayerNorm, 3 SiLU*Mul,
 * 4 Linear+ReLU), #nodes, nodes..., #inputs, inputs..., #outputs, outputs...};
 * *written receives the ints needed (TMC_ERR_INVALID when above capacity). The
 * reference's rejections (a cycle, a fused region with several results) come
 * back as TMC_ERR_INVALID with its message. Host only: no device work. */
int tmc_plan_regions(int input_count, const int32_t *nodes, size_t nodes_len, int node_count,
                     const int32_t *outputs, int output_count, const int32_t *contiguous, int32_t *order,
                     int32_t *regions, size_t capacity, size_t *written);
/* ---- graph compilation (replaces compileGraph / CompiledGraph::run,
 * src/runtime/GraphExecutor.hpp:16-46, GraphExecutor.cpp:346-431) ----
 * A typed tensor graph is analysed (types inferred, views aliased), split into
 * regions as formRegions does, and each region bound to one of this library's
 * kernels (tmc_kernel_lookup names); compile prepares them and captures them
 * as one CUDA graph. Encoding:
 *   input_types: per graph input {dtype (TMC_F16 or TMC_F32), rank (1..4),
 *                dims...}, concatenated;
 *   nodes:       per node {op, #operands, operands..., #attributes,
 *                attributes...}, op numbered as the reference's
 *                tensor::OpType, node i defining value input_count + i;
 *                attributes: RMSNorm / LayerNorm {epsilon as float bits}
 *                (none: 1e-5), Transpose {first, second} (a 2-D swap),
 *                Reshape / View {dims...}.
 * Supported: Add, Mul (equal shapes or a broadcast last-axis row), MatMul
 * (2-D; an fp16 right-hand operand is also accepted under an fp32 left-hand
 * one, an extension over TensorIR's matching-dtype rule so weights can stay
 * fp16), RMSNorm, LayerNorm (fused behind its residual Add), ReLU, SiLU,
 * Transpose, Reshape, View; other ops are refused with TMC_ERR_UNSUPPORTED
 * naming the op. An RMSNorm whose only use is a MatMul against a Transpose
 * view of an fp16 [N, K] weight, with fp32 rows <= 4, runs inside that GEMV's
 * prologue (the C1 graph becomes one rmsnorm_gemv_f32 launch).
 * tmc_graph_plan is host only: it writes the launch plan as text, one line
 * per launch "kernel(vA, vB, ...) -> vC [region]", and sets *needed to its
 * size + 1. tmc_graph_run writes every input from logical floats (element
 * counts from the types), replays the graph synchronously and reads every
 * declared output as logical floats; tmc_graph_value_info gives any value's
 * type (dims: 4 int64). tmc_graph_input_buffer returns a new handle on an
 * input's device storage (release it with tmc_buffer_destroy) and
 * tmc_graph_launch enqueues replays without synchronising, for device-side
 * inputs. */
typedef struct tmc_graph tmc_graph;
int tmc_graph_plan(int input_count, const int32_t *input_types, size_t input_types_len, const int32_t *nodes,
                   size_t nodes_len, int node_count, const int32_t *outputs, int output_count, char *text,
                   size_t size, size_t *needed);
int tmc_graph_compile(tmc_runtime *rt, int input_count, const int32_t *input_types, size_t input_types_len,
                      const int32_t *nodes, size_t nodes_len, int node_count, const int32_t *outputs,
                      int output_count, tmc_graph **out);
void tmc_graph_destroy(tmc_graph *graph);
int tmc_graph_describe(const tmc_graph *graph, char *text, size_t size, size_t *needed);
int tmc_graph_value_info(const tmc_graph *graph, int value, int *dtype, int *rank, int64_t *dims,
                         size_t *elements);
int tmc_graph_run(tmc_graph *graph, const float *const *inputs, float *const *outputs, double *gpu_us,
                  double *cpu_us);
int tmc_graph_input_buffer(tmc_graph *graph, int input, tmc_buffer **out);
int tmc_graph_launch(tmc_graph *graph, int replays);

/* planGraph's buffer and launch decisions (KernelPlan.cpp:11-59) for the same
 * graph encoding: roles[v] = 0 graph input, 1 intermediate, 2 declared output
 * (an input that is also an output stays 0); alias_of[v] = the data operand a
 * view's result aliases, else -1; launches[] = the non-view nodes in
 * topological order (*launch_count of them). The reference's per-launch
 * threadgroup sizes are Metal dispatch geometry and have no counterpart: this
 * library's launchers choose their own grids. Host only. */
int tmc_plan_buffers(int input_count, const int32_t *nodes, size_t nodes_len, int node_count,
                     const int32_t *outputs, int output_count, int32_t *roles, int32_t *alias_of,
                     int32_t *launches, int *launch_count);

/* compileDecoderLLM (DecoderLLMExecutor.hpp:99-101): allocate weights, KV pools
 * and activations on the runtime's device. Weights start at zero (norms at 1). */
int tmc_decoder_create(tmc_runtime *rt, const tmc_decoder_config *cfg, tmc_decoder **out);
void tmc_decoder_destroy(tmc_decoder *dec);
/* Weights by the reference manifest's logical names (export_decoder_llm.py:531-547):
 * "embedding.weight", "final_norm.weight", "lm_head.weight", "rope.cosine",
 * "rope.sine", "layer{i}.{input_norm,q,k,v,o,post_norm,gate,up,down}.weight".
 * Values are the full logical tensor; each rank keeps its tensor-parallel shard.
 * (DecoderLLMImporter.cpp:154-281 reads the same names.) */
int tmc_decoder_load_weight(tmc_decoder *dec, const char *name, const float *values, size_t count);
int tmc_decoder_load_weight_f16(tmc_decoder *dec, const char *name, const uint16_t *bits,
                                size_t count);
int tmc_decoder_load_manifest(tmc_decoder *dec, const tmc_manifest *m);
/* Rank-local window of a logical weight as floats (count must match it). */
int tmc_decoder_read_weight(tmc_decoder *dec, const char *name, float *out, size_t count);
/* Synthetic random init: every matrix ~N(0, stddev^2) from a counter-based
 * generator indexed by the logical element, so shards agree with TP=1. */
int tmc_decoder_init_random(tmc_decoder *dec, uint64_t seed, float stddev);
/* CompiledDecoderLLM::prefill / prefillChunked (DecoderLLMExecutor.hpp:55-58):
 * count tokens of one sequence in max_rows chunks. logits: NULL or
 * [count, local_vocab] floats; next_token: NULL or the greedy token after the
 * last position. */
int tmc_decoder_prefill(tmc_decoder *dec, int slot, const int32_t *tokens, int count,
                        float *logits, int32_t *next_token);
/* Timing of the last tmc_decoder_prefill (the reference's prefill timing in
 * DecoderLLMExecutor.cpp:982-1034): gpu_us = device time from the first
 * chunk's input copy to the last chunk's token readback (CUDA events on the
 * executor stream); cpu_us = host time of the whole call. */
int tmc_decoder_prefill_timing(tmc_decoder *dec, double *gpu_us, double *cpu_us);
/* CompiledDecoderLLM::decode (DecoderLLMExecutor.hpp:59-60) for `rows`
 * sequences at once (distinct slots): stage length+1, run the step graph,
 * commit. logits: NULL or [rows, local_vocab]; next_tokens: [rows]. */
int tmc_decoder_decode(tmc_decoder *dec, const int32_t *slots, const int32_t *tokens, int rows,
                       float *logits, int32_t *next_tokens);
/* Greedy loop on the device: `steps` replays of the step graph, each feeding
 * its argmax back (the apps' host loop, decoder_llm_main.cpp:135-162, without
 * host round trips). tokens_out: [steps, rows]; gpu_us: optional event time. */
int tmc_decoder_generate(tmc_decoder *dec, const int32_t *slots, const int32_t *tokens, int rows,
                         int steps, int32_t *tokens_out, double *gpu_us);
/* CompiledDecoderLLM::currentLength (DecoderLLMExecutor.hpp:62). */
size_t tmc_decoder_current_length(tmc_decoder *dec, int slot);
/* readKeyPrefix / readValuePrefix (DecoderLLMExecutor.hpp:63-64):
 * [local_kv_heads, length, head_dim] floats each; count = that size. */
int tmc_decoder_read_kv(tmc_decoder *dec, int layer, int slot, float *key, float *value,
                        size_t count);
/* restoreKVCache (DecoderLLMExecutor.hpp:83): keys/values are
 * [layers, local_kv_heads, length, head_dim] for an empty slot. */
int tmc_decoder_restore_kv(tmc_decoder *dec, int slot, size_t length, const float *keys,
                           const float *values);
/* kvBlockTable (DecoderLLMExecutor.hpp:79-80): allocated physical pages. */
int tmc_decoder_block_table(tmc_decoder *dec, int slot, int32_t *out, size_t capacity,
                            size_t *count);
/* stageKVLength / commitKVLength / rollbackKVLength / releaseKVCache
 * (DecoderLLMExecutor.hpp:81-86). */
int tmc_decoder_stage_length(tmc_decoder *dec, int slot, size_t length);
int tmc_decoder_commit_length(tmc_decoder *dec, int slot, size_t length);
int tmc_decoder_rollback_length(tmc_decoder *dec, int slot, size_t length);
int tmc_decoder_release(tmc_decoder *dec, int slot);
/* modelStorageBytes / kvStorageBytes / activationStorageBytes (DecoderLLMExecutor.hpp:72-74). */
int tmc_decoder_storage(tmc_decoder *dec, size_t *model_bytes, size_t *kv_bytes,
                        size_t *activation_bytes);
/* Rank-local sizes: heads, kv heads, intermediate, vocab slice and its offset. */
int tmc_decoder_local_dims(tmc_decoder *dec, int *heads, int *kv_heads, int *intermediate,
                           int *vocab, int *vocab_offset);
/* KVPagePool counters (KVCacheState.hpp:28-35): capacity, used, peak,
 * allocations, releases. */
int tmc_decoder_pool_stats(tmc_decoder *dec, size_t *capacity, size_t *used, size_t *peak,
                           size_t *allocations, size_t *releases);
/* Host-side failure injection for tests: the next n page allocations fail. */
int tmc_decoder_inject_page_failures(tmc_decoder *dec, size_t n);
/* Kernel launches in one step and the step's algorithmic HBM bytes (weights +
 * KV reads/appends for the given per-row context lengths). */
int tmc_decoder_kernels_per_step(tmc_decoder *dec, int rows);
double tmc_decoder_step_bytes(tmc_decoder *dec, int rows, const int32_t *context_lengths);

/* Time one kernel kind of the decode step in isolation (kind: 0 QKV, 1
 * attention, 2 O projection, 3 gate/up, 4 down, 5 LM head): a CUDA graph of
 * `rounds` passes over every layer's launch with the real weights, replayed
 * between CUDA events on the executor's stream. Outputs the mean launch
 * duration, the algorithmic HBM bytes of one launch and launches per step.
 * Call after a decode/generate so the step inputs are staged. */
int tmc_decoder_profile_kernel(tmc_decoder *dec, int kind, int rows, int rounds, double *avg_us,
                               double *bytes_per_launch, int *launches_per_step);

/* Step timeline: capacity > 0 makes every kernel of later steps append one
 * record per CTA (4 x uint64: tag = ((layer << 8) | kind) << 32 | CTA index,
 * then global-timer nanoseconds at entry, after the dependency wait and
 * prologue, and at exit); 0 turns it off. tmc_decoder_read_trace copies up to
 * `capacity` records into `out` (4 uint64 each), reports how many were
 * collected, and clears them. Tracing is a profiling aid with no reference
 * counterpart (the reference records one GPU duration per command buffer,
 * MetalRuntime.mm:253-258). */
int tmc_decoder_set_trace(tmc_decoder *dec, size_t capacity);
int tmc_decoder_read_trace(tmc_decoder *dec, uint64_t *out, size_t capacity, size_t *count);

/* ---- tensor parallelism (NCCL over NVLink; no reference counterpart: the
 * reference is single-device, README.md:321) ----
 * Rank 0 creates the id and shares it with the other ranks out of band
 * (e.g. torch.distributed broadcast); every rank then attaches its executor. */
int tmc_nccl_unique_id(uint8_t *id, size_t nbytes);
int tmc_decoder_attach_nccl(tmc_decoder *dec, const uint8_t *id, size_t nbytes, int world,
                            int rank);

/* Tensor parallelism over peer memory, fused into the kernels (no reference
 * counterpart). Each rank exports the CUDA IPC handle of its exchange window
 * (TMC_EXCHANGE_HANDLE_BYTES bytes), the ranks share them out of band, and
 * every rank attaches all of them in rank order. From then on the O and down
 * GEMVs store their fp32 partial sums straight into every rank's window over
 * NVLink and the next kernel sums them in rank order after bounded flag waits
 * (a timeout surfaces as TMC_ERR_DEVICE_STATUS); the LM head exchanges its
 * packed argmax keys the same way. No collective library call remains in the
 * step. All ranks must run the same sequence of steps; release every rank's
 * decoder only after all ranks have synchronised. */
#define TMC_EXCHANGE_HANDLE_BYTES 64
int tmc_decoder_exchange_handle(tmc_decoder *dec, uint8_t *handle, size_t nbytes);
int tmc_decoder_attach_peers(tmc_decoder *dec, const uint8_t *handles, size_t nbytes_each, int world,
                             int rank);
/* The same for ranks driven by one process: ranks[r] is rank r's decoder
 * (ranks[rank] == dec), each on a device with peer access to dec's; their
 * windows are used directly. Each rank attaches once. */
int tmc_decoder_attach_local_peers(tmc_decoder *dec, tmc_decoder *const *ranks, int world, int rank);
/* Budgets of the decoder kernels' bounded waits, in ns of global time (0: the
 * defaults, 10 s for another rank's exchange flags and 1 s for the tensor-core
 * GEMM's mbarrier and split-tile waits). A wait that runs out is recorded in
 * the device status block, the kernel drains its own copies in flight, frees
 * its tensor memory and returns, and the call returns TMC_ERR_DEVICE_STATUS;
 * the runtime stays usable. */
int tmc_decoder_set_wait_budgets(tmc_decoder *dec, uint64_t peer_wait_ns, uint64_t local_wait_ns);

/* ---- continuous batching (replaces runContinuousBatch,
 * src/runtime/ServingRuntime.hpp:73-76, ServingRuntime.cpp:513-930) ----
 * Serves `count` requests on a decoder's sequence slots (its weights loaded,
 * every slot empty; page_size > 0 for a shared paged pool). Request i has the
 * prompt prompt_tokens[prompt_offsets[i] .. prompt_offsets[i + 1]), asks for
 * decode_counts[i] greedy tokens, and arrives at scheduler tick
 * arrival_ticks[i]. Per tick: resume preempted requests that fit, admit
 * arrived requests that fit (chunked prefill), preempt the active request with
 * the most pages while the next token does not fit (KV snapshot to the host),
 * one batched decode step, release finished requests, audit page isolation.
 * Outputs in request order: generated tokens at offset i + sum_{j<i}
 * decode_counts[j] (1 + decode_counts[i] each: the prefill's next token, then
 * one per decode step), ttft_us[i] (arrival -> first token), finish_us[i]
 * (arrival -> last token); prefill_logits [sum of prompt lengths, local vocab]
 * and decode_logits [sum of decode_counts, local vocab] when not NULL. `log`
 * (optional) receives the scheduler's event log, truncated to log_size. All
 * tensor-parallel ranks must pass the same requests (decisions depend only on
 * ticks and page counts). */
typedef struct tmc_serving_metrics {
  double total_time_us, tokens_per_second, prefill_gpu_us, decode_gpu_us;
  double scheduler_overhead_us, kv_management_overhead_us, preemption_overhead_us;
  double average_active_batch;
  uint64_t max_active_batch, preemptions, resumes, peak_pages, page_allocations, page_releases;
  uint64_t decode_submissions, decoded_tokens, prefill_tokens, ticks;
  uint64_t model_bytes, kv_pool_bytes, activation_bytes;
} tmc_serving_metrics;
int tmc_serving_run(tmc_decoder *dec, int count, const int32_t *prompt_offsets,
                    const int32_t *prompt_tokens, const int32_t *decode_counts,
                    const int32_t *arrival_ticks, int32_t *generated, double *ttft_us,
                    double *finish_us, float *prefill_logits, float *decode_logits,
                    tmc_serving_metrics *metrics, char *log, size_t log_size);

/* ---- generated kernels: contract, admission gate, registry (replace
 * makeKernelContract / serializeKernelContract, src/llm/KernelContract.hpp:54-65,
 * DecoderKernelContracts.cpp:129-245; admitGeneratedKernel,
 * src/runtime/GeneratedKernelAdmission.hpp:10-13, .cpp:204-318; KernelRegistry /
 * writeAdmittedKernel, src/runtime/KernelRegistry.hpp:10-38) ----
 * Patterns: decoder_gemv_<K>_<N> (K*N <= 8M), decoder_rope,
 * decoder_residual_rmsnorm, decoder_gated_mlp, each optionally suffixed _fp16.
 * tmc_kernel_contract_json writes the contract (semantics, buffer interface,
 * kernel signature, legal block sizes, tolerances, minimum speedup) as JSON
 * and sets *needed to its size + 1. tmc_admit_generated_kernel compiles CUDA
 * C++ `source` with NVRTC for sm_100a, checks the parameter layout, validates
 * every contract case against its fp64 references, runs two paired timing
 * rounds against the built-in template kernel (each must reach the minimum
 * speedup), validates again, and writes feedback JSON (and, when admitted,
 * the artifact JSON) to the given paths (NULL or "" to skip). *admitted is 1
 * when admitted; *speedup is the worst round's speedup (0 if not timed).
 * The registry loads every admitted artifact of a directory (recompiling
 * it) and launches one with device pointers in contract order. */
int tmc_kernel_contract_json(const char *pattern, char *out, size_t size, size_t *needed);
int tmc_admit_generated_kernel(const char *pattern, const char *source, int block_size,
                               const char *feedback_path, const char *artifact_path, int *admitted,
                               double *speedup, char *log, size_t log_size);
/* Decode GEMV tuning (replaces tuneDecodeGEMV / DecodeGEMVSelection,
 * src/planner/DecodeGEMVTuner.hpp:13-25, DecodeGEMVTuner.cpp:162-304):
 * decode candidates (prefill == 0, rows <= 8) are decode GEMV configurations
 * (K-split team 1/2/4/8, dynamic row scheduling); the prefill candidate
 * (rows <= 128) is the tcgen05 GEMM. Each is validated against fp64 (<= 64M
 * MACs; else the baseline's output, 9 samples) and admitted only with
 * >= 1.05x over the generic linear baseline in two paired rounds; the fastest
 * admitted one is selected. input [rows, k] and weight [n, k] are logical
 * values stored as fp16 (fp16_storage != 0) or fp32 (the candidates read fp16
 * weights, so fp32 storage keeps the baseline). */
typedef struct tmc_gemv_selection {
  int success, use_baseline, ks, dynamic, tensor_core;
  double conservative_speedup;
} tmc_gemv_selection;
int tmc_tune_decode_gemv(int rows, int k, int n, const float *input, const float *weight, int fp16_storage,
                         int prefill, tmc_gemv_selection *out, char *log, size_t log_size);

/* RMSNorm tuning (replaces tuneRMSNorm / TuningResult, RMSNormTuner.hpp:14-44,
 * RMSNormTuner.cpp:159-309): block-size candidates against the frozen
 * 256-thread baseline, fp64-validated (fp32 atol 1e-5 / rtol 1e-4, fp16 2e-3),
 * admitted at >= 1.05x in two paired rounds. `output` (rows * width floats,
 * may be NULL) receives the final validated execution of the selection. */
typedef struct tmc_rmsnorm_selection {
  int success, used_baseline, selected_threads;
  double speedup, max_abs_error;
} tmc_rmsnorm_selection;
int tmc_tune_rmsnorm(int rows, int width, float eps, int fp16, const float *input, const float *weight,
                     const int *candidate_threads, int candidates, tmc_rmsnorm_selection *out, float *output,
                     char *log, size_t log_size);

typedef struct tmc_registry tmc_registry;
int tmc_registry_create(tmc_registry **out);
void tmc_registry_destroy(tmc_registry *reg);
int tmc_registry_load(tmc_registry *reg, const char *directory, int *loaded, char *log, size_t log_size);
int tmc_registry_launch(tmc_registry *reg, const char *pattern, void *const *buffers, int count,
                        unsigned work_items, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* TMC_CUDA_H */
