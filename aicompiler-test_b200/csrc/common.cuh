// Shared device helpers for the sm_100a decode kernels.
//
// Every kernel in this library follows three rules:
//  * weights are immutable and may be read before the programmatic-dependency
//    wait (griddepcontrol.wait); nothing that an earlier kernel writes is read,
//    and nothing is written, before that wait;
//  * range and validity failures never trap: they set a word in the device
//    status block (TmcDeviceStatus) and skip the access, and the host reads the
//    block after synchronising (the Metal kernels of the reference silently
//    `return` in the same situations, e.g. KVCacheMetalEmitter.cpp:149-150,268);
//  * every spin-wait is bounded by a clock budget and reports a timeout code.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace tmc {

// Device status block written by kernels (first error wins).
struct TmcDeviceStatus {
  int code;   // 0 = ok, else one of kStatus*
  int where;  // kernel id that reported it
  int info0;  // offending index / value
  int info1;
};

enum : int {
  kStatusOk = 0,
  kStatusTokenRange = 1,      // token id outside [0, vocabulary)
  kStatusLengthRange = 2,     // valid length outside [1, capacity]
  kStatusPageMissing = 3,     // block table entry < 0 for a used logical page
  kStatusPageRange = 4,       // physical page >= pool pages
  kStatusWaitTimeout = 5,     // a bounded mbarrier wait ran out
  kStatusShape = 6,           // launch-time shape mismatch caught on device
};

enum : int {
  kWhereGemv = 1,
  kWhereAttention = 2,
  kWhereEmbedding = 3,
  kWhereLMHead = 4,
  kWhereAppend = 5,
  kWhereMisc = 6,
  kWhereGemm = 7,
  kWhereExchange = 8,  // a peer's flag did not arrive in time (info0 = source rank)
};

__device__ __forceinline__ void report_status(TmcDeviceStatus *s, int code, int where,
                                              int info0, int info1 = 0) {
  if (s == nullptr) return;
  if (atomicCAS(&s->code, 0, code) == 0) {
    s->where = where;
    s->info0 = info0;
    s->info1 = info1;
  }
}

// ---- tracing ---------------------------------------------------------------------
// Optional per-CTA timeline of a decode step: when a kernel's `trace` pointer
// is set, thread 0 of every CTA appends one record (global nanosecond timer at
// entry, after the programmatic-dependency wait, and at exit).
struct TraceRecord {
  unsigned long long tag;      // (kernel tag << 32) | CTA linear index
  unsigned long long t_entry;
  unsigned long long t_ready;  // after griddepcontrol.wait and the prologue
  unsigned long long t_exit;
};

struct TraceSink {
  TraceRecord *records;
  unsigned int *count;
  unsigned int capacity;
  unsigned int tag;
};

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void trace_emit(const TraceSink &sink, unsigned long long t_entry,
                                           unsigned long long t_ready) {
  if (sink.records == nullptr || threadIdx.x != 0) return;
  const unsigned int i = atomicAdd(sink.count, 1u);
  if (i >= sink.capacity) return;
  const unsigned int cta = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
  TraceRecord r;
  r.tag = (static_cast<unsigned long long>(sink.tag) << 32) | cta;
  r.t_entry = t_entry;
  r.t_ready = t_ready;
  r.t_exit = global_ns();
  sink.records[i] = r;
}

// ---- programmatic dependent launch (PDL) -------------------------------------
// Both are no-ops when the kernel was not launched with the programmatic
// stream-serialization attribute.
__device__ __forceinline__ void pdl_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- system-scope flags (peer memory over NVLink) ----------------------------
__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int *p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(unsigned int *p, unsigned int v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Add with acquire-release semantics at GPU scope; returns the old value.
__device__ __forceinline__ unsigned int atomic_add_acq_rel_gpu(unsigned int *p, unsigned int v) {
  unsigned int old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
// Wait until *flag >= value (wrap-safe), at most budget_ns of global time.
__device__ __forceinline__ bool wait_flag_geq(const unsigned int *flag, unsigned int value,
                                              unsigned long long budget_ns) {
  const unsigned long long t0 = global_ns();
  while (static_cast<int>(ld_acquire_sys(flag) - value) < 0) {
    if (global_ns() - t0 > budget_ns) return false;
    __nanosleep(32);
  }
  return true;
}

// GPU-scope acquire load and bounded wait (counters shared by the CTAs of one
// kernel on one GPU).
__device__ __forceinline__ unsigned int ld_acquire_gpu(const unsigned int *p) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ bool wait_count_geq_gpu(const unsigned int *counter, unsigned int value,
                                                   unsigned long long budget_ns) {
  const unsigned long long t0 = global_ns();
  while (ld_acquire_gpu(counter) < value) {
    if (global_ns() - t0 > budget_ns) return false;
  }
  return true;
}

// ---- global loads ----------------------------------------------------------
// L2 policy for data read once per step (weights): its lines are replaced
// first, so the lines that are reused -- activations, KV pages, block tables,
// counters and the kernels' own code -- stay in L2 while gigabytes stream by.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
// Streaming 16-byte load of immutable data: read-only path, no L1 allocation,
// under the L2 cache policy `pol`.
__device__ __forceinline__ uint4 ldg_stream(const void *p, uint64_t pol) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p), "l"(pol));
  return v;
}

__device__ __forceinline__ float2 half2_bits_to_float2(uint32_t bits) {
  __half2 h = *reinterpret_cast<__half2 *>(&bits);
  return __half22float2(h);
}

// Round a float to fp16 storage and back (round-to-nearest-even).
__device__ __forceinline__ float round_half(float v) {
  return __half2float(__float2half_rn(v));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum for blockDim.x <= 1024; `scratch` holds >= 32 floats.
__device__ __forceinline__ float block_sum(float v, float *scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float r = lane < nwarps ? scratch[lane] : 0.0f;
  r = warp_sum(r);
  return r;
}

// Orderable 64-bit argmax key: larger value wins, then the smaller index
// (the tie rule of emitTokenArgmax, TransformerDecodeMetalEmitter.cpp:198-257,
// and of torch.argmax on the reference's fp16 logits). Key 0 is "empty".
__device__ __forceinline__ unsigned long long argmax_key(float value, int index) {
  uint32_t b = __float_as_uint(value);
  // NaN never wins: map it below every finite value.
  if ((b & 0x7fffffffu) > 0x7f800000u) b = 0xff800000u;  // -inf
  const uint32_t ordered = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return (static_cast<unsigned long long>(ordered) << 32) |
         static_cast<unsigned long long>(0xffffffffu - static_cast<uint32_t>(index));
}
__device__ __forceinline__ int argmax_key_index(unsigned long long key) {
  return static_cast<int>(0xffffffffu - static_cast<uint32_t>(key & 0xffffffffull));
}
__device__ __forceinline__ float argmax_key_value(unsigned long long key) {
  const uint32_t ordered = static_cast<uint32_t>(key >> 32);
  const uint32_t b = (ordered & 0x80000000u) ? (ordered & 0x7fffffffu) : ~ordered;
  return __uint_as_float(b);
}

__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, v, o);
    v = other > v ? other : v;
  }
  return v;
}

}  // namespace tmc
