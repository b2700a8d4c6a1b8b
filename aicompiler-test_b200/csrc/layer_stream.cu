// Layer streaming kernel for single-token decode (see layer_stream.cuh).
//
// Layout: one CTA per SM, 8 warps. Each warp owns a ring of S stages of 8 KB
// in shared memory (S = 3 when the staged activation vector leaves room, else
// 2), each stage with an mbarrier; lane 0 fills stages with cp.async.bulk
// copies of weight-row segments (a row of K fp16 values split into segments
// of at most 8 KB whose 16-byte chunk count is a multiple of 32) and the
// whole warp consumes them in the same order. Work units (one row, or the two
// rows of a RoPE / SwiGLU pair) are dealt to warps statically, unit u to the
// warp with global index u mod (8 x CTAs), warps numbered CTA-minor so every
// CTA gets an equal share of each phase to within one unit. A warp's fill
// sequence is all of its units of phase 0, then phase 1, ...; the fills for
// phase p + 1 are issued as soon as ring stages free up, i.e. while the warp
// still works on (or waits at the barrier after) phase p.
//
// Phase boundaries: a grid barrier (every warp of every CTA done with the
// phase: one arrival per CTA on a global counter, bounded acquire spin), then
// the next phase's prologue stages its activation vector into shared memory
// as fp16 (exact: every staged value is an fp16 storage value). Activations
// written in this kernel are read through L2 (ld.global.cg): other SMs wrote
// them, and this SM's L1 may hold older lines.
//
// Every wait is bounded (mbarrier waits about 1 s of SM clock, grid barriers
// 2 s of global time); a timeout reports kStatusWaitTimeout, the CTA stops
// computing, waits (bounded) for its own bulk copies still in flight, and
// exits.
#include "layer_stream.cuh"

#include <mutex>
#include <unordered_map>

#include "epilogue.cuh"
#include "mbarrier.cuh"

namespace tmc {
namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kStageBytes = 8192;
constexpr int kMaxStages = 3;
constexpr int kSegLaneChunks = kStageBytes / (32 * 16);  // 16-byte chunks per lane per stage
constexpr unsigned long long kBarrierBudgetNs = 2ull * 1000 * 1000 * 1000;
constexpr size_t kSmemLimit = 227 * 1024;

struct Shape {
  int N, K, C;     // rows, row length, 16-byte chunks per row
  int seg_chunks;  // chunks per segment (a multiple of 32)
  int nseg;        // segments per row
  int unit_rows;   // rows per work unit (2 for the pair epilogues)
  int units;
};

__device__ __forceinline__ Shape shape_of(const GemvParams &p) {
  Shape s;
  s.N = p.N;
  s.K = p.K;
  s.C = p.K >> 3;
  const int lane_chunks = (s.C + 31) >> 5;
  s.nseg = (lane_chunks + kSegLaneChunks - 1) / kSegLaneChunks;
  s.seg_chunks = ((lane_chunks + s.nseg - 1) / s.nseg) * 32;
  s.unit_rows = (p.epilogue == kEpiSwiGLU || p.epilogue == kEpiQKV) ? 2 : 1;
  s.units = (p.N + s.unit_rows - 1) / s.unit_rows;
  return s;
}

// Position in a warp's fill sequence.
struct Cursor {
  int ph;    // kStreamPhases once exhausted
  int unit;
  int r;     // row within the unit
  int seg;   // segment within the row
};

__device__ __forceinline__ void settle(Cursor &c, const Shape *sh, int gw) {
  while (c.ph < kStreamPhases && gw >= sh[c.ph].units) ++c.ph;
  c.unit = gw;
  c.r = 0;
  c.seg = 0;
}

__device__ __forceinline__ void advance(Cursor &c, const Shape *sh, int gw, int G) {
  const Shape &s = sh[c.ph];
  if (++c.seg < s.nseg) return;
  c.seg = 0;
  if (++c.r < s.unit_rows && c.unit * s.unit_rows + c.r < s.N) return;
  c.r = 0;
  c.unit += G;
  if (c.unit < s.units) return;
  ++c.ph;
  settle(c, sh, gw);
}

struct Smem {
  unsigned char *ring;       // [kWarps][S][kStageBytes]
  __half *xs;                // [max K] staged activations
  uint64_t *bars;            // [kWarps][S]
};

struct Warp {
  int w, lane, gw, G, S;
  unsigned int issued, consumed;  // fills of this warp
  Cursor prod, cons;
  float acc, first;               // running row sum; the pair's first row sum
  unsigned long long best;        // argmax key (LM head)
};

// Lane 0: fill the next stage of this warp's ring with the producer cursor's
// segment and advance the cursor.
__device__ __forceinline__ void issue_next(Warp &W, const Smem &sm, const Shape *sh, const __half *const *wptr) {
  if (W.prod.ph >= kStreamPhases) return;
  const Shape &s = sh[W.prod.ph];
  const int row = W.prod.unit * s.unit_rows + W.prod.r;
  const int c0 = W.prod.seg * s.seg_chunks;
  const int n = min(s.seg_chunks, s.C - c0);
  const int stage = static_cast<int>(W.issued % static_cast<unsigned int>(W.S));
  if (W.lane == 0) {
    const char *src = reinterpret_cast<const char *>(wptr[W.prod.ph] + (size_t)row * s.K) + (size_t)c0 * 16;
    uint64_t *bar = sm.bars + W.w * W.S + stage;
    mbar_arrive_expect_tx(bar, static_cast<uint32_t>(n) * 16u);
    bulk_g2s(sm.ring + ((size_t)W.w * W.S + stage) * kStageBytes, src, static_cast<uint32_t>(n) * 16u, bar);
  }
  ++W.issued;
  advance(W.prod, sh, W.gw, W.G);
}

// The CTA's grid barrier after `phase`: every thread's stores of the phase are
// ordered before one arrival per CTA; false if the others did not arrive in time.
__device__ __forceinline__ bool grid_barrier(const StreamParams &p, int phase, int *flag) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(p.sync, 1u);
    const unsigned int target = static_cast<unsigned int>(phase + 1) * gridDim.x;
    *flag = wait_count_geq_gpu(p.sync, target, kBarrierBudgetNs) ? 0 : 1;
    if (*flag) report_status(p.phase[0].status, kStatusWaitTimeout, kWhereStream, phase, blockIdx.x);
  }
  __syncthreads();
  return *flag == 0;
}

// Stage the phase's activation vector (fp16, exact) exactly as the decode
// GEMV's prologue computes it (stage_x, M = 1, 256 threads): kProF16 copies
// the fp16 input; kProF16Norm applies RMSNorm with the same per-thread sums,
// block reduction and rounding.
__device__ __forceinline__ void stage_vector(const GemvParams &p, __half *xs, float *red) {
  const int K = p.K;
  const int nvec = K >> 3;
  const uint4 *src = reinterpret_cast<const uint4 *>(static_cast<const __half *>(p.x));
  uint4 *dst = reinterpret_cast<uint4 *>(xs);
  if (p.prologue != kProF16Norm) {
    for (int v = threadIdx.x; v < nvec; v += blockDim.x) dst[v] = __ldcg(src + v);
    return;
  }
  float ss = 0.0f;
#pragma unroll 2
  for (int v = threadIdx.x; v < nvec; v += blockDim.x) {
    const uint4 raw = __ldcg(src + v);
    dst[v] = raw;
    float f[8];
    float2 t;
    t = half2_bits_to_float2(raw.x); f[0] = t.x; f[1] = t.y;
    t = half2_bits_to_float2(raw.y); f[2] = t.x; f[3] = t.y;
    t = half2_bits_to_float2(raw.z); f[4] = t.x; f[5] = t.y;
    t = half2_bits_to_float2(raw.w); f[6] = t.x; f[7] = t.y;
#pragma unroll
    for (int j = 0; j < 8; ++j) ss = fmaf(f[j], f[j], ss);
  }
  ss = block_sum(ss, red);
  const float inv = 1.0f / sqrtf(ss / static_cast<float>(K) + p.eps);
  const uint4 *g = static_cast<const uint4 *>(p.gamma);
#pragma unroll 2
  for (int v = threadIdx.x; v < nvec; v += blockDim.x) {
    const uint4 graw = g[v], xraw = dst[v];
    const uint32_t gw[4] = {graw.x, graw.y, graw.z, graw.w};
    const uint32_t xw[4] = {xraw.x, xraw.y, xraw.z, xraw.w};
    uint32_t out[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 gf = half2_bits_to_float2(gw[q]);
      const float2 xf = half2_bits_to_float2(xw[q]);
      __half2 h = __floats2half2_rn(round_half(__fmul_rn(__fmul_rn(xf.x, inv), gf.x)),
                                   round_half(__fmul_rn(__fmul_rn(xf.y, inv), gf.y)));
      out[q] = *reinterpret_cast<uint32_t *>(&h);
    }
    dst[v] = make_uint4(out[0], out[1], out[2], out[3]);
  }
}

// A finished row sum (all lanes hold it): the phase's epilogue.
template <int PH>
__device__ __forceinline__ void finish_row(const StreamParams &p, Warp &W, int row, int r, float sum) {
  const GemvParams &g = p.phase[PH];
  switch (g.epilogue) {
    case kEpiResidual:
      if (W.lane == 0) {
        // h = half(h + half(acc)); h was written by other CTAs earlier in this kernel.
        const __half res = __ldcg(g.residual + row);
        g.y_f16[row] = residual_value(res, sum);
      }
      break;
    case kEpiSwiGLU:
    case kEpiQKV:
      if (r == 0) {
        W.first = sum;
      } else if (W.lane == 0) {
        epilogue_pair(g, row - 1, 0, W.first, sum);
      }
      break;
    case kEpiArgmax: {
      const float v = round_half(sum);
      if (W.lane == 0 && g.y_f32 != nullptr) g.y_f32[row] = v;
      const unsigned long long key = argmax_key(v, g.vocab_offset + row);
      W.best = key > W.best ? key : W.best;
      break;
    }
    default:
      break;
  }
}

// Consume every fill of phase PH from this warp's ring (the phase's
// activations are staged in xs), refilling each stage with the next fill of
// the sequence. False on an mbarrier timeout.
template <int PH>
__device__ __forceinline__ bool consume_phase(const StreamParams &p, Warp &W, const Smem &sm, const Shape *sh,
                                              const __half *const *wptr) {
  const Shape &s = sh[PH];
  while (W.cons.ph == PH) {
    const int stage = static_cast<int>(W.consumed % static_cast<unsigned int>(W.S));
    const uint32_t parity = (W.consumed / static_cast<unsigned int>(W.S)) & 1u;
    if (!mbar_wait(sm.bars + W.w * W.S + stage, parity)) {
      if (W.lane == 0) report_status(p.phase[0].status, kStatusWaitTimeout, kWhereStream, PH, blockIdx.x);
      return false;
    }
    const uint4 *wv = reinterpret_cast<const uint4 *>(sm.ring + ((size_t)W.w * W.S + stage) * kStageBytes);
    const uint4 *xv4 = reinterpret_cast<const uint4 *>(sm.xs);
    const int c0 = W.cons.seg * s.seg_chunks;
    const int n = min(s.seg_chunks, s.C - c0);
    float acc = W.acc;
    for (int j = W.lane; j < n; j += 32) {
      const uint4 wq = wv[j];
      const uint4 xq = xv4[c0 + j];
      float xf[8];
      float2 t;
      t = half2_bits_to_float2(xq.x); xf[0] = t.x; xf[1] = t.y;
      t = half2_bits_to_float2(xq.y); xf[2] = t.x; xf[3] = t.y;
      t = half2_bits_to_float2(xq.z); xf[4] = t.x; xf[5] = t.y;
      t = half2_bits_to_float2(xq.w); xf[6] = t.x; xf[7] = t.y;
      acc = gemv_dot8(wq, xf, acc);
    }
    W.acc = acc;
    const bool row_done = W.cons.seg == s.nseg - 1;
    const int row = W.cons.unit * s.unit_rows + W.cons.r;
    const int r = W.cons.r;
    // The stage is free once every lane has read it: refill it (async-proxy
    // writes after generic-proxy reads of the same shared memory).
    __syncwarp();
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    ++W.consumed;
    issue_next(W, sm, sh, wptr);
    advance(W.cons, sh, W.gw, W.G);
    if (row_done) {
      const float sum = warp_sum(W.acc);
      W.acc = 0.0f;
      finish_row<PH>(p, W, row, r, sum);
    }
  }
  return true;
}

template <int PH>
__device__ __forceinline__ bool run_phase(const StreamParams &p, Warp &W, const Smem &sm, const Shape *sh,
                                          const __half *const *wptr, float *red, int *flag) {
  if (PH > 0 && !grid_barrier(p, PH - 1, flag)) return false;
  stage_vector(p.phase[PH], sm.xs, red);
  __syncthreads();
  const bool ok = consume_phase<PH>(p, W, sm, sh, wptr);
  // CTA-uniform outcome (a timed-out warp stops the CTA).
  if (!ok) *flag = 1;
  __syncthreads();
  return *flag == 0;
}

__global__ void __launch_bounds__(kThreads, 1) layer_stream_kernel(const StreamParams p, int stages) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  __shared__ Shape sh[kStreamPhases];
  __shared__ const __half *wptr[kStreamPhases];
  __shared__ float red[32];
  __shared__ unsigned long long warp_best[kWarps];
  __shared__ int flag, is_last;

  const unsigned long long t_entry = p.phase[0].trace.records ? global_ns() : 0ull;
  if (threadIdx.x < kStreamPhases) {
    sh[threadIdx.x] = shape_of(p.phase[threadIdx.x]);
    wptr[threadIdx.x] = p.phase[threadIdx.x].W;
  }
  if (threadIdx.x == 0) flag = 0;
  Smem sm;
  sm.ring = smem_raw;
  sm.xs = reinterpret_cast<__half *>(smem_raw + (size_t)kWarps * stages * kStageBytes);
  int max_k = 0;
#pragma unroll
  for (int q = 0; q < kStreamPhases; ++q) max_k = max(max_k, p.phase[q].K);
  sm.bars = reinterpret_cast<uint64_t *>(reinterpret_cast<unsigned char *>(sm.xs) + ((size_t)max_k * 2 + 15) / 16 * 16);

  Warp W;
  W.w = threadIdx.x >> 5;
  W.lane = threadIdx.x & 31;
  W.gw = W.w * gridDim.x + blockIdx.x;
  W.G = kWarps * gridDim.x;
  W.S = stages;
  W.issued = W.consumed = 0;
  W.acc = W.first = 0.0f;
  W.best = 0ull;
  if (W.lane == 0)
    for (int s = 0; s < stages; ++s) mbar_init(sm.bars + W.w * stages + s, 1);
  fence_barrier_init();
  __syncthreads();
  W.prod.ph = 0;
  settle(W.prod, sh, W.gw);
  W.cons = W.prod;
  // Weights never change: the first fills go out before the dependency wait.
  for (int s = 0; s < stages; ++s) issue_next(W, sm, sh, wptr);
  pdl_wait();
  pdl_launch_dependents();
  const unsigned long long t_ready = p.phase[0].trace.records ? global_ns() : 0ull;

  bool ok = run_phase<0>(p, W, sm, sh, wptr, red, &flag);
  ok = ok && run_phase<1>(p, W, sm, sh, wptr, red, &flag);
  ok = ok && run_phase<2>(p, W, sm, sh, wptr, red, &flag);
  ok = ok && run_phase<3>(p, W, sm, sh, wptr, red, &flag);

  const GemvParams &last = p.phase[kStreamPhases - 1];
  if (ok && last.epilogue == kEpiArgmax) {
    if (W.lane == 0) warp_best[W.w] = W.best;
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned long long b = 0ull;
      for (int w = 0; w < kWarps; ++w) b = warp_best[w] > b ? warp_best[w] : b;
      if (b != 0ull) atomicMax(last.argmax_keys, b);
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) is_last = atomicAdd(last.argmax_counter, 1u) == gridDim.x - 1 ? 1 : 0;
    __syncthreads();
    if (is_last) {
      __threadfence();
      argmax_finalize(last, threadIdx.x, [] { __syncthreads(); });
    }
  }
  // Drain: no bulk copy may still target this CTA's shared memory at exit
  // (only after a timeout are fills left unconsumed).
  while (W.consumed < W.issued) {
    const int stage = static_cast<int>(W.consumed % static_cast<unsigned int>(W.S));
    if (!mbar_wait(sm.bars + W.w * W.S + stage, (W.consumed / static_cast<unsigned int>(W.S)) & 1u)) break;
    ++W.consumed;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // The last CTA out resets the barrier for the next launch of this site.
    if (atomicAdd(p.sync + 32, 1u) == gridDim.x - 1) {
      atomicExch(p.sync, 0u);
      atomicExch(p.sync + 32, 0u);
    }
  }
  trace_emit(p.phase[0].trace, t_entry, t_ready);
}

int max_k_of(const StreamParams &p) {
  int k = 0;
  for (int q = 0; q < kStreamPhases; ++q) k = p.phase[q].K > k ? p.phase[q].K : k;
  return k;
}

int stages_for(const StreamParams &p) {
  const size_t xs = ((size_t)max_k_of(p) * 2 + 15) / 16 * 16;
  for (int s = kMaxStages; s >= 2; --s) {
    const size_t total = (size_t)kWarps * s * kStageBytes + xs + (size_t)kWarps * s * 8;
    if (total <= kSmemLimit - 2048) return s;  // room for the static shared memory
  }
  return 0;
}

}  // namespace

bool layer_stream_fits(const StreamParams &p) {
  for (int q = 0; q < kStreamPhases; ++q) {
    const GemvParams &g = p.phase[q];
    if (g.M != 1 || g.K <= 0 || (g.K & 7) != 0 || g.N <= 0 || g.W == nullptr) return false;
    if ((g.epilogue == kEpiSwiGLU || g.epilogue == kEpiQKV) && (g.N & 1)) return false;
    if (g.prologue != kProF16 && g.prologue != kProF16Norm) return false;
    if (g.xchg.world > 0) return false;
  }
  const GemvParams &o = p.phase[0], &d = p.phase[2];
  if (o.epilogue != kEpiResidual || d.epilogue != kEpiResidual || p.phase[1].epilogue != kEpiSwiGLU) return false;
  const int last = p.phase[3].epilogue;
  if (last != kEpiQKV && last != kEpiArgmax) return false;
  return stages_for(p) >= 2;
}

cudaError_t launch_layer_stream(const StreamParams &p, cudaStream_t stream, bool pdl, int num_sms) {
  if (!layer_stream_fits(p) || p.sync == nullptr) return cudaErrorInvalidValue;
  const int stages = stages_for(p);
  const size_t smem = (size_t)kWarps * stages * kStageBytes + ((size_t)max_k_of(p) * 2 + 15) / 16 * 16 +
                      (size_t)kWarps * stages * 8;
  static std::mutex mu;
  static std::unordered_map<int, size_t> configured;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (configured[dev] < smem) {
      e = cudaFuncSetAttribute(layer_stream_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
      configured[dev] = smem;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(num_sms);  // one CTA per SM: every CTA must be resident for the grid barriers
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, layer_stream_kernel, p, stages);
}

}  // namespace tmc
