// GQA split-K decode attention for sm_100a.
//
// Grid (max_splits, Hkv, rows), 128 threads. A CTA owns one KV head of one
// query row and a contiguous chunk of key positions, and serves all G = Hq/Hkv
// query heads of that KV head, so every K/V row is read from HBM once per
// query row (GQA reuse). K/V rows (D*2 bytes each) are gathered through the
// block table with 1-D TMA bulk copies (cp.async.bulk) into a two-stage
// shared-memory ring, completion tracked by mbarriers with bounded waits.
// Per tile: scores (one thread per (head, position), rotated chunk order so
// shared-memory reads are conflict-free), an online-softmax update per head,
// then P.V with each thread owning E output features of one head. Splits write
// (m, l, acc) partials; the last CTA of a (row, KV head) combines them
// (atomic ticket), so no second launch is needed.
#include "attention.cuh"

#include <cmath>
#include <mutex>
#include <string>
#include <unordered_map>

#include "api_util.hpp"
#include "tmc_cuda.h"

namespace tmc {
namespace {

constexpr int kThreads = 128;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// Bounded wait (about one second of SM clock); false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
  const long long start = clock64();
  const uint32_t addr = smem_u32(bar);
  while (true) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return true;
    if (clock64() - start > (1ll << 31)) return false;
  }
}

__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

template <int D, int G>
struct Cfg {
  static constexpr int T = (128 / G) > 64 ? 64 : (128 / G);  // positions per tile
  static constexpr int E = (G * D / kThreads) > 1 ? (G * D / kThreads) : 1;  // outputs per thread
  static constexpr int kChunks = D / 8;                       // 16-byte chunks per row
  static constexpr size_t kStageBytes = (size_t)T * D * 2;    // one of K or V per stage
  static constexpr size_t smem_bytes() {
    return 4 * kStageBytes                 // sK[2], sV[2]
           + (size_t)G * D * 4             // sQ
           + (size_t)G * T * 4             // sS
           + 3 * (size_t)G * 4 + 16        // sM, sL, sR (+pad)
           + 2 * (size_t)T * 4             // sValid[2]
           + 2 * 8 + 16;                   // bars
  }
};

template <int D, int G>
__global__ void __launch_bounds__(kThreads) attention_kernel(const AttentionParams p) {
  using C = Cfg<D, G>;
  constexpr int T = C::T, E = C::E;
  extern __shared__ __align__(128) unsigned char smem[];
  __half *sK = reinterpret_cast<__half *>(smem);
  __half *sV = sK + 2 * T * D;
  float *sQ = reinterpret_cast<float *>(sV + 2 * T * D);
  float *sS = sQ + G * D;
  float *sM = sS + G * T;
  float *sL = sM + G;
  float *sR = sL + G;
  int *sValid = reinterpret_cast<int *>(sR + G + 4);
  uint64_t *bars = reinterpret_cast<uint64_t *>(
      (reinterpret_cast<uintptr_t>(sValid + 2 * T) + 15) & ~uintptr_t(15));
  __shared__ int is_last;

  const int split = blockIdx.x, kvh = blockIdx.y, row = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  pdl_wait();
  pdl_launch_dependents();

  const int pos = p.positions[row];
  if (pos < 0 || pos >= p.capacity) {
    if (split == 0 && kvh == 0 && tid == 0)
      report_status(p.status, kStatusLengthRange, kWhereAttention, pos, row);
    return;
  }
  const int len = pos + 1;
  int nsplit = (len + p.min_chunk - 1) / p.min_chunk;
  if (nsplit > p.max_splits) nsplit = p.max_splits;
  if (nsplit < 1) nsplit = 1;
  int chunk = (len + nsplit - 1) / nsplit;
  chunk = (chunk + T - 1) / T * T;
  const int active = (len + chunk - 1) / chunk;
  if (split >= active) return;
  const int begin = split * chunk;
  const int end = min(len, begin + chunk);
  const int ntiles = (end - begin + T - 1) / T;
  const int *table = p.block_table + (size_t)p.table_rows[row] * p.table_stride;

  // Query heads of this KV head -> fp32 shared memory.
  for (int i = tid; i < G * D; i += kThreads) {
    const int g = i / D, d = i % D;
    sQ[i] = __half2float(p.q[(size_t)row * p.q_stride + (size_t)(kvh * G + g) * D + d]);
  }
  if (tid < G) {
    sM[tid] = -INFINITY;
    sL[tid] = 0.0f;
  }
  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  // Warp 0 gathers tile `t` into stage `t & 1`.
  auto issue = [&](int t) {
    const int stage = t & 1;
    const int p0 = begin + t * T;
    int ok[(T + 31) / 32];
    int nvalid = 0;
#pragma unroll
    for (int j = 0; j < (T + 31) / 32; ++j) {
      const int lp = lane + 32 * j;
      const int position = p0 + lp;
      int v = 0;
      if (lp < T && position < end) {
        const int logical = position / p.page_size;
        const int page = logical < p.table_stride ? table[logical] : -1;
        if (page < 0) {
          report_status(p.status, kStatusPageMissing, kWhereAttention, logical, row);
        } else if (page >= p.pool_pages) {
          report_status(p.status, kStatusPageRange, kWhereAttention, page, row);
        } else {
          v = 1;
        }
      }
      ok[j] = v;
      if (lp < T) sValid[stage * T + lp] = v;
      nvalid += __popc(__ballot_sync(0xffffffffu, v));
    }
    __syncwarp();  // sValid writes of all lanes precede the arrive (release)
    if (lane == 0) mbar_arrive_expect_tx(&bars[stage], static_cast<uint32_t>(nvalid) * D * 2 * 2);
    __syncwarp();
#pragma unroll
    for (int j = 0; j < (T + 31) / 32; ++j) {
      const int lp = lane + 32 * j;
      if (!ok[j]) continue;
      const int position = p0 + lp;
      const int page = table[position / p.page_size];
      const size_t off =
          (((size_t)page * p.hkv + kvh) * p.page_size + position % p.page_size) * D;
      bulk_g2s(sK + ((size_t)stage * T + lp) * D, p.k_pool + off, D * 2, &bars[stage]);
      bulk_g2s(sV + ((size_t)stage * T + lp) * D, p.v_pool + off, D * 2, &bars[stage]);
    }
  };

  if (warp == 0) {
    issue(0);
    if (ntiles > 1) issue(1);
  }

  // PV ownership: head pg, features [pd, pd + E).
  const int pg = tid / (D / E);
  const int pd = (tid % (D / E)) * E;
  const bool pv_active = pg < G;
  float acc[E];
#pragma unroll
  for (int e = 0; e < E; ++e) acc[e] = 0.0f;

  for (int t = 0; t < ntiles; ++t) {
    const int stage = t & 1;
    if (!mbar_wait(&bars[stage], (t >> 1) & 1)) {
      if (tid == 0) report_status(p.status, kStatusWaitTimeout, kWhereAttention, t, row);
      return;
    }
    const __half *k = sK + (size_t)stage * T * D;
    const __half *v = sV + (size_t)stage * T * D;
    // Scores.
    if (tid < G * T) {
      const int g = tid / T, lp = tid % T;
      float s = -INFINITY;
      if (sValid[stage * T + lp]) {
        const float *qg = sQ + g * D;
        const uint4 *krow = reinterpret_cast<const uint4 *>(k + (size_t)lp * D);
        float dot = 0.0f;
#pragma unroll
        for (int cc = 0; cc < C::kChunks; ++cc) {
          const int c = (cc + lp) % C::kChunks;
          const uint4 u = krow[c];
          const float4 qa = reinterpret_cast<const float4 *>(qg)[2 * c];
          const float4 qb = reinterpret_cast<const float4 *>(qg)[2 * c + 1];
          float2 f;
          f = half2_bits_to_float2(u.x); dot = fmaf(qa.x, f.x, dot); dot = fmaf(qa.y, f.y, dot);
          f = half2_bits_to_float2(u.y); dot = fmaf(qa.z, f.x, dot); dot = fmaf(qa.w, f.y, dot);
          f = half2_bits_to_float2(u.z); dot = fmaf(qb.x, f.x, dot); dot = fmaf(qb.y, f.y, dot);
          f = half2_bits_to_float2(u.w); dot = fmaf(qb.z, f.x, dot); dot = fmaf(qb.w, f.y, dot);
        }
        s = dot * p.scale;
      }
      sS[g * T + lp] = s;
    }
    __syncthreads();
    // Online softmax update, one warp per head.
    for (int g = warp; g < G; g += kThreads / 32) {
      float mx = -INFINITY;
      for (int lp = lane; lp < T; lp += 32) mx = fmaxf(mx, sS[g * T + lp]);
      mx = warp_max(mx);
      const float m_old = sM[g];
      const float m_new = fmaxf(m_old, mx);
      float sum = 0.0f;
      for (int lp = lane; lp < T; lp += 32) {
        const float s = sS[g * T + lp];
        const float e = (s == -INFINITY) ? 0.0f : expf(s - m_new);
        sS[g * T + lp] = e;
        sum += e;
      }
      sum = warp_sum(sum);
      if (lane == 0) {
        const float rescale = (m_old == -INFINITY) ? 0.0f : expf(m_old - m_new);
        sR[g] = rescale;
        sL[g] = sL[g] * rescale + sum;
        sM[g] = m_new;
      }
    }
    __syncthreads();
    // P.V
    if (pv_active) {
      const float r = sR[pg];
#pragma unroll
      for (int e = 0; e < E; ++e) acc[e] *= r;
      const float *pr = sS + pg * T;
      // Rows past the chunk end (and rows whose page was missing) were never
      // written this tile: skip them rather than multiply stale data by zero.
      const int nt = min(T, end - (begin + t * T));
      const int *valid = sValid + stage * T;
      for (int lp = 0; lp < nt; ++lp) {
        if (!valid[lp]) continue;
        const float w = pr[lp];
        const __half *vr = v + (size_t)lp * D + pd;
        if (E % 2 == 0) {
#pragma unroll
          for (int e = 0; e < E; e += 2) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(vr + e));
            acc[e] = fmaf(w, f.x, acc[e]);
            acc[e + 1] = fmaf(w, f.y, acc[e + 1]);
          }
        } else {
#pragma unroll
          for (int e = 0; e < E; ++e) acc[e] = fmaf(w, __half2float(vr[e]), acc[e]);
        }
      }
    }
    __syncthreads();
    if (warp == 0 && t + 2 < ntiles) issue(t + 2);
  }

  const size_t head_base = ((size_t)row * p.hkv + kvh);
  if (active == 1) {
    if (pv_active) {
      const float inv = 1.0f / sL[pg];
      __half *o = p.out + (size_t)row * p.out_stride + (size_t)(kvh * G + pg) * D + pd;
#pragma unroll
      for (int e = 0; e < E; ++e) o[e] = __float2half_rn(acc[e] * inv);
    }
    return;
  }
  // Write this split's partial, then the last CTA of the (row, KV head) combines.
  {
    float *wa = p.ws_acc + ((head_base * p.max_splits + split) * G) * D;
    if (pv_active) {
#pragma unroll
      for (int e = 0; e < E; ++e) wa[(size_t)pg * D + pd + e] = acc[e];
    }
    if (tid < G) {
      float *wm = p.ws_ml + ((head_base * p.max_splits + split) * G + tid) * 2;
      wm[0] = sM[tid];
      wm[1] = sL[tid];
    }
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned int prev = atomicAdd(p.counters + head_base, 1u);
    is_last = (prev == static_cast<unsigned int>(active - 1)) ? 1 : 0;
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  if (pv_active) {
    float mmax = -INFINITY;
    for (int s = 0; s < active; ++s) {
      const float *wm = p.ws_ml + ((head_base * p.max_splits + s) * G + pg) * 2;
      mmax = fmaxf(mmax, __ldcg(wm));
    }
    float den = 0.0f;
    float out[E];
#pragma unroll
    for (int e = 0; e < E; ++e) out[e] = 0.0f;
    for (int s = 0; s < active; ++s) {
      const float *wm = p.ws_ml + ((head_base * p.max_splits + s) * G + pg) * 2;
      const float ms = __ldcg(wm), ls = __ldcg(wm + 1);
      const float f = (ms == -INFINITY) ? 0.0f : expf(ms - mmax);
      den += ls * f;
      const float *wa = p.ws_acc + ((head_base * p.max_splits + s) * G + pg) * D + pd;
#pragma unroll
      for (int e = 0; e < E; ++e) out[e] = fmaf(__ldcg(wa + e), f, out[e]);
    }
    const float inv = 1.0f / den;
    __half *o = p.out + (size_t)row * p.out_stride + (size_t)(kvh * G + pg) * D + pd;
#pragma unroll
    for (int e = 0; e < E; ++e) o[e] = __float2half_rn(out[e] * inv);
  }
  if (tid == 0) atomicExch(p.counters + head_base, 0u);
}

template <int D, int G>
cudaError_t launch_instance(const AttentionParams &p, cudaStream_t stream, bool pdl) {
  auto kernel = attention_kernel<D, G>;
  const size_t smem = Cfg<D, G>::smem_bytes();
  static std::mutex mu;
  static std::unordered_map<int, bool> configured;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!configured[dev]) {
      e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(smem));
      if (e != cudaSuccess) return e;
      configured[dev] = true;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.max_splits, p.hkv, p.rows);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, p);
}

template <int D>
cudaError_t dispatch_g(const AttentionParams &p, cudaStream_t stream, bool pdl, int g) {
  switch (g) {
    case 1: return launch_instance<D, 1>(p, stream, pdl);
    case 2: return launch_instance<D, 2>(p, stream, pdl);
    case 4: return launch_instance<D, 4>(p, stream, pdl);
    case 8: return launch_instance<D, 8>(p, stream, pdl);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

size_t attention_workspace_bytes(int rows, int hq, int hkv, int head_dim, int max_splits) {
  (void)hkv;
  const size_t acc = (size_t)rows * hq * max_splits * head_dim * 4;
  const size_t ml = (size_t)rows * hq * max_splits * 2 * 4;
  return acc + ml;
}

cudaError_t launch_attention(const AttentionParams &p, cudaStream_t stream, bool pdl) {
  if (p.rows <= 0 || p.hkv <= 0 || p.hq <= 0 || p.hq % p.hkv != 0 || p.max_splits <= 0 ||
      p.min_chunk <= 0 || p.page_size <= 0 || p.rows > 65535 || p.hkv > 65535)
    return cudaErrorInvalidValue;
  const int g = p.hq / p.hkv;
  switch (p.head_dim) {
    case 16: return dispatch_g<16>(p, stream, pdl, g);
    case 32: return dispatch_g<32>(p, stream, pdl, g);
    case 64: return dispatch_g<64>(p, stream, pdl, g);
    case 128: return dispatch_g<128>(p, stream, pdl, g);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace tmc

// ---- allocation-free entry point ---------------------------------------------
//
// Some callers cannot allocate device memory when they call into this
// library: a host that reserved all of its device memory up front for its own
// pool, a runtime with a fixed memory plan that forbids allocation after
// start-up, or code on a latency-critical path where cudaMalloc's implicit
// device synchronisation is not acceptable. For them the split-K partials and
// tickets of the attention kernel live in this fixed array instead of a
// caller-provided workspace. Every GPU that loads the library holds the array
// (8 MiB) until the process exits.
namespace tmc {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;  // 8 MiB
static __device__ __align__(256) unsigned char g_attention_scratch[kNoAllocScratchBytes];

// Device address of the scratch array on the current device, resolved once per
// device (host code cannot use the symbol itself: on the host it names a
// stand-in, not device memory).
cudaError_t attention_scratch_address(void **out) {
  static std::mutex mu;
  static std::unordered_map<int, void *> addresses;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  auto it = addresses.find(dev);
  if (it == addresses.end()) {
    void *ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_attention_scratch);
    if (e != cudaSuccess) return e;
    it = addresses.emplace(dev, ptr).first;
  }
  *out = it->second;
  return cudaSuccess;
}

}  // namespace
}  // namespace tmc

extern "C" int tmc_k_paged_attention_f16_noalloc(
    const void *q, void *out, const void *k_pool, const void *v_pool, const int32_t *block_table,
    int table_stride, const int32_t *table_rows, const int32_t *positions, int rows, int hq, int hkv,
    int d, int page_size, int pool_pages, int capacity, int max_splits, int min_chunk, void *status,
    void *stream) {
  using namespace tmc_api;
  if (!q || !out || !k_pool || !v_pool || !block_table || !table_rows || !positions)
    return fail(TMC_ERR_INVALID, "null pointer");
  if (rows <= 0 || hq <= 0 || hkv <= 0 || d <= 0 || max_splits <= 0)
    return fail(TMC_ERR_INVALID, "rows, heads, head_dim and max_splits must be positive");
  // Scratch layout: split partials (acc, then m/l), then the tickets.
  const size_t partials = tmc::attention_workspace_bytes(rows, hq, hkv, d, max_splits);
  const size_t tickets_offset = (partials + 255) / 256 * 256;
  const size_t needed = tickets_offset + (size_t)rows * hkv * sizeof(uint32_t);
  if (needed > tmc::kNoAllocScratchBytes) {
    return fail(TMC_ERR_UNSUPPORTED,
                "paged attention (no-alloc): needs " + std::to_string(needed) +
                    " bytes of scratch, the fixed limit is " + std::to_string(tmc::kNoAllocScratchBytes) +
                    " (lower max_splits or rows, or use tmc_k_paged_attention_f16)");
  }
  void *scratch = nullptr;
  cudaError_t e = tmc::attention_scratch_address(&scratch);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(attention scratch)");
  auto *base = static_cast<unsigned char *>(scratch);
  auto *tickets = reinterpret_cast<unsigned int *>(base + tickets_offset);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // The array keeps the previous call's contents; the tickets must start at 0.
  e = cudaMemsetAsync(tickets, 0, (size_t)rows * hkv * sizeof(uint32_t), s);
  if (e != cudaSuccess) return cuda_fail(e, "clearing attention scratch tickets");
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
  p.ws_acc = reinterpret_cast<float *>(base);
  p.ws_ml = reinterpret_cast<float *>(base + (size_t)rows * hq * max_splits * d * sizeof(float));
  p.counters = tickets;
  p.status = static_cast<tmc::TmcDeviceStatus *>(status);
  e = tmc::launch_attention(p, s, false);
  if (e == cudaErrorInvalidValue) return fail(TMC_ERR_UNSUPPORTED, "attention: unsupported shape");
  return e == cudaSuccess ? ok() : cuda_fail(e, "attention (no-alloc) launch");
}
