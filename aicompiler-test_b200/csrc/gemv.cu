// Decode GEMV family for sm_100a (see gemv.cuh for the op list).
//
// Design (HBM-bound, arithmetic intensity ~1 flop/byte at M=1):
//  * one CTA = 8 warps; a warp owns a group of R=2 consecutive weight rows
//    and streams both rows with 16-byte `ld.global.nc.L1::no_allocate` loads,
//    U chunks per row in flight per lane (R*U*16 B = 256 B per lane);
//  * the grid is one wave (SMs x resident CTAs); row groups are dealt to
//    warps with the global warp id `warp * gridDim.x + blockIdx.x`, so every
//    CTA (hence every SM) gets the same number of rows to within one;
//  * the activation vector(s) are staged once per CTA in shared memory after
//    the fused prologue (RMSNorm / embedding gather), read back conflict-free;
//  * warp-shuffle reduction, then a scalar fused epilogue by lane 0;
//  * programmatic dependent launch: the CTA prefetches its first rows into L2
//    before griddepcontrol.wait, so weight streaming overlaps the tail of the
//    previous kernel in the decode graph.
#include "gemv.cuh"
#include "epilogue.cuh"

#include <mutex>
#include <unordered_map>

namespace tmc {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

// Bulk prefetch of [p, p + bytes) into L2 (16-byte aligned, size multiple of
// 16) under the L2 cache policy `pol`.
__device__ __forceinline__ void prefetch_bulk_l2(const void *p, uint32_t bytes, uint64_t pol) {
  asm volatile("cp.async.bulk.prefetch.L2.global.L2::cache_hint [%0], %1, %2;" ::"l"(p), "r"(bytes), "l"(pol)
               : "memory");
}

template <typename XS>
struct XLoad;
template <>
struct XLoad<float> {
  static __device__ __forceinline__ void get(const float *row, int c, float (&v)[8]) {
    const float4 a = reinterpret_cast<const float4 *>(row)[2 * c];
    const float4 b = reinterpret_cast<const float4 *>(row)[2 * c + 1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
  static __device__ __forceinline__ float cvt(float v) { return v; }
};
template <>
struct XLoad<__half> {
  static __device__ __forceinline__ void get(const __half *row, int c, float (&v)[8]) {
    unpack(reinterpret_cast<const uint4 *>(row)[c], v);
  }
  static __device__ __forceinline__ void unpack(const uint4 &u, float (&v)[8]) {
    float2 f;
    f = half2_bits_to_float2(u.x); v[0] = f.x; v[1] = f.y;
    f = half2_bits_to_float2(u.y); v[2] = f.x; v[3] = f.y;
    f = half2_bits_to_float2(u.z); v[4] = f.x; v[5] = f.y;
    f = half2_bits_to_float2(u.w); v[6] = f.x; v[7] = f.y;
  }
};

template <typename XS>
__device__ __forceinline__ XS to_xs(float v);
template <>
__device__ __forceinline__ float to_xs<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half to_xs<__half>(float v) { return __float2half_rn(v); }

// Vectorised store of 8 staged values (16 or 32 bytes).
__device__ __forceinline__ void store8(float *dst, const float (&f)[8]) {
  reinterpret_cast<float4 *>(dst)[0] = make_float4(f[0], f[1], f[2], f[3]);
  reinterpret_cast<float4 *>(dst)[1] = make_float4(f[4], f[5], f[6], f[7]);
}
__device__ __forceinline__ void store8(__half *dst, const float (&f)[8]) {
  uint4 u;
  __half2 h;
  h = __floats2half2_rn(f[0], f[1]); u.x = *reinterpret_cast<uint32_t *>(&h);
  h = __floats2half2_rn(f[2], f[3]); u.y = *reinterpret_cast<uint32_t *>(&h);
  h = __floats2half2_rn(f[4], f[5]); u.z = *reinterpret_cast<uint32_t *>(&h);
  h = __floats2half2_rn(f[6], f[7]); u.w = *reinterpret_cast<uint32_t *>(&h);
  *reinterpret_cast<uint4 *>(dst) = u;
}

// The RMSNorm weights of the fp16-gamma prologues do not depend on the
// previous kernel: each thread loads the first kGammaPre of the 8-element
// vectors it will scale (v = threadIdx.x + j blockDim.x) before the
// programmatic-dependency wait, so the norm's second pass does not wait on L2.
constexpr int kGammaPre = 2;
struct GammaPre {
  uint4 v[kGammaPre];
  bool ok;
};
__device__ __forceinline__ GammaPre load_gamma_pre(const GemvParams &p) {
  GammaPre g{};
  const int pro = p.prologue;
  g.ok = pro == kProF16Norm || pro == kProEmbedNorm || pro == kProResidualNorm;
  if (g.ok) {
    const int nvec = p.K >> 3;
#pragma unroll
    for (int j = 0; j < kGammaPre; ++j) {
      const int v = threadIdx.x + j * blockDim.x;
      g.v[j] = v < nvec ? reinterpret_cast<const uint4 *>(p.gamma)[v] : make_uint4(0, 0, 0, 0);
    }
  }
  return g;
}
// gamma[8 v .. 8 v + 7] for the j-th vector of this thread.
__device__ __forceinline__ void gamma8(const GemvParams &p, const GammaPre &pre, int j, int v, float (&gv)[8]) {
  if (pre.ok && j < kGammaPre) {
    XLoad<__half>::unpack(pre.v[j], gv);
  } else {
    XLoad<__half>::get(static_cast<const __half *>(p.gamma), v, gv);
  }
}

// Stage the M activation rows (after the fused prologue) into shared memory.
// K is a multiple of 8 (checked on the host).
// `writer`: this CTA writes the residual-stream rows back to h_out (one CTA
// of a GEMV launch; every CTA of the row-prologue kernel, one row each).
template <typename XS, int M>
__device__ __forceinline__ void stage_x(const GemvParams &p, XS *xs, float *red, bool writer, const GammaPre &pre) {
  const int K = p.K;
  const int nvec = K >> 3;
  const bool exchanged = p.prologue == kProResidualNorm && p.xchg.world > 0;
  if (exchanged) {
    // The reduced projection is the sum of every rank's slot: wait for each
    // rank's flag on this phase (one thread per source rank).
    if (p.xchg.wait && threadIdx.x < p.xchg.world) {
      const unsigned int value = *p.xchg.epoch * p.xchg.phases + p.xchg.phase + 1u;
      if (!wait_flag_geq(peer_flag(p.xchg, p.xchg.rank, p.xchg.phase & 1, threadIdx.x), value, peer_wait_budget(p)))
        report_status(p.status, kStatusWaitTimeout, kWhereExchange, threadIdx.x, (int)p.xchg.phase);
    }
    __syncthreads();
  }
  for (int m = 0; m < M; ++m) {
    XS *dst = xs + (size_t)m * K;
    if (m >= p.M) {
      for (int i = threadIdx.x; i < K; i += blockDim.x) dst[i] = to_xs<XS>(0.0f);
      continue;
    }
    const int pro = p.prologue;
    if (pro == kProF32 || pro == kProF32Norm) {
      // One vectorised pass from global memory into shared memory (sum of
      // squares on the way), then normalise in place.
      const float4 *src = reinterpret_cast<const float4 *>(static_cast<const float *>(p.x) +
                                                           (size_t)m * p.x_stride);
      float ss = 0.0f;
#pragma unroll 4
      for (int v = threadIdx.x; v < K / 4; v += blockDim.x) {
        const float4 f = src[v];
        ss = fmaf(f.x, f.x, ss);
        ss = fmaf(f.y, f.y, ss);
        ss = fmaf(f.z, f.z, ss);
        ss = fmaf(f.w, f.w, ss);
        dst[4 * v + 0] = to_xs<XS>(f.x);
        dst[4 * v + 1] = to_xs<XS>(f.y);
        dst[4 * v + 2] = to_xs<XS>(f.z);
        dst[4 * v + 3] = to_xs<XS>(f.w);
      }
      if (pro == kProF32Norm) {
        ss = block_sum(ss, red);
        const float inv = 1.0f / sqrtf(ss / static_cast<float>(K) + p.eps);
        const float4 *g = static_cast<const float4 *>(p.gamma);
#pragma unroll 4
        for (int v = threadIdx.x; v < K / 4; v += blockDim.x) {
          const float4 gv = g[v];
          // each thread rewrites exactly the elements it wrote above
          dst[4 * v + 0] = to_xs<XS>(__fmul_rn(__fmul_rn(static_cast<float>(dst[4 * v + 0]), inv), gv.x));
          dst[4 * v + 1] = to_xs<XS>(__fmul_rn(__fmul_rn(static_cast<float>(dst[4 * v + 1]), inv), gv.y));
          dst[4 * v + 2] = to_xs<XS>(__fmul_rn(__fmul_rn(static_cast<float>(dst[4 * v + 2]), inv), gv.z));
          dst[4 * v + 3] = to_xs<XS>(__fmul_rn(__fmul_rn(static_cast<float>(dst[4 * v + 3]), inv), gv.w));
        }
      }
    } else {
      // fp16 sources: plain, RMSNorm, or embedding gather + RMSNorm.
      const __half *src = nullptr;
      if (pro == kProResidualNorm) {
        // x = half(h + half(partial)): the residual add after a cross-rank
        // reduction, fused into the consumer's prologue. Staged into dst first.
        const __half *hrow = static_cast<const __half *>(p.x) + (size_t)m * p.x_stride;
        const float *prow = exchanged ? nullptr : p.partial + (size_t)m * K;
        const bool write_back = writer && p.h_out != nullptr;
        float ss = 0.0f;
        for (int v = threadIdx.x; v < nvec; v += blockDim.x) {
          float hv[8], f[8], pv[8];
          XLoad<__half>::get(hrow, v, hv);
          if (exchanged) {
            // Rank-ordered sum of the slots (L2 loads: peers wrote them).
#pragma unroll
            for (int j = 0; j < 8; ++j) pv[j] = 0.0f;
            for (int src = 0; src < p.xchg.world; ++src) {
              const float4 *sp = reinterpret_cast<const float4 *>(
                  peer_slot(p.xchg, p.xchg.rank, p.xchg.phase & 1, src, p.xchg.row0 + m));
              const float4 a = __ldcg(sp + 2 * v), b = __ldcg(sp + 2 * v + 1);
              pv[0] += a.x; pv[1] += a.y; pv[2] += a.z; pv[3] += a.w;
              pv[4] += b.x; pv[5] += b.y; pv[6] += b.z; pv[7] += b.w;
            }
          } else {
            const float4 a = reinterpret_cast<const float4 *>(prow)[2 * v];
            const float4 b = reinterpret_cast<const float4 *>(prow)[2 * v + 1];
            pv[0] = a.x; pv[1] = a.y; pv[2] = a.z; pv[3] = a.w;
            pv[4] = b.x; pv[5] = b.y; pv[6] = b.z; pv[7] = b.w;
          }
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            f[j] = round_half(__fadd_rn(hv[j], round_half(pv[j])));
            ss = fmaf(f[j], f[j], ss);
          }
          store8(dst + v * 8, f);
          if (write_back) {
            __half tmp[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) tmp[j] = __float2half_rn(f[j]);
            reinterpret_cast<uint4 *>(p.h_out + (size_t)m * K)[v] = *reinterpret_cast<uint4 *>(tmp);
          }
        }
        ss = block_sum(ss, red);
        const float inv = 1.0f / sqrtf(ss / static_cast<float>(K) + p.eps);
        int j = 0;
        for (int v = threadIdx.x; v < nvec; v += blockDim.x, ++j) {
          float gv[8], xv[8];
          gamma8(p, pre, j, v, gv);
          XLoad<XS>::get(dst, v, xv);
#pragma unroll
          for (int j = 0; j < 8; ++j) xv[j] = round_half(__fmul_rn(__fmul_rn(xv[j], inv), gv[j]));
          store8(dst + v * 8, xv);
        }
        continue;
      }
      if (pro == kProEmbedNorm) {
        const int tok = p.tokens[m];
        if (tok < 0 || tok >= p.vocab) {
          if (threadIdx.x == 0 && blockIdx.x == 0)
            report_status(p.status, kStatusTokenRange, kWhereEmbedding, tok, m);
        } else {
          src = p.embedding + (size_t)tok * K;
        }
      } else {
        src = static_cast<const __half *>(p.x) + (size_t)m * p.x_stride;
      }
      const bool norm = (pro == kProF16Norm || pro == kProEmbedNorm);
      const bool write_h = (pro == kProEmbedNorm) && writer && p.h_out != nullptr;
      if (pro == kProF16 && src != nullptr) {
        // A plain copy: each thread has all of its loads (up to kCopyVecs
        // 16-byte vectors) in flight before it stores any, one L2 round trip
        // for rows up to kCopyVecs x 8 x blockDim elements (a long row, e.g.
        // the down projection's 14336, would otherwise take four).
        constexpr int kCopyVecs = 8;
        const uint4 *s4 = reinterpret_cast<const uint4 *>(src);
        for (int v0 = threadIdx.x; v0 < nvec; v0 += kCopyVecs * blockDim.x) {
          uint4 buf[kCopyVecs];
#pragma unroll
          for (int j = 0; j < kCopyVecs; ++j) {
            const int v = v0 + j * blockDim.x;
            buf[j] = v < nvec ? s4[v] : make_uint4(0, 0, 0, 0);
          }
#pragma unroll
          for (int j = 0; j < kCopyVecs; ++j) {
            const int v = v0 + j * blockDim.x;
            if (v < nvec) {
              float f[8];
              XLoad<__half>::unpack(buf[j], f);
              store8(dst + v * 8, f);
            }
          }
        }
        continue;
      }
      // Pass 1: global -> shared (raw values; exact in XS), sum of squares.
      float ss = 0.0f;
#pragma unroll 2
      for (int v = threadIdx.x; v < nvec; v += blockDim.x) {
        const uint4 raw = src != nullptr ? reinterpret_cast<const uint4 *>(src)[v] : make_uint4(0, 0, 0, 0);
        if (write_h) reinterpret_cast<uint4 *>(p.h_out + (size_t)m * K)[v] = raw;
        float f[8];
        float2 t;
        t = half2_bits_to_float2(raw.x); f[0] = t.x; f[1] = t.y;
        t = half2_bits_to_float2(raw.y); f[2] = t.x; f[3] = t.y;
        t = half2_bits_to_float2(raw.z); f[4] = t.x; f[5] = t.y;
        t = half2_bits_to_float2(raw.w); f[6] = t.x; f[7] = t.y;
#pragma unroll
        for (int j = 0; j < 8; ++j) ss = fmaf(f[j], f[j], ss);
        store8(dst + v * 8, f);
      }
      if (norm) {
        ss = block_sum(ss, red);
        const float inv = 1.0f / sqrtf(ss / static_cast<float>(K) + p.eps);
        // Pass 2 (same elements per thread): half(x * inv * gamma).
        int j = 0;
#pragma unroll 2
        for (int v = threadIdx.x; v < nvec; v += blockDim.x, ++j) {
          float gv[8], xv[8];
          gamma8(p, pre, j, v, gv);
          XLoad<XS>::get(dst, v, xv);
#pragma unroll
          for (int j = 0; j < 8; ++j) xv[j] = round_half(__fmul_rn(__fmul_rn(xv[j], inv), gv[j]));
          store8(dst + v * 8, xv);
        }
      }
    }
  }
}

template <int R, int M>
__device__ __forceinline__ void epilogue(const GemvParams &p, int row0, float (&acc)[R][M],
                                         int lane, unsigned long long (&best)[M], const EpiPre &pre) {
  const int epi = p.epilogue;
  if (epi == kEpiArgmax) {
    // Every lane holds the full sums; all lanes track the key identically.
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int row = row0 + r;
      if (row >= p.N) continue;
#pragma unroll
      for (int m = 0; m < M; ++m) {
        if (m >= p.M) continue;
        const float v = round_half(acc[r][m]);
        if (lane == 0 && p.y_f32 != nullptr) p.y_f32[(size_t)m * p.y_stride + row] = v;
        const unsigned long long key = argmax_key(v, p.vocab_offset + row);
        best[m] = key > best[m] ? key : best[m];
      }
    }
    return;
  }
  if (lane != 0) return;
  if (epi == kEpiSwiGLU || epi == kEpiQKV) {
    // (row0, row0 + 1): a (gate, up) pair or an interleaved RoPE pair.
#pragma unroll
    for (int m = 0; m < M; ++m)
      if (m < p.M) epilogue_pair(p, row0, m, acc[0][m], acc[R - 1][m]);
    return;
  }
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int row = row0 + r;
    if (row >= p.N) continue;
#pragma unroll
    for (int m = 0; m < M; ++m)
      if (m < p.M) epilogue_one(p, row, m, acc[r][m], m == 0 && pre.ok, pre.res[r < 2 ? r : 0]);
  }
}

template <typename XS, int M, int R, int U, int KS>
__global__ void __launch_bounds__(kThreads) gemv_kernel(const GemvParams p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  XS *xs = reinterpret_cast<XS *>(smem_raw);
  __shared__ float red[32];
  __shared__ unsigned long long warp_best[kWarps][M];
  __shared__ float team_part[kWarps][R * M];
  __shared__ int is_last;

  // A team of KS warps shares each row group; warp `wt` of the team streams
  // the K-slice [c_lo, c_hi) of the group's rows (partials reduced in shared
  // memory). KS > 1 cuts each warp's chain of dependent load batches for
  // short-N / long-K shapes.
  constexpr int kTeams = kWarps / KS;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int team = warp / KS, wt = warp % KS;
  const int total_teams = kTeams * gridDim.x;
  const int gt = team * gridDim.x + blockIdx.x;
  const int ngroups = (p.N + R - 1) / R;
  const int nchunks = p.K >> 3;
  const int c_lo = (int)(((long long)nchunks * wt) / KS);
  const int c_hi = (int)(((long long)nchunks * (wt + 1)) / KS);

  // Weights are read once per step: evict-first in L2.
  const uint64_t wpol = l2_evict_first_policy();
  // Load a batch of U 16-byte chunks of each of the R rows of group g,
  // starting at chunk c0 (chunks at or past c_hi read as zero), into registers.
  auto load_batch = [&](int g, int c0, uint4 (&w)[R][U]) {
    const int row0 = g * R;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const bool rv = row0 + r < p.N;
      const uint4 *wr = reinterpret_cast<const uint4 *>(p.W + (size_t)(rv ? row0 + r : row0) * p.K);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = c0 + u * 32 + lane;
        w[r][u] = (c < c_hi && rv) ? ldg_stream(wr + c, wpol) : make_uint4(0, 0, 0, 0);
      }
    }
  };

  // Weights never change: the first batch is loaded into registers (and the
  // rest of this warp's slice of the first group warmed in L2) before waiting
  // on the producer of x, so HBM latency overlaps the previous kernel's tail
  // and the prologue.
  const unsigned long long t_entry = p.trace.records ? global_ns() : 0ull;
  uint4 w[R][U];
  int g = gt, c0 = c_lo;
  if (g < ngroups && c_lo < c_hi) load_batch(g, c_lo, w);
  // While the producer of x finishes, pull this warp's static share of the
  // weights (its slice of the groups gt, gt + total_teams, ...) into L2 with
  // bulk prefetches, up to a budget that keeps a whole launch's prefetch well
  // inside L2. CTAs of this kernel become resident as the previous kernel's
  // CTAs drain, so its tail streams this kernel's weights instead of idling.
  if (p.l2_prefetch_bytes > 0 && lane == 0 && c_lo < c_hi) {
    const long long per_warp = p.l2_prefetch_bytes / ((long long)total_teams * KS);
    const uint32_t slice = static_cast<uint32_t>(c_hi - c_lo) * 16u;
    long long budget = per_warp;
    for (int gg = gt; gg < ngroups && budget > 0; gg += total_teams) {
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const int row = gg * R + r;
        if (row >= p.N || budget <= 0) continue;
        const char *src = reinterpret_cast<const char *>(p.W + (size_t)row * p.K) + (size_t)c_lo * 16;
        prefetch_bulk_l2(src, slice, wpol);
        budget -= slice;
      }
    }
  }
  // (single-row launches: with more rows the registers are spoken for)
  const GammaPre gpre = M == 1 ? load_gamma_pre(p) : GammaPre{};
  // The first group's residual rows, when the caller marks them final (lane 0
  // runs the epilogue).
  EpiPre epre{};
  if (M == 1 && p.early_epilogue_inputs && lane == 0 && g < ngroups) epre = load_epi_pre<R>(p, g * R);
  pdl_wait();
  // Dynamic scheduling (one-warp teams): SMs do not get equal HBM bandwidth,
  // so equal static shares finish at different times. After its first (static)
  // group a warp takes groups from one of kGemvPools interleaved pools
  // (group = pool + kGemvPools * k), each with its own ticket counter on its
  // own cache line. Lane 0 takes the next ticket when it issues the loads of a
  // group's last batch and the warp uses it when the group ends, so the
  // atomic's round trip hides behind that batch, and a warp never holds a
  // second group when the tickets run out (a ticket taken a whole group ahead
  // left slow warps with two groups to finish at the end). A group's
  // arithmetic does not depend on the warp that runs it, so results stay
  // deterministic.
  const bool dynamic = KS == 1 && p.work_counter != nullptr && total_teams % kGemvPools == 0 &&
                       ngroups > 2 * total_teams;
  const int pool = gt % kGemvPools;
  const int pool_base = total_teams / kGemvPools;
  unsigned int *ticket = p.work_counter + pool * kGemvPoolStride;
  int g_next = gt + total_teams;
  int fetched = ngroups;
  // The first group is one batch long: its last batch is already loaded.
  if (dynamic && lane == 0 && c_lo + 32 * U >= c_hi)
    fetched = pool + kGemvPools * (pool_base + (int)atomicAdd(ticket, 1u));
  stage_x<XS, M>(p, xs, red, blockIdx.x == 0, gpre);
  __syncthreads();
  pdl_launch_dependents();
  const unsigned long long t_ready = p.trace.records ? global_ns() : 0ull;

  unsigned long long best[M];
#pragma unroll
  for (int m = 0; m < M; ++m) best[m] = 0ull;

  float acc[R][M];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int m = 0; m < M; ++m) acc[r][m] = 0.0f;

  while (g < ngroups) {
    // Consume the batch held in w (warps whose slice is empty skip).
    if (c0 < c_hi) {
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = c0 + u * 32 + lane;
        if (c < c_hi) {
#pragma unroll
          for (int m = 0; m < M; ++m) {
            float xv[8];
            XLoad<XS>::get(xs + (size_t)m * p.K, c, xv);
#pragma unroll
            for (int r = 0; r < R; ++r) acc[r][m] = gemv_dot8(w[r][u], xv, acc[r][m]);
          }
        }
      }
    }
    // Issue the next batch before reducing / running the epilogue.
    int ng = g, nc = c0 + 32 * U;
    if (nc >= c_hi) {
      nc = c_lo;
      if (dynamic) {
        ng = __shfl_sync(0xffffffffu, fetched, 0);
      } else {
        ng = g_next;
        g_next += total_teams;
      }
    }
    if (dynamic && lane == 0 && ng < ngroups && nc + 32 * U >= c_hi)
      fetched = pool + kGemvPools * (pool_base + (int)atomicAdd(ticket, 1u));
    if (ng < ngroups && c_lo < c_hi) load_batch(ng, nc, w);
    if (nc == c_lo) {
      // Group finished by every warp of the team (all walk the same groups).
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int m = 0; m < M; ++m) acc[r][m] = warp_sum(acc[r][m]);
      if (KS > 1) {
        if (lane == 0) {
#pragma unroll
          for (int r = 0; r < R; ++r)
#pragma unroll
            for (int m = 0; m < M; ++m) team_part[warp][r * M + m] = acc[r][m];
        }
        asm volatile("bar.sync %0, %1;" ::"r"(team + 1), "r"(KS * 32) : "memory");
        if (wt == 0) {
#pragma unroll
          for (int r = 0; r < R; ++r)
#pragma unroll
            for (int m = 0; m < M; ++m) {
              float t = 0.0f;
#pragma unroll
              for (int k = 0; k < KS; ++k) t += team_part[team * KS + k][r * M + m];
              acc[r][m] = t;
            }
          epilogue<R, M>(p, g * R, acc, lane, best, epre);
        }
        asm volatile("bar.sync %0, %1;" ::"r"(team + 1), "r"(KS * 32) : "memory");
      } else {
        epilogue<R, M>(p, g * R, acc, lane, best, epre);
      }
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int m = 0; m < M; ++m) acc[r][m] = 0.0f;
      epre.ok = false;  // the read-ahead inputs were the first group's
    }
    g = ng;
    c0 = nc;
  }

  if (dynamic) {
    // The last CTA to finish resets the tickets for the next launch.
    __syncthreads();
    if (threadIdx.x == 0) {
      const unsigned int done = atomicAdd(p.work_counter + kGemvPools * kGemvPoolStride, 1u);
      if (done == gridDim.x - 1) {
        for (int c = 0; c < kGemvPools; ++c) atomicExch(p.work_counter + c * kGemvPoolStride, 0u);
        atomicExch(p.work_counter + kGemvPools * kGemvPoolStride, 0u);
      }
    }
  }
  if (p.epilogue == kEpiF32Partial && p.xchg.world > 0) {
    // Causality chain, with one system-scope release per launch instead of a
    // system fence per CTA (which costs microseconds at every CTA's exit):
    // each thread's peer stores -> CTA barrier -> thread 0's GPU-scope
    // acq_rel arrival on the done counter -> the last CTA's acquire of it ->
    // its system-scope release store of this rank's flag in every window ->
    // the consumer's system-scope acquire of the flag.
    // The releases to the ranks go out in parallel, one lane each (a release
    // store waits for a system-scope round trip; serial ones add up).
    __syncthreads();
    if (threadIdx.x < 32) {
      int last = 0;
      if (threadIdx.x == 0) {
        const unsigned int done = atomic_add_acq_rel_gpu(p.xchg.done, 1u);
        last = done == gridDim.x - 1;
        if (last) atomicExch(p.xchg.done, 0u);
      }
      last = __shfl_sync(0xffffffffu, last, 0);
      __syncwarp();  // orders lane 0's acquire before the other lanes' releases
      if (last && p.xchg.signal && (int)threadIdx.x < p.xchg.world) {
        const unsigned int value = *p.xchg.epoch * p.xchg.phases + p.xchg.phase + 1u;
        st_release_sys(peer_flag(p.xchg, threadIdx.x, p.xchg.phase & 1, p.xchg.rank), value);
      }
    }
  }
  if (p.epilogue != kEpiArgmax) {
    if (p.trace.records) {
      __syncthreads();  // record the CTA's last warp, not warp 0
      trace_emit(p.trace, t_entry, t_ready);
    }
    return;
  }
  {
    if (lane == 0) {
#pragma unroll
      for (int m = 0; m < M; ++m) warp_best[warp][m] = best[m];
    }
    __syncthreads();
    if (threadIdx.x < M && threadIdx.x < p.M) {
      unsigned long long b = 0ull;
      for (int w = 0; w < kWarps; ++w) b = warp_best[w][threadIdx.x] > b ? warp_best[w][threadIdx.x] : b;
      if (b != 0ull) atomicMax(p.argmax_keys + threadIdx.x, b);
    }
    if (p.next_tokens == nullptr) {  // cross-rank reduction finalises
      trace_emit(p.trace, t_entry, t_ready);
      return;
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
      const unsigned int prev = atomicAdd(p.argmax_counter, 1u);
      is_last = (prev == gridDim.x - 1) ? 1 : 0;
    }
    __syncthreads();
    if (is_last) {
      __threadfence();
      argmax_finalize(p, threadIdx.x, [] { __syncthreads(); });
    }
    trace_emit(p.trace, t_entry, t_ready);
  }
}

// Row prologue for the batched tensor-core GEMM: one CTA per activation row
// runs the GEMV prologue (embedding gather, residual + reduced projection,
// RMSNorm; exchange waits included) and writes the fp16 row the GEMM's TMA
// reads. The rounding is the GEMV's own (same stage_x).
__global__ void __launch_bounds__(kThreads) row_prologue_kernel(const GemvParams p, __half *xn) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __half *xs = reinterpret_cast<__half *>(smem_raw);
  __shared__ float red[32];
  const int m = blockIdx.x;
  GemvParams q = p;
  q.M = 1;
  const bool f32_in = (p.prologue == kProF32 || p.prologue == kProF32Norm);
  if (p.x) q.x = f32_in ? static_cast<const void *>(static_cast<const float *>(p.x) + (size_t)m * p.x_stride)
                       : static_cast<const void *>(static_cast<const __half *>(p.x) + (size_t)m * p.x_stride);
  if (p.tokens) q.tokens = p.tokens + m;
  if (p.h_out) q.h_out = p.h_out + (size_t)m * p.K;
  if (p.partial) q.partial = p.partial + (size_t)m * p.K;
  q.xchg.row0 = p.xchg.row0 + m;
  const GammaPre gpre{};  // (reading gamma ahead slowed the batched steps' prologue)
  pdl_wait();
  pdl_launch_dependents();
  stage_x<__half, 1>(q, xs, red, true, gpre);
  __syncthreads();
  const uint4 *src = reinterpret_cast<const uint4 *>(xs);
  uint4 *dst = reinterpret_cast<uint4 *>(xn + (size_t)m * p.K);
  for (int v = threadIdx.x; v < (p.K >> 3); v += blockDim.x) dst[v] = src[v];
}

template <typename XS, int M, int R, int U, int KS>
cudaError_t launch_instance(const GemvParams &p, cudaStream_t stream, bool pdl, int num_sms) {
  auto kernel = gemv_kernel<XS, M, R, U, KS>;
  const size_t smem = (size_t)M * p.K * sizeof(XS);
  // Occupancy depends on the dynamic shared memory; cache it per (device, smem).
  static std::mutex mu;
  static std::unordered_map<long long, int> occ_cache;
  static size_t configured_smem = 0;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  int occ = 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (smem > 48 * 1024 && smem > configured_smem) {
      e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(smem));
      if (e != cudaSuccess) return e;
      configured_smem = smem;
    }
    const long long key = (static_cast<long long>(dev) << 40) | static_cast<long long>(smem);
    auto it = occ_cache.find(key);
    if (it != occ_cache.end()) {
      occ = it->second;
    } else {
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, kThreads, smem);
      if (e != cudaSuccess) return e;
      if (occ < 1) occ = 1;
      occ_cache[key] = occ;
    }
  }
  const int ngroups = (p.N + R - 1) / R;
  int grid = (ngroups + kWarps / KS - 1) / (kWarps / KS);
  const int wave = occ * num_sms;
  // Whole multiples of the SM count: teams take groups CTA-minor (group g goes
  // to CTA g % grid), so equal CTA counts per SM give every SM an equal share
  // of the rows (256 CTAs on 148 SMs would leave 108 SMs with twice the rows
  // of the other 40, and the launch would wait for them).
  if (grid > num_sms) grid = (grid + num_sms - 1) / num_sms * num_sms;
  if (grid > wave) grid = wave;
  if (grid < 1) grid = 1;

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
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

}  // namespace

namespace {

// Warps per row group: split K across a team when a row is several load
// batches long and there are too few row groups to keep every warp busy.
template <int M, int R, int U>
int choose_ks(const GemvParams &p, int num_sms) {
  // The team reduction makes a team's warps wait for their slowest member at
  // every group (barrier stalls dominate a K-split down projection), so K is
  // split only when there are too few row groups to occupy half the warps.
  const int ngroups = (p.N + R - 1) / R;
  const int batches = (p.K >> 3) / (32 * U);  // full load batches per row
  const int warps = num_sms * 16;             // two resident CTAs of 8 warps per SM
  int ks = 1;
  while (ks < 8 && ks * 2 <= batches && ngroups * ks * 2 <= warps) ks *= 2;
  // A tuned selection (DecodeGEMVTuner) overrides the rule when its team
  // still gets at least one load batch per warp.
  if (p.force_ks == 1 || ((p.force_ks == 2 || p.force_ks == 4 || p.force_ks == 8) && p.force_ks <= batches))
    ks = p.force_ks;
  return ks;
}

template <typename XS, int M, int R, int U>
cudaError_t launch_ks(const GemvParams &p, cudaStream_t stream, bool pdl, int num_sms) {
  switch (choose_ks<M, R, U>(p, num_sms)) {
    case 8: return launch_instance<XS, M, R, U, 8>(p, stream, pdl, num_sms);
    case 4: return launch_instance<XS, M, R, U, 4>(p, stream, pdl, num_sms);
    case 2: return launch_instance<XS, M, R, U, 2>(p, stream, pdl, num_sms);
    default: return launch_instance<XS, M, R, U, 1>(p, stream, pdl, num_sms);
  }
}

// One launch for M rows whose staged activations fit in shared memory.
cudaError_t launch_rows(const GemvParams &p, cudaStream_t stream, bool pdl, int num_sms) {
  const bool f32_in = (p.prologue == kProF32 || p.prologue == kProF32Norm);
  const size_t k = static_cast<size_t>(p.K);
  // fp32 staging keeps un-rounded fp32 activations exact (C1 graph); fp16 staging
  // is exact for the decoder's fp16-rounded activations and halves shared memory.
  if (p.M == 1) {
    if (f32_in || k * 4 <= 64 * 1024) return launch_ks<float, 1, 2, 8>(p, stream, pdl, num_sms);
    return launch_ks<__half, 1, 2, 8>(p, stream, pdl, num_sms);
  }
  if (p.M == 2) {
    if (k * 2 * 4 <= 112 * 1024) return launch_ks<float, 2, 2, 8>(p, stream, pdl, num_sms);
    if (f32_in) return cudaErrorInvalidValue;
    return launch_ks<__half, 2, 2, 8>(p, stream, pdl, num_sms);
  }
  if (p.M <= 4) {
    if (f32_in && k * 4 * 4 <= 200 * 1024) return launch_ks<float, 4, 2, 4>(p, stream, pdl, num_sms);
    if (f32_in || k * 4 * 2 > 200 * 1024) return cudaErrorInvalidValue;
    return launch_ks<__half, 4, 2, 4>(p, stream, pdl, num_sms);
  }
  if (f32_in || k * 8 * 2 > 200 * 1024) return cudaErrorInvalidValue;
  return launch_ks<__half, 8, 2, 4>(p, stream, pdl, num_sms);
}

// Largest row count per launch whose staging fits (see launch_rows).
int max_rows_per_launch(const GemvParams &p) {
  const bool f32_in = (p.prologue == kProF32 || p.prologue == kProF32Norm);
  const size_t k = static_cast<size_t>(p.K);
  const size_t budget = 200 * 1024;
  const size_t per_row = k * (f32_in ? 4 : 2);
  if (per_row > budget) return 0;
  int m = static_cast<int>(budget / per_row);
  if (m >= 8) return 8;
  if (m >= 4) return 4;
  if (m >= 2) return 2;
  return 1;
}

}  // namespace

cudaError_t launch_row_prologue(const GemvParams &p, __half *xn, cudaStream_t stream, bool pdl) {
  if (p.K <= 0 || (p.K & 7) != 0 || p.M <= 0 || p.prologue == kProF32 || p.prologue == kProF32Norm)
    return cudaErrorInvalidValue;
  const size_t smem = (size_t)p.K * sizeof(__half);
  static std::mutex mu;
  static std::unordered_map<int, bool> configured;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!configured[dev]) {
      e = cudaFuncSetAttribute(row_prologue_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
      if (e != cudaSuccess) return e;
      configured[dev] = true;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.M);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, row_prologue_kernel, p, xn);
}

cudaError_t launch_gemv(const GemvParams &p, cudaStream_t stream, bool pdl, int num_sms) {
  if (p.K <= 0 || (p.K & 7) != 0 || p.N <= 0 || p.M <= 0 || p.M > 8) return cudaErrorInvalidValue;
  if ((p.epilogue == kEpiQKV || p.epilogue == kEpiSwiGLU) && (p.N & 1)) return cudaErrorInvalidValue;
  const int cap = max_rows_per_launch(p);
  if (cap <= 0) return cudaErrorInvalidValue;
  if (p.M <= cap) return launch_rows(p, stream, pdl, num_sms);
  // Too many rows to stage at once: one launch per group of `cap` rows with
  // every row-indexed pointer offset (each launch streams the weights again).
  if (p.history != nullptr) return cudaErrorInvalidValue;  // greedy history indexes rows by M
  if (p.xchg.world > 0 && p.epilogue == kEpiArgmax) return cudaErrorInvalidValue;  // one key exchange per step
  for (int m0 = 0; m0 < p.M; m0 += cap) {
    GemvParams q = p;
    q.M = p.M - m0 < cap ? p.M - m0 : cap;
    const bool f32_in = (p.prologue == kProF32 || p.prologue == kProF32Norm);
    if (p.x) q.x = f32_in ? static_cast<const void *>(static_cast<const float *>(p.x) + m0 * p.x_stride)
                         : static_cast<const void *>(static_cast<const __half *>(p.x) + m0 * p.x_stride);
    if (p.tokens) q.tokens = p.tokens + m0;
    if (p.h_out) q.h_out = p.h_out + (size_t)m0 * p.K;
    if (p.partial) q.partial = p.partial + (size_t)m0 * p.K;
    if (p.y_f32) q.y_f32 = p.y_f32 + (size_t)m0 * p.y_stride;
    if (p.y_f16) q.y_f16 = p.y_f16 + (size_t)m0 * p.y_stride;
    if (p.residual) q.residual = p.residual + (size_t)m0 * p.y_stride;
    if (p.positions) q.positions = p.positions + m0;
    if (p.table_rows) q.table_rows = p.table_rows + m0;
    if (p.argmax_keys) q.argmax_keys = p.argmax_keys + m0;
    if (p.next_tokens) q.next_tokens = p.next_tokens + m0;
    if (p.feed_tokens) q.feed_tokens = p.feed_tokens + m0;
    if (p.feed_positions) q.feed_positions = p.feed_positions + m0;
    q.xchg.row0 = p.xchg.row0 + m0;
    q.xchg.signal = p.xchg.signal && m0 + cap >= p.M;  // flags once every row is stored
    cudaError_t e = launch_rows(q, stream, pdl, num_sms);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace tmc
