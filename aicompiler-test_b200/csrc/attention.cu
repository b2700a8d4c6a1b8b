// GQA decode attention for sm_100a, two schedules over one per-tile step.
//
// Per tile of 64 key positions of one (query row, KV head) pair: each of four
// warps takes 16 positions, computes the scores of all G = Hq/Hkv query heads
// of the KV head with mma.sync (query heads fill rows of the 16-row A tile),
// updates its online softmax and accumulates P.V; every K/V row is read from
// HBM once per query row (GQA reuse). K/V arrive through the block table as
// 16-position page boxes (TMA tensor maps, 128-byte swizzle) or, for other
// shapes, one bulk copy per position row, into an mbarrier ring with bounded
// waits.
// - Split schedule (latency: few pairs, bs1): grid (splits, Hkv, rows); a CTA
//   owns a chunk of one pair's positions; the CTAs of a pair merge through
//   distributed shared memory in a cluster, or through a workspace and an
//   atomic ticket when the pair spans several clusters.
// - Streaming schedule (throughput: many pairs, batched decode and serving):
//   one wave of persistent CTAs streams the concatenated tiles of all pairs
//   with a dedicated producer warp (attention_stream_kernel below).
#include "attention.cuh"
#include "gemm.cuh"

#include <cmath>
#include <mutex>
#include <string>
#include <unordered_map>

#include "api_util.hpp"
#include "mbarrier.cuh"
#include "tmc_cuda.h"

namespace tmc {
namespace {

constexpr int kThreads = 128;
constexpr int kPageCache = 512;  // page ids a CTA caches (longer chunks read the table per tile)
// Largest thread-block cluster (16 is the sm_100 opt-in, non-portable size; a
// device that cannot hold a 16-CTA cluster of this kernel falls back to 8).
constexpr int kMaxCluster = 16;
#ifndef TMC_ATTENTION_CLUSTER_LIMIT
#define TMC_ATTENTION_CLUSTER_LIMIT 16
#endif

__device__ __forceinline__ void ldmatrix_x2(uint32_t &r0, uint32_t &r1, const void *row_addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];"
               : "=r"(r0), "=r"(r1)
               : "r"(smem_u32(row_addr)));
}
__device__ __forceinline__ void ldmatrix_x2_trans(uint32_t &r0, uint32_t &r1, const void *row_addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0, %1}, [%2];"
               : "=r"(r0), "=r"(r1)
               : "r"(smem_u32(row_addr)));
}

// D = A(16x16, fp16, row) * B(16x8, fp16, col) + C, fp32 accumulate.
__device__ __forceinline__ void mma_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&h);
}

// BOX: K/V tiles arrive as 16-position page boxes through TMA tensor maps
// (128-byte swizzle, rows of 64 dims per half, no padding); otherwise one
// bulk copy per position row into padded rows.
template <int D, int G, bool BOX>
struct Cfg {
  static constexpr int kWarpsPerCta = kThreads / 32;     // 4
  static constexpr int kRowsPerWarp = 16;                // positions per warp per tile
  static constexpr int T = kWarpsPerCta * kRowsPerWarp;  // 64 positions per tile
  static constexpr int kRow = BOX ? D : D + 8;           // padded row (halves): conflict-free ldmatrix
  static constexpr size_t kStageBytes = (size_t)T * kRow * 2;  // one of K or V per stage
  static constexpr size_t kAlign = BOX ? 1024 : 0;       // swizzled stages start on 1024 bytes
  static constexpr int kStages = 2;
  static constexpr int kMaxSplits = kAttentionMaxSplits;
  static constexpr int kKSteps = D / 16;                 // QK^T k-steps
  static constexpr int kDTiles = D / 8;                  // PV n-tiles
  __host__ __device__ static constexpr size_t merge_bytes() { return (size_t)kWarpsPerCta * (G * D + 2 * G) * 4; }
  __host__ __device__ static constexpr size_t smem_bytes() {
    const size_t stages = (size_t)kStages * 2 * kStageBytes;
    return kAlign + (stages > merge_bytes() ? stages : merge_bytes())  // K/V ring, reused for the warp merge
           + (size_t)kStages * T * 4                            // sValid
           + (size_t)kMaxSplits * G * 4 * 2                     // combine weights (m then l)
           + (size_t)2 * kStages * 8 + 32;                      // full/empty barriers (+align)
  }
};

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_nctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}
// Shared-memory address of the same variable in cluster CTA `rank`.
__device__ __forceinline__ uint32_t map_cluster(const void *local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(local)), "r"(rank));
  return r;
}
// Asynchronous store into cluster CTA shared memory that completes as
// transaction bytes on an mbarrier of the receiving CTA (the sender does not
// wait for it to land).
__device__ __forceinline__ void st_async_f32(uint32_t addr, float v, uint32_t remote_bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(addr),
               "r"(__float_as_uint(v)), "r"(remote_bar)
               : "memory");
}
__device__ __forceinline__ void st_async_f32x2(uint32_t addr, float a, float b, uint32_t remote_bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.b32 [%0], {%1, %2}, [%3];" ::"r"(addr),
               "r"(__float_as_uint(a)), "r"(__float_as_uint(b)), "r"(remote_bar)
               : "memory");
}
// The two halves of a cluster barrier phase (a hardware barrier, not a spin):
// arriving after the mbarrier initialisation and waiting just before the
// first remote store proves every CTA of the cluster has started and made its
// barriers visible, at no cost in between.
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }

// One warp's 16 positions [p0, p0 + 16) of a K/V tile held in stage memory
// (sKs, sVs: the stage's K and V bytes; rows r0 .. r0 + 15 of the tile):
// scores against the query fragments qa, masking (positions >= end, rows
// whose page failed its checks), the online-softmax update of (m_run, l_run)
// and P.V into acc. BOX stages hold 128-byte-swizzled 64-dim halves, others
// padded rows. Returns true when V rows were zeroed (generic-proxy writes: a
// proxy fence is due before TMA refills the stage).
template <int D, int G, bool BOX>
__device__ __forceinline__ bool tile_step(unsigned char *sKs, unsigned char *sVs, int r0, int p0, int end,
                                          const int *valid, float scale, const uint32_t (&qa)[D / 16][4],
                                          float &m_run, float &l_run, float (&acc)[D / 8][4], int lane) {
  using C = Cfg<D, G, BOX>;
  constexpr int T = C::T, ROW = C::kRow;
  const int tq = lane & 3;
  const __half *k = reinterpret_cast<const __half *>(sKs) + (size_t)r0 * ROW;
  const __half *v = reinterpret_cast<const __half *>(sVs) + (size_t)r0 * ROW;
  (void)T;
  // BOX: a whole box landed; rows of positions past `end` (or of a missing
  // page) hold stale values: zero their V rows (P is 0 there, 0 * NaN is not).
  bool zeroed = false;
  if (BOX && p0 < end) {
    const int lp = lane & 15;
    const bool bad = !(p0 + lp < end && valid[lp]);
    if (__any_sync(0xffffffffu, bad)) {
      unsigned char *vs = sVs;
#pragma unroll
      for (int h = 0; h < D / 64; ++h) {
        // lanes 0-15 and 16-31 take the two 64-byte halves of row r0 + lp
        uint4 *dst = reinterpret_cast<uint4 *>(vs + h * T * 128 + (r0 + lp) * 128 + (lane >> 4) * 64);
        if (bad) {
#pragma unroll
          for (int c = 0; c < 4; ++c) dst[c] = make_uint4(0u, 0u, 0u, 0u);
        }
      }
      __syncwarp();
      zeroed = true;
    }
  }
  if (p0 < end) {
    // Scores S[16 heads x 16 positions] as two n-tiles of 8 positions.
    float sc[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.0f;
#pragma unroll
      for (int kk = 0; kk < C::kKSteps; ++kk) {
        uint32_t b0, b1;
        // matrices: rows = positions nt*8..+7, columns = dims kk*16..+7 and +8..+15
        const __half *addr;
        if (BOX) {
          const int R = r0 + nt * 8 + (lane & 7), d0 = kk * 16 + ((lane >> 3) & 1) * 8;
          addr = reinterpret_cast<const __half *>(sKs + (d0 >> 6) * T * 128 + R * 128 +
                                                  ((((d0 & 63) >> 3) ^ (R & 7)) << 4));
        } else {
          addr = k + (size_t)(nt * 8 + (lane & 7)) * ROW + kk * 16 + ((lane >> 3) & 1) * 8;
        }
        ldmatrix_x2(b0, b1, addr);
        mma_16816(sc[nt], qa[kk], b0, b1);
      }
    }
    // Scale, mask, online softmax (row gq owns c0/c1; c2/c3 are rows gq+8, unused).
    float mx = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int lp = nt * 8 + 2 * tq + j;
        const bool ok = p0 + lp < end && valid[lp];
        sc[nt][j] = ok ? sc[nt][j] * scale : -INFINITY;
        mx = fmaxf(mx, sc[nt][j]);
      }
    }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float m_new = fmaxf(m_run, mx);
    const float rescale = (m_run == -INFINITY) ? 0.0f : expf(m_run - m_new);
    float psum = 0.0f;
    float pr[2][2];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        pr[nt][j] = (sc[nt][j] == -INFINITY) ? 0.0f : expf(sc[nt][j] - m_new);
        psum += pr[nt][j];
      }
    }
    psum += __shfl_xor_sync(0xffffffffu, psum, 1);
    psum += __shfl_xor_sync(0xffffffffu, psum, 2);
    l_run = l_run * rescale + psum;
    m_run = m_new;
    // P as the A operand (16 heads x 16 positions) in two fp16 parts, hi + lo,
    // so the probabilities keep ~22 bits (the reference multiplies fp32
    // probabilities by the values).
    uint32_t pa[4], pl[4];
    {
      const __half2 h0 = __floats2half2_rn(pr[0][0], pr[0][1]);
      const __half2 h1 = __floats2half2_rn(pr[1][0], pr[1][1]);
      const float2 f0 = __half22float2(h0), f1 = __half22float2(h1);
      pa[0] = *reinterpret_cast<const uint32_t *>(&h0);
      pa[2] = *reinterpret_cast<const uint32_t *>(&h1);
      pl[0] = pack_half2(pr[0][0] - f0.x, pr[0][1] - f0.y);
      pl[2] = pack_half2(pr[1][0] - f1.x, pr[1][1] - f1.y);
      pa[1] = pa[3] = pl[1] = pl[3] = 0u;
    }
    // O[16 x D] += P . V[16 positions x D].
#pragma unroll
    for (int dt = 0; dt < C::kDTiles; ++dt) {
      acc[dt][0] *= rescale;
      acc[dt][1] *= rescale;
      uint32_t b0, b1;
      // matrices (transposed on load): rows = positions 0..7 and 8..15, columns = dims dt*8..+7
      const __half *addr;
      if (BOX) {
        const int R = r0 + (lane & 15), d0 = dt * 8;
        addr = reinterpret_cast<const __half *>(sVs + (d0 >> 6) * T * 128 + R * 128 +
                                                ((((d0 & 63) >> 3) ^ (R & 7)) << 4));
      } else {
        addr = v + (size_t)(lane & 15) * ROW + dt * 8;
      }
      ldmatrix_x2_trans(b0, b1, addr);
      mma_16816(acc[dt], pl, b0, b1);
      mma_16816(acc[dt], pa, b0, b1);
    }
  }
  return zeroed;
}

// Grid (max_splits, Hkv, rows), 4 warps, launched in clusters of `cluster`
// CTAs along the splits. A CTA owns one KV head of one query row and a chunk
// of key positions; each warp runs flash-decoding on its own 16 positions of
// every 64-position tile with tensor-core MMAs (the G query heads of the KV
// head fill rows of the 16-row A tile; unused rows are zero) and keeps its own
// online-softmax state; the warps merge in shared memory, then every CTA of a
// cluster pushes its (m, l, o) slices into the receive buffers of the CTAs
// that own them (remote stores, one cluster barrier) and each owner merges
// its slice from its own shared memory. Only when a (row, KV head) spans
// several clusters do the cluster results meet in the global workspace
// (atomic ticket, last CTA combines).
template <int D, int G, bool BOX>
__global__ void __launch_bounds__(kThreads)
    attention_kernel(const __grid_constant__ AttentionParams p, const __grid_constant__ CUtensorMap kmap,
                     const __grid_constant__ CUtensorMap vmap) {
  using C = Cfg<D, G, BOX>;
  constexpr int T = C::T, S = C::kStages, ROW = C::kRow;
  static_assert(G <= 8 && D % 16 == 0, "attention tile shape");
  static_assert(!BOX || D % 64 == 0, "page boxes are 64-dim halves");
  extern __shared__ __align__(128) unsigned char smem_raw[];
  unsigned char *smem = BOX ? reinterpret_cast<unsigned char *>(
                                  (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023))
                            : smem_raw;
  __half *sK = reinterpret_cast<__half *>(smem);
  __half *sV = sK + S * T * ROW;
  const size_t ring = (size_t)S * 2 * C::kStageBytes;
  unsigned char *after = smem + (ring > C::merge_bytes() ? ring : C::merge_bytes());
  int *sValid = reinterpret_cast<int *>(after);
  float *sW = reinterpret_cast<float *>(sValid + S * T);  // [kMaxSplits * G] weights, then l
  uint64_t *full = reinterpret_cast<uint64_t *>(
      (reinterpret_cast<uintptr_t>(sW + 2 * C::kMaxSplits * G) + 15) & ~uintptr_t(15));
  uint64_t *empty = full + S;
  __shared__ int is_last;
  __shared__ int sPages[kPageCache];  // the chunk's physical page ids
  __shared__ float xml[G * 2];  // this CTA's (m, l) per head
  // Receive buffers of this CTA's slice [crank * per, (crank + 1) * per) of the
  // G x D outputs: the o values of every CTA of the cluster, and each CTA's
  // (m, l) per head, written only by the cluster's asynchronous stores, which
  // complete on recv_bar (never aliasing the ring or the local merge area).
  __shared__ __align__(16) float recv_o[G * D + kMaxCluster];
  __shared__ __align__(16) float recv_ml[kMaxCluster * G * 2];
  __shared__ __align__(8) uint64_t recv_bar;
  __shared__ float merge_f[kMaxCluster * G];  // exp(m_c - max) per (CTA c, head)
  __shared__ float merge_md[G * 2];           // (max, denominator) per head

  const int split = blockIdx.x, kvh = blockIdx.y, row = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gq = lane >> 2, tq = lane & 3;  // mma fragment coordinates
  const uint32_t csize = cluster_nctarank(), crank = cluster_ctarank();
  const unsigned long long t_entry = p.trace.records ? global_ns() : 0ull;
  unsigned long long t_ready = 0ull;

  // Positions, table rows and the block table are final before the kernel that
  // produces q (and the newest K/V rows) starts: they are read, and the K/V rows
  // of older positions gathered, before the programmatic-dependency wait.
  const int pos = p.positions[row];
  const int trow = p.table_rows[row];  // loaded alongside pos: one round trip, not two
  if (pos < 0 || pos >= p.capacity) {  // the same for every CTA of the row
    if (split == 0 && kvh == 0 && tid == 0)
      report_status(p.status, kStatusLengthRange, kWhereAttention, pos, row);
    pdl_wait();
    return;
  }
  const int len = pos + 1;
  int nsplit = (len + p.min_chunk - 1) / p.min_chunk;
  if (p.max_chunk > 0 && nsplit > (int)csize) {
    // Fill one cluster before adding more: splits in other clusters meet only
    // through the global workspace and a ticket, a longer tail than the
    // distributed-shared-memory merge.
    const int wide = (len + p.max_chunk - 1) / p.max_chunk;
    nsplit = wide > (int)csize ? wide : (int)csize;
  }
  if (nsplit > p.max_splits) nsplit = p.max_splits;
  if (nsplit > C::kMaxSplits) nsplit = C::kMaxSplits;
  if (nsplit < 1) nsplit = 1;
  int chunk = (len + nsplit - 1) / nsplit;
  chunk = (chunk + 15) / 16 * 16;  // whole warp rows
  const int active = (len + chunk - 1) / chunk;
  const int first_split = split - (int)crank;
  if (first_split >= active) {  // the whole cluster is idle
    pdl_wait();
    trace_emit(p.trace, t_entry, t_entry);
    return;
  }
  const bool idle = split >= active;  // no positions, but joins the cluster merge
  const int begin = idle ? len : split * chunk;
  const int end = idle ? len : min(len, begin + chunk);
  const int ntiles = idle ? 0 : (end - begin + T - 1) / T;
  const int *table = p.block_table + (size_t)trow * p.table_stride;
  // Positions below `fresh` are never written by the producer kernel.
  const int fresh = p.early_mode == 2 ? end : (p.early_mode == 1 ? pos : begin);
  bool failed = false;

  // The chunk's physical page ids, looked up once (the block table is final
  // before the producer kernel starts): the per-tile gathers then read shared
  // memory instead of waiting on a dependent global load for every tile.
  const int lp0 = begin / p.page_size;
  const int npages = end > begin ? (end - 1) / p.page_size - lp0 + 1 : 0;
  const bool cached = npages <= kPageCache;
  if (cached) {
    for (int i = tid; i < npages; i += kThreads) {
      const int logical = lp0 + i;
      sPages[i] = logical < p.table_stride ? table[logical] : -1;
    }
  }
  auto page_of = [&](int logical) -> int {
    if (cached) return sPages[logical - lp0];
    return logical < p.table_stride ? table[logical] : -1;
  };

  if (tid == 0) {
#pragma unroll
    for (int st = 0; st < S; ++st) {
      mbar_init(&full[st], 1);
      mbar_init(&empty[st], C::kWarpsPerCta);
    }
    // The merge slice's bytes from every CTA of the cluster: its o values and
    // the (m, l) of every head.
    const int per = (G * D + (int)csize - 1) / (int)csize;
    const int lo = (int)crank * per, hi = min(G * D, lo + per);
    mbar_init(&recv_bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    mbar_arrive_expect_tx(&recv_bar, static_cast<uint32_t>(csize) * static_cast<uint32_t>(hi - lo + 2 * G) * 4u);
  }
  __syncthreads();
  // Phase 0 of the cluster barrier, waited on just before the first remote
  // store (the clusters that returned above are whole clusters).
  cluster_arrive_relaxed();

  // Warp 0: mark tile t's valid rows and arm its barrier with their bytes.
  auto arm = [&](int t) {
    const int stage = t % S;
    const int p0 = begin + t * T;
    int nvalid = 0;
#pragma unroll
    for (int j = 0; j < T / 32; ++j) {
      const int lp = lane + 32 * j;
      const int position = p0 + lp;
      int v = 0;
      if (position < end) {
        const int logical = position / p.page_size;
        const int page = page_of(logical);
        if (page < 0) {
          report_status(p.status, kStatusPageMissing, kWhereAttention, logical, row);
        } else if (page >= p.pool_pages) {
          report_status(p.status, kStatusPageRange, kWhereAttention, page, row);
        } else {
          v = 1;
        }
      }
      sValid[stage * T + lp] = v;
      if (!BOX && !v) {
        // No copy lands in this row: zero its V (P = 0 there, and 0 * NaN
        // from stale shared memory would poison the P.V product).
        uint4 *vrow = reinterpret_cast<uint4 *>(sV + ((size_t)stage * T + lp) * ROW);
#pragma unroll
        for (int c = 0; c < D / 8; ++c) vrow[c] = make_uint4(0u, 0u, 0u, 0u);
      }
      nvalid += __popc(__ballot_sync(0xffffffffu, v));
    }
    __syncwarp();
    if (BOX) {
      // One 16-position box per row group whose first position is valid (a
      // group lies in one page: group starts and page sizes are multiples of 16).
      int boxes = 0;
#pragma unroll
      for (int w = 0; w < C::kWarpsPerCta; ++w) boxes += sValid[stage * T + w * 16] ? 1 : 0;
      if (lane == 0) mbar_arrive_expect_tx(&full[stage], static_cast<uint32_t>(boxes) * 16 * D * 2 * 2);
    } else if (lane == 0) {
      mbar_arrive_expect_tx(&full[stage], static_cast<uint32_t>(nvalid) * D * 2 * 2);
    }
    __syncwarp();
  };
  // Warp 0: one bulk copy per valid row with position in [lo, hi) into the
  // padded shared-memory rows.
  auto copy = [&](int t, int lo, int hi) {
    const int stage = t % S;
    const int p0 = begin + t * T;
    if constexpr (BOX) {
      // Lane w issues group w's box (both 64-dim halves of K and of V) if its
      // valid positions all fall in [lo, hi): groups holding positions the
      // producer kernel still writes are requested after its completion.
      if (lane < C::kWarpsPerCta) {
        const int w = lane, g0 = p0 + w * 16;
        const int g_end = min(g0 + 16, end);
        if (g0 < end && sValid[stage * T + w * 16] && g0 >= lo && g_end <= hi) {
          const int page = page_of(g0 / p.page_size);
          const int y = (page * p.hkv + kvh) * p.page_size + g0 % p.page_size;
#pragma unroll
          for (int h = 0; h < D / 64; ++h) {
            tma_load_2d(reinterpret_cast<unsigned char *>(sK) + (size_t)stage * C::kStageBytes + h * T * 128 + w * 16 * 128,
                        &kmap, h * 64, y, &full[stage]);
            tma_load_2d(reinterpret_cast<unsigned char *>(sV) + (size_t)stage * C::kStageBytes + h * T * 128 + w * 16 * 128,
                        &vmap, h * 64, y, &full[stage]);
          }
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < T / 32; ++j) {
        const int lp = lane + 32 * j;
        const int position = p0 + lp;
        if (position < lo || position >= hi || position >= end || !sValid[stage * T + lp]) continue;
        const int page = page_of(position / p.page_size);
        const size_t off = (((size_t)page * p.hkv + kvh) * p.page_size + position % p.page_size) * D;
        bulk_g2s(sK + ((size_t)stage * T + lp) * ROW, p.k_pool + off, D * 2, &full[stage]);
        bulk_g2s(sV + ((size_t)stage * T + lp) * ROW, p.v_pool + off, D * 2, &full[stage]);
      }
    }
  };

  const int first = ntiles < S ? ntiles : S;
  int issued = first;  // tiles whose copies have been requested (warp 0's count)
  // Boxes (BOX) are all-or-nothing: a box holding any position at or past
  // `fresh` waits for the producer kernel.
  const int early_hi = fresh;
  if (warp == 0) {
    for (int t = 0; t < first; ++t) {
      arm(t);
      copy(t, begin, early_hi);
    }
  }
  pdl_wait();
  if (warp == 0) {
    for (int t = 0; t < first; ++t) {
      if (BOX) {
        // the boxes not issued early: those ending past `fresh`
        const int stage = t % S, p0 = begin + t * T;
        if (lane < C::kWarpsPerCta) {
          const int w = lane, g0 = p0 + w * 16, g_end = min(g0 + 16, end);
          if (g0 < end && sValid[stage * T + w * 16] && g_end > early_hi) {
            const int page = page_of(g0 / p.page_size);
            const int y = (page * p.hkv + kvh) * p.page_size + g0 % p.page_size;
#pragma unroll
            for (int h = 0; h < D / 64; ++h) {
              tma_load_2d(reinterpret_cast<unsigned char *>(sK) + (size_t)stage * C::kStageBytes + h * T * 128 + w * 16 * 128,
                          &kmap, h * 64, y, &full[stage]);
              tma_load_2d(reinterpret_cast<unsigned char *>(sV) + (size_t)stage * C::kStageBytes + h * T * 128 + w * 16 * 128,
                          &vmap, h * 64, y, &full[stage]);
            }
          }
        }
      } else {
        copy(t, fresh, end);
      }
    }
  }
  // Query A fragments: rows = the G query heads of this KV head (rows >= G are
  // zero), columns = head dimensions; fp16 values are exact.
  uint32_t qa[C::kKSteps][4];
  {
    const __half *q = p.q + (size_t)row * p.q_stride + (size_t)kvh * G * D;
#pragma unroll
    for (int kk = 0; kk < C::kKSteps; ++kk) {
      const int c0 = kk * 16 + 2 * tq;
      if (gq < G && !idle) {
        qa[kk][0] = *reinterpret_cast<const uint32_t *>(q + (size_t)gq * D + c0);
        qa[kk][2] = *reinterpret_cast<const uint32_t *>(q + (size_t)gq * D + c0 + 8);
      } else {
        qa[kk][0] = 0u;
        qa[kk][2] = 0u;
      }
      qa[kk][1] = 0u;  // rows 8..15: G <= 8
      qa[kk][3] = 0u;
    }
  }
  if (p.trace.records) t_ready = global_ns();

  // Per-warp flash-decoding state for fragment rows gq (valid when gq < G).
  float m_run = -INFINITY, l_run = 0.0f;
  float acc[C::kDTiles][4];
#pragma unroll
  for (int i = 0; i < C::kDTiles; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.0f;

  for (int t = 0; t < ntiles && !failed; ++t) {
    const int stage = t % S;
    // Warp-uniform outcome: the tile step below is warp-synchronous.
    if (!__all_sync(0xffffffffu, mbar_wait(&full[stage], (t / S) & 1))) {
      if (lane == 0) report_status(p.status, kStatusWaitTimeout, kWhereAttention, t, row);
      failed = true;
      break;
    }
    const int r0 = warp * 16;  // this warp's 16 rows of the tile
    const bool zeroed = tile_step<D, G, BOX>(reinterpret_cast<unsigned char *>(sK) + (size_t)stage * C::kStageBytes,
                                             reinterpret_cast<unsigned char *>(sV) + (size_t)stage * C::kStageBytes,
                                             r0, begin + t * T + r0, end, sValid + stage * T + r0, p.scale, qa,
                                             m_run, l_run, acc, lane);
    if (zeroed) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // before TMA refills
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);
    if (warp == 0 && t + S < ntiles) {
      // Every warp has finished this stage before it is refilled.
      if (!__all_sync(0xffffffffu, mbar_wait(&empty[stage], (t / S) & 1))) {
        if (lane == 0) report_status(p.status, kStatusWaitTimeout, kWhereAttention, t, row);
        failed = true;
        break;
      }
      arm(t + S);
      copy(t + S, begin, end);
      issued = t + S + 1;
    }
  }
  // Let the next kernel launch only now: its weight prefetch would otherwise
  // queue ahead of this kernel's latency-critical loads.
  pdl_launch_dependents();

  // After a wait ran out, copies may still be in flight into the ring: wait
  // (bounded) for the last S requested tiles before the ring is reused for
  // the merge or the CTA exits.
  if (__syncthreads_or(failed ? 1 : 0) && warp == 0 && lane == 0)
    for (int t = issued > S ? issued - S : 0; t < issued; ++t) (void)mbar_wait(&full[t % S], (t / S) & 1);

  // Merge the four warps' states (rows gq < G) in shared memory (the K/V ring
  // is free now): per warp [G][D] accumulators, then m and l per head.
  __syncthreads();
  float *mrg = reinterpret_cast<float *>(smem);
  float *mrg_ml = mrg + C::kWarpsPerCta * G * D;
  if (gq < G) {
#pragma unroll
    for (int dt = 0; dt < C::kDTiles; ++dt) {
      float *dst = mrg + ((size_t)warp * G + gq) * D + dt * 8 + 2 * tq;
      dst[0] = acc[dt][0];
      dst[1] = acc[dt][1];
    }
    if (tq == 0) {
      mrg_ml[(warp * G + gq) * 2] = m_run;
      mrg_ml[(warp * G + gq) * 2 + 1] = l_run;
    }
  }
  __syncthreads();
  // Thread -> (head hg, features [hd, hd + E)) over the merged result.
  constexpr int E = (G * D / kThreads) > 1 ? (G * D / kThreads) : 1;
  const int hg = tid / (D / E);
  const int hd = (tid % (D / E)) * E;
  const bool own = hg < G;
  float m_cta = -INFINITY, l_cta = 0.0f, o_cta[E];
#pragma unroll
  for (int e = 0; e < E; ++e) o_cta[e] = 0.0f;
  if (own) {
#pragma unroll
    for (int w = 0; w < C::kWarpsPerCta; ++w) m_cta = fmaxf(m_cta, mrg_ml[(w * G + hg) * 2]);
#pragma unroll
    for (int w = 0; w < C::kWarpsPerCta; ++w) {
      const float mw = mrg_ml[(w * G + hg) * 2];
      const float f = (mw == -INFINITY) ? 0.0f : expf(mw - m_cta);
      l_cta += mrg_ml[(w * G + hg) * 2 + 1] * f;
#pragma unroll
      for (int e = 0; e < E; ++e) o_cta[e] = fmaf(mrg[((size_t)w * G + hg) * D + hd + e], f, o_cta[e]);
    }
  }
  // Cluster merge: CTA `crank` owns outputs [lo, hi) of G*D. Every CTA sends
  // its (m, l) per head to all owners and each o value to the owner of its
  // output as asynchronous stores that complete on the owner's recv_bar; the
  // owner combines its slice from its own shared memory once all bytes have
  // landed (one one-way trip, no cluster-wide barrier after the sends).
  static_assert(kMaxCluster * G <= kThreads, "one (m, l) send per thread");
  if (own && hd == 0) {
    xml[hg * 2] = m_cta;
    xml[hg * 2 + 1] = l_cta;
  }
  const size_t head_base = ((size_t)row * p.hkv + kvh);
  const int nclusters = (active + (int)csize - 1) / (int)csize;
  const int cidx = split / (int)csize;       // this cluster along the splits
  const int stride = gridDim.x / (int)csize;  // cluster slots per (row, KV head)
  const int per = (G * D + (int)csize - 1) / (int)csize;
  const int lo = (int)crank * per, hi = min(G * D, lo + per);
  __syncthreads();  // xml complete
  cluster_wait();   // phase 0: every CTA of the cluster has started, its recv_bar armed
  if (tid < (int)csize * G) {
    const int q = tid / G, h = tid % G;
    st_async_f32x2(map_cluster(&recv_ml[((int)crank * G + h) * 2], q), xml[h * 2], xml[h * 2 + 1],
                   map_cluster(&recv_bar, q));
  }
  if (own) {
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const int i = hg * D + hd + e, q = i / per;
      st_async_f32(map_cluster(&recv_o[(int)crank * per + i - q * per], q), o_cta[e], map_cluster(&recv_bar, q));
    }
  }
  if (!mbar_wait(&recv_bar, 0)) {
    if (tid == 0) report_status(p.status, kStatusWaitTimeout, kWhereAttention, -1, row);
    // Stores may still be in flight into this CTA: wait once more (bounded)
    // before its shared memory goes away.
    (void)mbar_wait(&recv_bar, 0);
  }
  // Per head of the slice, lane c of a warp takes CTA c's (m, l): the head's
  // maximum and denominator come from warp shuffles and CTA c's weight
  // exp(m - max) goes to shared memory; each output is then one short
  // weighted sum over the CTAs (a once-per-launch path: little code, few
  // dependent steps).
  const int h_lo = lo / D, h_hi = hi > lo ? (hi - 1) / D : h_lo - 1;
  for (int h = h_lo + warp; h <= h_hi; h += C::kWarpsPerCta) {
    const bool in = lane < (int)csize;
    const float m = in ? recv_ml[(lane * G + h) * 2] : -INFINITY;
    const float l = in ? recv_ml[(lane * G + h) * 2 + 1] : 0.0f;
    const float mmax = warp_max(m);
    const float f = (m == -INFINITY) ? 0.0f : expf(m - mmax);
    const float den = warp_sum(l * f);
    if (in) merge_f[lane * G + h] = f;
    if (lane == 0) {
      merge_md[h * 2] = mmax;
      merge_md[h * 2 + 1] = den;
    }
  }
  __syncthreads();
  for (int i = lo + tid; i < hi; i += kThreads) {
    const int h = i / D;
    float num = 0.0f;
#pragma unroll
    for (int c = 0; c < kMaxCluster; ++c)
      if (c < (int)csize) num = fmaf(recv_o[c * per + i - lo], merge_f[c * G + h], num);
    if (nclusters == 1) {
      p.out[(size_t)row * p.out_stride + (size_t)kvh * G * D + i] = __float2half_rn(num / merge_md[h * 2 + 1]);
    } else {
      p.ws_acc[(head_base * stride + cidx) * G * D + i] = num;
      if (i % D == 0) {
        float *wm = p.ws_ml + ((head_base * stride + cidx) * G + h) * 2;
        wm[0] = merge_md[h * 2];
        wm[1] = merge_md[h * 2 + 1];
      }
    }
  }
  if (nclusters == 1) {
    trace_emit(p.trace, t_entry, t_ready);
    return;
  }

  // Several clusters: the last CTA of the (row, KV head) combines them.
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned int prev = atomicAdd(p.counters + head_base, 1u);
    is_last = (prev == static_cast<unsigned int>(nclusters * (int)csize - 1)) ? 1 : 0;
  }
  __syncthreads();
  if (!is_last) {
    trace_emit(p.trace, t_entry, t_ready);
    return;
  }
  __threadfence();
  const float2 *ml = reinterpret_cast<const float2 *>(p.ws_ml + (head_base * stride) * G * 2);
  float *sWl = sW + C::kMaxSplits * G;
  for (int i = tid; i < nclusters * G; i += kThreads) {
    const float2 v = __ldcg(ml + i);
    sW[i] = v.x;
    sWl[i] = v.y;
  }
  __syncthreads();
  for (int g = warp; g < G; g += kThreads / 32) {
    float mx = -INFINITY;
    for (int c = lane; c < nclusters; c += 32) mx = fmaxf(mx, sW[c * G + g]);
    mx = warp_max(mx);
    float den = 0.0f;
    for (int c = lane; c < nclusters; c += 32) {
      const int i = c * G + g;
      const float ms = sW[i];
      const float f = (ms == -INFINITY) ? 0.0f : expf(ms - mx);
      den += sWl[i] * f;
      sW[i] = f;
    }
    den = warp_sum(den);
    const float inv = 1.0f / den;
    for (int c = lane; c < nclusters; c += 32) sW[c * G + g] *= inv;
  }
  __syncthreads();
  for (int i = tid; i < G * D; i += kThreads) {
    const int h = i / D;
    float out = 0.0f;
    for (int c = 0; c < nclusters; ++c)
      out = fmaf(__ldcg(p.ws_acc + (head_base * stride + c) * G * D + i), sW[c * G + h], out);
    p.out[(size_t)row * p.out_stride + (size_t)kvh * G * D + i] = __float2half_rn(out);
  }
  if (tid == 0) atomicExch(p.counters + head_base, 0u);
  trace_emit(p.trace, t_entry, t_ready);
  (void)failed;
}

template <int D, int G, bool BOX>
cudaError_t launch_instance(const AttentionParams &p, cudaStream_t stream, bool pdl) {
  auto kernel = attention_kernel<D, G, BOX>;
  const size_t smem = Cfg<D, G, BOX>::smem_bytes();
  static std::mutex mu;
  static std::unordered_map<int, int> cluster_limit;  // per device, 0 = not configured
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  int limit = 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    limit = cluster_limit[dev];
    if (limit == 0) {
      e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(smem));
      if (e != cudaSuccess) return e;
      limit = 8;
      if (TMC_ATTENTION_CLUSTER_LIMIT > 8 &&
          cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) ==
              cudaSuccess) {
        cudaLaunchConfig_t probe = {};
        probe.gridDim = dim3(TMC_ATTENTION_CLUSTER_LIMIT, 1, 1);
        probe.blockDim = dim3(kThreads);
        probe.dynamicSmemBytes = smem;
        cudaLaunchAttribute ca;
        ca.id = cudaLaunchAttributeClusterDimension;
        ca.val.clusterDim.x = TMC_ATTENTION_CLUSTER_LIMIT;
        ca.val.clusterDim.y = 1;
        ca.val.clusterDim.z = 1;
        probe.attrs = &ca;
        probe.numAttrs = 1;
        int clusters = 0;
        if (cudaOccupancyMaxActiveClusters(&clusters, kernel, &probe) == cudaSuccess && clusters > 0)
          limit = TMC_ATTENTION_CLUSTER_LIMIT;
        (void)cudaGetLastError();
      }
      if (limit > TMC_ATTENTION_CLUSTER_LIMIT) limit = TMC_ATTENTION_CLUSTER_LIMIT;
      cluster_limit[dev] = limit;
    }
  }
  cudaLaunchConfig_t cfg = {};
  // Clusters along the splits; the grid covers whole clusters.
  const int splits = p.max_splits < Cfg<D, G, BOX>::kMaxSplits ? p.max_splits : Cfg<D, G, BOX>::kMaxSplits;
  int cluster = p.cluster;
  if (cluster <= 0) {
    // Clusters pay off for short splits (latency-bound decode, where the
    // merge is a large part of a CTA's life); with long splits (min_chunk >=
    // 512) rows shorter than the cluster would leave idle CTAs holding slots
    // at the cluster barrier, so those launches merge through the ticket.
    cluster = 1;
    while (p.min_chunk < 512 && cluster < splits && cluster < limit) cluster *= 2;
  } else if (cluster > limit) {
    return cudaErrorInvalidValue;
  }
  cfg.gridDim = dim3((splits + cluster - 1) / cluster * cluster, p.hkv, p.rows);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int n = 0;
  attr[n].id = cudaLaunchAttributeClusterDimension;
  attr[n].val.clusterDim.x = cluster;
  attr[n].val.clusterDim.y = 1;
  attr[n].val.clusterDim.z = 1;
  ++n;
  if (pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  CUtensorMap km{}, vm{};
  if (BOX) {
    km = *p.k_map;
    vm = *p.v_map;
  }
  return cudaLaunchKernelEx(&cfg, kernel, p, km, vm);
}

template <int D, bool BOX>
cudaError_t dispatch_g(const AttentionParams &p, cudaStream_t stream, bool pdl, int g) {
  switch (g) {
    case 1: return launch_instance<D, 1, BOX>(p, stream, pdl);
    case 2: return launch_instance<D, 2, BOX>(p, stream, pdl);
    case 4: return launch_instance<D, 4, BOX>(p, stream, pdl);
    case 8: return launch_instance<D, 8, BOX>(p, stream, pdl);
    default: return cudaErrorInvalidValue;
  }
}


// ---- streaming schedule for batched decode -----------------------------------
// With many (row, KV head) pairs (batched decode, serving) the split schedule
// above runs its CTAs in several partial waves and every CTA pays its own
// prologue and pipeline fill. Here one wave of persistent CTAs streams the
// concatenated 64-position tiles of all pairs: pair (r, h) owns the tiles
// [Q[r] + h nt(r), Q[r] + (h + 1) nt(r)) with nt(r) = ceil((pos_r + 1) / 64)
// and Q[r] = Hkv x (tiles of the rows before r); CTA c streams the run
// [W c / grid, W (c + 1) / grid) of the W tiles. A producer warp keeps an
// S-stage TMA ring full across pair boundaries (page lookups included); four
// consumer warps run the same per-tile step as the split kernel. At the end
// of a pair's segment the warps merge; a pair wholly inside the run is
// written out, a pair cut by a run boundary writes (acc, m, l) to its CTA's
// slot (0 for the run's first segment, 1 for its last) and takes a ticket;
// the last piece combines the pieces in CTA order (fixed for a given grid).
// Every wait, the consumer warps' merge barrier included, is a bounded
// mbarrier wait.
constexpr int kStreamRowsMax = 512;
constexpr int kStreamMaxCtas = 640;  // resident CTAs of the streaming schedule, any device
constexpr int kMaxPieces = 8;        // pieces of a cut pair combined through per-row weights

// QR query rows per pair: 1 for decode (one row per sequence; the G query
// heads fill G rows of the MMA's A tile), 16 / G for a row group of prefill
// (QR consecutive positions of one sequence, so all 16 rows are used and
// every K/V tile is read once for QR query rows).
template <int D, int G, int QR>
struct StreamCfg {
  using Tile = Cfg<D, G, true>;
  static constexpr int T = Tile::T;
  static constexpr int kRows = QR * G;  // used rows of the MMA's A tile
  static_assert(kRows <= 16, "a row group fills at most the 16 rows of the A tile");
  // Two CTAs per SM in both forms (registers capped at 168 so that three warps
  // of a partition fit its register file): 3 stages for decode (2 for G = 8),
  // 2 for row groups, whose merge buffer is four times larger. One CTA per SM
  // with a 5-stage ring ran the row groups ~20% slower (fewer math warps).
  static constexpr int kStages = QR == 1 ? (G <= 4 ? 3 : 2) : 2;
  static constexpr size_t kStageBytes = Tile::kStageBytes;  // one of K or V
  static constexpr int kConsumers = 4;
  static constexpr int kThreadsAll = (kConsumers + 1) * 32;
  static constexpr size_t kMergeFloats = (size_t)kConsumers * (kRows * D + 2 * kRows);
  __host__ __device__ static constexpr size_t smem_bytes() {
    return 1024 + (size_t)2 * kStages * kStageBytes + kMergeFloats * 4 + (size_t)kStages * T * 4 +
           (size_t)(kStreamRowsMax + 1) * 4 + (size_t)kStreamRowsMax * 4 * 2 + 128;  // + barriers, alignment
  }
};

// Workspace floats the streaming schedule needs for `grid` CTAs: two
// (acc [rows][D], m/l [rows][2]) slots per CTA, rows = used A-tile rows.
__host__ __device__ constexpr size_t stream_ws_floats(int grid, int rows, int d) {
  return (size_t)grid * 2 * rows * (d + 2);
}

// The CTA whose run holds tile i (runs [W c / grid, W (c + 1) / grid)).
__device__ __forceinline__ int stream_run_of(long long w, int grid, long long i) {
  return (int)(((i + 1) * grid + w - 1) / w) - 1;
}
__device__ __forceinline__ long long stream_run_begin(long long w, int grid, int c) { return w * c / grid; }

// A position in the tile space: row group, KV head, tile within the pair.
struct StreamCursor {
  int grp, h, t, nt;
  long long pair_start;  // global index of the pair's first tile
};

// Bounded barrier of the consumer warps (count = consumer warps) on `bar`.
__device__ __forceinline__ bool consumer_sync(uint64_t *bar, uint32_t &phase, int lane) {
  __threadfence_block();
  __syncwarp();
  if (lane == 0) mbar_arrive(bar);
  const bool ok = __all_sync(0xffffffffu, mbar_wait(bar, phase));
  phase ^= 1u;
  return ok;
}

// The per-tile step with all 16 rows of the A tile in use (row groups): row
// ri = j G + g is query head g of the group's j-th query row. Each row has its
// own end (the thread's rows gq and gq + 8 end at end0 and end1): positions
// past it are masked in the scores. V rows past the group's end (end_max) or
// of a missing page are zeroed, as in tile_step.
template <int D, int G>
__device__ __forceinline__ bool tile_step_rows16(unsigned char *sKs, unsigned char *sVs, int r0, int p0, int end_max,
                                                 int end0, int end1, const int *valid, float scale,
                                                 const uint32_t (&qa)[D / 16][4], float (&m_run)[2],
                                                 float (&l_run)[2], float (&acc)[D / 8][4], int lane) {
  using C = Cfg<D, G, true>;
  constexpr int T = C::T;
  const int tq = lane & 3;
  bool zeroed = false;
  if (p0 >= end_max) return false;
  {
    const int lp = lane & 15;
    const bool bad = !(p0 + lp < end_max && valid[lp]);
    if (__any_sync(0xffffffffu, bad)) {
#pragma unroll
      for (int h = 0; h < D / 64; ++h) {
        uint4 *dst = reinterpret_cast<uint4 *>(sVs + h * T * 128 + (r0 + lp) * 128 + (lane >> 4) * 64);
        if (bad) {
#pragma unroll
          for (int c = 0; c < 4; ++c) dst[c] = make_uint4(0u, 0u, 0u, 0u);
        }
      }
      __syncwarp();
      zeroed = true;
    }
  }
  // Scores S[16 rows x 16 positions] as two n-tiles of 8 positions; c0/c1 are
  // row gq, c2/c3 row gq + 8.
  float sc[2][4];
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.0f;
#pragma unroll
    for (int kk = 0; kk < C::kKSteps; ++kk) {
      uint32_t b0, b1;
      const int R = r0 + nt * 8 + (lane & 7), d0 = kk * 16 + ((lane >> 3) & 1) * 8;
      const __half *addr = reinterpret_cast<const __half *>(sKs + (d0 >> 6) * T * 128 + R * 128 +
                                                            ((((d0 & 63) >> 3) ^ (R & 7)) << 4));
      ldmatrix_x2(b0, b1, addr);
      mma_16816(sc[nt], qa[kk], b0, b1);
    }
  }
  float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int lp = nt * 8 + 2 * tq + j;
      const bool ok = valid[lp] != 0;
      sc[nt][j] = (ok && p0 + lp < end0) ? sc[nt][j] * scale : -INFINITY;
      sc[nt][2 + j] = (ok && p0 + lp < end1) ? sc[nt][2 + j] * scale : -INFINITY;
      mx[0] = fmaxf(mx[0], sc[nt][j]);
      mx[1] = fmaxf(mx[1], sc[nt][2 + j]);
    }
  }
  float rescale[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
    mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
    const float m_new = fmaxf(m_run[r], mx[r]);
    rescale[r] = (m_run[r] == -INFINITY) ? 0.0f : expf(m_run[r] - m_new);
    m_run[r] = m_new;
  }
  float pr[2][4], psum[2] = {0.0f, 0.0f};
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int r = c >> 1;
      pr[nt][c] = (sc[nt][c] == -INFINITY) ? 0.0f : expf(sc[nt][c] - m_run[r]);
      psum[r] += pr[nt][c];
    }
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    psum[r] += __shfl_xor_sync(0xffffffffu, psum[r], 1);
    psum[r] += __shfl_xor_sync(0xffffffffu, psum[r], 2);
    l_run[r] = l_run[r] * rescale[r] + psum[r];
  }
  // P as the A operand in two fp16 parts, hi + lo: a0 / a2 = row gq for
  // positions 0-7 / 8-15, a1 / a3 = row gq + 8.
  uint32_t pa[4], pl[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int nt = i >> 1, c = (i & 1) * 2;  // i: 0 -> (nt 0, row gq), 1 -> (nt 0, gq+8), 2 -> (nt 1, gq), 3 -> (nt 1, gq+8)
    const __half2 h = __floats2half2_rn(pr[nt][c], pr[nt][c + 1]);
    const float2 f = __half22float2(h);
    pa[i] = *reinterpret_cast<const uint32_t *>(&h);
    pl[i] = pack_half2(pr[nt][c] - f.x, pr[nt][c + 1] - f.y);
  }
  // mma_16816's A registers are {a0, a1, a2, a3} = {row gq k0-7, row gq+8 k0-7,
  // row gq k8-15, row gq+8 k8-15}: reorder (nt, row) -> register.
  const uint32_t ah[4] = {pa[0], pa[1], pa[2], pa[3]};
  const uint32_t al[4] = {pl[0], pl[1], pl[2], pl[3]};
#pragma unroll
  for (int dt = 0; dt < C::kDTiles; ++dt) {
    acc[dt][0] *= rescale[0];
    acc[dt][1] *= rescale[0];
    acc[dt][2] *= rescale[1];
    acc[dt][3] *= rescale[1];
    uint32_t b0, b1;
    const int R = r0 + (lane & 15), d0 = dt * 8;
    const __half *addr = reinterpret_cast<const __half *>(sVs + (d0 >> 6) * T * 128 + R * 128 +
                                                          ((((d0 & 63) >> 3) ^ (R & 7)) << 4));
    ldmatrix_x2_trans(b0, b1, addr);
    mma_16816(acc[dt], al, b0, b1);
    mma_16816(acc[dt], ah, b0, b1);
  }
  return zeroed;
}

template <int D, int G, int QR>
__global__ void __maxnreg__(168)  // two 160-thread CTAs per SM
    attention_stream_kernel(const __grid_constant__ AttentionParams p, const __grid_constant__ CUtensorMap kmap,
                            const __grid_constant__ CUtensorMap vmap) {
  using C = StreamCfg<D, G, QR>;
  using Tl = Cfg<D, G, true>;
  constexpr int T = C::T, S = C::kStages, NC = C::kConsumers, RW = C::kRows;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  unsigned char *base =
      reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char *sK = base;
  unsigned char *sV = base + (size_t)S * C::kStageBytes;
  float *mrg = reinterpret_cast<float *>(base + (size_t)2 * S * C::kStageBytes);
  float *mrg_ml = mrg + (size_t)NC * RW * D;
  int *sValid = reinterpret_cast<int *>(mrg + C::kMergeFloats);
  int *sPrefix = sValid + S * T;              // [groups + 1] tile starts of the groups (Q / Hkv)
  int *sEnd = sPrefix + kStreamRowsMax + 1;   // [groups] longest context of the group
  int *sTable = sEnd + kStreamRowsMax;        // [groups] block-table row of the group
  uint64_t *full = reinterpret_cast<uint64_t *>(
      (reinterpret_cast<uintptr_t>(sTable + kStreamRowsMax) + 15) & ~uintptr_t(15));
  uint64_t *empty = full + S;
  uint64_t *merge_bar = empty + S;
  __shared__ int s_last;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int hkv = p.hkv, rows = p.rows;
  const int groups = (rows + QR - 1) / QR;
  const unsigned long long t_entry = p.trace.records ? global_ns() : 0ull;
  unsigned long long t_ready = t_entry;

  // Tiles of the groups (positions and the block table are final before the
  // kernel that produces q starts): a group's tiles cover its longest context;
  // a row with a position outside the cache is reported and left out.
  for (int gi = tid; gi < groups; gi += blockDim.x) {
    int end = 0;
#pragma unroll 1
    for (int j = 0; j < QR; ++j) {
      const int r = gi * QR + j;
      if (r >= rows) break;
      const int pos = p.positions[r];
      if (pos < 0 || pos >= p.capacity) {
        report_status(p.status, kStatusLengthRange, kWhereAttention, pos, r);
      } else {
        end = max(end, pos + 1);
      }
    }
    sEnd[gi] = end;
    sTable[gi] = p.table_rows[gi * QR];  // the rows of a group share one block-table row
    sPrefix[gi + 1] = (end + T - 1) / T;
  }
  if (tid == 0) {
    sPrefix[0] = 0;
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NC);
    }
    mbar_init(merge_bar, NC);
    fence_barrier_init();
  }
  __syncthreads();
  if (warp == 0) {
    // Inclusive scan in chunks of 32 groups (each lane reads, then writes, its own entry).
    int carry = 0;
    for (int g0 = 0; g0 < groups; g0 += 32) {
      const int gi = g0 + lane;
      int v = gi < groups ? sPrefix[gi + 1] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += n;
      }
      if (gi < groups) sPrefix[gi + 1] = carry + v;
      carry += __shfl_sync(0xffffffffu, v, 31);
    }
  }
  __syncthreads();
  const long long W = (long long)sPrefix[groups] * hkv;
  // Runs over min(grid, W) CTAs, so every run is non-empty (the pieces of a
  // cut pair are then consecutive CTAs); the others have nothing to do.
  const int grid = (int)(W < (long long)gridDim.x ? W : (long long)gridDim.x);
  const bool has_run = W > 0 && (int)blockIdx.x < grid;
  const long long run_a = has_run ? stream_run_begin(W, grid, blockIdx.x) : 0;
  const long long run_b = has_run ? stream_run_begin(W, grid, blockIdx.x + 1) : 0;
  const int ntiles = (int)(run_b - run_a);

  // The cursor at global tile i: the last group whose tiles start at or before
  // i (that group has tiles), then the KV head and the tile within the pair.
  auto locate = [&](long long i) {
    int lo = 0, hi = groups - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if ((long long)sPrefix[mid] * hkv <= i) lo = mid; else hi = mid - 1;
    }
    StreamCursor c;
    c.grp = lo;
    c.nt = sPrefix[lo + 1] - sPrefix[lo];
    const long long off = i - (long long)sPrefix[lo] * hkv;
    c.h = (int)(off / c.nt);
    c.t = (int)(off % c.nt);
    c.pair_start = (long long)sPrefix[lo] * hkv + (long long)c.h * c.nt;
    return c;
  };
  auto advance = [&](StreamCursor &c) {
    if (++c.t < c.nt) return;
    c.t = 0;
    if (++c.h < hkv) {
      c.pair_start += c.nt;
      return;
    }
    c.h = 0;
    do {
      ++c.grp;
    } while (c.grp < groups && sPrefix[c.grp + 1] == sPrefix[c.grp]);
    if (c.grp < groups) {
      c.nt = sPrefix[c.grp + 1] - sPrefix[c.grp];
      c.pair_start = (long long)sPrefix[c.grp] * hkv;
    }
  };

  if (warp == NC) {
    // ---- producer warp: the ring, across pairs ----
    bool waited = false;
    int issued = 0;
    // Lane w < 4 looks up box group w's page for tile cursor c (16 positions,
    // one page); -1 when the group is past the context or its page is bad.
    auto lookup = [&](const StreamCursor &c) {
      int page = -1;
      if (lane < NC) {
        const int len = sEnd[c.grp], g0 = c.t * T + lane * 16;
        if (g0 < len) {
          const int logical = g0 / p.page_size;
          page = logical < p.table_stride ? p.block_table[(size_t)sTable[c.grp] * p.table_stride + logical] : -1;
          if (page < 0) {
            report_status(p.status, kStatusPageMissing, kWhereAttention, logical, c.grp * QR);
          } else if (page >= p.pool_pages) {
            report_status(p.status, kStatusPageRange, kWhereAttention, page, c.grp * QR);
            page = -1;
          }
        }
      }
      return page;
    };
    if (ntiles > 0) {
      StreamCursor c = locate(run_a);
      // The next tile's pages are looked up one tile ahead, so the table
      // load's latency overlaps the wait for a free stage and this tile's issue.
      int page_next = lookup(c);
      for (int k = 0; k < ntiles; ++k) {
        const int stage = k % S;
        const int page = page_next;
        StreamCursor cn = c;
        advance(cn);
        if (k + 1 < ntiles) page_next = lookup(cn);
        if (k >= S && !__all_sync(0xffffffffu, mbar_wait(&empty[stage], ((k / S) - 1) & 1))) {
          if (lane == 0) report_status(p.status, kStatusWaitTimeout, kWhereAttention, k, c.grp);
          break;
        }
        const int len = sEnd[c.grp], p0 = c.t * T;
        // Rows the preceding kernel still writes: the row's own newest
        // position (early_mode 1, one row per group), every row (0), none (2).
        const int fresh = p.early_mode == 2 ? len : (p.early_mode == 1 && QR == 1 ? len - 1 : 0);
        if (!waited && p0 + T > fresh) {
          pdl_wait();
          waited = true;
        }
        // Valid rows of the tile (positions before len in a valid page).
#pragma unroll
        for (int j = 0; j < T / 32; ++j) {
          const int lp = lane + 32 * j;
          const int gp = __shfl_sync(0xffffffffu, page, lp >> 4);
          sValid[stage * T + lp] = (p0 + lp < len && gp >= 0) ? 1 : 0;
        }
        const unsigned boxes = __popc(__ballot_sync(0xffffffffu, lane < NC && page >= 0));
        __syncwarp();
        if (lane == 0) mbar_arrive_expect_tx(&full[stage], boxes * 16u * D * 2u * 2u);
        __syncwarp();
        if (lane < NC && page >= 0) {
          const int g0 = p0 + lane * 16;
          const int y = (page * hkv + c.h) * p.page_size + g0 % p.page_size;
#pragma unroll
          for (int hh = 0; hh < D / 64; ++hh) {
            tma_load_2d(sK + (size_t)stage * C::kStageBytes + hh * T * 128 + lane * 16 * 128, &kmap, hh * 64, y,
                        &full[stage]);
            tma_load_2d(sV + (size_t)stage * C::kStageBytes + hh * T * 128 + lane * 16 * 128, &vmap, hh * 64, y,
                        &full[stage]);
          }
        }
        issued = k + 1;
        c = cn;
      }
    }
    if (!waited) pdl_wait();
    pdl_launch_dependents();
    // No copy may still be landing when the CTA exits: wait (bounded) for the
    // last S requested tiles (already consumed ones return at once).
    for (int k = issued > S ? issued - S : 0; k < issued; ++k) (void)mbar_wait(&full[k % S], (k / S) & 1);
    trace_emit(p.trace, t_entry, t_ready);
    return;
  }

  // ---- consumer warps ----
  const int gq = lane >> 2, tq = lane & 3;
  pdl_wait();  // q is written by the preceding kernel
  if (p.trace.records) t_ready = global_ns();
  uint32_t merge_phase = 0;
  bool failed = false;
  // The query row and head of A-tile row ri of group grp (row -1: none).
  auto row_of = [&](int grp, int ri) { return QR == 1 ? grp : (ri / G < QR ? grp * QR + ri / G : -1); };
  auto head_of = [&](int ri) { return QR == 1 ? ri : ri % G; };
  if (ntiles > 0) {
    StreamCursor c = locate(run_a);
    uint32_t qa[Tl::kKSteps][4];
    float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.0f, 0.0f};
    float acc[Tl::kDTiles][4];
    int end_r[2] = {0, 0};  // QR > 1: ends of the thread's rows gq and gq + 8
    long long seg_first = run_a;  // global index of the segment's first tile
    for (int k = 0; k < ntiles && !failed; ++k) {
      const long long gi = run_a + k;
      if (gi == seg_first) {
        // A new pair: the query fragments of its rows (unused rows zero) and a
        // fresh online-softmax state.
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int ri = gq + 8 * half;
          int row = -1;
          if (ri < RW) row = row_of(c.grp, ri);
          if (row >= rows) row = -1;
          if (QR > 1) {
            int e = 0;
            if (row >= 0) {
              const int pos = p.positions[row];
              e = (pos >= 0 && pos < p.capacity) ? pos + 1 : 0;
            }
            end_r[half] = e;
          }
          const __half *q = row >= 0 ? p.q + (size_t)row * p.q_stride + (size_t)(c.h * G + head_of(ri)) * D : nullptr;
#pragma unroll
          for (int kk = 0; kk < Tl::kKSteps; ++kk) {
            const int c0 = kk * 16 + 2 * tq;
            qa[kk][half] = q ? *reinterpret_cast<const uint32_t *>(q + c0) : 0u;
            qa[kk][2 + half] = q ? *reinterpret_cast<const uint32_t *>(q + c0 + 8) : 0u;
          }
        }
        m_run[0] = m_run[1] = -INFINITY;
        l_run[0] = l_run[1] = 0.0f;
#pragma unroll
        for (int i = 0; i < Tl::kDTiles; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.0f;
      }
      const int stage = k % S;
      if (!__all_sync(0xffffffffu, mbar_wait(&full[stage], (k / S) & 1))) {
        if (lane == 0) report_status(p.status, kStatusWaitTimeout, kWhereAttention, k, c.grp);
        failed = true;
        break;
      }
      const int len = sEnd[c.grp];
      const int r0 = warp * 16;
      bool zeroed;
      if constexpr (QR == 1) {
        zeroed = tile_step<D, G, true>(sK + (size_t)stage * C::kStageBytes, sV + (size_t)stage * C::kStageBytes,
                                       r0, c.t * T + r0, len, sValid + stage * T + r0, p.scale, qa, m_run[0],
                                       l_run[0], acc, lane);
      } else {
        zeroed = tile_step_rows16<D, G>(sK + (size_t)stage * C::kStageBytes, sV + (size_t)stage * C::kStageBytes,
                                        r0, c.t * T + r0, len, end_r[0], end_r[1], sValid + stage * T + r0, p.scale,
                                        qa, m_run, l_run, acc, lane);
      }
      if (zeroed) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // before TMA refills
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[stage]);

      const bool seg_end = c.t == c.nt - 1 || k == ntiles - 1;
      if (seg_end) {
        // Merge the warps' states (used rows), then write or hand over.
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int ri = gq + 8 * half;
          if (ri < RW && (QR > 1 || half == 0)) {
#pragma unroll
            for (int dt = 0; dt < Tl::kDTiles; ++dt) {
              float *dst = mrg + ((size_t)warp * RW + ri) * D + dt * 8 + 2 * tq;
              dst[0] = acc[dt][2 * half];
              dst[1] = acc[dt][2 * half + 1];
            }
            if (tq == 0) {
              mrg_ml[(warp * RW + ri) * 2] = m_run[half];
              mrg_ml[(warp * RW + ri) * 2 + 1] = l_run[half];
            }
          }
        }
        if (!consumer_sync(merge_bar, merge_phase, lane)) {
          failed = true;
          break;
        }
        const bool whole = seg_first == c.pair_start && c.t == c.nt - 1;
        const int slot = seg_first == run_a ? 0 : 1;
        const int ct = tid;  // 0 .. 127
        const size_t pair = (size_t)c.grp * hkv + c.h;
        float *ws_acc = p.ws_acc + ((size_t)blockIdx.x * 2 + slot) * RW * D;
        float *ws_ml = p.ws_ml + ((size_t)blockIdx.x * 2 + slot) * RW * 2;
        for (int i = ct; i < RW * D; i += NC * 32) {
          const int ri = i / D;
          float m_cta = -INFINITY;
#pragma unroll
          for (int w = 0; w < NC; ++w) m_cta = fmaxf(m_cta, mrg_ml[(w * RW + ri) * 2]);
          float l_cta = 0.0f, o = 0.0f;
#pragma unroll
          for (int w = 0; w < NC; ++w) {
            const float mw = mrg_ml[(w * RW + ri) * 2];
            const float f = (mw == -INFINITY) ? 0.0f : expf(mw - m_cta);
            l_cta += mrg_ml[(w * RW + ri) * 2 + 1] * f;
            o = fmaf(mrg[((size_t)w * RW + ri) * D + (i % D)], f, o);
          }
          if (whole) {
            const int row = row_of(c.grp, ri);
            if (row >= 0 && row < rows)
              p.out[(size_t)row * p.out_stride + (size_t)(c.h * G + head_of(ri)) * D + i % D] =
                  __float2half_rn(o / l_cta);
          } else {
            ws_acc[i] = o;
            if (i % D == 0) {
              ws_ml[ri * 2] = m_cta;
              ws_ml[ri * 2 + 1] = l_cta;
            }
          }
        }
        if (!whole) {
          // Every thread's partial stores, then the consumers' barrier, then
          // thread 0's GPU-scope acquire-release ticket: the last piece's
          // acquire (and its barrier) orders the other pieces' stores before
          // its loads, without a GPU-scope fence in every thread.
          if (!consumer_sync(merge_bar, merge_phase, lane)) {
            failed = true;
            break;
          }
          const long long pair_end = c.pair_start + c.nt;
          const int c_first = stream_run_of(W, grid, c.pair_start);
          const int c_last = stream_run_of(W, grid, pair_end - 1);
          if (ct == 0) {
            const unsigned int prev = atomic_add_acq_rel_gpu(p.counters + pair, 1u);
            s_last = prev == (unsigned int)(c_last - c_first) ? 1 : 0;
          }
          if (!consumer_sync(merge_bar, merge_phase, lane)) {
            failed = true;
            break;
          }
          if (s_last) {
            // The last piece: combine the pieces in CTA order. A piece sits in
            // slot 0 of a CTA whose run starts inside the pair (every CTA after
            // the first, and the first when its run starts at the pair), else
            // in slot 1. First one thread per row turns the pieces' (m, l)
            // into weights (in the merge buffer, free by now), then every
            // element sums its pieces' accumulators with all of its loads
            // independent -- loops of dependent L2 round trips per element
            // cost tens of microseconds per launch.
            const bool first_slot0 = stream_run_begin(W, grid, c_first) >= c.pair_start;
            const int np = c_last - c_first + 1;
            auto slot_of = [&](int q) { return (q > 0 || first_slot0) ? 0 : 1; };
            float *wts = mrg;  // [RW][kMaxPieces] combine weights
            if (np <= kMaxPieces) {
              if (ct < RW) {
                float m[kMaxPieces], mmax = -INFINITY;
#pragma unroll
                for (int q = 0; q < kMaxPieces; ++q) {
                  m[q] = q < np ? __ldcg(p.ws_ml + ((size_t)(c_first + q) * 2 + slot_of(q)) * RW * 2 + ct * 2)
                               : -INFINITY;
                  mmax = fmaxf(mmax, m[q]);
                }
                float den = 0.0f;
#pragma unroll
                for (int q = 0; q < kMaxPieces; ++q) {
                  const float f = (m[q] == -INFINITY) ? 0.0f : expf(m[q] - mmax);
                  if (q < np)
                    den = fmaf(__ldcg(p.ws_ml + ((size_t)(c_first + q) * 2 + slot_of(q)) * RW * 2 + ct * 2 + 1), f,
                               den);
                  m[q] = f;
                }
#pragma unroll
                for (int q = 0; q < kMaxPieces; ++q) wts[ct * kMaxPieces + q] = m[q] / den;
              }
              if (!consumer_sync(merge_bar, merge_phase, lane)) {
                failed = true;
                break;
              }
#pragma unroll
              for (int e = 0; e < (RW * D + NC * 32 - 1) / (NC * 32); ++e) {
                const int i = ct + e * NC * 32;
                if (i >= RW * D) break;
                const int ri = i / D;
                const int row = row_of(c.grp, ri);
                float num = 0.0f;
                for (int q = 0; q < np; ++q)
                  num = fmaf(__ldcg(p.ws_acc + ((size_t)(c_first + q) * 2 + slot_of(q)) * RW * D + i),
                             wts[ri * kMaxPieces + q], num);
                if (row >= 0 && row < rows)
                  p.out[(size_t)row * p.out_stride + (size_t)(c.h * G + head_of(ri)) * D + i % D] =
                      __float2half_rn(num);
              }
            } else {
              for (int i = ct; i < RW * D; i += NC * 32) {
                const int ri = i / D;
                const int row = row_of(c.grp, ri);
                if (row < 0 || row >= rows) continue;
                float mmax = -INFINITY;
                for (int q = 0; q < np; ++q)
                  mmax = fmaxf(mmax, __ldcg(p.ws_ml + ((size_t)(c_first + q) * 2 + slot_of(q)) * RW * 2 + ri * 2));
                float den = 0.0f, num = 0.0f;
                for (int q = 0; q < np; ++q) {
                  const size_t sl = (size_t)(c_first + q) * 2 + slot_of(q);
                  const float mc = __ldcg(p.ws_ml + sl * RW * 2 + ri * 2);
                  const float f = (mc == -INFINITY) ? 0.0f : expf(mc - mmax);
                  den = fmaf(__ldcg(p.ws_ml + sl * RW * 2 + ri * 2 + 1), f, den);
                  num = fmaf(__ldcg(p.ws_acc + sl * RW * D + i), f, num);
                }
                p.out[(size_t)row * p.out_stride + (size_t)(c.h * G + head_of(ri)) * D + i % D] =
                    __float2half_rn(num / den);
              }
            }
            if (ct == 0) atomicExch(p.counters + pair, 0u);
          }
        }
        // The merge buffer is free again once every warp has read it.
        if (!consumer_sync(merge_bar, merge_phase, lane)) {
          failed = true;
          break;
        }
        seg_first = gi + 1;
      }
      advance(c);
    }
  }
  pdl_launch_dependents();
  trace_emit(p.trace, t_entry, t_ready);
}

template <int D, int G, int QR>
cudaError_t launch_stream_instance(const AttentionParams &p, cudaStream_t stream, bool pdl, int grid) {
  auto kernel = attention_stream_kernel<D, G, QR>;
  const size_t smem = StreamCfg<D, G, QR>::smem_bytes();
  static std::mutex mu;
  static std::unordered_map<int, bool> configured;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!configured[dev]) {
      e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
      if (e != cudaSuccess) return e;
      configured[dev] = true;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(StreamCfg<D, G, QR>::kThreadsAll);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, p, *p.k_map, *p.v_map);
}

// Persistent CTAs the streaming schedule runs for this shape (one wave), or 0
// when it does not fit.
template <int D, int G, int QR>
int stream_grid_for(int num_sms) {
  static std::mutex mu;
  static std::unordered_map<int, int> per_sm;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  std::lock_guard<std::mutex> lock(mu);
  auto it = per_sm.find(dev);
  if (it == per_sm.end()) {
    auto kernel = attention_stream_kernel<D, G, QR>;
    const size_t smem = StreamCfg<D, G, QR>::smem_bytes();
    int blocks = 0;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
            cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, kernel, StreamCfg<D, G, QR>::kThreadsAll, smem) !=
            cudaSuccess)
      blocks = 0;
    (void)cudaGetLastError();
    it = per_sm.emplace(dev, blocks).first;
  }
  return it->second * num_sms;
}

}  // namespace

size_t attention_workspace_bytes(int rows, int hq, int hkv, int head_dim, int max_splits) {
  const size_t acc = (size_t)rows * hq * max_splits * head_dim * 4;
  const size_t ml = (size_t)rows * hq * max_splits * 2 * 4;
  // The streaming schedule's per-CTA slots, for up to kStreamMaxCtas resident
  // CTAs (a bound for any device: the grid is the occupancy times the SMs).
  const int g = hkv > 0 && hq % hkv == 0 ? hq / hkv : 1;
  const size_t stream = stream_ws_floats(kStreamMaxCtas, g, head_dim) * 4;
  return acc + ml > stream ? acc + ml : stream;
}

size_t attention_group_workspace_bytes(int head_dim) {
  return stream_ws_floats(kStreamMaxCtas, 16, head_dim) * 4;
}

cudaError_t launch_attention(const AttentionParams &p, cudaStream_t stream, bool pdl) {
  if (p.rows <= 0 || p.hkv <= 0 || p.hq <= 0 || p.hq % p.hkv != 0 || p.max_splits <= 0 ||
      p.min_chunk <= 0 || p.page_size <= 0 || p.rows > 65535 || p.hkv > 65535 ||
      p.cluster < 0 || p.cluster > kMaxCluster || (p.cluster & (p.cluster - 1)) != 0)
    return cudaErrorInvalidValue;
  const int g = p.hq / p.hkv;
  // Page boxes through tensor maps when the caller built them and the shape
  // allows (64-dim halves, pages of whole 16-position groups).
  const bool box = p.k_map != nullptr && p.v_map != nullptr && p.page_size % 16 == 0;
  // Many (row, KV head) pairs, or row groups: the streaming schedule, when the
  // caller's workspace holds its per-CTA slots.
  const bool grouped = p.row_group > 1;
  if (box && p.schedule != 1 && p.rows <= kStreamRowsMax && (p.head_dim == 64 || p.head_dim == 128) &&
      (g == 1 || g == 2 || g == 4 || g == 8)) {
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) !=
                                                   cudaSuccess)
      return cudaErrorInvalidValue;
    const int qr = grouped ? 16 / g : 1;
    const long long pairs = (long long)((p.rows + qr - 1) / qr) * p.hkv;
    // Measured at context 1280, 8 KV heads: streaming 59.7 vs split 16.8 us
    // at 1 row, equal at 8 rows (64 pairs), 36.7 vs 46.5 us at 16 rows.
    if (p.schedule == 2 || 2 * pairs >= sms) {
      int grid = 0;
#define TMC_STREAM_GRID(D_, G_)                                                          \
  if (p.head_dim == D_ && g == G_)                                                       \
    grid = grouped ? stream_grid_for<D_, G_, 16 / G_>(sms) : stream_grid_for<D_, G_, 1>(sms);
      TMC_STREAM_GRID(64, 1) TMC_STREAM_GRID(64, 2) TMC_STREAM_GRID(64, 4) TMC_STREAM_GRID(64, 8)
      TMC_STREAM_GRID(128, 1) TMC_STREAM_GRID(128, 2) TMC_STREAM_GRID(128, 4) TMC_STREAM_GRID(128, 8)
#undef TMC_STREAM_GRID
      const int used_rows = qr * g;
      if (grid > 0 && grid <= kStreamMaxCtas && p.ws_floats >= stream_ws_floats(grid, used_rows, p.head_dim)) {
        AttentionParams q = p;
        q.ws_ml = q.ws_acc + (size_t)grid * 2 * used_rows * p.head_dim;
#define TMC_STREAM_LAUNCH(D_, G_)                                                                     \
  if (p.head_dim == D_ && g == G_)                                                                    \
    return grouped ? launch_stream_instance<D_, G_, 16 / G_>(q, stream, pdl, grid)                    \
                   : launch_stream_instance<D_, G_, 1>(q, stream, pdl, grid);
        TMC_STREAM_LAUNCH(64, 1) TMC_STREAM_LAUNCH(64, 2) TMC_STREAM_LAUNCH(64, 4) TMC_STREAM_LAUNCH(64, 8)
        TMC_STREAM_LAUNCH(128, 1) TMC_STREAM_LAUNCH(128, 2) TMC_STREAM_LAUNCH(128, 4) TMC_STREAM_LAUNCH(128, 8)
#undef TMC_STREAM_LAUNCH
      }
      if (p.schedule == 2) return cudaErrorInvalidValue;
    }
  }
  switch (p.head_dim) {
    case 16: return dispatch_g<16, false>(p, stream, pdl, g);
    case 32: return dispatch_g<32, false>(p, stream, pdl, g);
    case 64: return box ? dispatch_g<64, true>(p, stream, pdl, g) : dispatch_g<64, false>(p, stream, pdl, g);
    case 128: return box ? dispatch_g<128, true>(p, stream, pdl, g) : dispatch_g<128, false>(p, stream, pdl, g);
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
// stand-in, not device memory). The address stays cached for the life of the
// process, so the entry point must not be used after cudaDeviceReset (or any
// other teardown of the device's primary context) in the same process.
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
  // The kernel never uses more than 64 splits, so the scratch is sized (and
  // the m/l partials placed) for the capped count: a request with a larger
  // max_splits runs exactly as the allocating entry point runs it.
  const int splits = max_splits < tmc::kAttentionMaxSplits ? max_splits : tmc::kAttentionMaxSplits;
  // Scratch layout: split partials (acc, then m/l), then the tickets.
  const size_t partials = tmc::attention_workspace_bytes(rows, hq, hkv, d, splits);
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
  p.max_splits = splits;
  p.min_chunk = min_chunk;
  p.early_mode = 2;  // standalone call: no kernel produces K/V concurrently
  p.ws_acc = reinterpret_cast<float *>(base);
  p.ws_ml = reinterpret_cast<float *>(base + (size_t)rows * hq * splits * d * sizeof(float));
  p.ws_floats = partials / sizeof(float);
  p.counters = tickets;
  p.status = static_cast<tmc::TmcDeviceStatus *>(status);
  // Same kernel variant as the allocating entry point: K/V as 16-position page
  // boxes through tensor maps when the shape allows. Encoding a tensor map
  // fills a host-side descriptor and allocates nothing.
  CUtensorMap km, vm;
  if ((d == 64 || d == 128) && page_size % 16 == 0 && (reinterpret_cast<uintptr_t>(k_pool) & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(v_pool) & 15) == 0) {
    const uint64_t pool_rows = (uint64_t)pool_pages * hkv * page_size;
    if (tmc::make_tensor_map_f16(&km, k_pool, pool_rows, d, 16) == cudaSuccess &&
        tmc::make_tensor_map_f16(&vm, v_pool, pool_rows, d, 16) == cudaSuccess) {
      p.k_map = &km;
      p.v_map = &vm;
    }
  }
  e = tmc::launch_attention(p, s, false);
  if (e == cudaErrorInvalidValue) return fail(TMC_ERR_UNSUPPORTED, "attention: unsupported shape");
  return e == cudaSuccess ? ok() : cuda_fail(e, "attention (no-alloc) launch");
}
