// Batched decode projections on tcgen05 tensor cores (see gemm.cuh).
//
// One persistent CTA per SM, 10 warps, warp-specialised:
//   warp 0    TMA producer: streams 128-row x (64 x atoms)-column weight
//             tiles (A, one 64-column swizzle atom per TMA box) and the
//             matching columns of the token rows (B) into a ring of
//             shared-memory stages (128-byte swizzle). Weight tiles do not
//             depend on earlier kernels, so the first ring-full is requested
//             before the programmatic-dependency wait;
//   warp 1    owns the tensor memory (four TN-column fp32 accumulators) and
//             issues the MMAs from one thread: 4 x atoms (M=128, N=TN,
//             K=16) per stage, tcgen05.commit frees the stage, a final commit hands the
//             accumulator to the epilogue;
//   warps 2-9 epilogue, two per 32-lane quarter of the accumulator (warp w
//             reads lanes 32 (w % 4) ..), taking alternate 16-token groups:
//             tcgen05.ld of their quarter of the
//             accumulator (one output feature per thread, TN tokens), then the
//             GEMV's per-element epilogues. With four accumulators the
//             epilogues of finished units overlap the MMAs of the next ones.
// Work division is stream-K (gemm.cuh): CTA c streams the iterations
// [W c / G, W (c + 1) / G) of the W = tiles x kblocks (tile, K block) space;
// each tile it touches is one piece. A piece that covers only part of its
// tile writes an fp32 partial to the CTA's workspace slot and counts itself
// in on the tile's arrival counter. The tile's "closers" -- the pieces whose
// runs end inside the tile, so their CTAs have nothing left to stream -- wait
// (bounded) for all pieces, then share the reduction: closer i sums groups
// i, i + closers, ... of 16 tokens over all partials in K order and applies
// the epilogue. Every CTA of the grid is resident before any closer waits
// (grid <= SMs, one CTA per SM, and the next kernel launches only after all of
// them passed their dependency trigger), so the waits end.
// Every mbarrier wait is bounded (mbarrier.cuh); a timeout is reported in the
// device status block and the CTA still releases its tensor memory and exits.
#include "gemm.cuh"

#include <mutex>
#include <unordered_map>

#include "epilogue.cuh"
#include "mbarrier.cuh"

namespace tmc {
namespace {

constexpr int kGemmThreads = 320;
constexpr int kEpiWarps = 8;
constexpr int kGroup = 16;      // token columns an epilogue step handles (one tcgen05.ld)
constexpr int kMaxTokens = 256;  // the largest TN
constexpr unsigned long long kTileWaitNs = 1000000000ull;  // a closer waits at most 1 s for the tile's pieces

// Epilogue kinds the kernel is specialised on: each instantiation carries one
// epilogue body, run by a non-unrolled loop over 16-token groups, so the
// kernel's code stays small enough for the instruction caches (a 64-token
// unrolled body of every kind made the code ~700 KB, and the tile's last,
// once-per-launch reduction ran out of cold instruction memory).
enum EpiKind : int { kEkQKV, kEkSwiGLU, kEkHalf, kEkF32, kEkArgmax };
constexpr int kTileBytesA = kGemmTileRows * kGemmKBlock * 2;  // 16 KB

template <int TN>
struct GemmCfg {
  static constexpr int kAtoms = gemm_k_atoms(TN);
  static constexpr int kBytesB = TN * kGemmKBlock * 2;  // one atom of token rows
  static constexpr int kStageBytes = kAtoms * (kTileBytesA + kBytesB);
  static constexpr int kStages = (216 * 1024 / kStageBytes) < 8 ? (216 * 1024 / kStageBytes) : 8;
  static_assert(kStages >= 2, "a pipeline needs two stages");
  // Accumulators in tensor memory (epilogues overlap later MMAs): four, two
  // for 256 tokens (512 columns, all of it).
  static constexpr int kAcc = TN >= 256 ? 2 : 4;
  static constexpr int kTmemCols = kAcc * TN < 32 ? 32 : kAcc * TN;  // a power of two, <= 512
  static constexpr size_t kSmem = 1024 + (size_t)kStages * kStageBytes + 256;
};

struct GemmWork {
  int tiles, kblocks;
  float *ws;
  unsigned int *tile_counters;
};

// First iteration of CTA c's run (iterations [run_begin(c), run_begin(c + 1))).
__device__ __forceinline__ long long run_begin(long long iters, int grid, int c) { return iters * c / grid; }
// The CTA whose run holds iteration i: the largest c with run_begin(c) <= i.
__device__ __forceinline__ int run_of(long long iters, int grid, long long i) {
  return (int)(((i + 1) * grid + iters - 1) / iters) - 1;
}

// The pieces of this CTA's run, in order: tile, K blocks [kb0, kb1), and its
// index among the run's pieces (partials use slot 0 for the first piece and
// 1 for the last; middle pieces always cover whole tiles).
struct Piece {
  int tile, kb0, kb1, index;
};
struct RunCursor {
  long long next, end;
  int kblocks, index;
  __device__ RunCursor(const GemmWork &w)
      : next(run_begin((long long)w.tiles * w.kblocks, gridDim.x, blockIdx.x)),
        end(run_begin((long long)w.tiles * w.kblocks, gridDim.x, blockIdx.x + 1)),
        kblocks(w.kblocks),
        index(0) {}
  __device__ bool get(Piece &pc) {
    if (next >= end) return false;
    pc.tile = (int)(next / kblocks);
    const long long t0 = (long long)pc.tile * kblocks;
    pc.kb0 = (int)(next - t0);
    pc.kb1 = (int)((end - t0) < kblocks ? (end - t0) : kblocks);
    pc.index = index++;
    next = t0 + pc.kb1;
    return true;
  }
};


// Shared-memory matrix descriptor of a K-major tile with 128-byte rows and
// 128-byte swizzle (the layout TMA writes with CU_TENSOR_MAP_SWIZZLE_128B):
// start address, leading offset 1 (unused when K fits one swizzle row),
// stride 1024 bytes between 8-row groups, descriptor version 1, layout 2.
__device__ __forceinline__ uint64_t sw128_desc(const void *smem) {
  uint64_t d = (uint64_t)((smem_u32(smem) >> 4) & 0x3FFFu);
  d |= (uint64_t)1u << 16;
  d |= (uint64_t)(1024u >> 4) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)2u << 61;
  return d;
}

__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 16 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float *v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Named barrier of the eight epilogue warps.
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

// The epilogue of 16 tokens (m0 .. m0 + 15 of the launch's rows) for this
// thread's output feature `row`, values in v: the arithmetic shared with the
// GEMV (epilogue.cuh). Values are computed unconditionally; loads and stores
// are predicated (M <= 0 for a warp half without a group this round). QKV
// reads the per-token position / KV slot staged in shared memory for the
// piece (tok_pos, tok_slot, indexed by token). The two warp halves (ew / 4)
// work on groups m0 and m0 +- 16 at the same time.
template <int EK>
__device__ __forceinline__ void apply_group(const GemvParams &p, const float (&v)[kGroup], int m0, bool active,
                                            int row, int lane, int ew, int t,
                                            unsigned long long (*red_keys)[kGroup], int *half_m0,
                                            const int *tok_pos, const long long *tok_slot) {
  const int M = active ? p.M - m0 : 0;
  const bool in_range = row < p.N;
  const long long ys = p.y_stride;
  if constexpr (EK == kEkArgmax) {
    float *y = p.y_f32 != nullptr ? p.y_f32 + (size_t)m0 * ys : nullptr;
    const int voff = p.vocab_offset;
    unsigned long long key[kGroup];
#pragma unroll
    for (int m = 0; m < kGroup; ++m) {
      const float h = round_half(v[m]);
      key[m] = in_range && m < M ? argmax_key(h, voff + row) : 0ull;
      if (y != nullptr && in_range && m < M) y[(size_t)m * ys + row] = h;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
      for (int m = 0; m < kGroup; ++m) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, key[m], o);
        key[m] = other > key[m] ? other : key[m];
      }
    }
    if (lane == 0) {
#pragma unroll
      for (int m = 0; m < kGroup; ++m) red_keys[ew][m] = key[m];
      if ((ew & 3) == 0) half_m0[ew >> 2] = active ? m0 : -1;
    }
    epi_sync();
    if (t < 2 * kGroup) {  // one thread per token of the two halves' groups
      const int hf = t / kGroup, tok = t % kGroup;
      const int mm = half_m0[hf] + tok;
      if (half_m0[hf] >= 0 && mm < p.M) {
        unsigned long long k = red_keys[hf * 4][tok];
#pragma unroll
        for (int e = 1; e < 4; ++e) k = red_keys[hf * 4 + e][tok] > k ? red_keys[hf * 4 + e][tok] : k;
        if (k != 0ull) atomicMax(p.argmax_keys + mm, k);
      }
    }
    epi_sync();
  } else if constexpr (EK == kEkSwiGLU) {
    __half *y = p.y_f16 + (size_t)m0 * ys + (row >> 1);
    const bool store = !(lane & 1) && in_range;
    __half out[kGroup];
#pragma unroll
    for (int m = 0; m < kGroup; ++m) {
      const float partner = __shfl_xor_sync(0xffffffffu, v[m], 1);
      out[m] = swiglu_value(v[m], partner);
    }
#pragma unroll
    for (int m = 0; m < kGroup; ++m)
      if (store && m < M) y[(size_t)m * ys] = out[m];
  } else if constexpr (EK == kEkQKV) {
    const int D = p.head_dim, q_rows = p.q_rows, kv_rows = p.kv_rows;
    const float *rc = p.rope_cos + ((row % D) >> 1), *rs = p.rope_sin + ((row % D) >> 1);
    __half *y = p.y_f16 + (size_t)m0 * ys + row;
    const bool rope = row < q_rows + kv_rows, is_q = row < q_rows;
    int local = row - q_rows;
    __half *pool = p.k_pool;
    if (local >= kv_rows) {
      local -= kv_rows;
      pool = p.v_pool;
    }
    const size_t head_off = (size_t)(local / D) * p.page_size * D + (local % D);
    const bool store = !(lane & 1) && in_range;
    float cs[kGroup], sn[kGroup];
#pragma unroll
    for (int m = 0; m < kGroup; ++m) {
      const int pos = m < M ? tok_pos[m0 + m] : -1;
      const bool use = rope && store && pos >= 0;
      cs[m] = use ? rc[(size_t)pos * (D >> 1)] : 0.0f;
      sn[m] = use ? rs[(size_t)pos * (D >> 1)] : 0.0f;
    }
    __half2 val[kGroup];
#pragma unroll
    for (int m = 0; m < kGroup; ++m) {
      const float partner = __shfl_xor_sync(0xffffffffu, v[m], 1);
      val[m] = rope ? rope_pair_value(v[m], partner, cs[m], sn[m])
                    : __floats2half2_rn(round_half(v[m]), round_half(partner));
    }
#pragma unroll
    for (int m = 0; m < kGroup; ++m) {
      if (!store || m >= M || tok_pos[m0 + m] < 0) continue;
      if (is_q) {
        *reinterpret_cast<__half2 *>(y + (size_t)m * ys) = val[m];
      } else if (tok_slot[m0 + m] >= 0) {
        *reinterpret_cast<__half2 *>(pool + (size_t)tok_slot[m0 + m] + head_off) = val[m];
      }
    }
  } else if constexpr (EK == kEkHalf) {
    __half *y = p.y_f16 + (size_t)m0 * ys + row;
    const __half *res = p.residual + (size_t)m0 * ys + row;
    const bool residual = p.epilogue == kEpiResidual;
    // All residual loads first: y and res are the same buffer (in place).
    __half out[kGroup];
#pragma unroll
    for (int m = 0; m < kGroup; ++m) out[m] = residual && in_range && m < M ? res[(size_t)m * ys] : __half(0.0f);
#pragma unroll
    for (int m = 0; m < kGroup; ++m) out[m] = residual ? residual_value(out[m], v[m]) : __float2half_rn(v[m]);
#pragma unroll
    for (int m = 0; m < kGroup; ++m)
      if (in_range && m < M) y[(size_t)m * ys] = out[m];
  } else {  // kEkF32: kEpiF32, kEpiF32Partial (optionally into every rank's exchange slot)
    if (p.epilogue == kEpiF32Partial && p.xchg.world > 0) {
      const int world = p.xchg.world, width = p.xchg.width;
      for (int q = 0; q < world; ++q) {
        float *dst = peer_slot(p.xchg, q, p.xchg.phase & 1, p.xchg.rank, p.xchg.row0 + m0) + row;
#pragma unroll
        for (int m = 0; m < kGroup; ++m)
          if (in_range && m < M) dst[(size_t)m * width] = v[m];
      }
    } else {
      float *y = p.y_f32 + (size_t)m0 * ys + row;
#pragma unroll
      for (int m = 0; m < kGroup; ++m)
        if (in_range && m < M) y[(size_t)m * ys] = v[m];
    }
  }
}

template <int TN, int EK>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap w_map, const __grid_constant__ CUtensorMap x_map,
                const GemvParams p, const GemmWork w) {
  using C = GemmCfg<TN>;
  constexpr int S = C::kStages;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char *base = reinterpret_cast<unsigned char *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int A = C::kAtoms;
  unsigned char *sA = base;                                  // [S][A] weight atoms
  unsigned char *sB = base + (size_t)S * A * kTileBytesA;    // [S][A] token atoms
  uint64_t *full = reinterpret_cast<uint64_t *>(sB + (size_t)S * A * C::kBytesB);
  uint64_t *empty = full + S;
  uint64_t *acc_full = empty + S;
  uint64_t *acc_empty = acc_full + C::kAcc;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + C::kAcc);
  __shared__ unsigned long long red_keys[kEpiWarps][kGroup];
  __shared__ int half_m0[2];
  __shared__ int tok_pos[kMaxTokens];          // QKV epilogue: per-token position (-1: skip)
  __shared__ long long tok_slot[kMaxTokens];   // ... and KV element offset of its page row
  __shared__ int s_last, s_fail;
  __shared__ unsigned long long s_ready;
  __shared__ uint64_t mma_drain;  // tracks the issuer's MMAs on a failure path
  const unsigned long long local_ns = p.local_wait_ns;
  const unsigned long long tile_ns = local_ns ? local_ns : kTileWaitNs;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const unsigned long long t_entry = p.trace.records ? global_ns() : 0ull;

  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < C::kAcc; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kEpiWarps);  // one arrival per epilogue warp
    }
    mbar_init(&mma_drain, 1);
    fence_barrier_init();
    s_fail = 0;
    s_ready = t_entry;
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(C::kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---- TMA producer ----
      int pending_kb[S];
      int last_it[S];  // the latest iteration loaded into each stage (-1: none)
#pragma unroll
      for (int s = 0; s < S; ++s) last_it[s] = -1;
      int it = 0;
      bool waited = false, ok = true;
      // Weight tiles are read once per launch: evict-first in L2, so the token
      // slab (read by every CTA) and the step's other reused lines stay.
      const uint64_t wpol = l2_evict_first_policy();
      // The token atoms of stage st, K block kb (A adjacent 64-column boxes).
      auto load_x = [&](int st, int kb) {
#pragma unroll
        for (int a = 0; a < A; ++a)
          tma_load_2d(sB + ((size_t)st * A + a) * C::kBytesB, &x_map, (kb * A + a) * kGemmKBlock, 0, &full[st]);
      };
      RunCursor run(w);
      Piece pc;
      while (ok && run.get(pc)) {
        const int tile = pc.tile;
        for (int kb = pc.kb0; kb < pc.kb1; ++kb, ++it) {
          const int st = it % S, round = it / S;
          if (it == S && !waited) {
            // The ring is full of weight tiles: wait for the producer of x,
            // then request the token slices of those stages.
            pdl_wait();
            if (p.trace.records) s_ready = global_ns();
            for (int j = 0; j < S; ++j) load_x(j, pending_kb[j]);
            waited = true;
          }
          if (round > 0 && !mbar_wait(&empty[st], (round - 1) & 1, local_ns)) {
            ok = false;
            break;
          }
          last_it[st] = it;
          // Atoms past K (a ragged last block) read as zeros and add nothing.
          mbar_arrive_expect_tx(&full[st], C::kStageBytes);
#pragma unroll
          for (int a = 0; a < A; ++a)
            tma_load_2d(sA + ((size_t)st * A + a) * kTileBytesA, &w_map, (kb * A + a) * kGemmKBlock,
                        tile * kGemmTileRows, &full[st], wpol);
          if (waited) {
            load_x(st, kb);
          } else {
            pending_kb[st] = kb;
          }
        }
      }
      if (!waited) {
        pdl_wait();
        if (p.trace.records) s_ready = global_ns();
        const int n = it < S ? it : S;
        for (int j = 0; j < n; ++j) load_x(j, pending_kb[j]);
      }
      pdl_launch_dependents();
      if (!ok) report_status(p.status, kStatusWaitTimeout, kWhereGemm, 0, blockIdx.x);
      // No copy may still be landing when the CTA exits (on a failure path
      // the MMA issuer stops consuming): wait, bounded, for each stage's last
      // load. On the normal path these phases have completed or are about to.
#pragma unroll 1
      for (int s = 0; s < S; ++s)
        if (last_it[s] >= 0) (void)mbar_wait(&full[s], (last_it[s] / S) & 1, local_ns);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA issuer: D[128 features x TN tokens] += W_tile . x_slice^T ----
      const uint32_t idesc = (1u << 4)                                  // D: fp32
                             | ((uint32_t)(TN >> 3) << 17)              // N
                             | ((uint32_t)(kGemmTileRows >> 4) << 24);  // M; A, B: fp16, K-major
      int it = 0;
      bool ok = true;
      RunCursor run(w);
      Piece pc;
      while (ok && run.get(pc)) {
        const int j = pc.index, kb0 = pc.kb0, kb1 = pc.kb1;
        const int buf = j % C::kAcc;
        if (j >= C::kAcc && !mbar_wait(&acc_empty[buf], ((j / C::kAcc) - 1) & 1, local_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(buf * TN);
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int st = it % S;
          if (!mbar_wait(&full[st], (it / S) & 1, local_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int a = 0; a < A; ++a) {
            const uint64_t da = sw128_desc(sA + ((size_t)st * A + a) * kTileBytesA);
            const uint64_t db = sw128_desc(sB + ((size_t)st * A + a) * C::kBytesB);
#pragma unroll
            for (int k = 0; k < kGemmKBlock / 16; ++k)  // +32 bytes along K per step
              umma_f16(d, da + 2u * k, db + 2u * k, idesc, (kb > kb0 || a > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&empty[st]);
        }
        if (ok) umma_commit(&acc_full[buf]);
      }
      if (!ok) {
        report_status(p.status, kStatusWaitTimeout, kWhereGemm, 1, blockIdx.x);
        // Every MMA issued so far completes before TMEM is freed.
        umma_commit(&mma_drain);
        (void)mbar_wait(&mma_drain, 0, local_ns);
      }
    }
  } else {
    // ---- epilogue warps ----
    pdl_wait();
    const int q = warp & 3;  // the TMEM lane quarter this warp may read
    const int ew = warp - 2;
    const int half = ew >> 2;  // this warp's 16-token groups: half, half + 2, ...
    const int t = threadIdx.x - 64;
    const int r = q * 32 + lane;
    if constexpr (EK == kEkQKV) {
      // One thread per token resolves its position and KV slot (page
      // lookup, range checks) once for the launch, off the tiles' critical
      // path (the step inputs are final once the dependency wait returned);
      // -1 marks a failed check.
      if (t < p.M) {
        const int pos = p.positions[t];
        long long slot = -1;
        const int ps = p.page_size;
        if (pos < 0 || pos >= p.capacity) {
          report_status(p.status, kStatusLengthRange, kWhereAppend, pos, t);
        } else {
          const int lp = pos / ps, off = pos % ps;
          if (lp >= p.table_stride) {
            report_status(p.status, kStatusLengthRange, kWhereAppend, pos, t);
          } else {
            const int page = p.block_table[(size_t)p.table_rows[t] * p.table_stride + lp];
            if (page < 0 || page >= p.pool_pages) {
              report_status(p.status, page < 0 ? kStatusPageMissing : kStatusPageRange, kWhereAppend,
                            page < 0 ? lp : page, t);
            } else {
              slot = ((long long)page * (p.kv_rows / p.head_dim) * ps + off) * p.head_dim;
            }
          }
        }
        tok_pos[t] = (pos < 0 || pos >= p.capacity) ? -1 : pos;  // q rows need only the position
        tok_slot[t] = slot;
      }
      epi_sync();
    }
    const long long iters = (long long)w.tiles * w.kblocks;
    RunCursor run(w);
    Piece pc;
    while (run.get(pc)) {
      const int tile = pc.tile, j = pc.index;
      const int buf = j % C::kAcc;
      if (!mbar_wait(&acc_full[buf], (j / C::kAcc) & 1, local_ns)) s_fail = 1;
      epi_sync();
      if (s_fail) break;
      tc_fence_after();
      const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * TN);
      const int row = tile * kGemmTileRows + r;
      const int groups = (p.M + kGroup - 1) / kGroup;
      const bool whole = pc.kb0 == 0 && pc.kb1 == w.kblocks;
      int c_first = 0, closers = 1, ci = 0;
      if (!whole) {
        // Part of the tile: store this piece's partial; the group barrier
        // plus one acquire-release arrival orders every thread's stores
        // before the closers' loads.
        float *part = w.ws + ((size_t)blockIdx.x * 2 + (j == 0 ? 0 : 1)) * TN * kGemmTileRows + r;
#pragma unroll 1
        for (int g = half; g < groups; g += 2) {
          float v[kGroup];
          tmem_ld16(tbase + (uint32_t)(g * kGroup), v);
          tmem_wait_ld();
#pragma unroll
          for (int m = 0; m < kGroup; ++m)
            if (g * kGroup + m < p.M) __stcg(part + (size_t)(g * kGroup + m) * kGemmTileRows, v[m]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[buf]);
        epi_sync();
        // The tile's pieces belong to the consecutive runs c_first .. c_last;
        // the closers are those whose runs end inside the tile.
        c_first = run_of(iters, gridDim.x, (long long)tile * w.kblocks);
        const int c_last = run_of(iters, gridDim.x, (long long)(tile + 1) * w.kblocks - 1);
        const long long tile_end = (long long)(tile + 1) * w.kblocks;
        const int c_close = run_begin(iters, gridDim.x, c_last + 1) <= tile_end ? c_last : c_last - 1;
        closers = c_close - c_first + 1;
        ci = (int)blockIdx.x - c_first;
        unsigned int *arrived = w.tile_counters + tile;
        if (t == 0) {
          atomic_add_acq_rel_gpu(arrived, 1u);
          if (ci < closers && !wait_count_geq_gpu(arrived, (unsigned int)(c_last - c_first + 1), tile_ns)) {
            report_status(p.status, kStatusWaitTimeout, kWhereGemm, 2, tile);
            s_fail = 1;
          }
        }
        epi_sync();
        if (ci >= closers) continue;  // not a closer: its run goes on
        if (s_fail) break;
      }
      // Groups this CTA applies: all of a whole tile, or a closer's share.
      const int assigned = whole ? groups : (ci < groups ? (groups - ci + closers - 1) / closers : 0);
#pragma unroll 1
      for (int j0 = 0; j0 < assigned; j0 += 2) {
        const int jj = j0 + half;
        const bool active = jj < assigned;
        const int g = whole ? jj : ci + jj * closers;
        float v[kGroup];
#pragma unroll
        for (int m = 0; m < kGroup; ++m) v[m] = 0.0f;
        if (!active) {
        } else if (whole) {
          tmem_ld16(tbase + (uint32_t)(g * kGroup), v);
          tmem_wait_ld();
        } else {
          // The partials in K order (run order), kBatch pieces' loads in flight.
          constexpr int kBatch = 4;
          const int c_last = run_of(iters, gridDim.x, (long long)(tile + 1) * w.kblocks - 1);
#pragma unroll 1
          for (int c2 = c_first; c2 <= c_last; c2 += kBatch) {
            float tmp[kBatch][kGroup];
#pragma unroll
            for (int e = 0; e < kBatch; ++e) {
              const int cc = c2 + e;
              if (cc <= c_last) {
                const bool first_piece = run_begin(iters, gridDim.x, cc) / w.kblocks == tile;
                const float *src = w.ws + ((size_t)cc * 2 + (first_piece ? 0 : 1)) * TN * kGemmTileRows + r +
                                   (size_t)g * kGroup * kGemmTileRows;
#pragma unroll
                for (int m = 0; m < kGroup; ++m)
                  tmp[e][m] = g * kGroup + m < p.M ? __ldcg(src + (size_t)m * kGemmTileRows) : 0.0f;
              }
            }
#pragma unroll
            for (int e = 0; e < kBatch; ++e)
              if (c2 + e <= c_last) {
#pragma unroll
                for (int m = 0; m < kGroup; ++m) v[m] += tmp[e][m];
              }
          }
        }
        apply_group<EK>(p, v, g * kGroup, active, row, lane, ew, t, red_keys, half_m0, tok_pos, tok_slot);
      }
      if (!whole) {
        // The last closer to finish resets the tile's counters.
        epi_sync();
        if (t == 0 && atomicAdd(w.tile_counters + w.tiles + tile, 1u) == (unsigned int)(closers - 1)) {
          w.tile_counters[tile] = 0u;
          w.tile_counters[w.tiles + tile] = 0u;
        }
      }
      if (whole) {  // the accumulator is free for the MMA warp
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[buf]);
      }
      if constexpr (EK == kEkQKV) epi_sync();  // the staging arrays are rewritten by the next piece
    }
    epi_sync();
    if (EK == kEkF32 && p.epilogue == kEpiF32Partial && p.xchg.world > 0 && t < 32) {
      // Same causality chain as the GEMV: epilogue stores -> group barrier ->
      // GPU-scope arrival -> the last CTA's per-rank system-scope releases.
      int last = 0;
      if (t == 0) {
        const unsigned int done = atomic_add_acq_rel_gpu(p.xchg.done, 1u);
        last = done == gridDim.x - 1;
        if (last) atomicExch(p.xchg.done, 0u);
      }
      last = __shfl_sync(0xffffffffu, last, 0);
      __syncwarp();
      if (last && p.xchg.signal && t < p.xchg.world) {
        const unsigned int value = *p.xchg.epoch * p.xchg.phases + p.xchg.phase + 1u;
        st_release_sys(peer_flag(p.xchg, t, p.xchg.phase & 1, p.xchg.rank), value);
      }
    }
    if (EK == kEkArgmax && p.next_tokens != nullptr) {
      __threadfence();
      epi_sync();
      if (t == 0) {
        const unsigned int prev = atomicAdd(p.argmax_counter, 1u);
        s_last = prev == gridDim.x - 1;
      }
      epi_sync();
      if (s_last) {
        __threadfence();
        argmax_finalize(p, t, [] { epi_sync(); });
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::kTmemCols)
                 : "memory");
  }
  trace_emit(p.trace, t_entry, s_ready);
}

template <int TN, int EK>
cudaError_t launch_tn(const GemvParams &p, const CUtensorMap &w_map, const CUtensorMap &x_map,
                      const GemmPlan &plan, float *ws, unsigned int *tile_counters, cudaStream_t stream, bool pdl) {
  using C = GemmCfg<TN>;
  auto kernel = gemm_kernel<TN, EK>;
  static std::mutex mu;
  static std::unordered_map<int, bool> configured;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!configured[dev]) {
      e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(C::kSmem));
      if (e != cudaSuccess) return e;
      configured[dev] = true;
    }
  }
  GemmWork w{plan.tiles, plan.kblocks, ws, tile_counters};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(plan.grid);
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = C::kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, w_map, x_map, p, w);
}

template <int EK>
cudaError_t launch_ek(const GemvParams &p, const CUtensorMap &w_map, const CUtensorMap &x_map, const GemmPlan &plan,
                      float *ws, unsigned int *tile_counters, cudaStream_t stream, bool pdl) {
  switch (plan.tn) {
    case 16: return launch_tn<16, EK>(p, w_map, x_map, plan, ws, tile_counters, stream, pdl);
    case 32: return launch_tn<32, EK>(p, w_map, x_map, plan, ws, tile_counters, stream, pdl);
    case 64: return launch_tn<64, EK>(p, w_map, x_map, plan, ws, tile_counters, stream, pdl);
    case 128: return launch_tn<128, EK>(p, w_map, x_map, plan, ws, tile_counters, stream, pdl);
    case 256: return launch_tn<256, EK>(p, w_map, x_map, plan, ws, tile_counters, stream, pdl);
    default: return cudaErrorInvalidValue;
  }
}

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

}  // namespace

GemmPlan plan_gemm(int N, int K, int M, int num_sms) {
  GemmPlan g{};
  g.tn = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 ? 128 : 256;
  g.tiles = (N + kGemmTileRows - 1) / kGemmTileRows;
  const int block = kGemmKBlock * gemm_k_atoms(g.tn);
  g.kblocks = (K + block - 1) / block;  // a ragged last block reads zeros
  const long long iters = (long long)g.tiles * g.kblocks;
  const int min_run = (kGemmMinRun + block - 1) / block;
  long long grid = iters / min_run;
  if (grid > num_sms) grid = num_sms;
  if (grid < 1) grid = 1;
  g.grid = (int)grid;
  return g;
}

size_t gemm_workspace_floats(const GemmPlan &plan) {
  const long long iters = (long long)plan.tiles * plan.kblocks;
  for (int c = 1; c < plan.grid; ++c)
    if (iters * c / plan.grid % plan.kblocks != 0) return (size_t)plan.grid * 2 * plan.tn * kGemmTileRows;
  return 0;
}

cudaError_t make_tensor_map_f16(CUtensorMap *map, const void *base, uint64_t rows, uint64_t cols,
                                uint32_t box_rows) {
  static std::mutex mu;
  static EncodeTiledFn encode = nullptr;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (encode == nullptr) {
      void *fn = nullptr;
      cudaDriverEntryPointQueryResult q;
      cudaError_t e = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q);
      if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || fn == nullptr)
        return e != cudaSuccess ? e : cudaErrorNotSupported;
      encode = reinterpret_cast<EncodeTiledFn>(fn);
    }
  }
  if (map == nullptr || base == nullptr || (reinterpret_cast<uintptr_t>(base) & 15) != 0 || cols % 8 != 0 ||
      box_rows == 0 || box_rows > 256)
    return cudaErrorInvalidValue;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kGemmKBlock, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims, strides, box,
                            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t launch_gemm(const GemvParams &p, const CUtensorMap &w_map, const CUtensorMap &x_map,
                        const GemmPlan &plan, float *ws, unsigned int *tile_counters, cudaStream_t stream,
                        bool pdl) {
  if (p.N <= 0 || p.K <= 0 || p.K % 8 != 0 || p.M <= 0 || p.M > plan.tn || plan.tn > 256 ||
      plan.tiles != (p.N + kGemmTileRows - 1) / kGemmTileRows ||
      plan.kblocks != (p.K + kGemmKBlock * gemm_k_atoms(plan.tn) - 1) / (kGemmKBlock * gemm_k_atoms(plan.tn)) ||
      plan.grid < 1 || plan.grid > (long long)plan.tiles * plan.kblocks ||  // every run non-empty
      tile_counters == nullptr || (gemm_workspace_floats(plan) > 0 && ws == nullptr))
    return cudaErrorInvalidValue;
  switch (p.epilogue) {
    case kEpiQKV:
    case kEpiSwiGLU:
      if (p.N & 1) return cudaErrorInvalidValue;
      break;
    case kEpiResidual:
    case kEpiF16:
    case kEpiF32:
    case kEpiF32Partial:
    case kEpiArgmax:
      break;
    default:
      return cudaErrorInvalidValue;
  }
  switch (p.epilogue) {
    case kEpiQKV: return launch_ek<kEkQKV>(p, w_map, x_map, plan, ws, tile_counters, stream, pdl);
    case kEpiSwiGLU: return launch_ek<kEkSwiGLU>(p, w_map, x_map, plan, ws, tile_counters, stream, pdl);
    case kEpiResidual:
    case kEpiF16: return launch_ek<kEkHalf>(p, w_map, x_map, plan, ws, tile_counters, stream, pdl);
    case kEpiArgmax: return launch_ek<kEkArgmax>(p, w_map, x_map, plan, ws, tile_counters, stream, pdl);
    default: return launch_ek<kEkF32>(p, w_map, x_map, plan, ws, tile_counters, stream, pdl);
  }
}

}  // namespace tmc
