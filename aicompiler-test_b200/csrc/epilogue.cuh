// Per-element epilogues shared by the decode GEMV (CUDA cores, M <= 8 rows)
// and the batched tcgen05 GEMM (tensor cores, up to 256 rows): both kernels
// hand every finished fp32 sum to these functions, so the two paths round
// and store identically.
//
// Rounding points follow the reference decoder (workloads/pytorch/decoder_llm.py):
// every linear output is rounded to fp16 storage before RoPE (:19-31),
// SiLU (:93-101) or the residual add (:104-118); RoPE and the residual add
// are computed in fp32 and rounded once more.
#pragma once

#include "gemv.cuh"

namespace tmc {

// ---- peer exchange addressing (layout in gemv.cuh) ----------------------------
constexpr unsigned long long kPeerWaitNs = 10ull * 1000 * 1000 * 1000;  // 10 s of global time
__host__ __device__ __forceinline__ unsigned long long peer_wait_budget(const GemvParams &p) {
  return p.peer_wait_ns ? p.peer_wait_ns : kPeerWaitNs;
}

__device__ __forceinline__ unsigned int *peer_flag(const PeerExchange &x, int owner, int set, int src) {
  return reinterpret_cast<unsigned int *>(x.window[owner]) + ((size_t)set * kMaxPeers + src) * kPeerFlagStride;
}
__device__ __forceinline__ unsigned long long *peer_key(const PeerExchange &x, int owner, int parity,
                                                        int src, int m) {
  return reinterpret_cast<unsigned long long *>(x.window[owner] + peer_key_offset()) +
         ((size_t)parity * kMaxPeers + src) * x.slot_rows + m;
}
__device__ __forceinline__ float *peer_slot(const PeerExchange &x, int owner, int parity, int src, int m) {
  return reinterpret_cast<float *>(x.window[owner] + peer_slot_offset(x.slot_rows)) +
         (((size_t)parity * kMaxPeers + src) * x.slot_rows + m) * x.width;
}

// ---- the arithmetic of each epilogue, shared by every kernel ---------------
// SwiGLU of one (gate, up) pair of fp32 sums: half(half(silu(half(g))) * half(u)).
__device__ __forceinline__ __half swiglu_value(float acc_gate, float acc_up) {
  const float g = round_half(acc_gate);
  const float u = round_half(acc_up);
  const float a = round_half(g / (1.0f + expf(-g)));
  return __float2half_rn(__fmul_rn(a, u));
}
// Interleaved RoPE of one (even, odd) pair of fp32 sums, rounded to fp16
// first; (c, s) = cos/sin of the pair's angle at the token's position.
__device__ __forceinline__ __half2 rope_pair_value(float acc_e, float acc_o, float c, float s) {
  const float e = round_half(acc_e);
  const float o = round_half(acc_o);
  return __floats2half2_rn(__fsub_rn(__fmul_rn(e, c), __fmul_rn(o, s)), __fadd_rn(__fmul_rn(e, s), __fmul_rn(o, c)));
}
// Residual add of a projection sum: half(residual + half(acc)).
__device__ __forceinline__ __half residual_value(__half residual, float acc) {
  return __float2half_rn(__fadd_rn(__half2float(residual), round_half(acc)));
}

// The residual rows of one row group of token 0, read ahead of the dependency
// wait (GemvParams::early_epilogue_inputs). ok == false: none.
struct EpiPre {
  bool ok;
  __half res[2];
};

template <int R>
__device__ __forceinline__ EpiPre load_epi_pre(const GemvParams &p, int row0) {
  EpiPre e{};
  if (p.epilogue == kEpiResidual && R <= 2) {
#pragma unroll
    for (int r = 0; r < R; ++r)
      if (row0 + r < p.N) e.res[r] = __ldcg(p.residual + row0 + r);
    e.ok = true;
  }
  return e;
}

// Rows (row0, row0 + 1) of token m, row0 even, with fp32 sums (acc_e, acc_o):
// kEpiSwiGLU: a (gate_i, up_i) pair, i = row0 / 2 -> y_f16[m, i];
// kEpiQKV: an interleaved RoPE pair inside one head of [q | k | v]; q goes to
// y_f16, k and v to the paged cache at the row's position.
__device__ __forceinline__ void epilogue_pair(const GemvParams &p, int row0, int m, float acc_e, float acc_o) {
  if (p.epilogue == kEpiSwiGLU) {
    p.y_f16[(size_t)m * p.y_stride + (row0 >> 1)] = swiglu_value(acc_e, acc_o);
    return;
  }
  // kEpiQKV
  const int D = p.head_dim;
  const int pos = p.positions[m];
  if (pos < 0 || pos >= p.capacity) {
    report_status(p.status, kStatusLengthRange, kWhereAppend, pos, m);
    return;
  }
  __half2 pair_value;
  if (row0 < p.q_rows + p.kv_rows) {
    const int pair = (row0 % D) >> 1;
    pair_value = rope_pair_value(acc_e, acc_o, p.rope_cos[(size_t)pos * (D >> 1) + pair],
                                 p.rope_sin[(size_t)pos * (D >> 1) + pair]);
  } else {
    pair_value = __floats2half2_rn(round_half(acc_e), round_half(acc_o));
  }
  if (row0 < p.q_rows) {
    *reinterpret_cast<__half2 *>(p.y_f16 + (size_t)m * p.y_stride + row0) = pair_value;
    return;
  }
  int local = row0 - p.q_rows;
  __half *pool = p.k_pool;
  if (local >= p.kv_rows) {
    local -= p.kv_rows;
    pool = p.v_pool;
  }
  const int kvh = local / D, d = local % D;
  const int lp = pos / p.page_size, off = pos % p.page_size;
  if (lp >= p.table_stride) {
    report_status(p.status, kStatusLengthRange, kWhereAppend, pos, m);
    return;
  }
  const int page = p.block_table[(size_t)p.table_rows[m] * p.table_stride + lp];
  if (page < 0) {
    report_status(p.status, kStatusPageMissing, kWhereAppend, lp, m);
    return;
  }
  if (page >= p.pool_pages) {
    report_status(p.status, kStatusPageRange, kWhereAppend, page, m);
    return;
  }
  const int hkv = p.kv_rows / D;
  const size_t addr = (((size_t)page * hkv + kvh) * p.page_size + off) * D + d;
  *reinterpret_cast<__half2 *>(pool + addr) = pair_value;
}

// One output (row, token m) with fp32 sum v: kEpiF32, kEpiF16, kEpiResidual,
// kEpiF32Partial (local partial buffer, or this rank's slot of every rank's
// exchange window).
// `has_res`: `res` is the residual read ahead (kEpiResidual, token 0).
__device__ __forceinline__ void epilogue_one(const GemvParams &p, int row, int m, float v, bool has_res,
                                             __half res) {
  const int epi = p.epilogue;
  const size_t idx = (size_t)m * p.y_stride + row;
  if (epi == kEpiF32Partial && p.xchg.world > 0) {
    for (int q = 0; q < p.xchg.world; ++q)
      peer_slot(p.xchg, q, p.xchg.phase & 1, p.xchg.rank, p.xchg.row0 + m)[row] = v;
  } else if (epi == kEpiF32 || epi == kEpiF32Partial) {
    p.y_f32[idx] = v;
  } else if (epi == kEpiF16) {
    p.y_f16[idx] = __float2half_rn(v);
  } else if (epi == kEpiResidual) {
    p.y_f16[idx] = residual_value(has_res ? res : p.residual[idx], v);
  }
}

// The LM-head argmax finalisation in the launch's last CTA: per row, the
// greedy token from the maximum packed key (under tensor parallelism after
// sending this rank's keys to every rank and waiting, bounded, for theirs),
// written to next_tokens and optionally fed back (tokens, positions + 1,
// history); the keys, the CTA counter and (TP) the step epoch are reset or
// advanced for the next launch. Run by a group of at least max(M, world)
// threads, index t, that synchronise with sync().
template <class Sync>
__device__ __forceinline__ void argmax_finalize(const GemvParams &p, int t, Sync sync) {
  const unsigned int step = p.history != nullptr ? *p.history_counter : 0u;
  unsigned long long key = 0ull;
  if (t < p.M) key = atomicExch(p.argmax_keys + t, 0ull);
  const PeerExchange &x = p.xchg;
  if (x.world > 0) {
    // Vocab-parallel head: send this rank's best key per row to every rank,
    // wait for every rank's keys, and finalise from their maximum.
    const unsigned int e = *x.epoch;
    const int parity = static_cast<int>(e & 1u);
    if (t < p.M)
      for (int q = 0; q < x.world; ++q) *peer_key(x, q, parity, x.rank, x.row0 + t) = key;
    sync();  // the key stores, then one system-scope release per rank (parallel threads)
    if (t < x.world) st_release_sys(peer_flag(x, t, 2 + parity, x.rank), e + 1u);
    if (t < x.world && !wait_flag_geq(peer_flag(x, x.rank, 2 + parity, t), e + 1u, peer_wait_budget(p)))
      report_status(p.status, kStatusWaitTimeout, kWhereExchange, t, -1);
    sync();
    if (t < p.M) {
      key = 0ull;
      for (int src = 0; src < x.world; ++src) {
        const unsigned long long k = __ldcg(peer_key(x, x.rank, parity, src, x.row0 + t));
        key = k > key ? k : key;
      }
    }
    if (t == 0) *x.epoch = e + 1u;
  }
  if (t < p.M) {
    const int tok = argmax_key_index(key);
    p.next_tokens[t] = tok;
    if (p.feed_tokens != nullptr) p.feed_tokens[t] = tok;
    if (p.feed_positions != nullptr) p.feed_positions[t] += 1;
    if (p.history != nullptr) p.history[(size_t)step * p.M + t] = tok;
  }
  sync();
  if (t == 0) {
    if (p.history != nullptr) *p.history_counter = step + 1;
    atomicExch(p.argmax_counter, 0u);
  }
}

}  // namespace tmc
