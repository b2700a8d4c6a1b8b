// Batched decode projections on the 5th-generation tensor cores (tcgen05).
//
// Replaces emitTiledGEMM (DecodeGEMVMetalEmitter.cpp:134-169), the
// reference's batched/prefill linear layer, for rows > 8: y = epilogue(W x^T)
// with W [N, K] fp16 row-major (the decoder's weights, unchanged) and x
// [M <= 256, K] fp16 rows, K % 8 == 0 (the GEMV prologue, written by launch_row_prologue,
// or an fp16 activation). The weight tile is the MMA's A operand (128 output
// features = the UMMA M dimension) and the token rows are its B operand
// (UMMA N = 16..128), so one weight byte feeds up to 128 tokens; the fp32
// accumulator lives in tensor memory. Epilogues are the GEMV's own
// (epilogue.cuh), so rows computed here round and store exactly as there.
#pragma once

#include <cuda.h>

#include "gemv.cuh"

namespace tmc {

constexpr int kGemmTileRows = 128;  // weight rows per tile (UMMA M)
constexpr int kGemmKBlock = 64;     // K elements of one 128-byte swizzle atom (one TMA box)
// Swizzle atoms per pipeline stage, adjacent along K: each stage fetches
// 64 * atoms contiguous weight elements of each of its 128 rows (512 B for
// up to 64 tokens, 256 B for 128), long enough runs for the DRAM pages (one
// 128-byte run per row per stage streamed ~20% slower). At 256 tokens the
// token slab dominates a stage and one atom (four 48 KB stages) measured
// ~4% faster than two.
__host__ __device__ constexpr int gemm_k_atoms(int tn) { return tn <= 64 ? 4 : tn <= 128 ? 2 : 1; }

// Stream-K work division: the tiles x kblocks (tile, K block) iterations, in
// tile-major order, are cut into `grid` contiguous equal runs, one per
// persistent CTA. A run covers whole tiles and at most two partial tiles (its
// first and its last); a partial tile's pieces are written as fp32 partials
// and summed in K order by the tile's last-arriving piece, so the result is
// fixed for a given plan and does not depend on timing.
struct GemmPlan {
  int tn;       // token columns per MMA (16, 32, 64, 128 or 256), >= M
  int tiles;    // ceil(N / 128)
  int kblocks;  // ceil(K / (64 * gemm_k_atoms(tn))): K blocks of one pipeline stage
  int grid;     // persistent CTAs (one per SM at most, each with >= kGemmMinRun iterations)
};

constexpr int kGemmMinRun = 256;  // fewest K elements a CTA streams (shorter runs cost more in partials)

GemmPlan plan_gemm(int N, int K, int M, int num_sms);
// fp32 elements of partial-tile workspace the plan needs (0 when every run is
// whole tiles): two [128 x tn] slots per CTA.
size_t gemm_workspace_floats(const GemmPlan &plan);

// 2-D tensor map of an fp16 row-major matrix [rows, cols] with a
// [box_rows, 64] box and 128-byte swizzle (the UMMA K-major SW128 layout).
cudaError_t make_tensor_map_f16(CUtensorMap *map, const void *base, uint64_t rows, uint64_t cols,
                                uint32_t box_rows);

// y = epilogue(W . x^T) for p.M rows. w_map: W with box_rows 128; x_map: the
// x rows with box_rows plan.tn. p.W/p.N/p.K/p.M and the epilogue fields are
// used as by launch_gemv; the prologue must already be applied (x is read as
// fp16 rows). ws: gemm_workspace_floats(plan) floats; tile_counters:
// 2 * plan.tiles zeroed words (left zeroed). Supported epilogues: kEpiQKV,
// kEpiSwiGLU, kEpiResidual, kEpiF16, kEpiF32, kEpiF32Partial (with or
// without peer exchange) and kEpiArgmax.
cudaError_t launch_gemm(const GemvParams &p, const CUtensorMap &w_map, const CUtensorMap &x_map,
                        const GemmPlan &plan, float *ws, unsigned int *tile_counters,
                        cudaStream_t stream, bool pdl);

}  // namespace tmc
