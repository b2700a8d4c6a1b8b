// Block-table-indexed GQA decode attention with split-K (flash-decoding).
//
// Replaces emitServingPagedKVAttention (KVCacheMetalEmitter.cpp:312-406),
// emitPagedKVAttention (:210-310) and emitKVAttention (:119-208): causal
// decode attention for one query token per row, scale 1/sqrt(D), softmax in
// fp32, context rounded to fp16. The reference is MHA only; here query head h
// reads KV head h / (Hq / Hkv) (grouped-query attention).
//
// KV layout in HBM: a pool of pages [page][Hkv][page_size][D] (fp16), the
// serving layout of emitServingPagedCacheAppend
// (DecoderLLMMetalEmitter.cpp:314-373). A contiguous per-sequence cache
// [B][H][capacity][D] is the special case page_size = capacity with block
// table row b = {b}.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace tmc {

struct AttentionParams {
  const __half *q;      // [rows, Hq, D], row stride q_stride elements
  long long q_stride;
  __half *out;          // [rows, Hq, D], row stride out_stride elements
  long long out_stride;
  const __half *k_pool;  // [pool_pages, Hkv, page_size, D]
  const __half *v_pool;
  const int *block_table;  // [table rows, table_stride]
  int table_stride;
  const int *table_rows;   // [rows] block-table row of each query row
  const int *positions;    // [rows] query position; keys [0, position] are attended
  int rows, hq, hkv, head_dim, page_size, pool_pages, capacity;
  float scale;
  int max_splits;  // splits actually used <= min(max_splits, 64)
  int cluster;     // CTAs per thread-block cluster along the splits (1..16, a power of two; 0 = auto)
  // Which K/V rows may be gathered before the programmatic-dependency wait:
  // 0 none, 1 positions below the row's own position (decode: only the newest
  // row is produced by the preceding kernel), 2 all (no concurrent producer).
  int early_mode;
  int min_chunk;   // positions per split at least this many
  // When > 0 and the splits need more than one cluster: use one full cluster
  // unless that gives splits longer than max_chunk positions.
  int max_chunk;
  float *ws_acc;   // [rows, hkv, <= max_splits cluster slots, G, D] (splits spanning clusters)
  float *ws_ml;    // [rows, hkv, <= max_splits cluster slots, G, 2]
  // Floats available from ws_acc on (ws_ml included); 0 = unknown. The
  // streaming schedule runs only when they hold its per-CTA slots.
  size_t ws_floats;
  // 0: automatic (streaming for many (row, KV head) pairs with page boxes,
  // else split); 1: the split schedule; 2: streaming (invalid when it does
  // not apply).
  int schedule;
  // > 1: the rows are prefill rows of one sequence at consecutive positions
  // (one block-table row), served in groups of 16 / G rows by the streaming
  // schedule so that each K/V tile is read once per group; the split schedule
  // treats the rows one by one.
  int row_group;
  unsigned int *counters;  // [rows, hkv], zero between launches
  TmcDeviceStatus *status;
  TraceSink trace;         // optional timeline (records == nullptr: off)
  // Optional (host pointers, copied into the launch): tensor maps of k_pool and
  // v_pool viewed as [pool_pages * hkv * page_size rows, head_dim] fp16 with a
  // [16 rows, 64 columns] box and 128-byte swizzle (make_tensor_map_f16 with
  // box_rows 16). With them, head_dim 64 or 128 and page_size % 16 == 0, K/V
  // tiles arrive as 16-position page boxes (8x fewer copies than per row).
  const CUtensorMap *k_map;
  const CUtensorMap *v_map;
};

// Most splits one (row, KV head) is ever cut into; larger max_splits values
// are capped to this.
constexpr int kAttentionMaxSplits = 64;

// Workspace bytes needed for a launch with these dimensions.
size_t attention_workspace_bytes(int rows, int hq, int hkv, int head_dim, int max_splits);
// Workspace bytes the streaming schedule needs for row groups (row_group > 1).
size_t attention_group_workspace_bytes(int head_dim);

cudaError_t launch_attention(const AttentionParams &p, cudaStream_t stream, bool pdl);

}  // namespace tmc
