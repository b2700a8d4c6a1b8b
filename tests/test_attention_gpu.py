"""Paged GQA decode attention on the GPU vs the CPU oracle (fp64 restatement of
emitServingPagedKVAttention, reference KVCacheMetalEmitter.cpp:312-406, plus the
GQA head map). Tolerance, per element after the reference's storage rounding
of the context to fp16: |gpu - ref| <= max(2e-3 x RMS(ref), one fp16 ulp of
ref) -- the context is stored in fp16, so an fp32 result a hair away from the
fp64 one can round to the neighbouring fp16 value near a rounding midpoint."""

import numpy as np
import pytest

from oracle import oracle

pytestmark = pytest.mark.gpu


def make_case(seed, rows, hq, hkv, d, page_size, lengths, pool_pages=None, share_table=False):
    rng = np.random.default_rng(seed)
    max_len = max(lengths)
    stride = (max_len + page_size - 1) // page_size
    need = sum((l + page_size - 1) // page_size for l in lengths)
    pool_pages = pool_pages or max(need + 3, 8)
    perm = rng.permutation(pool_pages).astype(np.int32)
    table = np.full((rows, stride), -1, dtype=np.int32)
    off = 0
    for r, l in enumerate(lengths):
        n = (l + page_size - 1) // page_size
        table[r, :n] = perm[off:off + n]
        off += n
    k_pool = rng.standard_normal((pool_pages, hkv, page_size, d)).astype(np.float16)
    v_pool = rng.standard_normal((pool_pages, hkv, page_size, d)).astype(np.float16)
    q = rng.standard_normal((rows, hq, d)).astype(np.float16)
    positions = np.array([l - 1 for l in lengths], dtype=np.int32)
    table_rows = np.arange(rows, dtype=np.int32)
    return q, k_pool, v_pool, table, table_rows, positions


def run_attention(rt, q, k_pool, v_pool, table, table_rows, positions, hkv, page_size, capacity,
                  max_splits=8, min_chunk=32, schedule=0, row_group=1):
    import tmc_cuda
    rows, hq, d = q.shape
    ws_bytes = tmc_cuda.attention_workspace_bytes(rows, hq, hkv, d, max_splits)
    qb, kb, vb = rt.upload(q), rt.upload(k_pool), rt.upload(v_pool)
    tb, trb, pb = rt.upload(table), rt.upload(table_rows), rt.upload(positions)
    out = rt.buffer(q.size, tmc_cuda.F16)
    ws = rt.buffer(max(ws_bytes // 4, 1), tmc_cuda.F32)
    counters = rt.upload(np.zeros(rows * hkv, dtype=np.int32))
    tmc_cuda.paged_attention_f16(rt, qb, out, kb, vb, tb, table.shape[1], trb, pb, rows, hq, hkv, d,
                                 page_size, k_pool.shape[0], capacity, max_splits, min_chunk, ws,
                                 counters, schedule, row_group)
    rt.synchronize()
    assert np.all(counters.read_raw() == 0), "split tickets must be left at zero"
    return out.read().reshape(rows, hq, d)


def check(got, ref):
    ref16 = oracle.round_f16(ref.astype(np.float32)).reshape(ref.shape)
    rms = float(np.sqrt(np.mean(ref ** 2)))
    ulp = np.spacing(np.abs(ref16).astype(np.float16)).astype(np.float64)
    err = np.abs(got.astype(np.float64) - ref16)
    bound = np.maximum(2e-3 * rms, ulp)
    worst = int(np.argmax(err - bound))
    assert np.all(err <= bound), (float(err.flat[worst]), float(bound.flat[worst]), rms)


CASES = [
    # (rows, hq, hkv, d, page, lengths)
    (1, 32, 8, 128, 16, [1]),
    (1, 32, 8, 128, 16, [1152]),
    (3, 32, 8, 128, 16, [17, 16, 300]),
    (4, 16, 16, 64, 2048, [513, 520, 576, 1]),   # contiguous MHA (C2 shape): one page per row
    (2, 4, 4, 16, 4, [9, 32]),                   # reference defaults: head_dim 16, page 4
    (2, 8, 2, 32, 8, [100, 7]),
    (2, 16, 2, 128, 16, [2000, 65]),             # G = 8
    (2, 4, 2, 64, 16, [64, 1000]),               # G = 2
]


@pytest.mark.parametrize("rows,hq,hkv,d,page,lengths", CASES)
@pytest.mark.parametrize("splits", [(1, 64), (16, 32)])
def test_paged_attention_matches_oracle(rt, rows, hq, hkv, d, page, lengths, splits):
    q, kp, vp, table, trows, pos = make_case(rows * 7 + d, rows, hq, hkv, d, page, lengths)
    capacity = table.shape[1] * page
    ref = oracle.paged_attention(q.astype(np.float32), kp.astype(np.float32), vp.astype(np.float32),
                                 table, trows, pos, hkv, page)
    got = run_attention(rt, q, kp, vp, table, trows, pos, hkv, page, capacity, *splits)
    check(got, ref)


@pytest.mark.parametrize("rows,hq,hkv,d,lengths,splits", [
    (1, 32, 8, 128, [5000], (64, 64)),     # 63 active splits: four 16-CTA clusters per head
    (2, 16, 2, 64, [3000, 40], (48, 64)),  # G = 8, head_dim 64: three clusters for the long
                                           # row; one active CTA and idle clusters for the short
])
def test_split_schedule_across_clusters_matches_oracle(rt, rows, hq, hkv, d, lengths, splits):
    # A pair wider than one cluster: each cluster merges its CTAs by pushes into
    # the owners' shared memory, then the last CTA combines the clusters'
    # results from the workspace.
    q, kp, vp, table, trows, pos = make_case(sum(lengths) + d, rows, hq, hkv, d, 16, lengths)
    ref = oracle.paged_attention(q.astype(np.float32), kp.astype(np.float32), vp.astype(np.float32),
                                 table, trows, pos, hkv, 16)
    got = run_attention(rt, q, kp, vp, table, trows, pos, hkv, 16, table.shape[1] * 16, *splits, schedule=1)
    check(got, ref)


def test_paged_attention_c4_subset(rt):
    # C4 shapes (32q/8kv x 128, 16-token pages, random pages of a large pool)
    # on 8 sequences with contexts drawn from U[128, 8192].
    from oracle import workloads
    ctx, table, positions, q = workloads.c4_inputs(seed=0, seqs=8, pool_pages=4608)
    rng = np.random.default_rng(1)
    kp = rng.standard_normal((4608, 8, 16, 128)).astype(np.float16)
    vp = rng.standard_normal((4608, 8, 16, 128)).astype(np.float16)
    trows = np.arange(8, dtype=np.int32)
    ref = oracle.paged_attention(q.astype(np.float32), kp.astype(np.float32), vp.astype(np.float32),
                                 table, trows, positions, 8, 16)
    got = run_attention(rt, q, kp, vp, table, trows, positions, 8, 16, 8192, 32, 256)
    check(got, ref)


# Batched launches: more (split, KV head, row) CTAs than fit on the GPU at
# once (several waves of clustered CTAs), ragged contexts.
ROWS_CASES = [
    # (rows, hq, hkv, d, lengths seed, max length, splits)
    (64, 32, 8, 128, 11, 1500, (8, 64)),
    (64, 32, 8, 128, 12, 1200, (4, 64)),
    (96, 16, 2, 128, 13, 700, (16, 32)),   # G = 8
    (200, 4, 2, 64, 14, 300, (8, 16)),     # G = 2, head_dim 64
]


@pytest.mark.parametrize("rows,hq,hkv,d,seed,max_len,splits", ROWS_CASES)
@pytest.mark.parametrize("schedule", [1, 2])  # split-K with cluster merges; streaming
def test_paged_attention_many_waves_matches_oracle(rt, rows, hq, hkv, d, seed, max_len, splits, schedule):
    rng = np.random.default_rng(seed)
    lengths = [int(x) for x in rng.integers(1, max_len, rows)]
    lengths[0], lengths[1], lengths[2] = 1, 64, 1024 if max_len > 1024 else 48
    q, kp, vp, table, trows, pos = make_case(seed, rows, hq, hkv, d, 16, lengths)
    capacity = table.shape[1] * 16
    ref = oracle.paged_attention(q.astype(np.float32), kp.astype(np.float32), vp.astype(np.float32),
                                 table, trows, pos, hkv, 16)
    got = run_attention(rt, q, kp, vp, table, trows, pos, hkv, 16, capacity, *splits, schedule=schedule)
    check(got, ref)


# The streaming schedule where it is not picked automatically: few pairs, so
# the runs are shorter than the pairs and most pairs are cut into several
# pieces (down to one tile per CTA) merged through the workspace; G = 1, 2, 4, 8.
STREAM_SMALL = [
    (3, 32, 8, 128, 16, [17, 16, 300]),
    (2, 16, 2, 128, 16, [2000, 65]),
    (2, 4, 2, 64, 16, [64, 1000]),
    (4, 16, 16, 64, 16, [513, 520, 576, 1]),
    (1, 32, 8, 128, 16, [8192]),
]


@pytest.mark.parametrize("rows,hq,hkv,d,page,lengths", STREAM_SMALL)
def test_streaming_schedule_with_cut_pairs_matches_oracle(rt, rows, hq, hkv, d, page, lengths):
    q, kp, vp, table, trows, pos = make_case(rows * 5 + d, rows, hq, hkv, d, page, lengths)
    ref = oracle.paged_attention(q.astype(np.float32), kp.astype(np.float32), vp.astype(np.float32),
                                 table, trows, pos, hkv, page)
    got = run_attention(rt, q, kp, vp, table, trows, pos, hkv, page, table.shape[1] * page, 64, 64, schedule=2)
    check(got, ref)


# Prefill rows: one sequence, consecutive positions, one block-table row. The
# streaming schedule serves them in groups of 16 / G rows that share each K/V
# tile (row_group 2); partial last groups, every G, pairs cut between CTAs.
PREFILL_CASES = [
    # (rows, hq, hkv, d, first position)
    (256, 32, 8, 128, 768),   # the bs1 decoder's last 256-row prefill chunk of a 1024-token prompt
    (37, 32, 8, 128, 100),    # G = 4: groups of 4, the last one partial
    (50, 16, 16, 64, 300),    # G = 1: groups of 16
    (21, 16, 2, 128, 2000),   # G = 8: groups of 2, long contexts
    (40, 4, 2, 64, 0),        # G = 2: groups of 8 from position 0
]


@pytest.mark.parametrize("rows,hq,hkv,d,first", PREFILL_CASES)
def test_prefill_row_groups_match_oracle(rt, rows, hq, hkv, d, first):
    page = 16
    rng = np.random.default_rng(rows + first)
    total = first + rows
    stride = (total + page - 1) // page
    pool_pages = stride + 5
    table = rng.permutation(pool_pages)[:stride].astype(np.int32).reshape(1, stride)
    kp = rng.standard_normal((pool_pages, hkv, page, d)).astype(np.float16)
    vp = rng.standard_normal((pool_pages, hkv, page, d)).astype(np.float16)
    q = rng.standard_normal((rows, hq, d)).astype(np.float16)
    trows = np.zeros(rows, np.int32)
    pos = (first + np.arange(rows)).astype(np.int32)
    ref = oracle.paged_attention(q.astype(np.float32), kp.astype(np.float32), vp.astype(np.float32),
                                 table, trows, pos, hkv, page)
    # The workspace size for these arguments must hold the row groups' slots
    # (640 x 2 x 16 x (d + 2) floats): pick max_splits accordingly.
    splits = max(1, -(-640 * 2 * 16 // (rows * hq)))
    got = run_attention(rt, q, kp, vp, table, trows, pos, hkv, page, stride * page, splits, 64, schedule=2,
                        row_group=2)
    check(got, ref)


@pytest.mark.parametrize("schedule", [1, 2])
def test_many_waves_missing_page_reports_device_status(rt, schedule):
    import tmc_cuda
    lengths = [700] * 64
    q, kp, vp, table, trows, pos = make_case(21, 64, 32, 8, 128, 16, lengths)
    table[40, 7] = -1
    with pytest.raises(tmc_cuda.TmcError) as err:
        run_attention(rt, q, kp, vp, table, trows, pos, 8, 16, table.shape[1] * 16, 8, 64, schedule=schedule)
    assert err.value.code == tmc_cuda.ERR_DEVICE_STATUS
    assert "no physical page" in err.value.message


def test_missing_page_reports_device_status(rt):
    import tmc_cuda
    q, kp, vp, table, trows, pos = make_case(3, 1, 4, 4, 16, 4, [20])
    table[0, 2] = -1
    with pytest.raises(tmc_cuda.TmcError) as err:
        run_attention(rt, q, kp, vp, table, trows, pos, 4, 4, table.shape[1] * 4)
    assert err.value.code == tmc_cuda.ERR_DEVICE_STATUS
    assert "no physical page" in err.value.message
    rt.synchronize()  # the status block was consumed; the context is still usable


def test_paged_attention_c4_full_size(rt):
    # The benchmarked C4 case itself (bench.c4_case: 64 sequences, contexts
    # U[128, 8192], 32q/8kv x 128, pages drawn at random from a 2^17-page pool
    # of 2 x 4.29 GB filled on the device, 8 splits of >= 1024 positions)
    # against the fp64 oracle. The oracle reads only the pages the block
    # tables name (copied back and renumbered densely).
    from concurrent.futures import ThreadPoolExecutor

    import bench
    import tmc_cuda
    from tests.parity_util import fp16_close
    c = bench.c4_case()
    rows, hq, hkv, d, page, pool_pages = c["rows"], c["hq"], c["hkv"], c["d"], c["page"], c["pool_pages"]
    table, ctx = c["table"], c["ctx"]
    kp = rt.buffer(pool_pages * hkv * page * d, tmc_cuda.F16)
    vp = rt.buffer(pool_pages * hkv * page * d, tmc_cuda.F16)
    tmc_cuda.fill_normal_f16(rt, kp, c["k_seed"], 0.0, 1.0)
    tmc_cuda.fill_normal_f16(rt, vp, c["v_seed"], 0.0, 1.0)
    qb, out = rt.upload(c["q"]), rt.buffer(c["q"].size, tmc_cuda.F16)
    tb, trb = rt.upload(table), rt.upload(np.arange(rows, dtype=np.int32))
    pb = rt.upload((ctx - 1).astype(np.int32))
    ws = rt.buffer(tmc_cuda.attention_workspace_bytes(rows, hq, hkv, d, c["max_splits"]) // 4 + 1, tmc_cuda.F32)
    counters = rt.upload(np.zeros(rows * hkv, dtype=np.int32))
    tmc_cuda.paged_attention_f16(rt, qb, out, kp, vp, tb, c["stride"], trb, pb, rows, hq, hkv, d, page,
                                 pool_pages, c["stride"] * page, c["max_splits"], c["min_chunk"], ws, counters)
    rt.synchronize()
    got = out.read().reshape(rows, hq, d).astype(np.float64)
    used = np.unique(table[table >= 0])
    dense = np.full(pool_pages, -1, np.int32)
    dense[used] = np.arange(used.size, dtype=np.int32)
    dtable = np.where(table >= 0, dense[np.maximum(table, 0)], -1).astype(np.int32)
    per_page = hkv * page * d
    kd = np.empty((used.size, per_page), np.float32)
    vd = np.empty((used.size, per_page), np.float32)
    for i, pg in enumerate(used):
        kd[i] = kp.read_raw_range(int(pg) * per_page * 2, per_page).astype(np.float32)
        vd[i] = vp.read_raw_range(int(pg) * per_page * 2, per_page).astype(np.float32)
    kd = kd.reshape(used.size, hkv, page, d)
    vd = vd.reshape(used.size, hkv, page, d)
    q32 = c["q"].astype(np.float32)
    pos = (ctx - 1).astype(np.int32)

    def one(r):
        return oracle.paged_attention(q32[r:r + 1], kd, vd, dtable, np.array([r], np.int32), pos[r:r + 1], hkv, page)

    import os
    with ThreadPoolExecutor(max_workers=max(1, min(16, os.cpu_count() or 1))) as ex:
        ref = np.concatenate(list(ex.map(one, range(rows))))
    print(f"[parity] C4 full size: {rows} sequences, sum ctx {int(ctx.sum())}, {used.size} pages read back")
    check(got, ref)
    fp16_close(got, oracle.round_f16(ref.astype(np.float32)).reshape(ref.shape), "C4 full-size attention output")
