"""The allocation-free paged-attention entry point (tmc_k_paged_attention_f16_noalloc).

It exists for callers that cannot allocate device memory at call time, e.g. a
host that gives all device memory to its own pool at start-up or a runtime
whose memory plan forbids allocation later: its split-K partials and tickets
live in a fixed device array inside the library. These tests call it through
the C ABI and compare it with the allocating entry point
(tmc_k_paged_attention_f16) and with the CPU oracle on the same inputs.

Two calls run back to back with different row and KV-head counts, with
min_chunk >= 512 so that every (row, KV head) is cut into several
single-CTA clusters: the splits then meet through the fixed array (partials,
then the ticket of the last CTA), and the second call reads partials and
tickets at other offsets than the first left behind. A request larger than
the fixed array is refused before anything runs; a max_splits above the
kernel's 64-split cap is sized for the cap. The file name sorts last so that a
stop-at-first-failure run has run every other test first.
"""

from ctypes import c_int, c_void_p

import numpy as np
import pytest

from oracle import oracle

pytestmark = pytest.mark.gpu


def noalloc_entry():
    import tmc_cuda
    fn = tmc_cuda.lib.tmc_k_paged_attention_f16_noalloc
    fn.restype = c_int
    fn.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_void_p,
                   c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p]
    return fn


def make_case(seed, hq, hkv, d, page, lengths):
    rng = np.random.default_rng(seed)
    rows = len(lengths)
    stride = (max(lengths) + page - 1) // page
    pool = sum((n + page - 1) // page for n in lengths) + 5
    perm = rng.permutation(pool).astype(np.int32)
    table = np.full((rows, stride), -1, np.int32)
    off = 0
    for r, n in enumerate(lengths):
        k = (n + page - 1) // page
        table[r, :k] = perm[off:off + k]
        off += k
    k_pool = rng.standard_normal((pool, hkv, page, d)).astype(np.float16)
    v_pool = rng.standard_normal((pool, hkv, page, d)).astype(np.float16)
    q = rng.standard_normal((rows, hq, d)).astype(np.float16)
    positions = np.array([n - 1 for n in lengths], np.int32)
    return q, k_pool, v_pool, table, np.arange(rows, dtype=np.int32), positions


def oracle_check(got, q, kp, vp, table, trows, pos, hkv, page):
    """Per element within max(2e-3 x RMS, one fp16 ulp) of the fp64 oracle
    after its fp16 storage rounding (the test_attention_gpu.py bound)."""
    ref = oracle.paged_attention(q.astype(np.float32), kp.astype(np.float32), vp.astype(np.float32),
                                 table, trows, pos, hkv, page)
    ref16 = oracle.round_f16(ref.astype(np.float32)).reshape(ref.shape)
    rms = float(np.sqrt(np.mean(ref ** 2)))
    ulp = np.spacing(np.abs(ref16).astype(np.float16)).astype(np.float64)
    err = np.abs(got - ref16)
    assert np.all(err <= np.maximum(2e-3 * rms, ulp)), (float(err.max()), rms)


def run_pair(rt, case, splits, chunk):
    """The allocating entry point, then the allocation-free one, on one case;
    returns (allocating output, allocation-free output) as float64."""
    import tmc_cuda
    q, kp, vp, table, trows, pos, hkv, page = case
    rows, hq, d = q.shape
    capacity = table.shape[1] * page
    qb, kb, vb = rt.upload(q), rt.upload(kp), rt.upload(vp)
    tb, trb, pb = rt.upload(table), rt.upload(trows), rt.upload(pos)
    # The allocating entry point's contract: a workspace for the full max_splits.
    ws = rt.buffer(tmc_cuda.attention_workspace_bytes(rows, hq, hkv, d, splits) // 4 + 1, tmc_cuda.F32)
    counters = rt.upload(np.zeros(rows * hkv, np.int32))
    ref_out = rt.buffer(q.size, tmc_cuda.F16)
    tmc_cuda.paged_attention_f16(rt, qb, ref_out, kb, vb, tb, table.shape[1], trb, pb, rows, hq, hkv, d,
                                 page, kp.shape[0], capacity, splits, chunk, ws, counters)
    rt.synchronize()
    out = rt.buffer(q.size, tmc_cuda.F16)
    code = noalloc_entry()(qb.ptr, out.ptr, kb.ptr, vb.ptr, tb.ptr, table.shape[1], trb.ptr, pb.ptr, rows, hq,
                           hkv, d, page, kp.shape[0], capacity, splits, chunk, rt.status_ptr, rt.stream)
    assert code == tmc_cuda.OK, tmc_cuda.last_error()
    rt.synchronize()
    return (ref_out.read().reshape(q.shape).astype(np.float64), out.read().reshape(q.shape).astype(np.float64))


def test_noalloc_attention_merges_across_clusters_through_the_fixed_array_twice(rt):
    # Call 1: 3 rows x 8 KV heads, contexts of a few thousand positions cut into
    # up to 12 splits of >= 512 positions (one CTA per cluster: partials and
    # tickets in the fixed array). Call 2: other rows / KV heads / splits, so
    # its partials and tickets sit at other offsets than call 1 left them.
    cases = [
        ((*make_case(21, 32, 8, 128, 16, [3000, 5100, 700]), 8, 16), 12, 512),
        ((*make_case(22, 16, 2, 128, 16, [4097, 1800, 2600, 1030, 6000]), 2, 16), 16, 640),
    ]
    for call, (case, splits, chunk) in enumerate(cases):
        ref, got = run_pair(rt, case, splits, chunk)
        rms = float(np.sqrt(np.mean(ref ** 2)))
        err = float(np.max(np.abs(got - ref)))
        print(f"no-alloc call {call}: max|err| vs allocating entry {err:.3e} (rms {rms:.3f})")
        assert err <= 2e-3 * rms, (call, err, rms)
        oracle_check(got, *case)


def test_noalloc_attention_page_boxes_match_allocating_entry(rt):
    # Short splits (clusters of up to 16 CTAs merging through distributed
    # shared memory) on the C4 head shape; the same kernel variant as the
    # allocating entry point (16-position page boxes through tensor maps).
    case = (*make_case(23, 32, 8, 128, 16, [1152, 17, 300]), 8, 16)
    ref, got = run_pair(rt, case, 16, 32)
    assert np.array_equal(ref, got)
    oracle_check(got, *case)


def test_noalloc_attention_caps_max_splits_at_the_kernel_limit(rt):
    # max_splits 200 would need 200-split partials; the kernel uses at most 64,
    # so the request is sized for 64 and runs like the allocating entry point.
    case = (*make_case(24, 8, 2, 64, 16, [9000, 40]), 2, 16)
    ref, got = run_pair(rt, case, 200, 128)
    assert np.array_equal(ref, got)
    oracle_check(got, *case)


def test_noalloc_attention_refuses_requests_beyond_the_fixed_scratch(rt):
    import tmc_cuda
    hq, hkv, d = 32, 8, 128
    rows, splits = 64, 64  # 64*32*64*130*4 bytes of partials, far above 8 MiB
    q, kp, vp, table, trows, pos = make_case(3, hq, hkv, d, 16, [40] * rows)
    qb, kb, vb = rt.upload(q), rt.upload(kp), rt.upload(vp)
    tb, trb, pb = rt.upload(table), rt.upload(trows), rt.upload(pos)
    out = rt.buffer(q.size, tmc_cuda.F16)
    fn = noalloc_entry()
    code = fn(qb.ptr, out.ptr, kb.ptr, vb.ptr, tb.ptr, table.shape[1], trb.ptr, pb.ptr, rows, hq, hkv, d,
              16, kp.shape[0], table.shape[1] * 16, splits, 32, rt.status_ptr, rt.stream)
    assert code == tmc_cuda.ERR_UNSUPPORTED
    assert "fixed limit" in tmc_cuda.last_error()
    rt.synchronize()
