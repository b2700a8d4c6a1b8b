"""The allocation-free paged-attention entry point (tmc_k_paged_attention_f16_noalloc).

It exists for callers that cannot allocate device memory at call time, e.g. a
host that gives all device memory to its own pool at start-up or a runtime
whose memory plan forbids allocation later: its split-K partials and tickets
live in a fixed device array inside the library. These tests call it through
the C ABI and compare it with the allocating entry point
(tmc_k_paged_attention_f16) on the same inputs, twice in a row (the second call
starts from the array contents the first call left), and check that a request
larger than the fixed array is refused before anything runs. The file name
sorts last so that a stop-at-first-failure run has run every other test first.
"""

import ctypes
from ctypes import c_int, c_void_p

import numpy as np
import pytest

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


def test_noalloc_attention_matches_allocating_entry_point_twice(rt):
    import tmc_cuda
    hq, hkv, d, page, splits, chunk = 32, 8, 128, 16, 16, 32
    lengths = [1152, 17, 300]
    q, kp, vp, table, trows, pos = make_case(21, hq, hkv, d, page, lengths)
    rows = len(lengths)
    capacity = table.shape[1] * page
    qb, kb, vb = rt.upload(q), rt.upload(kp), rt.upload(vp)
    tb, trb, pb = rt.upload(table), rt.upload(trows), rt.upload(pos)

    # Existing entry point with a caller-allocated workspace.
    ws = rt.buffer(tmc_cuda.attention_workspace_bytes(rows, hq, hkv, d, splits) // 4 + 1, tmc_cuda.F32)
    counters = rt.upload(np.zeros(rows * hkv, np.int32))
    ref_out = rt.buffer(q.size, tmc_cuda.F16)
    tmc_cuda.paged_attention_f16(rt, qb, ref_out, kb, vb, tb, table.shape[1], trb, pb, rows, hq, hkv, d,
                                 page, kp.shape[0], capacity, splits, chunk, ws, counters)
    rt.synchronize()
    ref = ref_out.read().astype(np.float64)
    rms = float(np.sqrt(np.mean(ref ** 2)))

    fn = noalloc_entry()
    for call in range(2):
        out = rt.buffer(q.size, tmc_cuda.F16)
        code = fn(qb.ptr, out.ptr, kb.ptr, vb.ptr, tb.ptr, table.shape[1], trb.ptr, pb.ptr, rows, hq, hkv,
                  d, page, kp.shape[0], capacity, splits, chunk, rt.status_ptr, rt.stream)
        assert code == tmc_cuda.OK, tmc_cuda.last_error()
        rt.synchronize()
        got = out.read().astype(np.float64)
        err = float(np.max(np.abs(got - ref)))
        assert err <= 2e-3 * rms, (call, err, rms)


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
