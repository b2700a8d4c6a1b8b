"""Host KV page pool and per-sequence cache state on the CPU
(aicompiler-test_b200/csrc/KVCacheState.cpp, compiled with g++ together with
tests/kv_state_shim.cpp; reference KVPagePool / KVCacheState,
src/runtime/KVCacheState.cpp:30-86,153-216,355-379):
- the free list is LIFO seeded in ascending order, so the first allocation is
  the highest page id and a released page is the next one handed out;
- peak / allocation / release counters; releasing a page that is not allocated
  is rejected;
- stageLength allocates all or nothing: on pool exhaustion (or an injected
  allocation failure) the pages it took are returned and the state is unchanged;
- a failing block-table upload unwinds the allocation and re-sends the old row;
- rollbackLength releases pages beyond the new length; commitLength rejects 0
  and lengths above capacity; destroying a state returns its pages.
By design (not in the reference): rollbackLength also lowers the committed
length when it releases pages that held committed positions, and the block
table is sent only when the page list changed."""

import ctypes
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(ROOT, "aicompiler-test_b200", "csrc")


@pytest.fixture(scope="module")
def kv(tmp_path_factory):
    if shutil.which("g++") is None:
        pytest.skip("g++ not available")
    out = str(tmp_path_factory.mktemp("kvshim") / "libkvshim.so")
    subprocess.run(["g++", "-std=c++17", "-O1", "-shared", "-fPIC", "-I", CSRC,
                    os.path.join(ROOT, "tests", "kv_state_shim.cpp"), os.path.join(CSRC, "KVCacheState.cpp"),
                    "-o", out], check=True, capture_output=True)
    lib = ctypes.CDLL(out)
    P, S, Z, I = ctypes.c_void_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t), ctypes.POINTER(ctypes.c_int)
    sig = {
        "kv_last_error": (ctypes.c_char_p, []),
        "kv_pool_new": (P, [S, S]), "kv_pool_free": (None, [P]), "kv_pool_stats": (None, [P, Z]),
        "kv_pool_allocate": (ctypes.c_int, [P]), "kv_pool_release": (ctypes.c_int, [P, ctypes.c_int]),
        "kv_pool_is_allocated": (ctypes.c_int, [P, ctypes.c_int]), "kv_pool_fail_next": (None, [P, S]),
        "kv_state_new": (P, [P, S, ctypes.c_int, ctypes.c_int]), "kv_state_free": (None, [P]),
        "kv_state_stage": (ctypes.c_int, [P, S]), "kv_state_rollback": (ctypes.c_int, [P, S]),
        "kv_state_reset": (ctypes.c_int, [P]), "kv_state_commit": (ctypes.c_int, [P, S]),
        "kv_state_length": (S, [P]), "kv_state_max_pages": (S, [P]),
        "kv_state_pages": (S, [P, I, S]), "kv_state_row": (S, [P, I, S]),
        "kv_sink_fail_next": (None, [P, ctypes.c_int]), "kv_sink_count": (S, [P]),
        "kv_sink_row": (S, [P, S, I, S]),
    }
    for name, (res, args) in sig.items():
        f = getattr(lib, name)
        f.restype, f.argtypes = res, args
    return lib


def stats(kv, pool):
    out = (ctypes.c_size_t * 6)()
    kv.kv_pool_stats(pool, out)
    return dict(zip(("capacity", "used", "available", "peak", "allocations", "releases"), list(out)))


def ints(fn, *args, cap=64):
    buf = (ctypes.c_int * cap)()
    n = fn(*args, buf, cap)
    return list(buf[:n])


def err(kv):
    return kv.kv_last_error().decode()


def test_pool_is_lifo_and_counts(kv):
    pool = kv.kv_pool_new(16, 4)
    assert [kv.kv_pool_allocate(pool) for _ in range(3)] == [3, 2, 1]
    assert kv.kv_pool_release(pool, 2) == 0
    assert kv.kv_pool_allocate(pool) == 2          # the released page comes back first
    assert kv.kv_pool_allocate(pool) == 0
    assert kv.kv_pool_allocate(pool) == -1         # exhausted
    assert stats(kv, pool) == dict(capacity=4, used=4, available=0, peak=4, allocations=5, releases=1)
    assert kv.kv_pool_release(pool, 7) == -1 and "invalid page" in err(kv)
    assert kv.kv_pool_release(pool, 1) == 0
    assert kv.kv_pool_release(pool, 1) == -1       # not allocated any more
    assert kv.kv_pool_is_allocated(pool, 1) == 0 and kv.kv_pool_is_allocated(pool, 3) == 1
    kv.kv_pool_free(pool)


def test_pool_and_state_reject_bad_dimensions(kv):
    assert kv.kv_pool_new(0, 4) is None and kv.kv_pool_new(16, 0) is None
    pool = kv.kv_pool_new(4, 2)
    assert kv.kv_state_new(pool, 12, 0, 0) is None    # 3 pages can never fit in 2
    assert "full capacity" in err(kv)
    assert kv.kv_state_new(pool, 0, 0, 0) is None
    kv.kv_pool_free(pool)


def test_stage_commit_rollback_and_block_table_rows(kv):
    pool = kv.kv_pool_new(4, 8)
    st = kv.kv_state_new(pool, 20, 3, 1)
    assert kv.kv_state_max_pages(st) == 5
    assert kv.kv_state_stage(st, 5) == 0
    assert ints(kv.kv_state_pages, st) == [7, 6]
    assert ints(kv.kv_state_row, st) == [7, 6, -1, -1, -1]
    assert kv.kv_sink_count(st) == 1 and ints(kv.kv_sink_row, st, 0) == [7, 6, -1, -1, -1]
    assert kv.kv_state_length(st) == 0                 # staging does not commit
    assert kv.kv_state_commit(st, 5) == 0 and kv.kv_state_length(st) == 5
    assert kv.kv_state_stage(st, 8) == 0 and kv.kv_sink_count(st) == 1   # same pages: no upload
    assert kv.kv_state_stage(st, 13) == 0
    assert ints(kv.kv_state_pages, st) == [7, 6, 5, 4] and kv.kv_sink_count(st) == 2
    # Roll back the uncommitted positions: pages past the committed length go back.
    assert kv.kv_state_rollback(st, 5) == 0
    assert ints(kv.kv_state_pages, st) == [7, 6] and kv.kv_state_length(st) == 5
    assert ints(kv.kv_sink_row, st, 2) == [7, 6, -1, -1, -1]
    assert stats(kv, pool)["used"] == 2 and stats(kv, pool)["peak"] == 4
    # Length checks (KVCacheState.cpp:170-175,198-202,242-247).
    assert kv.kv_state_stage(st, 0) == -1 and "outside the configured capacity" in err(kv)
    assert kv.kv_state_stage(st, 21) == -1
    assert kv.kv_state_rollback(st, 21) == -1 and "beyond its configured capacity" in err(kv)
    assert kv.kv_state_commit(st, 0) == -1 and kv.kv_state_commit(st, 21) == -1
    assert kv.kv_state_length(st) == 5
    # Rolling back below the committed length lowers it (by design, see the docstring).
    assert kv.kv_state_rollback(st, 3) == 0 and kv.kv_state_length(st) == 3
    assert ints(kv.kv_state_pages, st) == [7]
    assert kv.kv_state_reset(st) == 0 and kv.kv_state_length(st) == 0
    assert ints(kv.kv_state_pages, st) == [] and stats(kv, pool)["used"] == 0
    kv.kv_state_free(st)
    kv.kv_pool_free(pool)


def test_stage_is_all_or_nothing_on_exhaustion(kv):
    pool = kv.kv_pool_new(4, 4)
    a = kv.kv_state_new(pool, 16, 0, 1)
    b = kv.kv_state_new(pool, 16, 1, 1)
    assert kv.kv_state_stage(a, 12) == 0               # 3 of 4 pages
    assert kv.kv_state_stage(b, 4) == 0                # the last page
    assert kv.kv_state_stage(b, 8) == -1 and "exhausted" in err(kv)
    assert ints(kv.kv_state_pages, b) == [0] and kv.kv_sink_count(b) == 1   # unchanged, no upload
    kv.kv_state_free(a)                                # destroying a state returns its pages
    assert stats(kv, pool)["available"] == 3
    assert kv.kv_state_stage(b, 16) == 0
    assert ints(kv.kv_state_pages, b) == [0, 1, 2, 3]
    kv.kv_state_free(b)
    # a: 3, b: 1 then 3 more; every page released again.
    assert stats(kv, pool) == dict(capacity=4, used=0, available=4, peak=4, allocations=7, releases=7)
    kv.kv_pool_free(pool)


def test_partial_allocation_is_returned(kv):
    pool = kv.kv_pool_new(4, 4)
    a = kv.kv_state_new(pool, 16, 0, 0)
    b = kv.kv_state_new(pool, 16, 1, 1)
    assert kv.kv_state_stage(a, 1) == 0                # page 3
    # b needs 4 pages, 3 are free: it takes 2, 1, 0, misses the fourth, returns all three.
    assert kv.kv_state_stage(b, 16) == -1 and "exhausted" in err(kv)
    assert ints(kv.kv_state_pages, b) == [] and kv.kv_sink_count(b) == 0
    assert stats(kv, pool) == dict(capacity=4, used=1, available=3, peak=4, allocations=4, releases=3)
    # LIFO: the unwound pages went back newest-first, so the same ids come out again.
    assert kv.kv_state_stage(b, 12) == 0 and ints(kv.kv_state_pages, b) == [2, 1, 0]
    kv.kv_state_free(a)
    kv.kv_state_free(b)
    kv.kv_pool_free(pool)


def test_injected_allocation_failure_unwinds(kv):
    pool = kv.kv_pool_new(2, 8)
    st = kv.kv_state_new(pool, 16, 0, 1)
    assert kv.kv_state_stage(st, 2) == 0
    kv.kv_pool_fail_next(pool, 1)
    # The next allocation fails as if the pool were empty: the state keeps its page.
    before = stats(kv, pool)
    assert kv.kv_state_stage(st, 8) == -1 and "exhausted" in err(kv)
    assert stats(kv, pool) == before and ints(kv.kv_state_pages, st) == [7]
    assert kv.kv_sink_count(st) == 1
    assert kv.kv_state_stage(st, 8) == 0 and ints(kv.kv_state_pages, st) == [7, 6, 5, 4]
    kv.kv_state_free(st)
    kv.kv_pool_free(pool)


def test_failed_block_table_upload_unwinds(kv):
    pool = kv.kv_pool_new(4, 6)
    st = kv.kv_state_new(pool, 24, 2, 1)
    assert kv.kv_state_stage(st, 4) == 0
    kv.kv_sink_fail_next(st, 1)
    assert kv.kv_state_stage(st, 12) == -1 and "upload failed" in err(kv)
    assert ints(kv.kv_state_pages, st) == [5] and stats(kv, pool)["used"] == 1
    # The failed row, then the old row re-sent so the device table matches the state.
    n = kv.kv_sink_count(st)
    assert n == 3 and ints(kv.kv_sink_row, st, 1)[:3] == [5, 4, 3]
    assert ints(kv.kv_sink_row, st, 2) == [5, -1, -1, -1, -1, -1]
    kv.kv_state_free(st)
    kv.kv_pool_free(pool)
