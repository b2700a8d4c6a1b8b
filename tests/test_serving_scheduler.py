"""The continuous-batching scheduler on the CPU (runServingScheduler,
aicompiler-test_b200/csrc/ServingScheduler.hpp; reference runContinuousBatch,
src/runtime/ServingRuntime.cpp:513-930), instantiated with a host executor
(tests/serving_shim.cpp) that keeps the real page pool and cache states but
makes each next token a hash of the sequence's own history. The reference's
serving check (serving_main.cpp:69-140) then becomes exact: every request's
tokens equal its sequential chain, whatever the batching, admission order,
preemption or resume. Also checked: preemption under page pressure and a
resume for every preemption, every page returned, maxRows respected by
splitting a tick's decode into several calls, late arrivals, zero-token
requests, and the reference's rejections of invalid requests."""

import ctypes
import os
import shutil
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(ROOT, "aicompiler-test_b200", "csrc")
STATS = ("preemptions", "resumes", "peak_pages", "allocations", "releases", "decode_calls", "decoded",
         "prefilled", "ticks", "max_batch", "max_rows_seen", "pages_in_use")


@pytest.fixture(scope="module")
def lib(tmp_path_factory):
    if shutil.which("g++") is None:
        pytest.skip("g++ not available")
    out = str(tmp_path_factory.mktemp("servingshim") / "libservingshim.so")
    subprocess.run(["g++", "-std=c++17", "-O1", "-shared", "-fPIC", "-I", CSRC,
                    os.path.join(ROOT, "tests", "serving_shim.cpp"), os.path.join(CSRC, "KVCacheState.cpp"),
                    "-o", out], check=True, capture_output=True)
    lib = ctypes.CDLL(out)
    I, I32, S = ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_size_t)
    lib.serving_run.restype = ctypes.c_int
    lib.serving_run.argtypes = [ctypes.c_int, I, I32, I, I] + [ctypes.c_int] * 6 + [I32, S]
    lib.serving_last_error.restype = ctypes.c_char_p
    lib.serving_log.restype = ctypes.c_char_p
    return lib


def next_token(history, vocab):
    # FNV-1a over the tokens, as the shim's next_token.
    x = 1469598103934665603
    for t in history:
        x ^= t & 0xFFFFFFFF
        x = (x * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return x % vocab


def sequential(prompt, decode_count, vocab):
    hist = list(prompt)
    toks = [next_token(hist, vocab)]
    for _ in range(decode_count):
        hist.append(toks[-1])
        toks.append(next_token(hist, vocab))
    return toks


def serve(lib, prompts, decodes, arrivals, max_slots, capacity, max_rows, page_size, pool_pages, vocab=1000):
    n = len(prompts)
    arr = lambda v, t: (t * len(v))(*v)
    lens = [len(p) for p in prompts]
    flat = [int(t) for p in prompts for t in p]
    out = (ctypes.c_int32 * sum(1 + d for d in decodes))()
    stats = (ctypes.c_size_t * len(STATS))()
    rc = lib.serving_run(n, arr(lens, ctypes.c_int), arr(flat, ctypes.c_int32), arr(decodes, ctypes.c_int),
                         arr(arrivals, ctypes.c_int), max_slots, capacity, max_rows, page_size, pool_pages, vocab,
                         out, stats)
    if rc != 0:
        raise RuntimeError(lib.serving_last_error().decode())
    toks, o = [], 0
    for d in decodes:
        toks.append(list(out[o:o + 1 + d]))
        o += 1 + d
    return toks, dict(zip(STATS, list(stats))), lib.serving_log().decode()


def workload(seed, n, vocab=1000, prompt=(3, 40), decode=(0, 30), spread=6):
    rng = np.random.default_rng(seed)
    prompts = [rng.integers(0, vocab, int(rng.integers(*prompt))).tolist() for _ in range(n)]
    decodes = [int(rng.integers(*decode)) for _ in range(n)]
    arrivals = [int(rng.integers(0, spread)) for _ in range(n)]
    return prompts, decodes, arrivals


def check_sequential(toks, prompts, decodes, vocab=1000):
    for i, (p, d) in enumerate(zip(prompts, decodes)):
        assert toks[i] == sequential(p, d, vocab), f"request {i}"


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_ample_pages_match_sequential_without_preemption(lib, seed):
    prompts, decodes, arrivals = workload(seed, 12)
    toks, st, _ = serve(lib, prompts, decodes, arrivals, max_slots=16, capacity=128, max_rows=16, page_size=8,
                        pool_pages=512)
    check_sequential(toks, prompts, decodes)
    assert st["preemptions"] == st["resumes"] == 0
    assert st["decoded"] == sum(decodes) and st["prefilled"] == sum(len(p) for p in prompts)
    assert st["allocations"] == st["releases"] and st["pages_in_use"] == 0
    assert st["ticks"] > max(arrivals)


@pytest.mark.parametrize("seed,pool", [(3, 14), (4, 12), (5, 20)])
def test_page_pressure_preempts_and_resumes_exactly(lib, seed, pool):
    # Pools of 12-20 pages of 8 (one full sequence needs 12) for ten requests of
    # up to 11 pages: the scheduler must preempt the request holding the most
    # pages and resume it later with its KV state intact.
    prompts, decodes, arrivals = workload(seed, 10, prompt=(10, 30), decode=(20, 60), spread=2)
    toks, st, log = serve(lib, prompts, decodes, arrivals, max_slots=8, capacity=96, max_rows=8, page_size=8,
                          pool_pages=pool)
    check_sequential(toks, prompts, decodes)
    assert st["preemptions"] > 0 and st["resumes"] == st["preemptions"]
    assert "preempted for page pressure" in log and "resumed at length" in log
    assert st["peak_pages"] <= pool and st["pages_in_use"] == 0
    assert st["allocations"] == st["releases"]


def test_more_active_rows_than_max_rows_split_the_step(lib):
    prompts, decodes, arrivals = workload(6, 20, decode=(10, 20), spread=1)
    toks, st, _ = serve(lib, prompts, decodes, arrivals, max_slots=20, capacity=128, max_rows=3, page_size=8,
                        pool_pages=1024)
    check_sequential(toks, prompts, decodes)
    assert st["max_rows_seen"] == 3 and st["max_batch"] > 3
    assert st["decode_calls"] > st["ticks"]


def test_slots_are_reused_and_late_arrivals_wait(lib):
    # Two slots for seven requests, one arriving at tick 40.
    prompts, decodes, arrivals = workload(7, 7, decode=(1, 6), spread=3)
    arrivals[-1] = 40
    toks, st, log = serve(lib, prompts, decodes, arrivals, max_slots=2, capacity=64, max_rows=2, page_size=4,
                          pool_pages=64)
    check_sequential(toks, prompts, decodes)
    assert st["max_batch"] <= 2 and st["ticks"] > 40
    assert log.count("prefill complete") == 7 and log.count("finished") == sum(1 for d in decodes if d > 0)


def test_zero_decode_requests_finish_at_prefill(lib):
    prompts = [[1, 2, 3], [4, 5], [6]]
    toks, st, _ = serve(lib, prompts, [0, 0, 0], [0, 1, 2], max_slots=1, capacity=16, max_rows=1, page_size=4,
                        pool_pages=4)
    assert toks == [sequential(p, 0, 1000) for p in prompts]
    assert st["decode_calls"] == 0 and st["pages_in_use"] == 0


@pytest.mark.parametrize("case,match", [
    ("long_prompt", "dimensions are invalid"),
    ("too_many_tokens", "dimensions are invalid"),
    ("empty_prompt", "dimensions are invalid"),
    ("small_pool", "cannot hold"),
])
def test_invalid_requests_are_rejected(lib, case, match):
    prompts, decodes, arrivals, pool = [[1, 2, 3]], [4], [0], 16
    if case == "long_prompt":
        prompts = [list(range(32))]                 # prompt must be shorter than the capacity
    if case == "too_many_tokens":
        decodes = [30]                              # 3 + 30 > capacity 32
    if case == "empty_prompt":
        prompts = [[]]
    if case == "small_pool":
        decodes, pool = [20], 2                     # 23 tokens need 6 pages of 4
    with pytest.raises(RuntimeError, match=match):
        serve(lib, prompts, decodes, arrivals, max_slots=2, capacity=32, max_rows=2, page_size=4, pool_pages=pool)
