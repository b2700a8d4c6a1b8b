"""Timing statistics (aicompiler-test_b200/csrc/timing_stats.hpp, used by the
tuners' paired measurements) against the reference's definitions
(benchmark::summarizeTimings, Benchmark.cpp:10-25): median as the mean of the
two middle samples for an even count, the 90th percentile interpolated
linearly between ranks floor(0.9 (n-1)) and the next, which is numpy's median
and its default linear percentile; minimum, maximum; no statistics for no
samples."""

import ctypes
import os
import shutil
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(ROOT, "aicompiler-test_b200", "csrc")


@pytest.fixture(scope="module")
def summarize(tmp_path_factory):
    if shutil.which("g++") is None:
        pytest.skip("g++ not available")
    out = str(tmp_path_factory.mktemp("timingshim") / "libtimingshim.so")
    subprocess.run(["g++", "-std=c++17", "-O1", "-shared", "-fPIC", "-I", CSRC,
                    os.path.join(ROOT, "tests", "timing_shim.cpp"), "-o", out], check=True, capture_output=True)
    lib = ctypes.CDLL(out)
    lib.summarize.restype = ctypes.c_int
    lib.summarize.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]

    def run(values):
        v = np.ascontiguousarray(values, np.float64)
        out = np.zeros(5)
        ok = lib.summarize(v.ctypes.data, v.size, out.ctypes.data)
        return tuple(out) if ok else None
    return run


@pytest.mark.parametrize("n", [1, 2, 3, 4, 9, 10, 31, 32, 100])
def test_statistics_match_the_reference_definitions(summarize, n):
    rng = np.random.default_rng(n)
    for _ in range(20):
        v = rng.exponential(10.0, n) + rng.integers(0, 3, n)   # ties included
        got = summarize(v)
        ref = (n, np.median(v), np.percentile(v, 90), v.min(), v.max())
        np.testing.assert_allclose(got, ref, rtol=1e-15, atol=0)


def test_no_samples_have_no_statistics(summarize):
    assert summarize([]) is None
