"""Standalone RMSNorm (RMSNormOp, src/tensor/TensorIR.hpp:98-104; emitRMSNorm,
src/backend/metal/MetalEmitter.cpp:12-76) and its tuner (tuneRMSNorm,
src/planner/RMSNormTuner.cpp:159-309) on the GPU, against the reference's
golden vectors and the fp64 oracle.

Tolerances are the tuner's own (RMSNormTuner.cpp:19-20,75-76): fp32 storage
atol 1e-5 / rtol 1e-4, fp16 storage atol 2e-3 / rtol 2e-3.
"""

import os

import numpy as np
import pytest

from oracle import oracle

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
THREADS = [0, 32, 64, 128, 256, 512, 1024]  # 0 = the frozen 256-thread baseline


def gamma_for(width):
    return (0.5 + (np.arange(width) % 31) / 32.0).astype(np.float32)


def run(rt, x, gamma, eps, fp16, threads):
    import tmc_cuda
    rows, width = x.shape
    dt = np.float16 if fp16 else np.float32
    xb = rt.upload(x.astype(dt))
    gb = rt.upload(gamma.astype(dt))
    yb = rt.buffer(rows * width, tmc_cuda.F16 if fp16 else tmc_cuda.F32)
    tmc_cuda.rmsnorm(rt, xb, gb, yb, rows, width, eps, threads)
    rt.synchronize()
    return yb.read().reshape(rows, width).astype(np.float32)


def tol(fp16):
    return (2e-3, 2e-3) if fp16 else (1e-5, 1e-4)


@pytest.mark.parametrize("threads", THREADS)
@pytest.mark.parametrize("case,width,fp16", [("r1x4096", 4096, False), ("r3x4097", 4097, False),
                                             ("h1x257", 257, True)])
def test_rmsnorm_matches_reference_golden(rt, case, width, fp16, threads):
    g = np.load(os.path.join(GOLDEN, "rmsnorm.npz"))
    x = g[f"{case}_x"]
    gamma = gamma_for(width)
    if fp16:
        x = oracle.round_f16(x).reshape(x.shape)
        gamma = oracle.round_f16(gamma)
    y = run(rt, x, gamma, 1e-5, fp16, threads)
    ok, worst, bad, first = oracle.compare(y, g[f"{case}_y"], *tol(fp16))
    assert ok, (worst, bad, first)


@pytest.mark.parametrize("threads", [0, 128, 512])
@pytest.mark.parametrize("rows,width,fp16", [(64, 4096, True), (7, 5120, False), (33, 4104, True), (2, 6, False)])
def test_rmsnorm_matches_oracle(rt, rows, width, fp16, threads):
    rng = np.random.default_rng(rows * 7 + width)
    x = rng.standard_normal((rows, width)).astype(np.float32)
    gamma = (1.0 + 0.1 * rng.standard_normal(width)).astype(np.float32)
    if fp16:
        x = oracle.round_f16(x).reshape(x.shape)
        gamma = oracle.round_f16(gamma)
    y = run(rt, x, gamma, 1e-6, fp16, threads)
    ok, worst, bad, first = oracle.compare(y, oracle.rmsnorm(x, gamma, 1e-6), *tol(fp16))
    assert ok, (worst, bad, first)


def test_rmsnorm_rejects_bad_block_size(rt):
    import tmc_cuda
    b = rt.buffer(64, tmc_cuda.F32)
    with pytest.raises(tmc_cuda.TmcError):
        tmc_cuda.rmsnorm(rt, b, b, b, 1, 64, 1e-5, 96)


@pytest.mark.parametrize("rows,width,fp16", [(1, 4096, False), (64, 4096, True), (3, 4097, False)])
def test_rmsnorm_tuner_selection_is_validated(rows, width, fp16):
    import tmc_cuda
    rng = np.random.default_rng(width + rows)
    x = rng.standard_normal((rows, width)).astype(np.float32)
    gamma = gamma_for(width)
    sel = tmc_cuda.tune_rmsnorm(x, gamma, 1e-5, fp16=fp16, candidate_threads=(64, 128, 256, 512, 96))
    assert sel["success"], sel["log"]
    assert "candidate_96 | Hardware Filter FAIL" in sel["log"]
    assert "Final numerical validation: PASS" in sel["log"]
    if not sel["used_baseline"]:
        assert sel["speedup"] >= 1.05 and sel["threads"] in (64, 128, 256, 512)
    else:
        assert sel["threads"] == 256
    if fp16:
        x = oracle.round_f16(x).reshape(x.shape)
        gamma = oracle.round_f16(gamma)
    ok, worst, bad, first = oracle.compare(sel["output"], oracle.rmsnorm(x, gamma, 1e-5), *tol(fp16))
    assert ok, (worst, bad, first)
