"""Batched projection on tcgen05 tensor cores (the decoder's path for more
than 8 rows; replaces emitTiledGEMM, DecodeGEMVMetalEmitter.cpp:134-169)
against an fp64 restatement of the same product on the fp16 inputs.

Tolerance: max |gpu - ref| <= 1e-4 x RMS(ref) (fp32 accumulation of fp16
products; far inside the north-star 2e-3 x RMS), and two launches give
bit-identical results (split-K partials are summed in a fixed order)."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CASES = [
    # rows, k, n
    (9, 4096, 4096),      # 16-token tile, one weight tile per CTA
    (16, 1024, 2816),     # single-layer FFN shape (C2)
    (33, 4096, 6144),     # 64-token tile, 8B QKV shape
    (64, 4096, 4096),     # bs64 O projection
    (64, 14336, 4096),    # bs64 down projection: K split across CTAs
    (100, 2048, 1000),    # 128-token tile, ragged last weight tile
    (128, 512, 384),
    (200, 4096, 6144),    # 256-token tile (prefill chunks), QKV shape
    (256, 1024, 2816),    # 256-token tile, C2 FFN shape
    (1, 64, 128),
]


def run(rt, x, w):
    import tmc_cuda
    rows, k = x.shape
    n = w.shape[0]
    xb, wb = rt.upload(x), rt.upload(w)
    yb = rt.buffer(rows * n, tmc_cuda.F32)
    ws = rt.buffer(max(tmc_cuda.batched_gemm_workspace_bytes(n, k, rows) // 4, 1), tmc_cuda.F32)
    tmc_cuda.batched_gemm_f16(rt, xb, wb, yb, rows, k, n, ws)
    rt.synchronize()
    first = yb.read().reshape(rows, n)
    tmc_cuda.batched_gemm_f16(rt, xb, wb, yb, rows, k, n, ws)
    rt.synchronize()
    second = yb.read().reshape(rows, n)
    return first, second


@pytest.mark.parametrize("rows,k,n", CASES)
def test_batched_gemm_matches_fp64(rt, rows, k, n):
    rng = np.random.default_rng(rows * 131 + k + n)
    x = rng.standard_normal((rows, k)).astype(np.float16)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float16)
    got, again = run(rt, x, w)
    ref = x.astype(np.float64) @ w.astype(np.float64).T
    rms = float(np.sqrt(np.mean(ref ** 2)))
    err = float(np.max(np.abs(got.astype(np.float64) - ref)))
    assert err <= 1e-4 * rms, (err, rms)
    assert np.array_equal(got, again), "batched gemm is not deterministic"
