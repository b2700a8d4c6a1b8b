"""The prepared-execution surface on the GPU: built-in kernels bound to buffers
and constants (tmc_prepare, the reference's MetalRuntime::prepareBuffers,
MetalRuntime.mm:594-648), run with NaN sentinels and executed
(PreparedExecution, MetalRuntime.mm:197-277), and chained into one CUDA graph
(prepareSequence, MetalRuntime.mm:751-781).

- the C1 RMSNorm -> GEMV bound through tmc_prepare matches the reference's
  evaluateGraph golden; run() and execute() agree;
- the reference's rejections: an input aliasing an output, duplicate outputs,
  dispatch beyond the device limits, wrong binding counts; plus this backend's
  interface checks (element types, sizes);
- a sequence (fp16 RMSNorm, then a GEMV reading its output) equals the two
  executions run one by one, and replays launched without synchronising give
  the same result; GEMV steps start before their predecessor ends
  (programmatic dependent launch) only when no earlier step writes the weights
  they read early: a sequence whose first step writes the second's weights
  still equals its steps run one by one;
- the tensor-core GEMM and the paged attention bound through tmc_prepare equal
  their direct C-ABI entry points bit for bit.
"""

import os

import numpy as np
import pytest

from oracle import oracle, workloads

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def test_prepared_c1_matches_reference_golden(rt):
    import tmc_cuda
    x, gamma, w = workloads.c1_inputs(seed=0)
    g = np.load(os.path.join(GOLDEN, "c1_full.npz"))
    xb, gb, wb = rt.upload(x), rt.upload(gamma), rt.upload(w.astype(np.float16))
    yb = rt.buffer(4096, tmc_cuda.F32)
    p = tmc_cuda.Prepared(rt, "rmsnorm_gemv_f32", [xb, gb, wb], [yb], [1, 4096, 4096, tmc_cuda.float_bits(1e-5)])
    y, gpu_us, cpu_us = p.run()
    assert gpu_us > 0 and cpu_us >= gpu_us * 0.5
    ref = g["y"].reshape(-1)
    rms = float(np.sqrt(np.mean(ref ** 2)))
    assert float(np.max(np.abs(y - ref))) <= 2e-3 * rms
    ok, worst, bad, first = oracle.compare(y, ref, 1e-5, 1e-4)
    assert ok, (worst, bad, first)
    yb.write(np.full(4096, np.nan, np.float32))
    p.execute()
    assert np.array_equal(yb.read(), y)


def test_prepare_rejects_what_prepare_buffers_rejects(rt):
    import tmc_cuda
    a = rt.buffer(64, tmc_cuda.F32)
    g = rt.buffer(64, tmc_cuda.F32)
    y = rt.buffer(64, tmc_cuda.F32)
    eps = tmc_cuda.float_bits(1e-5)
    cases = [
        (([a, g], [a], [1, 64, eps], 1, 64), "aliases an output"),
        (([a, g], [y, y], [1, 64, eps], 1, 64), "distinct"),
        (([a, g], [y], [1, 64, eps], 1, 4096), "exceeds device or pipeline limits"),
        (([a, g], [y], [1, 64, eps], 0, 64), "exceeds device or pipeline limits"),
        (([a], [y], [1, 64, eps], 1, 64), "binds 2 inputs"),
        (([a, g], [y], [1, 128, eps], 1, 64), "needs 128"),
        (([a, g], [y], [1, 64, eps], 1, 48), "power of two"),
    ]
    for (ins, outs, consts, groups, threads), fragment in cases:
        with pytest.raises(tmc_cuda.TmcError) as err:
            tmc_cuda.Prepared(rt, "rmsnorm", ins, outs, consts, groups, threads)
        assert fragment in err.value.message, (fragment, err.value.message)
    h = rt.buffer(64, tmc_cuda.F16)
    with pytest.raises(tmc_cuda.TmcError, match="must be fp32"):
        tmc_cuda.Prepared(rt, "rmsnorm", [a, h], [y], [1, 64, eps], 1, 64)
    with pytest.raises(tmc_cuda.TmcError, match="no built-in kernel"):
        tmc_cuda.Prepared(rt, "no_such_kernel", [a], [y])


def test_sequence_equals_its_steps_run_one_by_one(rt):
    import tmc_cuda
    rng = np.random.default_rng(3)
    rows, k, n = 4, 1024, 768
    x = rng.standard_normal((rows, k)).astype(np.float16)
    gamma = rng.uniform(0.5, 1.5, k).astype(np.float16)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float16)
    xb, gb, wb = rt.upload(x), rt.upload(gamma), rt.upload(w)
    hb = rt.buffer(rows * k, tmc_cuda.F16)
    yb = rt.buffer(rows * n, tmc_cuda.F32)
    norm = tmc_cuda.Prepared(rt, "rmsnorm", [xb, gb], [hb], [rows, k, tmc_cuda.float_bits(1e-5)], rows, 128)
    gemv = tmc_cuda.Prepared(rt, "gemv_f16", [hb, wb], [yb], [rows, k, n])
    h_ref, _, _ = norm.run()
    y_ref, _, _ = gemv.run()
    ref = oracle.gemv(h_ref.reshape(rows, k), w.astype(np.float32)).reshape(-1)
    assert float(np.max(np.abs(y_ref - ref))) <= 2e-3 * float(np.sqrt(np.mean(ref ** 2)))
    seq = tmc_cuda.Sequence(rt, [norm, gemv])
    hb.write(np.zeros(rows * k, np.float32))
    yb.write(np.full(rows * n, np.nan, np.float32))
    gpu_us, _ = seq.execute()
    assert gpu_us > 0 and np.array_equal(yb.read(), y_ref)
    yb.write(np.full(rows * n, np.nan, np.float32))
    seq.launch(5)
    rt.synchronize()
    assert np.array_equal(yb.read(), y_ref)


def test_sequence_keeps_weights_written_by_an_earlier_step_ordered(rt):
    import tmc_cuda
    rng = np.random.default_rng(4)
    rows, k, n = 2, 2048, 4096
    x = rng.standard_normal((rows, k)).astype(np.float16)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float16)
    xb, wb = rt.upload(x), rt.upload(w)
    zero = rt.upload(np.zeros(k, np.float16))
    w2 = rt.buffer(n * k, tmc_cuda.F16)
    y1 = rt.buffer(rows * n, tmc_cuda.F32)
    y2 = rt.buffer(rows * n, tmc_cuda.F32)
    direct = tmc_cuda.Prepared(rt, "gemv_f16", [xb, wb], [y1], [rows, k, n])
    copy = tmc_cuda.Prepared(rt, "add", [wb, zero], [w2], [n, k, 1])  # w2 = w + 0: writes the next step's weights
    gemv = tmc_cuda.Prepared(rt, "gemv_f16", [xb, w2], [y2], [rows, k, n])
    ref, _, _ = direct.run()
    for _ in range(3):
        w2.write(np.full(n * k, np.nan, np.float32))
        y2.write(np.full(rows * n, np.nan, np.float32))
        seq = tmc_cuda.Sequence(rt, [copy, gemv])
        seq.execute()
        assert np.array_equal(y2.read(), ref)
        seq.close()


def test_prepared_gemm_and_attention_equal_their_entry_points(rt):
    import tmc_cuda
    rng = np.random.default_rng(9)
    rows, k, n = 40, 4096, 1536
    x = rng.standard_normal((rows, k)).astype(np.float16)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float16)
    xb, wb = rt.upload(x), rt.upload(w)
    direct = rt.buffer(rows * n, tmc_cuda.F32)
    ws = rt.buffer(tmc_cuda.batched_gemm_workspace_bytes(n, k, rows) // 4 + 1, tmc_cuda.F32)
    tmc_cuda.batched_gemm_f16(rt, xb, wb, direct, rows, k, n, ws)
    yb = rt.buffer(rows * n, tmc_cuda.F32)
    p = tmc_cuda.Prepared(rt, "batched_gemm_f16", [xb, wb], [yb], [rows, k, n])
    y, _, _ = p.run()
    y2, _, _ = p.run()  # the retained tickets were left at zero
    assert np.array_equal(y, direct.read()) and np.array_equal(y, y2)

    from tests.test_attention_gpu import make_case, run_attention
    q, kp, vp, table, trows, pos = make_case(5, 3, 32, 8, 128, 16, [700, 33, 1500])
    cap = table.shape[1] * 16
    ref = run_attention(rt, q, kp, vp, table, trows, pos, 8, 16, cap, 8, 64)
    bufs = [rt.upload(a) for a in (q, kp, vp, table, trows, pos)]
    out = rt.buffer(q.size, tmc_cuda.F16)
    att = tmc_cuda.Prepared(rt, "paged_attention_f16", bufs, [out],
                            [3, 32, 8, 128, 16, kp.shape[0], cap, table.shape[1], 8, 64])
    got, _, _ = att.run()
    assert np.array_equal(got.reshape(ref.shape), ref)
