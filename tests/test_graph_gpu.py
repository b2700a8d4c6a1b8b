"""Compiled tensor graphs on the GPU (tmc_graph_compile / tmc_graph_run, the
reference's compileGraph + CompiledGraph::run) against the reference's own CPU
evaluator, evaluateGraph, compiled from its sources into oracle/_ref.

Tolerances are those compileGraph validates with (GraphExecutor.cpp tolerance():
fp32 atol 1e-5 / rtol 1e-4, fp16 atol = rtol = 2e-3), checked with the
reference's Validator::compare restatement (oracle.compare), plus the north
star max|err| <= 2e-3 x RMS for the C1 graph."""

import os

import numpy as np
import pytest

from oracle import oracle, workloads

pytestmark = pytest.mark.gpu
F16, F32 = 0, 1
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def tolerance(dtype):
    return (2e-3, 2e-3) if dtype == F16 else (1e-5, 1e-4)


def storage(a, dtype):
    """Host values as the graph stores them (fp16 rounding for fp16 inputs)."""
    a = np.asarray(a, np.float32)
    return a.astype(np.float16).astype(np.float32) if dtype == F16 else a


def check_against_reference(rt, inputs, nodes, outputs, values, expect_kernels=None):
    import tmc_cuda
    values = [storage(v, d) for v, (d, _) in zip(values, inputs)]
    g = tmc_cuda.Graph(rt, inputs, nodes, outputs)
    if expect_kernels is not None:
        assert [s.split("(")[0] for s in g.plan()] == expect_kernels
    outs, gpu_us = g.run(*values)
    # The reference refuses an fp16 weight under fp32 (TensorIR's matching-dtype
    # rule): give it the same values declared fp32 (exact).
    base = inputs[0][0]
    ref_inputs = [(F32 if (base == F32 and d == F16) else d, s) for d, s in inputs]
    ref = oracle.ref_evaluate_graph(ref_inputs, nodes, outputs, values)
    at = 0
    for v, out in zip(outputs, outs):
        n = out.size
        atol, rtol = tolerance(base)
        ok, worst, bad, first = oracle.compare(out.reshape(-1), ref[at:at + n], atol, rtol)
        assert ok, (v, worst, bad, first)
        at += n
    again, _ = g.run(*values)
    for a, b in zip(outs, again):
        assert np.array_equal(a, b)
    g.close()
    return outs


@pytest.mark.parametrize("dtype", [F32, F16])
def test_fused_regions_match_evaluate_graph(rt, dtype):
    rng = np.random.default_rng(3)
    x = rng.standard_normal((6, 96))
    b = rng.standard_normal((96,))
    w = rng.uniform(0.5, 1.5, 96)
    c = rng.standard_normal(96) * 0.1
    X, R = (dtype, (6, 96)), (dtype, (96,))
    check_against_reference(rt, [X, R, R], [("Add", [0, 1]), ("RMSNorm", [3, 2], [1e-5])], [4], [x, b, w],
                            ["fused_add_rmsnorm"])
    check_against_reference(rt, [X, X, R, R], [("Add", [0, 1]), ("LayerNorm", [4, 2, 3], [1e-5])], [5],
                            [x, rng.standard_normal((6, 96)), w, c], ["fused_add_layernorm"])
    check_against_reference(rt, [X, R], [("SiLU", [0]), ("Mul", [1, 2])], [3], [x, b], ["fused_silu_mul"])
    check_against_reference(rt, [X, (dtype, (96, 40)), (dtype, (40,))],
                            [("MatMul", [0, 1]), ("Add", [3, 2]), ("ReLU", [4])], [5],
                            [x, rng.standard_normal((96, 40)) * 0.1, rng.standard_normal(40) * 0.1],
                            ["fused_linear_relu"])


@pytest.mark.parametrize("dtype", [F32, F16])
def test_unfused_graph_matches_evaluate_graph(rt, dtype):
    # Norm -> projection through a Transpose view -> view -> elementwise chain,
    # with two declared outputs (one of them an intermediate).
    rng = np.random.default_rng(5)
    rows, k, n = 3, 128, 96
    inputs = [(dtype, (rows, k)), (dtype, (k,)), (dtype, (n, k)), (dtype, (rows * n,))]
    nodes = [("RMSNorm", [0, 1], [1e-5]),          # v4
             ("Transpose", [2], [0, 1]),            # v5
             ("MatMul", [4, 5]),                    # v6
             ("Reshape", [6], [rows * n]),          # v7 (alias)
             ("Add", [7, 3]),                       # v8
             ("ReLU", [8]),                         # v9
             ("Mul", [9, 9]),                       # v10
             ("SiLU", [10])]                        # v11
    kernels = ["rmsnorm", "gemv_f16" if dtype == F16 else "matmul", "add", "relu", "mul", "silu"]
    check_against_reference(rt, inputs, nodes, [6, 11],
                            [rng.standard_normal((rows, k)), rng.uniform(0.5, 1.5, k),
                             rng.standard_normal((n, k)) * 0.05, rng.standard_normal(rows * n) * 0.1], kernels)


def test_c1_graph_fp32_weight_matches_evaluate_graph(rt):
    # The reference's C1 graph as it declares it (W fp32 holding fp16-rounded
    # values): RMSNorm then a tiled MatMul through the Transpose view.
    import tmc_cuda
    x, gamma, w = workloads.c1_inputs(seed=2, k=1024, n=512)
    g = tmc_cuda.Graph(rt, [(F32, (1, 1024)), (F32, (1024,)), (F32, (512, 1024))],
                       [("RMSNorm", [0, 1], [1e-5]), ("Transpose", [2], [0, 1]), ("MatMul", [3, 4])], [5])
    assert [s.split("(")[0] for s in g.plan()] == ["rmsnorm", "matmul"]
    (y,), _ = g.run(x, gamma, w.astype(np.float32))
    ref = oracle.ref_rmsnorm_matmul(x, gamma, w.astype(np.float32))
    ok, worst, bad, first = oracle.compare(y.reshape(-1), ref.reshape(-1), 1e-5, 1e-4)
    assert ok, (worst, bad, first)
    g.close()


def test_graph_inputs_on_the_device_and_replays(rt):
    # Inputs written straight into the compiled graph's device buffers, replays
    # enqueued without synchronising (the benchmark's path).
    import ctypes

    import tmc_cuda
    x, gamma, w = workloads.c1_inputs(seed=4, k=512, n=256)
    g = tmc_cuda.Graph(rt, [(F32, (1, 512)), (F32, (512,)), (F16, (256, 512))],
                       [("RMSNorm", [0, 1], [1e-5]), ("Transpose", [2], [0, 1]), ("MatMul", [3, 4])], [5])
    (y,), _ = g.run(x, gamma, w)
    h = ctypes.c_void_p()
    tmc_cuda.check(tmc_cuda.lib.tmc_graph_input_buffer(g.handle, 0, ctypes.byref(h)))
    tmc_cuda.check(tmc_cuda.lib.tmc_buffer_write(h, x.reshape(-1).ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                                                 x.size, 0))
    tmc_cuda.check(tmc_cuda.lib.tmc_graph_launch(g.handle, 3))
    rt.synchronize()
    tmc_cuda.lib.tmc_buffer_destroy(h)
    (y2,), _ = g.run(x, gamma, w)
    assert np.array_equal(y, y2)
    g.close()
