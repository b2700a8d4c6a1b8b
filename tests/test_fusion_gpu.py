"""Fused graph regions on the GPU (emitFusion, FusionMetalEmitter.cpp:81-214:
Add -> RMSNorm, residual Add -> LayerNorm, SiLU -> Mul, Linear -> ReLU)
against the reference's evaluateGraph outputs (tests/golden/fusion.npz). The
tolerance is the graph suite's own (tensor_graph_examples.cpp:55-58): fp32
atol 1e-5 / rtol 1e-4, fp16 2e-3 / 2e-3."""

import os

import numpy as np
import pytest

from oracle import oracle

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def names():
    g = np.load(os.path.join(GOLDEN, "fusion.npz"))
    return sorted({k.rsplit("_", 1)[0] for k in g.files if k.endswith("_y")})


@pytest.mark.parametrize("name", names())
def test_fused_region_matches_reference(rt, name):
    import tmc_cuda
    g = np.load(os.path.join(GOLDEN, "fusion.npz"))
    fp16 = "_h" in name
    dt, code = (np.float16, tmc_cuda.F16) if fp16 else (np.float32, tmc_cuda.F32)
    x, b, y_ref = g[f"{name}_x"], g[f"{name}_b"], g[f"{name}_y"]
    up = lambda a: rt.upload(np.ascontiguousarray(a.astype(dt)))  # noqa: E731
    y = rt.buffer(y_ref.size, code)
    kind = name.split("_")[0]
    if kind == "linrelu":
        m, k = x.shape
        tmc_cuda.fused_linear_relu(rt, up(x), up(b), up(g[f"{name}_c"]), y, m, k, y_ref.shape[1])
    elif kind == "silumul":
        tmc_cuda.fused_silu_mul(rt, up(x), up(b), y, x.shape[0], x.shape[1], 1 if b.ndim == 1 else b.shape[0])
    else:
        c = up(g[f"{name}_c"]) if kind == "addln" else None
        tmc_cuda.fused_add_norm(rt, up(x), up(b), up(g[f"{name}_w"]), y, x.shape[0], x.shape[1],
                                1 if b.ndim == 1 else b.shape[0], 1e-5, c)
    rt.synchronize()
    got = y.read().reshape(y_ref.shape).astype(np.float32)
    atol, rtol = (2e-3, 2e-3) if fp16 else (1e-5, 1e-4)
    ok, worst, bad, first = oracle.compare(got, y_ref, atol, rtol)
    assert ok, (name, worst, bad, first)
