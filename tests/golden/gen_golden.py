"""Generate the committed golden vectors for the oracle pin tests.

Run where the reference project's sources are present (the oracle Makefile's
REFERENCE variable names the checkout) after `make -C oracle` built
oracle/_ref/libtmcref.so, the reference's own evaluateGraph compiled from its
sources:

    python tests/golden/gen_golden.py

Outputs (small .npz files beside this script):
  c1_small.npz   RMSNorm -> Transpose(W) -> MatMul, rows 1 and 3, k=n=256, with
                 the graph suite's data() pattern and seeded N(0,1) inputs; y from
                 the reference's evaluateGraph.
  c1_full.npz    the BASELINE C1 case (seed 0, 4096 x 4096): y from evaluateGraph
                 (inputs are regenerated from the seed by oracle.workloads.c1_inputs).
  rmsnorm.npz    the graph suite's RMSNorm cases ([1,4096]; [3,4097] with a zero row
                 and a x1e-4 row; fp16 [1,257]), apps/tensor_graph_examples.cpp:79-123.
  fusion.npz     the graph suite's fused regions (Add -> RMSNorm [3,4097], Residual
                 Add -> LayerNorm [3,17], SiLU -> Mul [3,17], Linear -> ReLU [3,7]x[7,5]),
                 plus fp32 / fp16 seeded variants of each; y from evaluateGraph.
"""

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import oracle, workloads  # noqa: E402


def rms_weight(width):
    # tensor_graph_examples.cpp:98-101
    return (0.5 + (np.arange(width) % 31) / 32.0).astype(np.float32)


def main():
    if not oracle.reference_available():
        raise SystemExit("oracle/_ref/libtmcref.so missing: run `make -C oracle` with the reference mounted")
    out = {}
    for rows in (1, 3):
        k = n = 256
        x = workloads.graph_pattern(rows * k, seed=0).reshape(rows, k)
        gamma = rms_weight(k)
        w = workloads.graph_pattern(n * k, seed=5, scale=0.05).reshape(n, k)
        w = oracle.round_f16(w).reshape(n, k)
        out[f"pattern{rows}_x"], out[f"pattern{rows}_gamma"], out[f"pattern{rows}_w"] = x, gamma, w
        out[f"pattern{rows}_y"] = oracle.ref_rmsnorm_matmul(x, gamma, w, 1e-5)
        xs, gs, ws = workloads.c1_inputs(seed=7, k=k, n=n, rows=rows)
        ws = ws.astype(np.float32)
        out[f"seeded{rows}_x"], out[f"seeded{rows}_gamma"], out[f"seeded{rows}_w"] = xs, gs, ws
        out[f"seeded{rows}_y"] = oracle.ref_rmsnorm_matmul(xs, gs, ws, 1e-5)
    np.savez_compressed(os.path.join(HERE, "c1_small.npz"), **out)

    x, gamma, w = workloads.c1_inputs(seed=0)
    y = oracle.ref_rmsnorm_matmul(x, gamma, w.astype(np.float32), 1e-5)
    np.savez_compressed(os.path.join(HERE, "c1_full.npz"), y=y, x_head=x[0, :8], w_head=w[0, :8].astype(np.float32))

    cases = {}
    x = workloads.graph_pattern(4096).reshape(1, 4096)
    cases["r1x4096_x"] = x
    cases["r1x4096_y"] = oracle.ref_rmsnorm(x, rms_weight(4096), 1e-5, dtype=1)
    x = workloads.graph_pattern(3 * 4097).reshape(3, 4097)
    x[0, :] = 0.0
    x[1, :] *= np.float32(1e-4)
    cases["r3x4097_x"] = x
    cases["r3x4097_y"] = oracle.ref_rmsnorm(x, rms_weight(4097), 1e-5, dtype=1)
    x = workloads.graph_pattern(257).reshape(1, 257)
    cases["h1x257_x"] = x
    cases["h1x257_y"] = oracle.ref_rmsnorm(x, rms_weight(257), 1e-5, dtype=0)
    np.savez_compressed(os.path.join(HERE, "rmsnorm.npz"), **cases)

    # Fused regions of the graph suite (tensor_graph_examples.cpp:79-143,210-225),
    # fp32 as there, then fp16 and larger seeded variants of each.
    fz = {}

    def put(name, kind, x, b, w=None, c=None, fp16=False, n=0):
        if fp16:
            x, b = oracle.round_f16(x).reshape(x.shape), oracle.round_f16(b).reshape(b.shape)
            w = None if w is None else oracle.round_f16(w).reshape(w.shape)
            c = None if c is None else oracle.round_f16(c).reshape(c.shape)
        fz[f"{name}_x"], fz[f"{name}_b"] = x, b
        if w is not None:
            fz[f"{name}_w"] = w
        if c is not None:
            fz[f"{name}_c"] = c
        fz[f"{name}_y"] = oracle.ref_fusion(kind, x, b, w, c, 1e-5, fp16, n)

    pat = workloads.graph_pattern
    x = pat(3 * 4097).reshape(3, 4097)
    x[0, :] = 0.0
    x[1, :] *= np.float32(1e-4)
    put("addrms", "add_rmsnorm", x, pat(4097, seed=3, scale=0.1), rms_weight(4097))
    ln_w = pat(17, seed=3, scale=0.2) + np.float32(1.0)
    put("addln", "add_layernorm", pat(3 * 17).reshape(3, 17), pat(17, seed=1, scale=0.1), ln_w,
        pat(17, seed=2, scale=0.05))
    put("silumul", "silu_mul", pat(3 * 17).reshape(3, 17), pat(17, seed=2))
    put("linrelu", "linear_relu", pat(3 * 7).reshape(3, 7), pat(7 * 5, seed=1, scale=0.25).reshape(7, 5), None,
        pat(5, seed=2, scale=0.1), n=5)
    rng = np.random.default_rng(11)
    r = lambda *s: rng.standard_normal(s).astype(np.float32)  # noqa: E731
    for fp16 in (False, True):
        t = "h" if fp16 else "f"
        put(f"addrms_{t}8", "add_rmsnorm", r(8, 4096), r(8, 4096), 1 + 0.1 * r(4096), fp16=fp16)
        put(f"addln_{t}9", "add_layernorm", r(9, 1000), r(1000), 1 + 0.1 * r(1000), 0.1 * r(1000), fp16=fp16)
        put(f"silumul_{t}8", "silu_mul", 3 * r(8, 1024), r(8, 1024), fp16=fp16)
        put(f"linrelu_{t}40", "linear_relu", r(40, 96), 0.2 * r(96, 72), None, 0.1 * r(72), fp16=fp16, n=72)
    np.savez_compressed(os.path.join(HERE, "fusion.npz"), **fz)
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
