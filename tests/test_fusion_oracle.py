"""The C restatement of the fused graph regions (oracle/graph_ref.c
oracle_fusion, following GraphReference.cpp:129-199 node by node) against the
golden vectors the reference's own evaluateGraph produced
(tests/golden/gen_golden.py): bit-exact fp64."""

import os

import numpy as np
import pytest

from oracle import oracle

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
KINDS = {"addrms": "add_rmsnorm", "addln": "add_layernorm", "silumul": "silu_mul", "linrelu": "linear_relu"}


def cases():
    g = np.load(os.path.join(GOLDEN, "fusion.npz"))
    names = sorted({k.rsplit("_", 1)[0] for k in g.files if k.endswith("_y")})
    return names


@pytest.mark.parametrize("name", cases())
def test_fusion_restatement_matches_reference_golden(name):
    g = np.load(os.path.join(GOLDEN, "fusion.npz"))
    kind = KINDS[name.split("_")[0]]
    fp16 = "_h" in name
    y = g[f"{name}_y"]
    got = oracle.fusion(kind, g[f"{name}_x"], g[f"{name}_b"], g[f"{name}_w"] if f"{name}_w" in g else None,
                        g[f"{name}_c"] if f"{name}_c" in g else None, 1e-5, fp16, n=y.shape[1])
    assert np.array_equal(got, y)


@pytest.mark.skipif(not oracle.reference_available(), reason="oracle/_ref not built here")
@pytest.mark.parametrize("kind", ["add_rmsnorm", "add_layernorm", "silu_mul", "linear_relu"])
@pytest.mark.parametrize("fp16", [False, True])
def test_fusion_restatement_matches_live_reference(kind, fp16):
    rng = np.random.default_rng(5)
    x = rng.standard_normal((5, 40)).astype(np.float32)
    b = rng.standard_normal((40, 9) if kind == "linear_relu" else (5, 40)).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(40)).astype(np.float32)
    c = rng.standard_normal(9 if kind == "linear_relu" else 40).astype(np.float32)
    if fp16:
        x, b, w, c = (oracle.round_f16(a).reshape(a.shape) for a in (x, b, w, c))
    n = 9 if kind == "linear_relu" else 0
    assert np.array_equal(oracle.fusion(kind, x, b, w, c, 1e-5, fp16, n), oracle.ref_fusion(kind, x, b, w, c, 1e-5, fp16, n))


def test_storage_rounding_follows_the_reference_tie_rule():
    # GraphReference.cpp:38-59 rounds fp16 ties away from zero; inputs convert
    # with round-to-nearest-even (the GPU's rule).
    tie = 1.0 + 2.0 ** -11          # halfway between fp16 1.0 and 1.0 + 2^-10
    assert oracle._lib.oracle_store(tie, 0) == np.float32(1.0 + 2.0 ** -10)
    assert oracle._lib.oracle_store(-tie, 0) == np.float32(-(1.0 + 2.0 ** -10))
    assert oracle.round_f16(np.array([tie], np.float32))[0] == np.float32(1.0)
    assert oracle._lib.oracle_store(1.0 + 2.0 ** -12, 0) == np.float32(1.0)
    assert oracle._lib.oracle_store(70000.0, 0) == np.float32(np.inf)
