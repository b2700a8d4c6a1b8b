"""Pin the CPU oracle (oracle/graph_ref.c) to the reference's own CPU path.

The golden vectors under tests/golden/ were produced by the reference's
evaluateGraph (reference src/validation/GraphReference.cpp:98) compiled from its
sources (tests/golden/gen_golden.py). These tests run on CPU only.
"""

import os

import numpy as np
import pytest

from oracle import oracle, workloads

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")

pytestmark = pytest.mark.skipif(not oracle.available(), reason="run `make -C oracle` first")


def test_f16_rounding_exhaustive_against_ieee():
    # Every fp16 bit pattern round-trips; fp32 values round like IEEE RNE (numpy).
    bits = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16)
    halves = bits.view(np.float16)
    finite = np.isfinite(halves)
    as32 = halves[finite].astype(np.float32)
    assert np.array_equal(oracle.round_f16(as32), as32)
    rng = np.random.default_rng(3)
    vals = np.concatenate([
        rng.standard_normal(200000).astype(np.float32) * np.float32(10.0) ** rng.integers(-9, 5, 200000),
        np.array([65504.0, 65519.99, 65520.0, 1e-8, 2.0 ** -25, 2.0 ** -24, 5.96e-8, -0.0], np.float32),
    ]).astype(np.float32)
    with np.errstate(over="ignore"):
        expected = vals.astype(np.float16).astype(np.float32)
    got = oracle.round_f16(vals)
    assert np.array_equal(np.isinf(got), np.isinf(expected))
    fin = np.isfinite(expected)
    assert np.array_equal(got[fin], expected[fin])
    assert np.array_equal(oracle.f32_to_f16_bits(vals[fin]), vals[fin].astype(np.float16).view(np.uint16))


@pytest.mark.parametrize("kind", ["pattern", "seeded"])
@pytest.mark.parametrize("rows", [1, 3])
def test_c1_small_restatement_matches_reference_golden(kind, rows):
    g = np.load(os.path.join(GOLDEN, "c1_small.npz"))
    x, gamma, w, y = (g[f"{kind}{rows}_{n}"] for n in ("x", "gamma", "w", "y"))
    got = oracle.rmsnorm_matmul(x, gamma, w, 1e-5)
    # Same fp64 expression order as evaluateGraph: identical to the last bit.
    assert np.array_equal(got, y)


def test_c1_full_restatement_matches_reference_golden():
    g = np.load(os.path.join(GOLDEN, "c1_full.npz"))
    x, gamma, w = workloads.c1_inputs(seed=0)
    assert np.array_equal(x[0, :8], g["x_head"]) and np.array_equal(w[0, :8].astype(np.float32), g["w_head"])
    got = oracle.rmsnorm_matmul(x, gamma, w.astype(np.float32), 1e-5)
    assert np.array_equal(got, g["y"])


@pytest.mark.parametrize("case,width,dtype", [("r1x4096", 4096, 1), ("r3x4097", 4097, 1), ("h1x257", 257, 0)])
def test_rmsnorm_restatement_matches_reference_golden(case, width, dtype):
    g = np.load(os.path.join(GOLDEN, "rmsnorm.npz"))
    x = g[f"{case}_x"]
    if dtype == 0:
        x = oracle.round_f16(x).reshape(x.shape)  # evaluateGraph stores fp16 inputs first
    gamma = (0.5 + (np.arange(width) % 31) / 32.0).astype(np.float32)
    if dtype == 0:
        gamma = oracle.round_f16(gamma)
    got = oracle.rmsnorm(x, gamma, 1e-5)
    assert np.array_equal(got, g[f"{case}_y"])


@pytest.mark.skipif(not oracle.reference_available(), reason="oracle/_ref not built here")
@pytest.mark.parametrize("rows,k,n,seed", [(1, 64, 40, 1), (2, 136, 97, 2), (4, 512, 33, 3)])
def test_restatement_matches_live_reference(rows, k, n, seed):
    x, gamma, w = workloads.c1_inputs(seed=seed, k=k, n=n, rows=rows)
    w = w.astype(np.float32)
    assert np.array_equal(oracle.rmsnorm_matmul(x, gamma, w), oracle.ref_rmsnorm_matmul(x, gamma, w))


def test_compare_matches_validator_semantics():
    ref = np.array([1.0, 2.0, 3.0, np.inf], dtype=np.float64)
    ok, worst, bad, first = oracle.compare(np.array([1.0, 2.0, 3.0, 1.0], np.float32), ref, 1e-5, 1e-4)
    assert not ok and bad == 1 and first == 3 and worst == np.inf
    ok, worst, bad, first = oracle.compare(np.array([1.0, 2.0002, 3.0], np.float32), ref[:3], 1e-5, 1e-4)
    assert ok and first == -1


def test_paged_attention_oracle_reduces_to_dense_softmax():
    # A contiguous cache expressed as one page per sequence must equal plain
    # softmax(q k^T / sqrt(d)) v.
    rng = np.random.default_rng(0)
    hq, hkv, d, length = 4, 2, 16, 37
    k = rng.standard_normal((1, hkv, length, d)).astype(np.float32)
    v = rng.standard_normal((1, hkv, length, d)).astype(np.float32)
    q = rng.standard_normal((1, hq, d)).astype(np.float32)
    out = oracle.paged_attention(q, k, v, np.array([[0]], np.int32), np.array([0], np.int32),
                                 np.array([length - 1], np.int32), hkv, length)
    for h in range(hq):
        s = k[0, h // 2].astype(np.float64) @ q[0, h].astype(np.float64) / np.sqrt(d)
        p = np.exp(s - s.max())
        p /= p.sum()
        np.testing.assert_allclose(out[0, h], p @ v[0, h // 2].astype(np.float64), rtol=1e-10, atol=1e-12)


@pytest.mark.parametrize("hq,hkv,page", [(32, 8, 16), (4, 4, 4), (8, 2, 5)])
def test_paged_attention_oracle_matches_the_decoder_oracle(hq, hkv, page):
    # The C restatement of the serving kernel (scattered pages, GQA head map,
    # several rows of different lengths) against the decoder oracle's attention
    # (causal_gqa_attention, pinned bit for bit to the reference exporter) on the
    # same fp16-valued data: the C path sums in fp64, the decoder oracle in fp32.
    import torch
    from oracle.decoder_ref import causal_gqa_attention
    rng = np.random.default_rng(hq * 100 + page)
    d, lengths = 32, [1, page, 3 * page + 2, 70]
    pages_per = [(n + page - 1) // page for n in lengths]
    npages = sum(pages_per) + 3
    perm = rng.permutation(npages).astype(np.int32)
    stride = max(pages_per)
    table = np.full((len(lengths), stride), -1, np.int32)
    off = 0
    for r, n in enumerate(pages_per):
        table[r, :n] = perm[off:off + n]
        off += n
    f16 = lambda *shape: rng.standard_normal(shape).astype(np.float16).astype(np.float32)
    kp, vp, q = f16(npages, hkv, page, d), f16(npages, hkv, page, d), f16(len(lengths), hq, d)
    pos = np.array(lengths, np.int32) - 1
    out = oracle.paged_attention(q, kp, vp, table, np.arange(len(lengths), dtype=np.int32), pos, hkv, page)
    for r, n in enumerate(lengths):
        ids = table[r, :pages_per[r]]
        # Gather the sequence's pages back into a contiguous [1, hkv, n, d] cache.
        k = torch.from_numpy(kp[ids].transpose(1, 0, 2, 3).reshape(hkv, -1, d)[:, :n][None].copy())
        v = torch.from_numpy(vp[ids].transpose(1, 0, 2, 3).reshape(hkv, -1, d)[:, :n][None].copy())
        ref = causal_gqa_attention(torch.from_numpy(q[r][None, :, None, :].copy()), k, v, n - 1)[0, :, 0].numpy()
        np.testing.assert_allclose(out[r], ref, rtol=2e-5, atol=2e-6)
