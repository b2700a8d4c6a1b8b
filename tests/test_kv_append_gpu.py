"""KV-cache appends bit-exact against the CPU oracle.

A cache append is a copy of the K/V projection (after RoPE for K) into the
slot the block table names (emitDecoderCacheAppend /
emitDecoderPagedCacheAppend / emitServingPagedCacheAppend,
DecoderLLMMetalEmitter.cpp:160-258,314-373). To check the copy and its
placement bit for bit, the projection values themselves are made exact: every
embedding entry is +-1 with unit norms, so the RMS-normalised input rounds to
the same +-1 in fp16 on both sides (1/sqrt(1 + 1e-5) is within half an ulp of
1), and every K/V weight row holds four entries from {+-1, +-0.5, +-0.25}, so
each projection is an exact dyadic sum. RoPE then runs the same fp32
multiply/subtract on the same tables (read back from the decoder) on both
sides. Layer 0's cache after prefill (GEMV chunks of 8 rows, or tensor-core
chunks of 32 rows) and decode steps must equal the oracle's fp16 cache exactly,
for contiguous and 16-position paged caches and several sequences.
"""

import numpy as np
import pytest
import torch

from oracle.decoder_ref import DecoderOracle, DecoderSpec, random_weights

pytestmark = pytest.mark.gpu

H, HEADS, KV, INTER, VOCAB, CAP = 256, 4, 2, 512, 48, 128
D = H // HEADS
SPEC = DecoderSpec(hidden=H, heads=HEADS, kv_heads=KV, intermediate=INTER, vocab=VOCAB, layers=2,
                   capacity=CAP, rope_theta=5e5)


def exact_weights(seed):
    rng = np.random.default_rng(seed)
    w = random_weights(SPEC, seed, std=0.05)
    w["embedding.weight"] = rng.choice(np.array([-1.0, 1.0], np.float16), size=(VOCAB, H))
    for name in ("layer0.k.weight", "layer0.v.weight"):
        m = np.zeros((KV * D, H), np.float16)
        for r in range(KV * D):
            cols = rng.choice(H, 4, replace=False)
            m[r, cols] = rng.choice(np.array([-1.0, -0.5, -0.25, 0.25, 0.5, 1.0], np.float16), 4)
        w[name] = m
    return w


@pytest.mark.parametrize("page_size,max_rows", [(0, 8), (16, 8), (16, 32)])
def test_kv_appends_are_bit_exact(rt, page_size, max_rows):
    import tmc_cuda
    w = exact_weights(41)
    slots = 3
    dec = tmc_cuda.Decoder(rt, H, HEADS, INTER, VOCAB, SPEC.layers, CAP, kv_heads=KV, rope_theta=5e5,
                           page_size=page_size, max_rows=max_rows, max_slots=slots)
    dec.load_weights(w)
    cos = torch.from_numpy(dec.read_weight("rope.cosine", CAP * D // 2).reshape(CAP, D // 2))
    sin = torch.from_numpy(dec.read_weight("rope.sine", CAP * D // 2).reshape(CAP, D // 2))
    oracle = DecoderOracle(SPEC, w, cos, sin)
    rng = np.random.default_rng(42)
    toks = []
    for s, n in enumerate((40, 17, 70)):
        prompt = rng.integers(0, VOCAB, n).astype(np.int32)
        _, t = dec.prefill(prompt, slot=s, logits=False)
        oracle.forward(s, prompt)
        toks.append(t)
    for _ in range(5):
        _, nxt = dec.decode(toks, slots=list(range(slots)))
        for s in range(slots):
            oracle.forward(s, [toks[s]])  # the same inputs as the GPU (layer 0 sees only the embedding)
        toks = [int(x) for x in nxt]
    for s in range(slots):
        k, v = dec.read_kv(0, slot=s)
        rk, rv = oracle.caches[s][0]
        assert k.shape == tuple(rk.shape)
        assert np.array_equal(k, rk.float().numpy()), f"slot {s}: key cache differs"
        assert np.array_equal(v, rv.float().numpy()), f"slot {s}: value cache differs"
        assert np.count_nonzero(k) > 0.9 * k.size  # the check is not vacuous
    dec.close()
