"""Pin the decoder oracle (oracle/decoder_ref.py) to the reference's own PyTorch
model: the golden vectors were recorded by the reference exporter
(tools/export_decoder_llm.py, tests/golden/gen_decoder_golden.py). With
kv_heads == heads and theta = 1e4 the restatement must reproduce every recorded
logit, token and KV cache bit for bit. CPU only."""

import json
import os

import numpy as np
import pytest
import torch

from oracle.decoder_ref import DecoderOracle, DecoderSpec, random_weights, rope_tables, spec_from_golden

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def load(name):
    g = np.load(os.path.join(GOLDEN, name))
    meta = json.loads(str(g["meta"]))
    return g, meta


def golden_weights(g, meta):
    from oracle.decoder_ref import weight_names
    return {n: g[n].astype(np.float32) for n in weight_names(meta["layers"])}


@pytest.mark.parametrize("name", ["decoder_default_fp16.npz", "decoder_wide_fp16.npz"])
def test_oracle_reproduces_reference_exporter_bit_exactly(name):
    g, meta = load(name)
    spec = spec_from_golden(meta)
    cos, sin = torch.from_numpy(g["rope.cosine"]), torch.from_numpy(g["rope.sine"])
    # The exporter's tables equal the oracle's own construction (decoder_llm.py:48-55).
    c2, s2 = rope_tables(spec.capacity, spec.head_dim, 10000.0)
    assert torch.equal(cos, c2) and torch.equal(sin, s2)
    oracle = DecoderOracle(spec, golden_weights(g, meta), cos, sin)
    tokens = g["prefill.tokens"][0]
    logits, nxt = oracle.forward(0, tokens)
    assert np.array_equal(logits.float().numpy(), g["prefill.logits"][0].astype(np.float32))
    assert nxt == int(g["prefill.next_tokens"][0])
    for layer in range(meta["layers"]):
        k, v = oracle.caches[0][layer]
        assert np.array_equal(k.float().numpy(), g[f"prefill.layer{layer}.key_cache"][0].astype(np.float32))
        assert np.array_equal(v.float().numpy(), g[f"prefill.layer{layer}.value_cache"][0].astype(np.float32))
    for step in range(meta["decode_count"]):
        cur = g[f"decode{step}.tokens"][0]
        assert int(cur[0]) == nxt
        logits, nxt = oracle.forward(0, cur)
        assert np.array_equal(logits.float().numpy(), g[f"decode{step}.logits"][0].astype(np.float32))
        assert nxt == int(g[f"decode{step}.next_tokens"][0])
    last = meta["decode_count"] - 1
    for layer in range(meta["layers"]):
        k, v = oracle.caches[0][layer]
        assert np.array_equal(k.float().numpy(), g[f"decode{last}.layer{layer}.key_cache"][0].astype(np.float32))
        assert np.array_equal(v.float().numpy(), g[f"decode{last}.layer{layer}.value_cache"][0].astype(np.float32))


def test_gqa_extension_with_replicated_kv_heads_equals_mha():
    # A GQA model whose KV heads are copies of each other's groups equals the MHA
    # model with repeated K/V projections: checks the head map h -> h // group.
    spec_g = DecoderSpec(hidden=64, heads=4, kv_heads=2, intermediate=96, vocab=50, layers=1, capacity=16)
    w = random_weights(spec_g, 3)
    spec_m = DecoderSpec(hidden=64, heads=4, kv_heads=4, intermediate=96, vocab=50, layers=1, capacity=16)
    wm = dict(w)
    D = 16
    for kind in ("k", "v"):
        kv = w[f"layer0.{kind}.weight"].reshape(2, D, 64)
        wm[f"layer0.{kind}.weight"] = np.repeat(kv, 2, axis=0).reshape(4 * D, 64)
    a = DecoderOracle(spec_g, w)
    b = DecoderOracle(spec_m, wm)
    la, ta = a.forward(0, [1, 2, 3, 4, 5])
    lb, tb = b.forward(0, [1, 2, 3, 4, 5])
    assert torch.equal(la, lb) and ta == tb
    la, _ = a.forward(0, [ta])
    lb, _ = b.forward(0, [tb])
    assert torch.equal(la, lb)


def test_incremental_decode_equals_one_shot_prefill():
    spec = DecoderSpec(hidden=64, heads=4, kv_heads=1, intermediate=64, vocab=40, layers=2, capacity=12,
                       rope_theta=500000.0)
    w = random_weights(spec, 9)
    a = DecoderOracle(spec, w)
    b = DecoderOracle(spec, w)
    toks = [3, 7, 1, 9, 4, 2]
    la, _ = a.forward(0, toks)
    for i, t in enumerate(toks):
        lb, _ = b.forward(0, [t])
        torch.testing.assert_close(la[i].float(), lb[0].float(), rtol=0, atol=2e-3)
