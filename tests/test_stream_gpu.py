"""The layer streaming kernel (layer_stream.cu) against the per-projection
GEMV path, bit for bit.

Single-token steps without tensor parallelism run, per layer, one attention
kernel and one streaming kernel (O, gate/up, down and the next layer's QKV, or
the LM head after the last layer) instead of five GEMV launches. Every row is
computed with the GEMV's own arithmetic (prologue sums, lane chunk order,
reductions, epilogues), so a decoder with use_stream=True must reproduce a
decoder with use_stream=False exactly: logits, greedy tokens, the device
greedy loop and every KV-cache row. Checked on the reference exporter's two
golden models (contiguous and paged caches), a grouped-query model with RoPE
base 5e5, and the full C3 width (hidden 4096, 32q/8kv x 128, SwiGLU 14336,
vocab 128256) with 2 layers. Parity of the GEMV path itself against the
oracle and the reference exporter is in test_decoder_gpu.py and
test_c3_width_gpu.py; those tests now run their single-token steps through
this kernel as well.
"""

import numpy as np
import pytest

from tests.test_decoder_gpu import load, load_golden_weights, make_decoder

pytestmark = pytest.mark.gpu


def decode_run(dec, prompt, steps):
    logits, tok = dec.prefill(prompt)
    outs, toks = [logits], [tok]
    for _ in range(steps):
        lg, n = dec.decode([toks[-1]])
        outs.append(lg)
        toks.append(int(n[0]))
    return outs, toks


@pytest.mark.parametrize("name", ["decoder_default_fp16.npz", "decoder_wide_fp16.npz"])
@pytest.mark.parametrize("page_size", [0, 4])
def test_stream_equals_gemv_path_on_golden_models(rt, name, page_size):
    g, meta = load(name)
    runs = []
    for stream in (True, False):
        dec = make_decoder(rt, meta, page_size=page_size, use_stream=stream)
        load_golden_weights(dec, g, meta)
        assert dec.kernels_per_step(1) == (1 + 2 * meta["layers"] if stream else 5 * meta["layers"] + 1)
        prompt = g["prefill.tokens"][0]
        # One token more than a multiple of max_rows (8): the last prefill
        # chunk is a single-token step as well.
        prompt = np.concatenate([prompt, prompt])[: (len(prompt) // 8) * 8 + 1]
        outs, toks = decode_run(dec, prompt, 10)
        kv = [dec.read_kv(l) for l in range(meta["layers"])]
        gen, _ = dec.generate([toks[-1]], 6)
        runs.append((outs, toks, kv, gen[:, 0].tolist()))
        dec.close()
    (oa, ta, ka, ga), (ob, tb, kb, gb) = runs
    assert ta == tb and ga == gb
    for x, y in zip(oa, ob):
        assert np.array_equal(x, y)
    for (k0, v0), (k1, v1) in zip(ka, kb):
        assert np.array_equal(k0, k1) and np.array_equal(v0, v1)


def test_stream_equals_gemv_path_gqa(rt):
    import tmc_cuda
    from oracle.decoder_ref import DecoderSpec, random_weights
    spec = DecoderSpec(hidden=1024, heads=8, kv_heads=2, intermediate=2816, vocab=1000, layers=3, capacity=96,
                       rope_theta=5e5)
    w = random_weights(spec, 17, std=0.05)
    prompt = np.random.default_rng(1).integers(0, spec.vocab, 33)
    runs = []
    for stream in (True, False):
        dec = tmc_cuda.Decoder(rt, spec.hidden, spec.heads, spec.intermediate, spec.vocab, spec.layers,
                               spec.capacity, kv_heads=2, rope_theta=5e5, page_size=16, use_stream=stream)
        dec.load_weights(w)
        outs, toks = decode_run(dec, prompt, 12)
        runs.append((outs, toks, [dec.read_kv(l) for l in range(spec.layers)]))
        dec.close()
    assert runs[0][1] == runs[1][1]
    for x, y in zip(runs[0][0], runs[1][0]):
        assert np.array_equal(x, y)
    for (k0, v0), (k1, v1) in zip(runs[0][2], runs[1][2]):
        assert np.array_equal(k0, k1) and np.array_equal(v0, v1)


def test_stream_equals_gemv_path_at_c3_width(rt):
    import tmc_cuda
    H, HEADS, KV, INTER, VOCAB, LAYERS, CAP = 4096, 32, 8, 14336, 128256, 2, 96
    prompt = np.random.default_rng(41).integers(0, VOCAB, 17).astype(np.int32)
    runs = []
    for stream in (True, False):
        dec = tmc_cuda.Decoder(rt, H, HEADS, INTER, VOCAB, LAYERS, CAP, kv_heads=KV, rope_theta=5e5, page_size=16,
                               use_stream=stream)
        dec.init_random(seed=5, std=0.02)
        outs, toks = decode_run(dec, prompt, 8)
        gen, _ = dec.generate([toks[-1]], 8)
        runs.append((outs, toks, [dec.read_kv(l) for l in range(LAYERS)], gen[:, 0].tolist()))
        dec.close()
    assert runs[0][1] == runs[1][1] and runs[0][3] == runs[1][3]
    for x, y in zip(runs[0][0], runs[1][0]):
        assert np.array_equal(x, y)
    for (k0, v0), (k1, v1) in zip(runs[0][2], runs[1][2]):
        assert np.array_equal(k0, k1) and np.array_equal(v0, v1)
