"""BASELINE config C2 against the CPU oracle: one decoder layer, single-token
decode over a contiguous fixed-capacity KV cache.

Layer: d_model 1024, 16 heads x 64 (MHA), RMSNorm eps 1e-5, RoPE theta 1e4,
SwiGLU 2816, fp16 weights ~N(0, 0.02). Cache: capacity 2048, prefilled to 512
valid positions with K/V ~N(0, 1) (written through restoreKVCache, the
reference's past_key / past_value path of decoder_llm.py:61). Steps: 64 decode
steps whose input embeddings are ~N(0, 1).

The executor takes token ids, so the 64 step inputs are the 64 rows of the
embedding table (step t feeds token t: its embedding row IS the step's N(0, 1)
input vector), and the layer's output is read through the final RMSNorm and a
64-row LM head (~N(0, 0.02)) -- 64 projections of the hidden state per step,
compared with the oracle (oracle/decoder_ref.py) under the tolerances of
tests/parity_util.py, with the 64 appended K/V rows and the argmax.
"""

import numpy as np
import pytest
import torch

from oracle.decoder_ref import DecoderOracle, DecoderSpec, weight_names
from tests.parity_util import TokenCheck, fp16_close

pytestmark = pytest.mark.gpu

H, HEADS, INTER, CAP, PREFIX, STEPS = 1024, 16, 2816, 2048, 512, 64
D = H // HEADS
SPEC = DecoderSpec(hidden=H, heads=HEADS, kv_heads=HEADS, intermediate=INTER, vocab=STEPS, layers=1,
                   capacity=CAP, rope_theta=1e4)


def c2_decoder(rt, seed=11):
    """The C2 layer with its cache prefilled; returns (decoder, oracle)."""
    import tmc_cuda
    dec = tmc_cuda.Decoder(rt, H, HEADS, INTER, STEPS, 1, CAP, kv_heads=HEADS, rope_theta=1e4, page_size=0)
    dec.init_random(seed=seed, std=0.02)
    rng = np.random.default_rng(seed)
    inputs = rng.standard_normal((STEPS, H), dtype=np.float32).astype(np.float16)  # step inputs ~N(0, 1)
    dec.load_weight("embedding.weight", inputs)
    keys = rng.standard_normal((1, HEADS, PREFIX, D), dtype=np.float32).astype(np.float16)
    values = rng.standard_normal((1, HEADS, PREFIX, D), dtype=np.float32).astype(np.float16)
    dec.restore_kv(0, keys.astype(np.float32), values.astype(np.float32))
    sizes = {"embedding.weight": (STEPS, H), "final_norm.weight": (H,), "lm_head.weight": (STEPS, H),
             "layer0.input_norm.weight": (H,), "layer0.post_norm.weight": (H,), "layer0.q.weight": (H, H),
             "layer0.k.weight": (H, H), "layer0.v.weight": (H, H), "layer0.o.weight": (H, H),
             "layer0.gate.weight": (INTER, H), "layer0.up.weight": (INTER, H), "layer0.down.weight": (H, INTER)}
    weights = {n: dec.read_weight(n, int(np.prod(sizes[n]))).reshape(sizes[n]).astype(np.float16)
               for n in weight_names(1)}
    cos = torch.from_numpy(dec.read_weight("rope.cosine", CAP * D // 2).reshape(CAP, D // 2))
    sin = torch.from_numpy(dec.read_weight("rope.sine", CAP * D // 2).reshape(CAP, D // 2))
    oracle = DecoderOracle(SPEC, weights, cos, sin)
    oracle.caches[0] = [(torch.from_numpy(keys[0]), torch.from_numpy(values[0]))]
    return dec, oracle


def test_c2_layer_64_steps_match_oracle(rt):
    dec, oracle = c2_decoder(rt)
    assert dec.length() == PREFIX
    twin = oracle.fork(summation_order_seed=3, caches=oracle.caches)
    tokens = TokenCheck("C2 layer")
    for t in range(STEPS):
        lo, to = oracle.forward(0, [t])
        lt, _ = twin.forward(0, [t])
        lg, nxt = dec.decode([t])
        ref = lo[0].float().numpy()
        fp16_close(lg[0], ref, f"C2 step {t} (context {PREFIX + t + 1}) head logits", twin=lt[0].float().numpy())
        tokens.check(int(nxt[0]), to, ref, lg[0])
    tokens.report()
    assert dec.length() == PREFIX + STEPS
    k, v = dec.read_kv(0)
    rk, rv = oracle.caches[0][0]
    # The restored prefix is an exact copy; the 64 appended rows are projections.
    assert np.array_equal(k[:, :PREFIX], rk[:, :PREFIX].float().numpy())
    assert np.array_equal(v[:, :PREFIX], rv[:, :PREFIX].float().numpy())
    fp16_close(k[:, PREFIX:], rk[:, PREFIX:].float().numpy(), "C2 appended keys (64 positions)")
    fp16_close(v[:, PREFIX:], rv[:, PREFIX:].float().numpy(), "C2 appended values (64 positions)")
    dec.close()


def test_c2_device_loop_matches_host_loop(rt):
    # The same 64 steps through the device greedy loop (the bench's C2 timing
    # path) give the host loop's tokens.
    a, _ = c2_decoder(rt)
    b, _ = c2_decoder(rt)
    t = 0
    host = []
    for _ in range(STEPS):
        _, n = a.decode([t], logits=False)
        t = int(n[0])
        host.append(t)
    dev, gpu_us = b.generate([0], STEPS)
    assert dev[:, 0].tolist() == host and gpu_us > 0
    a.close()
    b.close()
