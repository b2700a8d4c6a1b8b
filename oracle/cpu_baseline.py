"""CPU baseline of the decode path -- TEST / BENCHMARK INFRASTRUCTURE ONLY.

Times the reference's own algorithm (the PyTorch decoder of
workloads/pytorch/decoder_llm.py, restated in oracle/decoder_ref.py with the
GQA / rope-theta extensions) on the host cores, on a bounded sample of the
Llama-3-8B-shaped decode workload:

  sample = `steps` single-token decode steps of ONE 8B-shaped decoder layer
           (hidden 4096, 32 q / 8 kv heads x 128, SwiGLU 14336, fp16 storage)
           over a `context`-token KV cache, plus `head_calls` LM-head GEMVs
           (128256 x 4096 fp16) with the final RMSNorm and argmax;
  tokens/s = 1 / (32 x mean layer time + mean LM-head time).

The layer weights are random (values do not change the time).
"""

from __future__ import annotations

import time

import numpy as np
import torch
import torch.nn.functional as F

from .decoder_ref import DecoderOracle, DecoderSpec


def llama8b_spec(layers=32):
    return DecoderSpec(hidden=4096, heads=32, kv_heads=8, intermediate=14336, vocab=128256,
                       layers=layers, capacity=2048, epsilon=1e-5, rope_theta=500000.0)


def decode_tokens_per_second(steps: int = 6, context: int = 1024, head_calls: int = 3,
                             threads: int | None = None, seed: int = 0):
    if threads:
        torch.set_num_threads(threads)
    full = llama8b_spec()
    one = DecoderSpec(hidden=full.hidden, heads=full.heads, kv_heads=full.kv_heads,
                      intermediate=full.intermediate, vocab=8, layers=1, capacity=context + steps + 8,
                      epsilon=full.epsilon, rope_theta=full.rope_theta)
    g = torch.Generator().manual_seed(seed)
    H, D, I = one.hidden, one.head_dim, one.intermediate

    def mat(r, c):
        return (torch.randn(r, c, generator=g) * 0.02).to(torch.float16).numpy()

    w = {"embedding.weight": mat(8, H), "final_norm.weight": np.ones(H, np.float16),
         "lm_head.weight": mat(8, H), "layer0.input_norm.weight": np.ones(H, np.float16),
         "layer0.post_norm.weight": np.ones(H, np.float16), "layer0.q.weight": mat(one.heads * D, H),
         "layer0.k.weight": mat(one.kv_heads * D, H), "layer0.v.weight": mat(one.kv_heads * D, H),
         "layer0.o.weight": mat(H, one.heads * D), "layer0.gate.weight": mat(I, H),
         "layer0.up.weight": mat(I, H), "layer0.down.weight": mat(H, I)}
    oracle = DecoderOracle(one, w)
    k = (torch.randn(one.kv_heads, context, D, generator=g)).to(torch.float16)
    v = (torch.randn(one.kv_heads, context, D, generator=g)).to(torch.float16)
    oracle.caches[0] = [(k, v)]
    oracle.forward(0, [1])  # warm-up
    t0 = time.perf_counter()
    for i in range(steps):
        oracle.forward(0, [i % 8])
    layer_s = (time.perf_counter() - t0) / steps

    head = (torch.randn(full.vocab, H, generator=g) * 0.02).to(torch.float16)
    norm = torch.ones(H, dtype=torch.float16)
    x = torch.randn(1, H, generator=g).to(torch.float16)

    def head_call():
        scale = torch.rsqrt(x.float().pow(2).mean(dim=-1, keepdim=True) + full.epsilon)
        hn = (x.float() * scale * norm.float()).to(torch.float16)
        return int(F.linear(hn, head).argmax())

    head_call()
    t0 = time.perf_counter()
    for _ in range(head_calls):
        head_call()
    head_s = (time.perf_counter() - t0) / head_calls
    per_token = full.layers * layer_s + head_s
    return {
        "tokens_per_s": 1.0 / per_token,
        "layer_ms": layer_s * 1e3,
        "lm_head_ms": head_s * 1e3,
        "threads": torch.get_num_threads(),
        "sample": (f"{steps} decode steps of one Llama-3-8B-shaped layer (fp16, GQA 32/8, ctx {context}) "
                   f"+ {head_calls} LM-head GEMVs (128256x4096); per token = 32 layers + head"),
    }
