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


def paged_attention_gbs(sequences: int = 12, threads: int | None = None, seed: int = 4):
    """C4 paged GQA decode attention on the host: the C restatement of the
    serving kernel (oracle_paged_attention, KVCacheMetalEmitter.cpp:312-406)
    over `sequences` seeded sequences with contexts ~U[128, 8192], 32 q / 8 kv
    heads x 128, 16-token pages drawn from a shuffled pool. Timed on one thread
    and on `threads` threads (sequences split across them; the C call releases
    the GIL). GB/s counts the same algorithmic bytes as the GPU measurement:
    fp16 K and V of every context position (4096 B per position) + q + out."""
    import os
    from concurrent.futures import ThreadPoolExecutor

    from . import oracle

    threads = threads or os.cpu_count() or 1
    rng = np.random.default_rng(seed)
    hq, hkv, d, page = 32, 8, 128, 16
    ctx = rng.integers(128, 8193, sequences)
    pages_per = (ctx + page - 1) // page
    stride = int(pages_per.max())
    npages = int(pages_per.sum())
    perm = rng.permutation(npages).astype(np.int32)
    table = np.full((sequences, stride), -1, dtype=np.int32)
    off = 0
    for r in range(sequences):
        table[r, : pages_per[r]] = perm[off: off + pages_per[r]]
        off += pages_per[r]
    kp = rng.standard_normal((npages, hkv, page, d), dtype=np.float32).astype(np.float16).astype(np.float32)
    vp = rng.standard_normal((npages, hkv, page, d), dtype=np.float32).astype(np.float16).astype(np.float32)
    q = rng.standard_normal((sequences, hq, d), dtype=np.float32).astype(np.float16).astype(np.float32)
    pos = (ctx - 1).astype(np.int32)
    nbytes = 4096.0 * float(ctx.sum()) + 2.0 * sequences * hq * d * 2

    def run(rows):
        rows = np.asarray(rows)
        return oracle.paged_attention(q[rows], kp, vp, table, rows.astype(np.int32), pos[rows], hkv, page)

    t0 = time.perf_counter()
    run(np.arange(sequences))
    one_s = time.perf_counter() - t0
    workers = min(threads, sequences)
    # One task per sequence, longest first, so the threads finish together.
    order = [[int(r)] for r in np.argsort(-ctx)]
    with ThreadPoolExecutor(max_workers=workers) as ex:
        t0 = time.perf_counter()
        list(ex.map(run, order))
        many_s = time.perf_counter() - t0
    return {
        "gbs_1_thread": nbytes / one_s / 1e9,
        "gbs_all_threads": nbytes / many_s / 1e9,
        "threads": workers,
        "sample": (f"{sequences} sequences, contexts U[128,8192] (sum {int(ctx.sum())}), 32q/8kv x 128, "
                   f"16-token pages; C restatement of the serving kernel (fp64 softmax), once on 1 thread "
                   f"and once with one task per sequence on {workers} threads"),
    }


C1_BYTES = 33_603_584  # W fp16 4096x4096 + x, gamma, y fp32 [4096]


def c1_gbs(calls: int = 3, seed: int = 0):
    """C1 RMSNorm -> GEMV on one host core through the reference's OWN
    evaluateGraph (src/validation/GraphReference.cpp:98, compiled from the
    reference sources into oracle/_ref by oracle/Makefile) when it was built,
    else the C restatement (oracle/graph_ref.c); GB/s counts the same
    algorithmic bytes as the GPU measurement."""
    from . import oracle, workloads
    x, gamma, w = workloads.c1_inputs(seed=seed)
    w32 = w.astype(np.float32)
    kind = "reference" if oracle.reference_available() else "port"
    fn = oracle.ref_rmsnorm_matmul if kind == "reference" else oracle.rmsnorm_matmul
    fn(x, gamma, w32)  # warm-up
    t0 = time.perf_counter()
    for _ in range(calls):
        fn(x, gamma, w32)
    per_call = (time.perf_counter() - t0) / calls
    return {"gbs": C1_BYTES / per_call / 1e9, "us_per_call": per_call * 1e6, "cores": 1, "kind": kind,
            "sample": (f"{calls} calls of the C1 graph (RMSNorm -> Transpose(W) -> MatMul, 4096 x 4096, seed 0) "
                       + ("through the reference's own evaluateGraph (fp64 accumulation), single-threaded"
                          if kind == "reference" else "through the C restatement of evaluateGraph, single-threaded"))}


def c2_steps_per_second(steps: int = 64, threads: int | None = None, seed: int = 11):
    """C2 on the host: the oracle port of the reference's decoder_llm.py (one
    layer, d 1024, 16 x 64 MHA, SwiGLU 2816, fp16 weights, a 512-position
    N(0,1) KV prefix, capacity 2048) for `steps` decode steps with N(0,1)
    input embeddings; reports steps/s and GB/s over the C2 algorithmic bytes
    (weights once + KV read and append per step)."""
    if threads:
        torch.set_num_threads(threads)
    spec = DecoderSpec(hidden=1024, heads=16, kv_heads=16, intermediate=2816, vocab=steps, layers=1,
                       capacity=2048, epsilon=1e-5, rope_theta=1e4)
    g = torch.Generator().manual_seed(seed)
    H, D, I = 1024, 64, 2816

    def mat(r, c, std=0.02):
        return (torch.randn(r, c, generator=g) * std).to(torch.float16).numpy()

    w = {"embedding.weight": mat(steps, H, 1.0), "final_norm.weight": np.ones(H, np.float16),
         "lm_head.weight": mat(steps, H), "layer0.input_norm.weight": np.ones(H, np.float16),
         "layer0.post_norm.weight": np.ones(H, np.float16), "layer0.q.weight": mat(H, H),
         "layer0.k.weight": mat(H, H), "layer0.v.weight": mat(H, H), "layer0.o.weight": mat(H, H),
         "layer0.gate.weight": mat(I, H), "layer0.up.weight": mat(I, H), "layer0.down.weight": mat(H, I)}
    oracle = DecoderOracle(spec, w)
    k = torch.randn(16, 512, D, generator=g).to(torch.float16)
    v = torch.randn(16, 512, D, generator=g).to(torch.float16)
    oracle.caches[0] = [(k, v)]
    t0 = time.perf_counter()
    for t in range(steps):
        oracle.forward(0, [t])
    dt = time.perf_counter() - t0
    weights = 2 * (4 * H * H + 3 * H * I + 2 * H) + 2 * steps * H
    kv = sum(2 * 2 * H * (512 + t + 1) for t in range(steps))
    return {"steps_per_s": steps / dt, "gbs": (weights * steps + kv) / dt / 1e9, "threads": torch.get_num_threads(),
            "sample": f"all {steps} C2 decode steps through the oracle port of decoder_llm.py (torch CPU)"}
