"""One tensor-parallel rank of the decoder, run as a spawned child process by
tests/test_tp_gpu.py (one process per GPU, NCCL between them).

The rank loads the unsharded golden weights (the decoder keeps its own shard:
column-parallel Q/K/V/gate/up, row-parallel O/down, vocab-parallel LM head),
replays the reference exporter's prefill and decode tokens, and returns its
local logits slice, its local KV heads and the greedy tokens it saw."""

import json
import os
import sys
import traceback

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def decode_worker(rank, world, uid, npz, page_size, generate_steps, queue, mode="nccl", port=0):
    """mode "nccl": reductions through the NCCL collective (uid = its unique
    id); mode "p2p": the fused peer exchange, IPC handles shared over a gloo
    group on 127.0.0.1:port."""
    dist = None
    try:
        sys.path.insert(0, ROOT)
        sys.path.insert(0, os.path.join(ROOT, "aicompiler-test_b200"))
        import tmc_cuda
        from oracle.decoder_ref import weight_names

        g = np.load(os.path.join(HERE, "golden", npz))
        meta = json.loads(str(g["meta"]))
        rt = tmc_cuda.Runtime(rank)
        dec = tmc_cuda.Decoder(rt, meta["hidden_size"], meta["heads"], meta["intermediate_size"],
                               meta["vocabulary_size"], meta["layers"], meta["capacity"],
                               epsilon=meta["epsilon"], page_size=page_size, max_rows=8,
                               tp_rank=rank, tp_size=world)
        if mode == "p2p":
            import torch.distributed as dist
            dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                    world_size=world)
            handles = [None] * world
            dist.all_gather_object(handles, dec.exchange_handle())
            dec.attach_peers(handles, rank)
        else:
            dec.attach_nccl(uid, world, rank)
        for n in weight_names(meta["layers"]):
            dec.load_weight(n, g[n])
        dec.load_weight("rope.cosine", g["rope.cosine"])
        dec.load_weight("rope.sine", g["rope.sine"])
        out = {"rank": rank, "local_vocab": dec.local_vocab, "local_kv_heads": dec.local_kv_heads}
        logits, nxt = dec.prefill(g["prefill.tokens"][0])
        out["prefill.logits"] = logits
        out["prefill.next"] = int(nxt)
        for step in range(meta["decode_count"]):
            lg, n = dec.decode(g[f"decode{step}.tokens"][0])
            out[f"decode{step}.logits"] = lg[0]
            out[f"decode{step}.next"] = int(n[0])
        out["kv"] = [dec.read_kv(layer) for layer in range(meta["layers"])]
        toks, _ = dec.generate([out[f"decode{meta['decode_count'] - 1}.next"]], generate_steps)
        out["generate"] = toks[:, 0].tolist()
        rt.synchronize()
        if dist is not None:
            dist.barrier()  # no rank unmaps its window while a peer may still write into it
        dec.close()  # step graphs (which hold NCCL calls) go before the communicator
        rt.close()
        queue.put(out)
    except Exception:
        queue.put({"rank": rank, "error": traceback.format_exc()})
    finally:
        if dist is not None and dist.is_initialized():
            dist.destroy_process_group()


def batched_worker(rank, world, uid, queue, mode="nccl", port=0, rows=12, steps=3):
    """Batched tensor-parallel decode of a seeded random model: `rows`
    sequences prefilled (chunks of up to 16 rows) and `steps` batched decode
    steps through the tensor-core projections; returns the rank's logits slices
    and the greedy tokens. world == 1 is the single-GPU reference."""
    dist = None
    try:
        sys.path.insert(0, ROOT)
        sys.path.insert(0, os.path.join(ROOT, "aicompiler-test_b200"))
        import tmc_cuda

        rt = tmc_cuda.Runtime(rank)
        dec = tmc_cuda.Decoder(rt, 1024, 16, 2816, 8000, 2, 256, kv_heads=4, page_size=16, max_rows=16,
                               max_slots=16, tp_rank=rank, tp_size=world)
        if world > 1 and mode == "p2p":
            import torch.distributed as dist
            dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                    world_size=world)
            handles = [None] * world
            dist.all_gather_object(handles, dec.exchange_handle())
            dec.attach_peers(handles, rank)
        elif world > 1:
            dec.attach_nccl(uid, world, rank)
        dec.init_random(seed=3, std=0.05)
        rng = np.random.default_rng(7)
        toks = []
        for s in range(rows):
            prompt = rng.integers(0, 8000, 20 + 3 * s).astype(np.int32)
            toks.append(dec.prefill(prompt, slot=s, logits=False)[1])
        out = {"rank": rank, "local_vocab": dec.local_vocab, "logits": [], "tokens": []}
        slots = list(range(rows))
        for _ in range(steps):
            lg, nxt = dec.decode(toks, slots=slots)
            out["logits"].append(np.asarray(lg))
            toks = [int(t) for t in nxt]
            out["tokens"].append(toks)
        rt.synchronize()
        if dist is not None:
            dist.barrier()
        dec.close()
        rt.close()
        queue.put(out)
    except Exception:
        queue.put({"rank": rank, "error": traceback.format_exc()})
    finally:
        if dist is not None and dist.is_initialized():
            dist.destroy_process_group()


GQA = dict(hidden=4096, heads=32, kv_heads=8, intermediate=1024, vocab=4096, layers=2, capacity=128,
           rope_theta=5e5, seed=9, std=0.02)


def gqa_decoder(tmc_cuda, rt, rank=0, world=1, page_size=16):
    g = GQA
    dec = tmc_cuda.Decoder(rt, g["hidden"], g["heads"], g["intermediate"], g["vocab"], g["layers"],
                           g["capacity"], kv_heads=g["kv_heads"], rope_theta=g["rope_theta"],
                           page_size=page_size, max_rows=8, tp_rank=rank, tp_size=world)
    return dec


def gqa_worker(rank, world, uid, queue, mode, port, prompt, feed):
    """One rank of a grouped-query model at the C3 head shape (32 query / 8 KV
    heads x 128, so one KV head per rank at world 8), seeded random weights:
    prefill `prompt`, then one decode step per token of `feed` (the oracle's
    greedy tokens: teacher-forced); returns the rank's logits slices, its greedy
    tokens and its KV heads."""
    dist = None
    try:
        sys.path.insert(0, ROOT)
        sys.path.insert(0, os.path.join(ROOT, "aicompiler-test_b200"))
        import tmc_cuda

        rt = tmc_cuda.Runtime(rank)
        dec = gqa_decoder(tmc_cuda, rt, rank, world)
        if world > 1 and mode == "p2p":
            import torch.distributed as dist
            dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                    world_size=world)
            handles = [None] * world
            dist.all_gather_object(handles, dec.exchange_handle())
            dec.attach_peers(handles, rank)
        elif world > 1:
            dec.attach_nccl(uid, world, rank)
        dec.init_random(seed=GQA["seed"], std=GQA["std"])
        out = {"rank": rank, "local_vocab": dec.local_vocab, "local_kv_heads": dec.local_kv_heads,
               "logits": [], "tokens": []}
        lg, t = dec.prefill(np.asarray(prompt, np.int32))
        out["logits"].append(lg)
        out["tokens"].append(int(t))
        for tok in feed:
            lg, n = dec.decode([int(tok)])
            out["logits"].append(lg)
            out["tokens"].append(int(n[0]))
        out["kv"] = [dec.read_kv(layer) for layer in range(GQA["layers"])]
        rt.synchronize()
        if dist is not None:
            dist.barrier()
        dec.close()
        rt.close()
        queue.put(out)
    except Exception:
        queue.put({"rank": rank, "error": traceback.format_exc()})
    finally:
        if dist is not None and dist.is_initialized():
            dist.destroy_process_group()
