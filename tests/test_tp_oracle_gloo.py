"""The tensor-parallel decomposition on CPU: two or four `gloo` ranks each run
one shard of the golden decoder (oracle.decoder_ref.TensorParallelOracle -- the
same column/row/vocab split, fp32 partial-sum allreduce points and packed-key
argmax max-reduction as the device decoder), and the result must equal the
reference exporter's recorded outputs (export_decoder_llm.py:446-551):
greedy tokens bit for bit, logits within 2e-3 x RMS. The packed argmax key is
also checked against torch.argmax's min-index tie rule directly."""

import json
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle.decoder_ref import TensorParallelOracle, argmax_key, argmax_key_index, spec_from_golden

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, npz, out_dir):
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        g = np.load(os.path.join(GOLDEN, npz))
        meta = json.loads(str(g["meta"]))
        weights = {k: g[k] for k in g.files if k.endswith(".weight")}

        def reduce_sum(t):
            t = t.contiguous()
            dist.all_reduce(t, op=dist.ReduceOp.SUM)
            return t

        def reduce_max(t):
            t = t.contiguous()
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return t

        o = TensorParallelOracle(spec_from_golden(meta), weights,
                                 rope_cos=torch.as_tensor(g["rope.cosine"]).float(),
                                 rope_sin=torch.as_tensor(g["rope.sine"]).float(),
                                 rank=rank, world=world, all_reduce_sum=reduce_sum, all_reduce_max=reduce_max)
        res = {}
        logits, nxt = o.forward(0, g["prefill.tokens"][0])
        res["prefill.logits"] = logits.float().numpy()
        res["prefill.next"] = nxt
        for step in range(meta["decode_count"]):
            logits, nxt = o.forward(0, g[f"decode{step}.tokens"][0])
            res[f"decode{step}.logits"] = logits[-1].float().numpy()
            res[f"decode{step}.next"] = nxt
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), **{k: np.asarray(v) for k, v in res.items()})
    finally:
        dist.destroy_process_group()


def rms_close(got, ref, what):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    rms = float(np.sqrt(np.mean(ref ** 2)))
    err = float(np.max(np.abs(got - ref)))
    assert err <= 2e-3 * rms, f"{what}: max err {err} > {2e-3 * rms}"


@pytest.mark.parametrize("npz,world", [("decoder_default_fp16.npz", 2), ("decoder_wide_fp16.npz", 2),
                                       ("decoder_default_fp16.npz", 4)])
def test_gloo_ranks_match_reference_exporter(tmp_path, npz, world):
    mp.spawn(_rank, args=(world, _free_port(), npz, str(tmp_path)), nprocs=world, join=True)
    g = np.load(os.path.join(GOLDEN, npz))
    meta = json.loads(str(g["meta"]))
    ranks = [np.load(tmp_path / f"rank{r}.npz") for r in range(world)]
    rms_close(np.concatenate([r["prefill.logits"] for r in ranks], -1), g["prefill.logits"][0], "prefill")
    for r in ranks:
        assert int(r["prefill.next"]) == int(g["prefill.next_tokens"][0])
    for step in range(meta["decode_count"]):
        rms_close(np.concatenate([r[f"decode{step}.logits"] for r in ranks], -1),
                  g[f"decode{step}.logits"][0, 0], f"decode{step}")
        for r in ranks:
            assert int(r[f"decode{step}.next"]) == int(g[f"decode{step}.next_tokens"][0])


def test_packed_argmax_key_tie_rule():
    v = torch.tensor([[1.0, 3.0, -2.0, 3.0, float("-inf")], [-5.0, -1.0, -1.0, -7.0, -1.0]], dtype=torch.float16)
    for row in range(2):
        whole = argmax_key(v[row:row + 1], 0)
        # split into shards [0, 2) and [2, 5): the max of the shard keys is the whole-row key
        a = argmax_key(v[row:row + 1, :2], 0)
        b = argmax_key(v[row:row + 1, 2:], 2)
        assert int(torch.maximum(a, b)[0]) == int(whole[0])
        assert int(argmax_key_index(whole)[0]) == int(torch.argmax(v[row].float()))
