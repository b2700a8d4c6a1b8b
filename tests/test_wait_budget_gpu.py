"""Bounded waits that run out, on one GPU, without a fault or a hang.

Two tensor-parallel shards of a small model are created in this process on
the same GPU and rank 0 attaches both exchange windows
(tmc_decoder_attach_local_peers). Only rank 0 ever launches a kernel, so rank
1's exchange flags are never raised: rank 0's first wait for them is a wait on
a flag that nothing sets. With its peer budget set to 5 ms
(tmc_decoder_set_wait_budgets) every such wait gives up, the kernels record
the timeout in the runtime's device status block, drain their own copies,
free their tensor memory and return, and the call fails with
TMC_ERR_DEVICE_STATUS:

- a 16-row prefill: projections on the tcgen05 GEMM, whose LM-head launch
  waits for the peer's argmax keys while it holds tensor memory;
- a 4-row prefill: the GEMV path, whose prologues wait for the peer's
  partial sums.

Afterwards the same runtime still works: the tensor-core GEMM (which
allocates tensor memory on every SM it runs on) matches its fp64 reference,
and a single-GPU decoder on the runtime prefills and decodes.
"""

import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

H, HEADS, INTER, VOCAB, LAYERS, CAP = 256, 4, 512, 512, 2, 64
BUDGET_NS = 5_000_000


def shard(rt, rank, rows):
    import tmc_cuda
    d = tmc_cuda.Decoder(rt, H, HEADS, INTER, VOCAB, LAYERS, CAP, max_rows=rows, tp_rank=rank, tp_size=2)
    d.init_random(seed=1, std=0.02)
    return d


@pytest.mark.parametrize("rows", [16, 4])
def test_peer_flag_wait_runs_out_and_the_runtime_stays_usable(rt, rows):
    import tmc_cuda
    ranks = [shard(rt, r, rows) for r in range(2)]
    ranks[0].attach_local_peers(ranks, 0)
    ranks[0].set_wait_budgets(peer_ns=BUDGET_NS)
    prompt = np.arange(rows, dtype=np.int32) + 3
    t0 = time.perf_counter()
    with pytest.raises(tmc_cuda.TmcError) as err:
        ranks[0].prefill(prompt, logits=False)
    elapsed = time.perf_counter() - t0
    print(f"[timeout] {rows}-row prefill: {err.value.message!r} after {elapsed * 1e3:.1f} ms")
    assert err.value.code == tmc_cuda.ERR_DEVICE_STATUS
    assert "timed out" in err.value.message
    assert elapsed < 10.0  # a handful of 5 ms waits (and the 1 s defaults were not reached)
    assert ranks[0].length(0) == 0  # the failed prefill rolled back
    for d in ranks:
        d.close()

    # The runtime is usable: tensor memory was released and the status block cleared.
    rng = np.random.default_rng(5)
    m, k, n = 64, 4096, 4096
    x = rng.standard_normal((m, k)).astype(np.float16)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float16)
    xb, wb = rt.upload(x), rt.upload(w)
    yb = rt.buffer(m * n, tmc_cuda.F32)
    ws = rt.buffer(max(tmc_cuda.batched_gemm_workspace_bytes(n, k, m) // 4, 1), tmc_cuda.F32)
    tmc_cuda.batched_gemm_f16(rt, xb, wb, yb, m, k, n, ws)
    rt.synchronize()
    ref = x.astype(np.float64) @ w.astype(np.float64).T
    got = yb.read().reshape(m, n)
    assert float(np.max(np.abs(got - ref))) <= 1e-4 * float(np.sqrt(np.mean(ref ** 2)))

    single = tmc_cuda.Decoder(rt, H, HEADS, INTER, VOCAB, LAYERS, CAP, max_rows=rows)
    single.init_random(seed=1, std=0.02)
    _, tok = single.prefill(prompt, logits=False)
    _, nxt = single.decode([tok], logits=False)
    assert 0 <= tok < VOCAB and 0 <= int(nxt[0]) < VOCAB
    single.close()
