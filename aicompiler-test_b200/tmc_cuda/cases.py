"""Standalone kernel cases for timing and profiling one kernel in isolation.

    python -m tmc_cuda.cases gemm --rows 64 --n 28672 --k 4096 [--reps 20]
    python -m tmc_cuda.cases attention --rows 64 --ctx 1152 [--hq 32 --hkv 8 --d 128 --page 16]
    python -m tmc_cuda.cases gemv --rows 1 --n 28672 --k 4096
    python -m tmc_cuda.cases rmsnorm --rows 16384 --k 4096 [--fp16] [--threads 256]

Each case builds seeded inputs on the device (larger than L2 where the shape
allows), launches the kernel `--warmup` times, then `--reps` times between
CUDA events on the runtime's stream, and prints one JSON line with the mean
launch time and the algorithmic bytes. Run from `aicompiler-test_b200/` (or
with it on PYTHONPATH); `ncu --clock-control none --metrics gpu__time_duration.sum
-k regex:<kernel> -s <warmup> -c <n>` captures the first timed launches
(without --clock-control none ncu locks the GPU clocks, which the next user of
a shared GPU inherits); keep a full-set capture on one kernel and a few
launches of a small case.
"""

from __future__ import annotations

import argparse
import json

import numpy as np


def _timer(rt):
    import torch
    stream = torch.cuda.ExternalStream(rt.stream)
    return stream, torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def _time(rt, launch, warmup, reps):
    import torch
    for _ in range(warmup):
        launch()
    rt.synchronize()
    stream, e0, e1 = _timer(rt)
    e0.record(stream)
    for _ in range(reps):
        launch()
    e1.record(stream)
    torch.cuda.synchronize()
    rt.synchronize()
    return e0.elapsed_time(e1) * 1e3 / reps


def case_gemm(rt, a):
    import tmc_cuda
    w = rt.buffer(a.n * a.k, tmc_cuda.F16)
    tmc_cuda.fill_normal_f16(rt, w, 1, 0.0, 0.02)
    x = rt.upload(np.random.default_rng(0).standard_normal((a.rows, a.k)).astype(np.float16))
    y = rt.buffer(a.rows * a.n, tmc_cuda.F32)
    ws = rt.buffer(max(tmc_cuda.batched_gemm_workspace_bytes(a.n, a.k, a.rows) // 4, 1), tmc_cuda.F32)
    us = _time(rt, lambda: tmc_cuda.batched_gemm_f16(rt, x, w, y, a.rows, a.k, a.n, ws), a.warmup, a.reps)
    nbytes = 2 * a.n * a.k + 2 * a.rows * a.k + 4 * a.rows * a.n
    return {"kernel": "gemm_kernel (tcgen05)", "rows": a.rows, "n": a.n, "k": a.k, "us": us,
            "bytes": nbytes, "gbs": nbytes / us / 1e3, "tflops": 2 * a.rows * a.n * a.k / us / 1e6}


def case_gemv(rt, a):
    import tmc_cuda
    w = rt.buffer(a.n * a.k, tmc_cuda.F16)
    tmc_cuda.fill_normal_f16(rt, w, 1, 0.0, 0.02)
    x = rt.upload(np.random.default_rng(0).standard_normal((a.rows, a.k)).astype(np.float16))
    y = rt.buffer(a.rows * a.n, tmc_cuda.F32)
    us = _time(rt, lambda: tmc_cuda.gemv_f16(rt, x, w, y, a.rows, a.k, a.n), a.warmup, a.reps)
    nbytes = 2 * a.n * a.k + 2 * a.rows * a.k + 4 * a.rows * a.n
    return {"kernel": "gemv_kernel", "rows": a.rows, "n": a.n, "k": a.k, "us": us, "bytes": nbytes,
            "gbs": nbytes / us / 1e3}


def case_rmsnorm(rt, a):
    """RMSNormOp (emitRMSNorm) over [rows, k]: x, gamma and y all fp32 or all
    fp16 (--fp16); one CTA per row with --threads threads (0: the baseline)."""
    import tmc_cuda
    dt = tmc_cuda.F16 if a.fp16 else tmc_cuda.F32
    size = 2 if a.fp16 else 4
    x = rt.buffer(a.rows * a.k, dt)
    if a.fp16:
        tmc_cuda.fill_normal_f16(rt, x, 4, 0.0, 1.0)
    else:
        x.write(np.random.default_rng(0).standard_normal(a.rows * a.k).astype(np.float32))
    g = rt.upload(np.random.default_rng(1).uniform(0.5, 1.5, a.k).astype(np.float16 if a.fp16 else np.float32))
    y = rt.buffer(a.rows * a.k, dt)
    us = _time(rt, lambda: tmc_cuda.rmsnorm(rt, x, g, y, a.rows, a.k, 1e-5, a.threads), a.warmup, a.reps)
    nbytes = 2 * size * a.rows * a.k + size * a.k
    return {"kernel": "rmsnorm_kernel", "rows": a.rows, "width": a.k, "dtype": "f16" if a.fp16 else "f32",
            "threads": a.threads, "us": us, "bytes": nbytes, "gbs": nbytes / us / 1e3}


def case_attention(rt, a):
    import tmc_cuda
    rng = np.random.default_rng(0)
    # contexts: all a.ctx, or ~U[a.ctx, a.ctx_max] when --ctx-max is given
    ctx = np.full(a.rows, a.ctx) if a.ctx_max <= a.ctx else rng.integers(a.ctx, a.ctx_max + 1, a.rows)
    pages_per_seq = int((ctx.max() + a.page - 1) // a.page)
    pool_pages = max(a.rows * pages_per_seq + 8, a.pool_pages)
    kp = rt.buffer(pool_pages * a.hkv * a.page * a.d, tmc_cuda.F16)
    vp = rt.buffer(pool_pages * a.hkv * a.page * a.d, tmc_cuda.F16)
    tmc_cuda.fill_normal_f16(rt, kp, 2, 0.0, 1.0)
    tmc_cuda.fill_normal_f16(rt, vp, 3, 0.0, 1.0)
    perm = rng.permutation(pool_pages)[: a.rows * pages_per_seq].astype(np.int32)
    table = rt.upload(perm.reshape(a.rows, pages_per_seq))
    trows = rt.upload(np.arange(a.rows, dtype=np.int32))
    pos = rt.upload((ctx - 1).astype(np.int32))
    q = rt.upload(rng.standard_normal((a.rows, a.hq, a.d)).astype(np.float16))
    out = rt.buffer(a.rows * a.hq * a.d, tmc_cuda.F16)
    # The decoder's split policy (DecoderExecutor.cpp, attention launch).
    sms = 148
    splits = max(1, min(64, (2 * sms + a.rows * a.hkv - 1) // (a.rows * a.hkv)))
    if a.rows * a.hkv >= sms:
        splits = 1
        while splits < 16 and 2 * splits * a.rows * a.hkv <= 8 * sms:
            splits *= 2
    if a.splits > 0:
        splits = a.splits
    ws = rt.buffer(max(tmc_cuda.attention_workspace_bytes(a.rows, a.hq, a.hkv, a.d, splits) // 4, 1),
                   tmc_cuda.F32)
    counters = rt.upload(np.zeros(a.rows * a.hkv, dtype=np.int32))

    def launch():
        tmc_cuda.paged_attention_f16(rt, q, out, kp, vp, table, pages_per_seq, trows, pos, a.rows, a.hq,
                                     a.hkv, a.d, a.page, pool_pages, pages_per_seq * a.page, splits,
                                     a.min_chunk, ws, counters, a.schedule)

    us = _time(rt, launch, a.warmup, a.reps)
    nbytes = 2 * 2 * int(ctx.sum()) * a.hkv * a.d + 2 * 2 * a.rows * a.hq * a.d
    return {"kernel": "attention_kernel", "rows": a.rows, "ctx": a.ctx, "ctx_max": a.ctx_max, "hq": a.hq,
            "hkv": a.hkv, "d": a.d, "splits": splits, "min_chunk": a.min_chunk, "schedule": a.schedule,
            "us": us, "bytes": nbytes,
            "gbs": nbytes / us / 1e3}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=("gemm", "gemv", "attention", "rmsnorm"))
    ap.add_argument("--rows", type=int, default=64)
    ap.add_argument("--n", type=int, default=28672)
    ap.add_argument("--k", type=int, default=4096)
    ap.add_argument("--ctx", type=int, default=1152)
    ap.add_argument("--hq", type=int, default=32)
    ap.add_argument("--hkv", type=int, default=8)
    ap.add_argument("--d", type=int, default=128)
    ap.add_argument("--page", type=int, default=16)
    ap.add_argument("--ctx-max", type=int, default=0, help="contexts ~U[ctx, ctx_max] (attention)")
    ap.add_argument("--splits", type=int, default=0, help="attention max splits (0: the decoder's policy)")
    ap.add_argument("--min-chunk", type=int, default=64, help="attention positions per split at least")
    ap.add_argument("--pool-pages", type=int, default=0, help="attention page pool size (at least what fits)")
    ap.add_argument("--schedule", type=int, default=0,
                    help="attention schedule: 0 automatic, 1 split-K with cluster merges, 2 streaming")
    ap.add_argument("--fp16", action="store_true", help="rmsnorm: fp16 x, gamma and y (default fp32)")
    ap.add_argument("--threads", type=int, default=256, help="rmsnorm: threads per row (0: the baseline)")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--reps", type=int, default=20)
    a = ap.parse_args(argv)
    import tmc_cuda
    rt = tmc_cuda.Runtime(0)
    fn = {"gemm": case_gemm, "gemv": case_gemv, "attention": case_attention, "rmsnorm": case_rmsnorm}[a.case]
    print(json.dumps(fn(rt, a)), flush=True)
    rt.close()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
