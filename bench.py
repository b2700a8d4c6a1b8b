#!/usr/bin/env python3
"""Decode benchmark of the B200 backend.

Workload: Llama-3-8B-shaped decoder (32 layers, hidden 4096, 32 query / 8 KV
heads x 128, SwiGLU 14336, vocab 128256, RoPE theta 5e5), fp16 random-init
weights ~N(0, 0.02), batch 1, a 1024-token random prompt (prefilled untimed),
then greedy decode. One "step" = one decode token (all 32 layers + LM head).

    python bench.py [--gpus N] [--steps K] [--warmup W]
    torchrun --nproc-per-node N bench.py --gpus N ...      (tensor parallel, NCCL)
    python bench.py --impl reference                        (CPU reference arm)

value  = K / device time of K graph replays of the greedy decode loop (CUDA
         events on the executor stream, max over ranks); weights (15 GB) exceed
         the 126 MB L2, so every step streams them from HBM.
e2e    = the same metric through the public per-step API (tmc_decoder_decode):
         each step copies its input token from pinned host memory and reads the
         next token back, wall-clock timed.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "aicompiler-test_b200"))

METRIC = "decode tok/s (8B-shape, bs1 & bs64) + GEMV/attn HBM GB/s vs peak"
CFG = dict(hidden=4096, heads=32, kv_heads=8, intermediate=14336, vocab=128256, layers=32,
           rope_theta=500000.0, epsilon=1e-5)


def parse(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256, help="timed decode steps (C3: 256, contexts 1025..1280)")
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--prompt", type=int, default=1024)
    ap.add_argument("--layers", type=int, default=CFG["layers"])
    ap.add_argument("--no-kernels", action="store_true", help="skip the per-kernel timing")
    ap.add_argument("--batch", type=int, default=64, help="rows of the batched decode measurement (bs64)")
    ap.add_argument("--batch-steps", type=int, default=32)
    ap.add_argument("--no-batch", action="store_true", help="skip the batched decode measurement")
    ap.add_argument("--no-c4", action="store_true", help="skip the C4 paged-attention measurement")
    ap.add_argument("--serving", type=int, default=48,
                    help="serve this many requests (C5: Poisson 20 req/s, prompts U[128,2048], "
                         "outputs U[64,512], max batch 128; 1000 in the full config; 0 skips)")
    ap.add_argument("--no-c1", action="store_true", help="skip the C1 RMSNorm -> GEMV measurement")
    ap.add_argument("--no-c2", action="store_true", help="skip the C2 single-layer measurement")
    ap.add_argument("--no-prefill", action="store_true", help="skip the prefill / TTFT measurement")
    ap.add_argument("--collective", choices=("p2p", "nccl"), default="p2p",
                    help="TP reductions: peer exchange fused into the kernels, or NCCL allreduce")
    return ap.parse_args(argv)


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            m = json.load(f)
        return float(m["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "100", "-f", self.path],
                stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.2)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        try:
            with open(self.path) as f:
                lines = f.readlines()
            os.unlink(self.path)
        except Exception:
            return None
        return summarize_clocks(lines)


def summarize_clocks(lines):
    """Median SM clock, the largest max clock and the throttle reasons seen
    Active in `nvidia-smi --format=csv,noheader,nounits` lines of
    ClockSampler.QUERY; None without a complete line. Unreadable values
    ("[N/A]") are skipped."""
    rows = [[p.strip() for p in line.split(",")] for line in lines]
    rows = [r for r in rows if len(r) >= 9]
    if not rows:
        return None

    def num(text):
        try:
            return float(text)
        except ValueError:
            return None

    sm = sorted(v for v in (num(r[1]) for r in rows) if v is not None)
    mx = [v for v in (num(r[2]) for r in rows) if v is not None]
    names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
    return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": max(mx) if mx else None,
            "reasons": reasons, "samples": len(rows)}


def dist_info():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def emit(obj):
    print(json.dumps(obj), flush=True)


def headline_config(args, world):
    """The headline workload; both arms print this same `config`."""
    return {"workload": "C3 Llama-3-8B-shaped greedy decode, batch 1, prompt 1024",
            "layers": args.layers, "hidden": CFG["hidden"], "heads": CFG["heads"],
            "kv_heads": CFG["kv_heads"], "intermediate": CFG["intermediate"],
            "vocab": CFG["vocab"], "batch": 1, "prompt": args.prompt,
            "parallelism": f"tp{world}",
            "tp_reduction": (args.collective if world > 1 else None),
            "l2": "inputs larger than L2: 15 GB of weights streamed per step"}


def run_reference(args, world, rank):
    """CPU reference arm: the reference's PyTorch decoder algorithm on the host."""
    if rank != 0:
        return 0
    import torch

    from oracle import cpu_baseline
    torch.set_num_threads(os.cpu_count() or 1)
    # Each step = one decode step of one 8B-shaped layer; per-token time is
    # extrapolated to 32 layers + LM head (see oracle/cpu_baseline.py).
    r = cpu_baseline.decode_tokens_per_second(steps=max(1, args.steps), context=args.prompt, head_calls=2)
    value = r["tokens_per_s"]
    emit({"metric": METRIC, "impl": "reference", "value": value, "unit": "tok/s", "n_gpus": args.gpus,
          "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 / value, "higher_is_better": True,
          "scaling": "strong", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
          "config": headline_config(args, world),
          "cpu_baseline": {"value": value, "unit": "tok/s", "cores": r["threads"], "kind": "port",
                           "sample": r["sample"]},
          "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})
    return 0


def run_ours(args, world, rank, local):
    import numpy as np
    import torch

    import tmc_cuda

    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device("cuda", local))

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        if dist is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    rt = tmc_cuda.Runtime(local)
    W, K = max(3, args.warmup), args.steps
    E = K
    SAMPLES, SAMPLE_STEPS = 31, 8
    capacity = ((args.prompt + W + K + E + SAMPLES * SAMPLE_STEPS + 32 + 15) // 16) * 16
    dec = tmc_cuda.Decoder(rt, CFG["hidden"], CFG["heads"], CFG["intermediate"], CFG["vocab"], args.layers,
                           capacity, kv_heads=CFG["kv_heads"], epsilon=CFG["epsilon"],
                           rope_theta=CFG["rope_theta"], max_rows=PREFILL_ROWS, max_slots=1, page_size=16,
                           tp_rank=rank, tp_size=world)
    if world > 1 and args.collective == "p2p":
        handles = [None] * world
        dist.all_gather_object(handles, dec.exchange_handle())
        dec.attach_peers(handles, rank)
    elif world > 1:
        uid = [tmc_cuda.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        dec.attach_nccl(uid[0], world, rank)
    dec.init_random(seed=0, std=0.02)
    prompt = np.random.default_rng(0).integers(0, CFG["vocab"], args.prompt).astype(np.int32)
    # Decode steps run the GEMVs (1 row); the prompt is prefilled in
    # PREFILL_ROWS-row chunks on the tcgen05 GEMMs.
    _, tok = dec.prefill(prompt, logits=False)

    # warm-up (also builds the step graph)
    out, _ = dec.generate([tok], W)
    tok = int(out[-1, 0])

    clocks = ClockSampler(local) if rank == 0 else None
    if clocks:
        clocks.start()
    barrier()
    out, gpu_us = dec.generate([tok], K)
    barrier()
    clk = clocks.stop() if clocks else None
    gpu_us = max_over_ranks(gpu_us)
    tok = int(out[-1, 0])
    value = K / (gpu_us * 1e-6)
    launches = dec.kernels_per_step(1) * K

    # Per-sample statistics as the reference's Benchmark reports them
    # (median / p90 over >= 31 samples): 31 device loops of 8 steps each.
    per_step = []
    for _ in range(SAMPLES):
        o, us = dec.generate([tok], SAMPLE_STEPS)
        tok = int(o[-1, 0])
        per_step.append(us / SAMPLE_STEPS / 1e3)
    samples = {"n": SAMPLES, "steps_each": SAMPLE_STEPS,
               "ms_per_step_median": max_over_ranks(float(np.median(per_step))),
               "ms_per_step_p90": max_over_ranks(float(np.percentile(per_step, 90))),
               "ms_per_step_min": max_over_ranks(float(np.min(per_step)))}

    # e2e through the per-step public API with host buffers
    barrier()
    t0 = time.perf_counter()
    for _ in range(E):
        _, n = dec.decode([tok], logits=False)
        tok = int(n[0])
    barrier()
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    e2e = {"value": E / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": 3 * PREFILL_ROWS * 4, "d2h_bytes_per_step": 4,
           "api": "tmc_decoder_decode (token in from pinned host memory, next token out)"}

    # Bytes of the mean timed step: the KV read grows with the context, which
    # runs from prompt + W + 1 to prompt + W + K over the timed steps.
    step_bytes = dec.step_bytes([args.prompt + W + (K + 1) // 2])
    hbm, peak_kind = measured_peaks()
    kernels = {}
    roofline = None
    if not args.no_kernels:
        for kind in ("qkv", "attention", "o_proj", "gate_up", "down", "lm_head"):
            if world > 1 and kind in ("o_proj", "down"):
                continue
            us, b, n = dec.profile_kernel(kind, rows=1, rounds=4)
            kernels[kind] = {"us": round(us, 3), "bytes": int(b), "launches_per_step": n,
                             "gbs": round(b / us / 1e3, 1), "frac_of_peak": round(b / us / 1e3 / hbm, 3)}
        dom = max(kernels, key=lambda k: kernels[k]["us"] * kernels[k]["launches_per_step"])
        d = kernels[dom]
        # DRAM bytes of one launch of the dominant kernel from a committed ncu
        # summary under profiles/ (a "traffic_bytes_per_launch <kind>: N" line).
        traffic = None
        if world == 1:
            import glob
            for tpath in sorted(glob.glob(os.path.join(ROOT, "profiles", "*.md"))):
                for line in open(tpath):
                    if line.startswith(f"traffic_bytes_per_launch {dom}:"):
                        traffic = int(line.split(":")[1])
        roofline = {"kernel": f"gemv {dom}" if dom != "attention" else "attention", "bound": "hbm",
                    "achieved": d["gbs"], "peak": hbm, "unit": "GB/s", "frac": d["frac_of_peak"],
                    "traffic": traffic, "peak_source": f"{peak_kind} hbm_gbs (MEASURED_PEAKS.json)",
                    "bytes_per_launch": d["bytes"], "launch_us": d["us"]}

    def guarded(name, fn):
        # The secondary measurements must not take the headline line with them:
        # a failure is reported in the line as that measurement's "error".
        try:
            return fn()
        except Exception as exc:  # noqa: BLE001
            print(f"[bench] {name} failed on rank {rank}: {exc}", file=sys.stderr, flush=True)
            return {"error": f"{type(exc).__name__}: {exc}"[:400]}

    prefill = None
    if not args.no_prefill:
        prefill = guarded("prefill", lambda: measure_prefill(dec, prompt, args, world, barrier, max_over_ranks))

    batched = None
    if not args.no_batch:
        dec.close()  # release the bs1 model before building the batched one
        batched = guarded("bs64", lambda: measure_batched(args, world, rank, local, dist, barrier, max_over_ranks,
                                                           hbm, peak_kind))

    c4 = None
    if not args.no_c4:
        c4 = guarded("c4", lambda: measure_c4(args, world, rank, local, barrier, max_over_ranks, hbm, peak_kind))

    c1 = None
    if not args.no_c1:
        c1 = guarded("c1", lambda: measure_c1(args, world, rank, local, barrier, max_over_ranks, hbm, peak_kind))

    c2 = None
    if not args.no_c2:
        c2 = guarded("c2", lambda: measure_c2(args, world, rank, local, barrier, max_over_ranks, hbm, peak_kind))

    serving = None
    if args.serving > 0:
        tick_s = batched.get("ms_per_step", 10.0) * 1e-3 if batched else 0.01
        serving = guarded("serving", lambda: measure_serving(args, world, rank, local, dist, barrier, hbm, tick_s))

    cpu = None
    if rank == 0 and world == 1:
        from oracle import cpu_baseline
        r = cpu_baseline.decode_tokens_per_second(steps=6, context=args.prompt, head_calls=2)
        cpu = {"value": r["tokens_per_s"], "unit": "tok/s", "cores": r["threads"], "kind": "port",
               "sample": r["sample"]}
        if isinstance(serving, dict) and "error" not in serving:
            # The port decodes one request's token at a time (no batching on
            # the host), so its serving throughput is its decode rate.
            serving["cpu_baseline"] = {"value": r["tokens_per_s"], "unit": "output tok/s", "cores": r["threads"],
                                       "kind": "port",
                                       "sample": r["sample"] + "; requests decoded one token at a time"}

    if rank == 0:
        step_ms = gpu_us / K / 1e3
        emit({
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": step_ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f16", "data": "synthetic (random-init N(0,0.02) fp16 weights, random prompt ids)",
            "config": headline_config(args, world),
            # Whole-job bytes: every rank streams its own shard (step_bytes is one rank's).
            "step_roofline": {"bytes_per_step": step_bytes * world,
                              "bytes_per_step_per_rank": step_bytes,
                              "achieved_gbs": step_bytes * world / (step_ms * 1e-3) / 1e9,
                              "aggregate_peak_gbs": hbm * world,
                              "frac": step_bytes / (step_ms * 1e-3) / 1e9 / hbm},
            "e2e": e2e,
            "samples": samples,
            "timed_contexts": [args.prompt + W + 1, args.prompt + W + K],
            "gpu_launches": launches,
            "roofline": roofline,
            "kernels": kernels,
            "prefill": prefill,
            "bs64": batched,
            "c1": c1,
            "c2": c2,
            "c4": c4,
            "serving": serving,
            "cpu_baseline": cpu,
            "clocks": clk,
        })
    if dist is not None:
        dist.barrier()
        dec.close()
        dist.destroy_process_group()
    return 0


PREFILL_ROWS = 256  # prompt rows per prefill chunk (tcgen05 GEMM token columns)


def prefill_flops(n, layers=None):
    """Algorithmic FLOPs of prefilling an n-token prompt and producing its
    first token: every linear layer for all n rows (2 flops per weight per
    row), causal attention (QK^T and PV over positions 0..t for row t), and
    the LM head for the last row only."""
    L = CFG["layers"] if layers is None else layers
    H, I, V = CFG["hidden"], CFG["intermediate"], CFG["vocab"]
    D = H // CFG["heads"]
    qkv = H * (CFG["heads"] + 2 * CFG["kv_heads"]) * D
    per_row = 2 * L * (qkv + H * H + 3 * I * H)
    attn = L * CFG["heads"] * 4 * D * (n * (n + 1) // 2)
    return per_row * n + attn + 2 * V * H


def measure_prefill(dec, prompt, args, world, barrier, max_over_ranks):
    """TTFT of the headline model: the 1024-token prompt prefilled into an
    empty slot in PREFILL_ROWS-row chunks on the tcgen05 GEMMs (chunks queued
    back to back), through tmc_decoder_prefill with the prompt in host memory
    and the first token read back. 1 untimed + 7 timed prefills; medians.
    value = prompt tokens / device time; the roofline is tensor-bound
    (prefill_flops over the measured sustained bf16 dense peak; fp16 and bf16
    run at the same tensor rate)."""
    import numpy as np
    reps = 7
    gpu, wall = [], []
    for i in range(reps + 1):
        dec.release(0)
        barrier()
        t0 = time.perf_counter()
        dec.prefill(prompt, logits=False)
        barrier()
        w = max_over_ranks(time.perf_counter() - t0)
        g = max_over_ranks(dec.prefill_timing()[0])
        if i:
            gpu.append(g)
            wall.append(w)
    gpu_us = float(np.median(gpu))
    wall_s = float(np.median(wall))
    flops = prefill_flops(len(prompt), args.layers)
    tflops = flops / (gpu_us * 1e-6) / 1e12
    peak = measured_tensor_peak()
    return {"metric": "prefill tok/s (TTFT of a 1024-token prompt)", "value": len(prompt) / (gpu_us * 1e-6),
            "unit": "tok/s", "ttft_ms": wall_s * 1e3, "gpu_ms": gpu_us / 1e3,
            "ttft_ms_samples": [round(x * 1e3, 3) for x in wall], "chunk_rows": PREFILL_ROWS,
            "roofline": {"bound": "tensor", "achieved": tflops, "peak": peak[0] * world, "unit": "TFLOP/s",
                         "frac": tflops / (peak[0] * world), "flops": flops, "peak_source": peak[1]},
            "e2e": {"value": len(prompt) / wall_s, "unit": "tok/s", "h2d_bytes_per_step": 4 * len(prompt),
                    "d2h_bytes_per_step": 4, "api": "tmc_decoder_prefill (prompt from host memory, first token out)"},
            "config": {"workload": "C3 prefill: 1024-token random prompt, batch 1, empty cache", "reps": reps,
                       "statistic": "median"}}


def measured_tensor_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            m = json.load(f)
        return float(m["bf16_tflops_sustained"]), "measured bf16_tflops_sustained (MEASURED_PEAKS.json)"
    except Exception:
        return 1400.0, "fallback sustained bf16 dense"


def events(rt):
    """CUDA events on the runtime's own stream (torch's events see only the
    stream they are recorded on)."""
    import torch
    stream = torch.cuda.ExternalStream(rt.stream)
    return stream, torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def measure_c1(args, world, rank, local, barrier, max_over_ranks, hbm, peak_kind):
    """C1: RMSNorm -> GEMV (x fp32 [1, 4096] ~N(0,1), gamma fp32 ~U(0.5,1.5),
    W fp16 [4096, 4096] ~N(0,0.02), y fp32), through the prepared-execution
    surface: 10 executions over 10 independent weight copies (335 MB, more
    than twice the 126 MB L2, so every call streams its weights from HBM),
    captured as one sequence (CUDA graph) and replayed between CUDA events.
    value = algorithmic bytes per call (W + x + gamma + y = 33,603,584 B) /
    device time per call; every rank measures its own copies (the graph path
    is single-GPU: replicas only). cpu_baseline: the reference's own
    evaluateGraph on one host core (oracle/_ref)."""
    import numpy as np

    import tmc_cuda
    from oracle import workloads  # seeded inputs only (the C1 distributions)
    copies, reps = 10, 20
    x, gamma, w = workloads.c1_inputs(seed=0)
    rt = tmc_cuda.Runtime(local)
    eps = tmc_cuda.float_bits(1e-5)
    keep, steps = [], []
    for c in range(copies):
        wb = rt.buffer(4096 * 4096, tmc_cuda.F16)
        tmc_cuda.fill_normal_f16(rt, wb, 100 + c, 0.0, 0.02)
        xb, gb, yb = rt.upload(x), rt.upload(gamma), rt.buffer(4096, tmc_cuda.F32)
        keep += [wb, xb, gb, yb]
        steps.append(tmc_cuda.Prepared(rt, "rmsnorm_gemv_f32", [xb, gb, wb], [yb], [1, 4096, 4096, eps]))
    seq = tmc_cuda.Sequence(rt, steps)
    seq.launch(3)
    rt.synchronize()
    stream, e0, e1 = events(rt)
    barrier()
    e0.record(stream)
    seq.launch(reps)
    e1.record(stream)
    rt.synchronize()
    us = max_over_ranks(e0.elapsed_time(e1) * 1e3 / (reps * copies))
    nbytes = 33_603_584
    single_us = steps[0].execute()[0]  # one call submitted alone (launch latency included)
    seq.close()
    for p in steps:
        p.close()
    rt.close()
    cpu = None
    if rank == 0 and world == 1:
        try:
            from oracle import cpu_baseline
            r = cpu_baseline.c1_gbs(calls=3)
            cpu = {"value": r["gbs"], "unit": "GB/s", "cores": r["cores"], "kind": r["kind"], "sample": r["sample"],
                   "us_per_call": r["us_per_call"]}
        except Exception as e:  # the GPU measurement above stands without it
            cpu = {"error": f"{type(e).__name__}: {e}"}
    achieved = nbytes / us / 1e3
    return {"metric": "RMSNorm -> GEMV HBM GB/s", "value": achieved * world, "unit": "GB/s",
            "us_per_call": us, "us_single_call_submitted_alone": single_us, "bytes_per_call": nbytes,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                         "frac": achieved / hbm, "peak_source": f"{peak_kind} hbm_gbs (MEASURED_PEAKS.json)"},
            "cpu_baseline": cpu,
            "config": {"workload": "C1 RMSNorm -> GEMV 4096 x 4096 (x fp32, W fp16, y fp32), seed 0 inputs",
                       "api": "tmc_prepare + tmc_sequence_launch (kernel rmsnorm_gemv_f32)",
                       "l2": f"{copies} weight copies = {copies * 33.55:.0f} MB > 2 x L2, rotated",
                       "parallelism": f"replicas x{world}"}}


def measure_c2(args, world, rank, local, barrier, max_over_ranks, hbm, peak_kind):
    """C2: one decoder layer (d 1024, 16 x 64 MHA, SwiGLU 2816, fp16 weights
    ~N(0,0.02), RoPE theta 1e4), a contiguous cache of capacity 2048 with 512
    N(0,1) positions restored, 64 single-token decode steps (the device greedy
    loop; step inputs are rows of a 64-row N(0,1) embedding table and the layer
    output is read through a 64-row head). The layer's 25.7 MB of weights fit
    in L2, so two numbers: warm = the one-layer decoder's 64 steps; cold = 16
    independently initialised copies of the layer chained in one step (411 MB
    of weights per step, more than twice L2), value = its per-layer GB/s.
    Algorithmic bytes per layer-step: weights + norms + K/V read of the
    context + K/V append (the 64-row head's 128 KB counted in the step)."""
    import numpy as np

    import tmc_cuda
    H, HEADS, INTER, CAP, PREFIX, STEPS = 1024, 16, 2816, 2048, 512, 64
    D = H // HEADS
    rng = np.random.default_rng(11)
    inputs = rng.standard_normal((STEPS, H), dtype=np.float32).astype(np.float16)
    prefix_k = rng.standard_normal((1, HEADS, PREFIX, D), dtype=np.float32)
    prefix_v = rng.standard_normal((1, HEADS, PREFIX, D), dtype=np.float32)
    rt = tmc_cuda.Runtime(local)
    out = {}
    for name, layers in (("warm", 1), ("cold", 16)):
        dec = tmc_cuda.Decoder(rt, H, HEADS, INTER, STEPS, layers, CAP, kv_heads=HEADS, rope_theta=1e4, page_size=0)
        dec.init_random(seed=11, std=0.02)
        dec.load_weight("embedding.weight", inputs)
        dec.restore_kv(0, np.repeat(prefix_k, layers, axis=0), np.repeat(prefix_v, layers, axis=0))
        dec.generate([0], 4)  # warm-up (builds the step graph); context 516
        dec.rollback(0, PREFIX)
        barrier()
        _, gpu_us = dec.generate([0], STEPS)
        gpu_us = max_over_ranks(gpu_us)
        ctx = [PREFIX + STEPS // 2]
        step_bytes = dec.step_bytes(ctx)
        per_layer = (step_bytes - 2.0 * (STEPS * H + H)) / layers
        step_us = gpu_us / STEPS
        out[name] = {"us_per_step": step_us, "us_per_layer": step_us / layers, "layers_per_step": layers,
                     "bytes_per_step": step_bytes, "gbs": step_bytes / step_us / 1e3,
                     "frac_of_peak": step_bytes / step_us / 1e3 / hbm, "bytes_per_layer_step": per_layer}
        dec.close()
    rt.close()
    cpu = None
    if rank == 0 and world == 1:
        try:
            import torch

            from oracle import cpu_baseline
            torch.set_num_threads(os.cpu_count() or 1)
            r = cpu_baseline.c2_steps_per_second(steps=STEPS)
            cpu = {"value": r["gbs"], "unit": "GB/s", "cores": r["threads"], "kind": "port", "sample": r["sample"],
                   "steps_per_s": r["steps_per_s"]}
        except Exception as e:
            cpu = {"error": f"{type(e).__name__}: {e}"}
    cold = out["cold"]
    return {"metric": "single decoder layer decode HBM GB/s", "value": cold["gbs"] * world, "unit": "GB/s",
            "steps_per_s_one_layer_warm": 1e6 / out["warm"]["us_per_step"],
            "warm": out["warm"], "cold": cold,
            "roofline": {"bound": "hbm", "achieved": cold["gbs"], "peak": hbm, "unit": "GB/s",
                         "frac": cold["frac_of_peak"], "peak_source": f"{peak_kind} hbm_gbs (MEASURED_PEAKS.json)"},
            "cpu_baseline": cpu,
            "config": {"workload": "C2 one layer d1024 16x64 MHA FFN 2816, cache 2048 with 512 N(0,1) positions, "
                                   "64 decode steps",
                       "l2": "cold: 16 chained copies of the layer (411 MB of weights per step); warm: L2-resident",
                       "parallelism": f"replicas x{world}"}}


def c4_case(world=1, rank=0):
    """The C4 inputs every rank measures (and tests/test_attention_gpu.py
    checks against the oracle): 64 sequences with contexts ~U[128, 8192] drawn
    from a seeded generator, this rank's 32/world query and 8/world KV heads of
    dimension 128, 16-token pages, each block table a run of a random draw of
    distinct pages from a 2^17-page pool, fp16 queries ~N(0, 1); the K/V pools
    are filled on the device with the counter-based N(0, 1) generator and the
    seeds given. The launch policy (8 splits of at least 1024 positions) is the
    one timed: long splits amortise each CTA's setup and merge."""
    import numpy as np
    rows, hq, hkv, d, page = 64, 32 // world, 8 // world, 128, 16
    pool_pages = 1 << 17
    rng = np.random.default_rng(4)
    ctx = rng.integers(128, 8193, rows)
    pages_per = (ctx + page - 1) // page
    stride = int(pages_per.max())
    perm = rng.permutation(pool_pages)[: int(pages_per.sum())].astype(np.int32)
    table = np.full((rows, stride), -1, dtype=np.int32)
    off = 0
    for r in range(rows):
        table[r, : pages_per[r]] = perm[off: off + pages_per[r]]
        off += pages_per[r]
    q = rng.standard_normal((rows, hq, d)).astype(np.float16)
    return {"rows": rows, "hq": hq, "hkv": hkv, "d": d, "page": page, "pool_pages": pool_pages, "ctx": ctx,
            "table": table, "stride": stride, "q": q, "k_seed": 10 + rank, "v_seed": 20 + rank,
            "max_splits": 8, "min_chunk": 1024}


def measure_c4(args, world, rank, local, barrier, max_over_ranks, hbm, peak_kind):
    """C4: block-table GQA decode attention, 64 sequences with contexts ~U[128, 8192],
    32 q / 8 kv heads x 128 (sharded by KV head across the ranks), fp16 K/V ~N(0,1)
    in 16-token pages, each block table a random draw of distinct pages from a
    2^17-page pool (2 x 4.29 GB at TP1), one fp16 query per sequence.
    value = algorithmic bytes (4096 x sum(ctx) + q + out) / device time, max over
    ranks; K/V (> L2) are re-read from HBM by every launch."""
    import numpy as np
    import torch

    import tmc_cuda
    c = c4_case(world, rank)
    rows, hq, hkv, d, page, pool_pages = c["rows"], c["hq"], c["hkv"], c["d"], c["page"], c["pool_pages"]
    ctx, table, stride = c["ctx"], c["table"], c["stride"]
    rt = tmc_cuda.Runtime(local)
    kp = rt.buffer(pool_pages * hkv * page * d, tmc_cuda.F16)
    vp = rt.buffer(pool_pages * hkv * page * d, tmc_cuda.F16)
    tmc_cuda.fill_normal_f16(rt, kp, c["k_seed"], 0.0, 1.0)
    tmc_cuda.fill_normal_f16(rt, vp, c["v_seed"], 0.0, 1.0)
    tb, trows = rt.upload(table), rt.upload(np.arange(rows, dtype=np.int32))
    pos = rt.upload((ctx - 1).astype(np.int32))
    q = rt.upload(c["q"])
    out = rt.buffer(rows * hq * d, tmc_cuda.F16)
    max_splits, min_chunk = c["max_splits"], c["min_chunk"]
    ws = rt.buffer(tmc_cuda.attention_workspace_bytes(rows, hq, hkv, d, max_splits) // 4 + 1, tmc_cuda.F32)
    counters = rt.upload(np.zeros(rows * hkv, dtype=np.int32))

    def launch():
        tmc_cuda.paged_attention_f16(rt, q, out, kp, vp, tb, stride, trows, pos, rows, hq, hkv, d, page,
                                     pool_pages, stride * page, max_splits, min_chunk, ws, counters)

    for _ in range(3):
        launch()
    rt.synchronize()
    stream = torch.cuda.ExternalStream(rt.stream)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 20
    barrier()
    e0.record(stream)
    for _ in range(reps):
        launch()
    e1.record(stream)
    torch.cuda.synchronize()
    rt.synchronize()
    us = max_over_ranks(e0.elapsed_time(e1) * 1e3 / reps)
    nbytes = (4096 * int(ctx.sum()) + 2 * rows * 32 * d * 2) + 0.0  # whole job (all KV heads)
    rt.close()
    cpu = None
    if rank == 0 and world == 1:
        # The C restatement of the reference's serving kernel on the host cores
        # (a bounded sample of the same distribution; one thread and all threads).
        try:
            from oracle import cpu_baseline
            r = cpu_baseline.paged_attention_gbs(sequences=8)
            cpu = {"value": r["gbs_all_threads"], "unit": "GB/s", "cores": r["threads"], "kind": "port",
                   "value_1_thread": r["gbs_1_thread"], "sample": r["sample"]}
        except Exception as e:  # the GPU measurement above stands without it
            cpu = {"error": f"{type(e).__name__}: {e}"}
    return {"metric": "paged GQA attention HBM GB/s", "value": nbytes / us / 1e3, "unit": "GB/s",
            "cpu_baseline": cpu,
            "us_per_call": us, "bytes_per_call": nbytes, "sum_ctx": int(ctx.sum()),
            "frac_of_peak": nbytes / us / 1e3 / (hbm * world), "peak_gbs": hbm * world,
            "peak_source": f"{peak_kind} hbm_gbs (MEASURED_PEAKS.json)",
            "config": {"sequences": rows, "ctx": "U[128,8192]", "heads": "32q/8kv x 128", "page": page,
                       "pool_pages": pool_pages, "max_splits": max_splits, "min_chunk": min_chunk,
                       "parallelism": f"kv-head shards x{world}"}}


def measure_serving(args, world, rank, local, dist, barrier, hbm, tick_s):
    """C5: continuous batching (tmc_serving_run) of `args.serving` seeded
    requests: prompts ~U[128, 2048] random ids, outputs ~U[64, 512] greedy
    tokens, Poisson arrivals at 20 req/s mapped onto scheduler ticks of about
    one decode step (`tick_s`, measured), max batch 128, KV page pool = 80% of
    the HBM left after the weights. Reports output tok/s (decoded tokens / wall
    time of the whole run), TTFT and TPOT percentiles, and the decode steps'
    fraction of the HBM roofline (weights + KV bytes of every step / their
    device time)."""
    import numpy as np
    import torch

    import tmc_cuda
    n = args.serving
    rng = np.random.default_rng(0)
    prompts = [rng.integers(0, CFG["vocab"], int(rng.integers(128, 2049))).astype(np.int32) for _ in range(n)]
    outputs = [int(rng.integers(64, 513)) for _ in range(n)]
    arrival_s = np.cumsum(rng.exponential(1.0 / 20.0, n))
    arrivals = np.floor(arrival_s / max(tick_s, 1e-4)).astype(np.int32)
    capacity = 2048 + 512 + 16
    rt = tmc_cuda.Runtime(local)
    free, _ = torch.cuda.mem_get_info(local)
    weights = 2 * (CFG["vocab"] * CFG["hidden"] * (1 + 1.0 / world)
                   + args.layers * (CFG["hidden"] * (CFG["heads"] + 2 * CFG["kv_heads"]) * 128
                                    + CFG["hidden"] * CFG["heads"] * 128 + 3 * CFG["hidden"] * CFG["intermediate"])
                   / world)
    page_bytes = 2 * 2 * (CFG["kv_heads"] // world) * 16 * 128 * args.layers
    pool_pages = int(0.8 * (free - weights - (4 << 30)) / page_bytes)
    dec = tmc_cuda.Decoder(rt, CFG["hidden"], CFG["heads"], CFG["intermediate"], CFG["vocab"], args.layers,
                           capacity, kv_heads=CFG["kv_heads"], epsilon=CFG["epsilon"],
                           rope_theta=CFG["rope_theta"], max_rows=128, max_slots=128, page_size=16,
                           pool_pages=pool_pages, tp_rank=rank, tp_size=world)
    if world > 1 and args.collective == "p2p":
        handles = [None] * world
        dist.all_gather_object(handles, dec.exchange_handle())
        dec.attach_peers(handles, rank)
    elif world > 1:
        uid = [tmc_cuda.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        dec.attach_nccl(uid[0], world, rank)
    dec.init_random(seed=0, std=0.02)
    barrier()
    served = tmc_cuda.serve(dec, prompts, outputs, arrivals)
    barrier()
    m = served["metrics"]
    ttft = served["ttft_us"] / 1e3
    tpot = (served["finish_us"] - served["ttft_us"]) / np.maximum(1, np.array(outputs)) / 1e3
    weight_step = dec.step_bytes([])
    kv_row = 2 * 2 * (CFG["kv_heads"] // world) * 128 * args.layers
    kv_bytes = sum(kv_row * (len(p) * o + o * (o + 1) // 2) for p, o in zip(prompts, outputs))
    step_bytes = m["decode_submissions"] * weight_step + kv_bytes
    frac = step_bytes / (m["decode_gpu_us"] * 1e-6) / 1e9 / hbm if m["decode_gpu_us"] else None
    result = {"requests": n, "value": m["decoded_tokens"] / (m["total_time_us"] * 1e-6), "unit": "output tok/s",
              "ttft_ms": {"p50": float(np.percentile(ttft, 50)), "p90": float(np.percentile(ttft, 90))},
              "tpot_ms": {"p50": float(np.percentile(tpot, 50)), "p90": float(np.percentile(tpot, 90))},
              "decode_step_roofline_frac": frac, "average_active_batch": m["average_active_batch"],
              "max_active_batch": m["max_active_batch"], "preemptions": m["preemptions"],
              "decode_steps": m["decode_submissions"], "prefill_tokens": m["prefill_tokens"],
              "decoded_tokens": m["decoded_tokens"], "wall_s": m["total_time_us"] * 1e-6,
              "pool_pages": pool_pages, "tick_ms": tick_s * 1e3,
              "config": {"arrivals": "Poisson 20 req/s mapped to ticks", "prompts": "U[128,2048]",
                         "outputs": "U[64,512]", "max_batch": 128, "page_budget": "80% of free HBM",
                         "parallelism": f"tp{world}"}}
    dec.close()
    return result


def measure_batched(args, world, rank, local, dist, barrier, max_over_ranks, hbm, peak_kind):
    """bs64 of the metric: `args.batch` sequences, each prefilled with its own
    seeded 1024-token prompt (untimed), then the device greedy loop with all
    rows in every step (tensor-core projections, batched paged attention).
    value = rows x steps / device time of the steps (max over ranks)."""
    import numpy as np

    import tmc_cuda
    B, W, K = args.batch, max(3, args.warmup), args.batch_steps
    capacity = ((args.prompt + W + K + 16 + 15) // 16) * 16
    rt = tmc_cuda.Runtime(local)
    dec = tmc_cuda.Decoder(rt, CFG["hidden"], CFG["heads"], CFG["intermediate"], CFG["vocab"], args.layers,
                           capacity, kv_heads=CFG["kv_heads"], epsilon=CFG["epsilon"],
                           rope_theta=CFG["rope_theta"], max_rows=B, max_slots=B, page_size=16,
                           tp_rank=rank, tp_size=world)
    if world > 1 and args.collective == "p2p":
        handles = [None] * world
        dist.all_gather_object(handles, dec.exchange_handle())
        dec.attach_peers(handles, rank)
    elif world > 1:
        uid = [tmc_cuda.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        dec.attach_nccl(uid[0], world, rank)
    dec.init_random(seed=0, std=0.02)
    toks = []
    for s in range(B):
        prompt = np.random.default_rng(1000 + s).integers(0, CFG["vocab"], args.prompt).astype(np.int32)
        toks.append(dec.prefill(prompt, slot=s, logits=False)[1])
    slots = list(range(B))
    out, _ = dec.generate(toks, W, slots=slots)
    toks = [int(t) for t in out[-1]]
    barrier()
    out, gpu_us = dec.generate(toks, K, slots=slots)
    barrier()
    gpu_us = max_over_ranks(gpu_us)
    ctx = [args.prompt + W + K // 2] * B
    step_bytes = dec.step_bytes(ctx)
    step_ms = gpu_us / K / 1e3
    kernels = {}
    if not args.no_kernels:
        for kind in ("qkv", "attention", "o_proj", "gate_up", "down", "lm_head"):
            if world > 1 and kind in ("o_proj", "down"):
                continue
            us, b, n = dec.profile_kernel(kind, rows=B, rounds=2)
            kernels[kind] = {"us": round(us, 3), "bytes": int(b), "launches_per_step": n,
                             "gbs": round(b / us / 1e3, 1), "frac_of_peak": round(b / us / 1e3 / hbm, 3)}
    result = {"value": B * K / (gpu_us * 1e-6), "unit": "tok/s", "rows": B, "steps": K, "warmup": W,
              "ms_per_step": step_ms, "config": {"prompt": args.prompt, "sequences": B,
                                                 "parallelism": f"tp{world}"},
              "step_roofline": {"bytes_per_step": step_bytes * world, "bytes_per_step_per_rank": step_bytes,
                                "achieved_gbs": step_bytes * world / (step_ms * 1e-3) / 1e9,
                                "peak_gbs": hbm * world, "frac": step_bytes / (step_ms * 1e-3) / 1e9 / hbm,
                                "peak_source": f"{peak_kind} hbm_gbs (MEASURED_PEAKS.json)"},
              "gpu_launches": dec.kernels_per_step(B) * K, "kernels": kernels}
    barrier()
    dec.close()
    return result


def main():
    args = parse()
    world, rank, local = dist_info()
    if args.impl == "reference":
        return run_reference(args, world, rank)
    return run_ours(args, world, rank, local)


if __name__ == "__main__":
    sys.exit(main())
