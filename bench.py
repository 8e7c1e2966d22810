#!/usr/bin/env python
"""bench.py -- BASELINE.json's metric on its batch-64 config (C2), one JSON line on rank 0.

Workload (per GPU): GPT-2 124M base2 (seeded random-init weights, converted exactly as base2_convert.py does),
64 independent streams, each a 32-id uniform-random prompt (numpy default_rng(1), the ids of rank r are rows
[64r, 64r+64) of one [64N, 32] draw), then greedy words. A STEP is one decode step: one new position for each of the
64 streams (first word from the prompt pass). C2 asks for 128 words per stream, i.e. 127 decode steps with the
key/value store growing 33 -> 160 positions; the timed loop runs those 127 steps as a cycle, rewinding the streams
to their prompt (b2_rewind, part of the timed work) after each cycle, so any --steps replays C2 exactly.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config c2|c4|c5]

--config c4 (the prompt pass, 32 x 512-id prompts, seed 3; a step = one whole prompt pass; roofline = the bank
products' int8 tensor operations against twice the measured dense bf16 rate) and --config c5 (Pythia-160M decode,
512 streams of 64-id prompts, seed 4, 128 words; a step = one decode step of all 512 streams) measure the other two
workloads the same way; the driver's default is C2.

value = 64 * N * K / (max over ranks of the CUDA-event time of the K steps). Weights (247 MB) exceed L2 (126 MB)
and are streamed every step, so no L2 flush is needed between steps. e2e = the same K steps through b2_step_host
(host buffers: the 64 words copied in and out every step). The reference arm (--impl reference) times the CPU
port of base2.py's own loop (oracle/, prefix recomputed for every word) on this box's cores.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "greedy tokens/sec/GPU at batch 64 (bit-exact vs base2.py); % HBM roofline"
UNIT = "tokens/s"
B, P, WORDS, SEED, V = 64, 32, 128, 1, 50257
CYCLE = WORDS - 1                      # decode steps in one C2 job
WEIGHT_BYTES = 247_064_064             # 48 banks + head, int16, read once per step
KV_BYTES_PER_KEY = 55_872              # per stream per attended key: 12 x (K 768x2 + V 768x4 + 12 exponents x 4)
WORKLOAD = ("C2: GPT-2 124M base2 greedy decode, 64 streams per GPU, 32-id prompts (seed 1), 128 words each "
            "(127 decode steps, key/value store 33->160 positions)")


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return float(j["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def env_rank():
    from streaming_machine_b200.shard import rank_env
    return rank_env()


# ---------------------------------------------------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------------------------------------------------
def clocks_start(local_rank):
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    idx = vis.split(",")[local_rank] if vis else str(local_rank)
    fd, path = tempfile.mkstemp(suffix=".csv")
    os.close(fd)
    q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")
    try:
        proc = subprocess.Popen(["nvidia-smi", "-i", idx, f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                 "-lms", "100"], stdout=open(path, "w"), stderr=subprocess.DEVNULL)
    except OSError:
        return None, path
    time.sleep(0.25)
    return proc, path


def clocks_stop(proc, path):
    if proc is None:
        return None
    proc.terminate()
    try:
        proc.wait(5)
    except subprocess.TimeoutExpired:
        proc.kill()
    rows = []
    with open(path) as f:
        for line in f:
            c = [x.strip() for x in line.split(",")]
            if len(c) >= 9 and c[1].isdigit():
                rows.append(c)
    os.unlink(path)
    if not rows:
        return None
    sm = [int(r[1]) for r in rows]
    mx = max(int(r[2]) for r in rows)
    names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
    loaded = [s for s in sm if s > 0.5 * mx] or sm
    return {"sm_mhz": int(statistics.median(loaded)), "sm_max_mhz": mx, "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------------------------------------------------------------
# the CPU port of base2.py's loop (reference arm and cpu_baseline)
# ---------------------------------------------------------------------------------------------------------------------
def cpu_sample(M, steps: int, warmup: int, budget_s: float):
    """Words/s of base2.py's own algorithm (oracle/, prefix recomputed for every word, streams in parallel over all
    cores) on C2 words at the job's average key count: each sampled stream extends prompt + 64 greedy words by one
    word (97 positions through the machine). Returns (value, cores, sample text, timed steps)."""
    import numpy as np

    from oracle.oracle import Oracle
    cores = os.cpu_count() or 1
    orc = Oracle(M)
    nb = min(B, cores)
    ids = np.random.default_rng(SEED).integers(0, V, (B, P))[:nb]
    prefix = np.concatenate([ids, orc.generate(ids, 64)], 1)       # untimed: the real greedy prefix
    for _ in range(max(0, warmup)):
        orc.generate_recompute(prefix[:1], 1)
    times = []
    t_all = time.perf_counter()
    for _ in range(max(1, steps)):
        t0 = time.perf_counter()
        orc.generate_recompute(prefix, 1, threads=cores)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_all > budget_s:
            break
    value = nb * len(times) / sum(times)
    sample = (f"{nb} C2 streams x 1 word per step at 96 attended keys (prompt + 64 greedy words, prefix "
              f"recomputed as base2.py:123 does), {len(times)} step(s), {cores} threads")
    return value, cores, sample, len(times)


def run_reference(args):
    rank, world, _ = env_rank()
    if rank != 0:
        return
    from streaming_machine_b200 import convert
    M = convert.load_gpt2(0)
    value, cores, sample, steps = cpu_sample(M, args.steps, min(args.warmup, 1), budget_s=150.0)
    line = {"metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": args.gpus, "steps": steps,
            "warmup": min(args.warmup, 1), "ms_per_step": round(1000 * min(B, cores) / value, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int64",
            "data": "synthetic", "impl": "reference",
            "config": {"workload": WORKLOAD, "streams_per_gpu": B, "prompt": P, "words": WORDS},
            "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------------------------------------------------
def run_ours(args):
    import numpy as np
    import torch

    rank, world, local_rank = env_rank()
    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))

    def barrier():
        if dist:
            dist.barrier(device_ids=[local_rank])

    def max_over_ranks(x: float) -> float:
        from streaming_machine_b200.shard import max_over_ranks as mor
        return mor(x, dist, device="cuda")

    from streaming_machine_b200 import convert, engine
    if rank == 0:
        M = convert.load_gpt2(0)
        barrier()
    else:
        barrier()
        M = convert.load_gpt2(0)
    eng = engine.Engine(M, device=local_rank, n_streams=B, max_ctx=P + CYCLE + 1)
    from streaming_machine_b200.shard import stream_ids
    ids = stream_ids(SEED, B, P, rank, world, V)
    lens = torch.full((B,), P, dtype=torch.int32, device="cuda")
    buf = torch.empty(B * CYCLE, dtype=torch.int32, device="cuda")

    class Cursor:
        pos = 0

    def run_steps(n, first_t, cur, host=False, host_tok=None):
        """n decode steps in C2 cycles (rewind to the prompt after 127)."""
        while n > 0:
            seg = min(n, CYCLE - cur.pos)
            if host:
                for _ in range(seg):
                    host_tok = eng.step_host(host_tok)
            else:
                eng.generate_device(B, seg, buf[:B * seg].view(B, seg))
            cur.pos += seg
            n -= seg
            if cur.pos == CYCLE:
                eng.rewind(lens, first_t)
                cur.pos = 0
                if host:
                    host_tok = first_t.cpu().numpy()
        return host_tok

    # ---- one full C2 job, untimed: the words (checked below against the reference machine) ----
    first = eng.prefill(ids)
    first_t = torch.as_tensor(first, device="cuda")
    parity = {}
    if args.quick:                           # profiling aid: prompt pass + W + K steps, one JSON line, nothing else
        cur = Cursor()
        run_steps(args.warmup, first_t, cur)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        run_steps(args.steps, first_t, cur)
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        if rank == 0:
            print(json.dumps({"quick": True, "steps": args.steps, "ms_per_step": round(1000 * dt / args.steps, 4)}))
        eng.close()
        return
    eng.generate_device(B, CYCLE, buf.view(B, CYCLE))
    words = np.concatenate([first[:, None], buf.view(B, CYCLE).cpu().numpy()], 1)
    if rank == 0:
        with open(os.path.join(ROOT, "tests", "golden", "gpt2_seed0.json")) as f:
            gold = json.load(f)["c2"]
        parity["golden_streams_equal"] = all(words[int(s), :4].tolist() == g["tokens"] for s, g in gold.items())
    eng.rewind(lens, first_t)

    # ---- pass 1: the device-timed value ----
    cur = Cursor()
    run_steps(args.warmup, first_t, cur)
    torch.cuda.synchronize()
    eng.profile(False)                       # reset the launch counter
    barrier()
    torch.cuda.synchronize()
    clk_proc, clk_path = clocks_start(local_rank)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    run_steps(args.steps, first_t, cur)
    ev1.record()
    ev1.synchronize()
    torch.cuda.synchronize()
    clocks = clocks_stop(clk_proc, clk_path)
    barrier()
    launches, _ = eng.profile_read()
    t_ms = max_over_ranks(ev0.elapsed_time(ev1))
    value = B * world * args.steps / (t_ms / 1000.0)

    # ---- pass 2: end to end through the C ABI with host buffers ----
    eng.prefill(ids)
    cur = Cursor()
    tok = run_steps(args.warmup, first_t, cur, host=True, host_tok=first.astype(np.int32))
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    run_steps(args.steps, first_t, cur, host=True, host_tok=tok)
    e1.record()
    e1.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    e2e = {"value": round(B * world * args.steps / (e2e_ms / 1000.0), 2), "unit": UNIT,
           "h2d_bytes_per_step": 4 * B, "d2h_bytes_per_step": 4 * B}

    # ---- pass 3: per-kernel-class event timing over one C2 cycle (same positions as the timed loop) ----
    eng.prefill(ids)
    eng.profile(True)
    eng.generate_device(B, CYCLE, buf.view(B, CYCLE))
    n_prof, by = eng.profile_read()
    eng.profile(False)
    bank_n, bank_ms = by["bank"]
    att_n, att_ms = by["attend"]
    peak, peak_kind = peaks()
    steps_prof = CYCLE
    bank_bytes = WEIGHT_BYTES * steps_prof
    bank_gbs = bank_bytes / (bank_ms / 1000.0) / 1e9
    keys = sum(P + 1 + t for t in range(CYCLE))                    # keys attended per stream over the cycle
    att_bytes = B * KV_BYTES_PER_KEY * keys
    att_gbs = att_bytes / (att_ms / 1000.0) / 1e9
    traffic = None       # DRAM bytes per bank launch from the committed ncu summary of the same kernel
    tp = os.path.join(ROOT, "profiles", "bank_wide_decode_c2.md")
    if os.path.exists(tp):
        import re
        mt = re.search(r"bank_dram_bytes_per_launch_avg:\s*(\d+)", open(tp).read())
        traffic = int(mt.group(1)) if mt else None
    roofline = {"bound": "hbm", "achieved": round(bank_gbs, 1), "peak": peak, "unit": "GB/s",
                "frac": round(bank_gbs / peak, 4), "traffic": traffic,
                "kernel": "bank product (49 launches per step: 48 banks + head)",
                "algorithmic_bytes_per_launch": round(WEIGHT_BYTES / 49), "avg_launch_us": round(1000 * bank_ms / bank_n, 2),
                "peak_kind": peak_kind}
    step_bytes = (WEIGHT_BYTES * steps_prof + att_bytes) / steps_prof
    line = {"metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(t_ms / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int64", "data": "synthetic",
            "config": {"workload": WORKLOAD, "streams_per_gpu": B, "prompt": P, "words": WORDS,
                       "parallelism": f"stream sharding over {world} GPU(s), no collective",
                       "l2": "no flush: 247 MB of weights streamed per step exceed the 126 MB L2"},
            "roofline": roofline,
            "roofline_attend": {"bound": "hbm", "achieved": round(att_gbs, 1), "peak": peak, "unit": "GB/s",
                                "frac": round(att_gbs / peak, 4)},
            "step_hbm_frac": round(step_bytes / (t_ms / args.steps / 1000.0) / 1e9 / peak, 4),
            "e2e": e2e, "clocks": clocks, "gpu_launches": int(launches),
            "kernel_ms_per_step": {k: round(v[1] / steps_prof, 4) for k, v in by.items()},
            "parity": parity}
    if rank == 0 and world == 1 and not args.no_cpu:
        cv, cores, sample, _ = cpu_sample(M, 2, 0, budget_s=30.0)
        line["cpu_baseline"] = {"value": round(cv, 4), "unit": UNIT, "cores": cores, "kind": "port", "sample": sample}
    eng.close()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist:
        dist.destroy_process_group()



# ---------------------------------------------------------------------------------------------------------------------
# C4: the prompt pass (int8 tensor-pipe bound) and C5: Pythia-160M decode at 512 streams
# ---------------------------------------------------------------------------------------------------------------------
C4_B, C4_P, C4_SEED = 32, 512, 3
C4_MACS_PER_ROW = 84_934_656            # int16 multiply-adds of the 48 layer banks per position
C5_B, C5_P, C5_WORDS, C5_SEED, C5_V = 512, 64, 128, 4, 50304
C5_WEIGHT_BYTES = 247_136_256


def _dist(local_rank, world):
    if world <= 1:
        return None
    import datetime

    import torch.distributed as dist
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))
    return dist


def run_c4(args):
    import numpy as np
    import torch

    rank, world, local_rank = env_rank()
    torch.cuda.set_device(local_rank)
    dist = _dist(local_rank, world)
    from streaming_machine_b200 import convert, engine
    from streaming_machine_b200.shard import max_over_ranks, stream_ids
    M = convert.load_gpt2(0)
    eng = engine.Engine(M, device=local_rank, n_streams=C4_B, max_ctx=C4_P)
    ids = stream_ids(C4_SEED, C4_B, C4_P, rank, world, V)
    ids_t = torch.as_tensor(ids.astype(np.int32).ravel(), device="cuda")
    lens_t = torch.full((C4_B,), C4_P, dtype=torch.int32, device="cuda")
    nxt = torch.empty(C4_B, dtype=torch.int32, device="cuda")

    def one():
        eng._call("b2_prefill", eng.h, ids_t.data_ptr(), lens_t.data_ptr(), C4_B, nxt.data_ptr(), None, eng._stream())

    for _ in range(max(args.warmup, 1)):
        one()
    torch.cuda.synchronize()
    eng.profile(False)
    if dist:
        dist.barrier(device_ids=[local_rank])
    clk_proc, clk_path = clocks_start(local_rank)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(args.steps):
        one()
    ev1.record()
    ev1.synchronize()
    clocks = clocks_stop(clk_proc, clk_path)
    launches, _ = eng.profile_read()
    t_ms = max_over_ranks(ev0.elapsed_time(ev1), dist, device="cuda")
    tokens = C4_B * C4_P * world * args.steps
    value = tokens / (t_ms / 1000.0)
    # end to end: host ids in, the next words back (Engine.prefill)
    e0 = time.perf_counter()
    for _ in range(args.steps):
        eng.prefill(ids)
    e2e_s = max_over_ranks(time.perf_counter() - e0, dist, device="cuda")
    # per-class event time of one pass: the bank products' share
    eng.profile(True)
    one()
    _, by = eng.profile_read()
    eng.profile(False)
    bank_ms = by["bank"][1]
    ops = C4_B * C4_P * C4_MACS_PER_ROW * 4 * 2 + C4_B * 768 * V * 4 * 2      # int8 ops: 4 per int16 MAC, x2
    with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
        pk = json.load(f)
    peak = 2.0 * float(pk["bf16_tflops"])
    achieved = ops / (bank_ms / 1000.0) / 1e12
    line = {"metric": "prompt-pass tokens/sec/GPU (C4, bit-exact vs base2.py); % int8 tensor roofline",
            "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(t_ms / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int64", "data": "synthetic",
            "config": {"workload": "C4: GPT-2 124M base2 prompt pass, 32 streams x 512 ids per GPU (seed 3)",
                       "l2": "no flush: each pass streams 2 x 247 MB of weight planes and ~1 GB of activations"},
            "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": peak, "unit": "TOPS (int8)",
                         "frac": round(achieved / peak, 4), "traffic": None,
                         "kernel": "bank products (k_bank_tiles), int8 ops per pass / their summed event time",
                         "peak_kind": "2 x measured dense bf16 (int8 tensor rate is twice bf16's)",
                         "bank_ms_per_pass": round(bank_ms, 3)},
            "e2e": {"value": round(tokens / e2e_s, 1), "unit": "tokens/s",
                    "h2d_bytes_per_step": 4 * C4_B * C4_P, "d2h_bytes_per_step": 4 * C4_B},
            "clocks": clocks, "gpu_launches": int(launches),
            "kernel_ms_per_step": {k: round(v[1], 4) for k, v in by.items()}}
    if rank == 0 and world == 1 and not args.no_cpu:
        from oracle.oracle import Oracle
        orc = Oracle(M)
        n = 96
        t0 = time.perf_counter()
        orc.scores(ids[0][:n], n - 1, n)
        dt = time.perf_counter() - t0
        line["cpu_baseline"] = {"value": round(n / dt, 3), "unit": "tokens/s", "cores": os.cpu_count() or 1,
                                "kind": "port", "sample": f"stream 0's first {n} prompt positions through the machine "
                                                          "(teacher-forced, banks split over all threads)"}
    eng.close()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist:
        dist.destroy_process_group()


def run_c5(args):
    import numpy as np
    import torch

    rank, world, local_rank = env_rank()
    torch.cuda.set_device(local_rank)
    dist = _dist(local_rank, world)
    from streaming_machine_b200 import convert, engine
    from streaming_machine_b200.shard import max_over_ranks, stream_ids
    PM = convert.load_pythia(0)
    eng = engine.Engine(PM, device=local_rank, n_streams=C5_B, max_ctx=C5_P + C5_WORDS)
    ids = stream_ids(C5_SEED, C5_B, C5_P, rank, world, C5_V)
    cycle = C5_WORDS - 1
    lens = torch.full((C5_B,), C5_P, dtype=torch.int32, device="cuda")
    buf = torch.empty(C5_B * cycle, dtype=torch.int32, device="cuda")
    first_t = torch.as_tensor(eng.prefill(ids), device="cuda")
    pos = [0]

    def steps(n):
        while n > 0:
            seg = min(n, cycle - pos[0])
            eng.generate_device(C5_B, seg, buf[:C5_B * seg].view(C5_B, seg))
            pos[0] += seg
            n -= seg
            if pos[0] == cycle:
                eng.rewind(lens, first_t)
                pos[0] = 0

    steps(args.warmup)
    torch.cuda.synchronize()
    eng.profile(False)
    if dist:
        dist.barrier(device_ids=[local_rank])
    clk_proc, clk_path = clocks_start(local_rank)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    steps(args.steps)
    ev1.record()
    ev1.synchronize()
    clocks = clocks_stop(clk_proc, clk_path)
    launches, _ = eng.profile_read()
    t_ms = max_over_ranks(ev0.elapsed_time(ev1), dist, device="cuda")
    value = C5_B * world * args.steps / (t_ms / 1000.0)
    eng.prefill(ids)
    pos[0] = 0
    eng.profile(True)
    eng.generate_device(C5_B, cycle, buf.view(C5_B, cycle))
    _, by = eng.profile_read()
    eng.profile(False)
    bank_gbs = C5_WEIGHT_BYTES * cycle / (by["bank"][1] / 1000.0) / 1e9
    peak, peak_kind = peaks()
    line = {"metric": "Pythia-160M greedy tokens/sec/GPU (C5, bit-exact vs pythia_base2.py); % HBM roofline",
            "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(t_ms / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int64", "data": "synthetic",
            "config": {"workload": "C5: Pythia-160M base2 greedy decode, 512 streams per GPU, 64-id prompts (seed 4), "
                                   "128 words (127 decode steps, store 65->192 positions)",
                       "l2": "no flush: 247 MB of weights streamed per step exceed the 126 MB L2"},
            "roofline": {"bound": "hbm", "achieved": round(bank_gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(bank_gbs / peak, 4), "traffic": None,
                         "kernel": "bank products, weight bytes per step / their summed event time",
                         "peak_kind": peak_kind},
            "clocks": clocks, "gpu_launches": int(launches),
            "kernel_ms_per_step": {k: round(v[1] / cycle, 4) for k, v in by.items()}}
    eng.close()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist:
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=40 * CYCLE)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline leg")
    ap.add_argument("--config", choices=("c2", "c4", "c5"), default="c2",
                    help="c2 (default): the metric's batch-64 decode; c4: the prompt pass; c5: Pythia-160M decode")
    ap.add_argument("--quick", action="store_true",
                    help="profiling aid: prompt pass, --warmup and --steps decode steps, no other pass")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    elif args.config == "c4":
        run_c4(args)
    elif args.config == "c5":
        run_c5(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
