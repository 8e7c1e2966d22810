#!/usr/bin/env python
"""bench.py -- BASELINE.json's metric on its batch-64 config (C2), one JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config c1|c2|c3|c4|c5]

Decode configs (a STEP is one decode step: one new position for every stream of this rank; the first word of a
stream comes from the prompt pass):
  c2 (default) GPT-2 124M base2, 64 streams per GPU, 32-id prompts (seed 1), 128 words: 127 decode steps with the
               key/value store growing 33 -> 160 positions
  c1           GPT-2, 1 stream per GPU, 8-id prompt (seed 0), 16 words
  c3           GPT-2, 16 streams per GPU, 960-id prompts (seed 2), 64 words: the store fills 1,024 positions
  c5           Pythia-160M, 512 streams (64-id prompts, seed 4, 128 words) PARTITIONED over the N GPUs (512/N each)
Weak scaling for c1-c3 (each rank has its own streams: rows [rB, rB + B) of one [NB, P] draw, so rank 0 always holds
the single-GPU streams); strong scaling for c5 (one fixed set of 512 streams shared out).
  c4           the prompt pass of 32 x 512-id prompts (seed 3); a step = one whole pass

Timing. Each job is a cycle of words - 1 decode steps; the timed loop replays it, rewinding every stream to its prompt
(b2_rewind, inside the timed work) at the end of a cycle. K steps that are not a whole number of cycles are CENTRED on
the cycle (a window at the job's mean context), whole cycles start at its first step. value = (streams of all ranks)
x K / (max over ranks of the CUDA-event time of the K steps): the whole-job aggregate; value_per_gpu = value / N is the
metric's per-GPU figure. Weights (247 MB) exceed L2 (126 MB) and are streamed every step, so no L2 flush is needed.

A second, identical pass runs with in-kernel stamps (b2_profile mode 2: every bank / arrival / quantisation launch
stamps when its dependent work starts, inside the same CUDA graph with programmatic launches); `roofline` is the bank
product (the dominant kernel class): weight bytes per launch / average launch duration. `step_hbm_frac` is the step's
algorithmic bytes (weights + the keys and values the timed steps attend) over the timed step.

e2e = the same K steps through b2_step_host (host buffers: the words copied in and out every step). parity = the
untimed first job's words against the oracle's whole-job digests (tests/golden). The reference arm (--impl
reference) times the CPU port of base2.py's own loop (oracle/, prefix recomputed for every word) on this box's cores.
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

C2_METRIC = "greedy tokens/sec/GPU at batch 64 (bit-exact vs base2.py); % HBM roofline"
UNIT = "tokens/s"
KV_BYTES_PER_KEY = 55_872              # per stream per attended key: 12 x (K 768x2 + V 768x4 + 12 exponents x 4)
WEIGHT_BYTES = {"gpt2": 247_064_064, "pythia": 247_136_256}   # 48 banks + head, int16, read once per step
BANK_LAUNCHES = 49                     # 48 layer banks + the head per decode step
# DRAM bytes per bank launch of a decode step, (12 x (qkv + proj + fc + mproj) + head) / 49, from ncu captures of
# single launches (dram__bytes_read.sum + dram__bytes_write.sum; commands and per-bank figures in the decode-bank
# summary under profiles/). Not measured in this run; None where no capture was made (C5's 512-row path).
BANK_TRAFFIC = {"c1": 5_175_824, "c2": 6_096_274, "c3": 5_472_705}
BANK_TRAFFIC_SOURCE = "ncu: dram__bytes_read.sum + dram__bytes_write.sum of single bank launches (profiles/)"
VOCAB = {"gpt2": 50257, "pythia": 50304}

DECODE = {
    "c1": dict(model="gpt2", seed=0, streams=1, prompt=8, words=16, scaling="weak",
               metric="greedy tokens/sec/GPU at batch 1 (C1, bit-exact vs base2.py); % HBM roofline",
               workload="C1: GPT-2 124M base2 greedy decode, 1 stream per GPU, 8-id prompt (seed 0), 16 words"),
    "c2": dict(model="gpt2", seed=1, streams=64, prompt=32, words=128, scaling="weak", metric=C2_METRIC,
               workload="C2: GPT-2 124M base2 greedy decode, 64 streams per GPU, 32-id prompts (seed 1), 128 words "
                        "each (127 decode steps, key/value store 33->160 positions)"),
    "c3": dict(model="gpt2", seed=2, streams=16, prompt=960, words=64, scaling="weak",
               metric="greedy tokens/sec/GPU at batch 16, 1,024-position contexts (C3, bit-exact vs base2.py); "
                      "% HBM roofline",
               workload="C3: GPT-2 124M base2 greedy decode, 16 streams per GPU, 960-id prompts (seed 2), 64 words "
                        "(key/value store 961->1024 positions)"),
    "c5": dict(model="pythia", seed=4, streams=512, prompt=64, words=128, scaling="strong",
               metric="Pythia-160M greedy tokens/sec, 512 streams partitioned over the GPUs (C5, bit-exact vs "
                      "pythia_base2.py); % HBM roofline",
               workload="C5: Pythia-160M base2 greedy decode, 512 streams in total split 512/N over N GPUs, 64-id "
                        "prompts (seed 4), 128 words (store 65->192 positions)"),
}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return j, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


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
# the CPU port of the reference's loop (reference arm and cpu_baseline)
# ---------------------------------------------------------------------------------------------------------------------
def cpu_sample(name: str, steps: int, warmup: int, budget_s: float):
    """Words/s of the reference's own algorithm (oracle/: every word recomputes the whole prefix, base2.py:123,
    pythia_base2.py:175) on words at the job's average attended-key count. GPT-2: up to one stream per core in
    parallel (one stream for C3, its banks split over the cores); Pythia: one stream, banks split over the cores.
    Returns (value, cores, sample text, timed steps)."""
    import numpy as np

    from oracle.oracle import Oracle, PythiaOracle
    from streaming_machine_b200 import convert
    cfg = DECODE[name]
    cores = os.cpu_count() or 1
    V = VOCAB[cfg["model"]]
    half = (cfg["words"] - 1) // 2                      # words before the sampled one: the job's mean context
    ids_all = np.random.default_rng(cfg["seed"]).integers(0, V, (cfg["streams"], cfg["prompt"]))
    if cfg["model"] == "pythia":
        orc = PythiaOracle(convert.load_pythia(0))
        nb = 1
    else:
        orc = Oracle(convert.load_gpt2(0))
        nb = 1 if cfg["prompt"] > 256 else min(cfg["streams"], cores)
    ids = ids_all[:nb]
    prefix = np.concatenate([ids, orc.generate(ids, half)], 1) if half else ids   # untimed: the real greedy prefix

    def one():
        if cfg["model"] == "pythia":
            orc.scores(prefix[0], prefix.shape[1] - 1, prefix.shape[1])
        else:
            orc.generate_recompute(prefix, 1, threads=cores)

    for _ in range(max(0, warmup)):
        one()
    times = []
    t_all = time.perf_counter()
    for _ in range(max(1, steps)):
        t0 = time.perf_counter()
        one()
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_all > budget_s:
            break
    value = nb * len(times) / sum(times)
    sample = (f"{nb} {name.upper()} stream(s) x 1 word per step at {prefix.shape[1] + 1} attended keys (prompt + "
              f"{half} greedy words, the whole prefix recomputed as the reference's loop does), {len(times)} step(s), "
              f"{cores} threads")
    return value, cores, sample, len(times)


def run_reference(args):
    rank, world, _ = env_rank()
    if rank != 0:
        return
    name = args.config if args.config in DECODE else "c2"
    cfg = DECODE[name]
    value, cores, sample, steps = cpu_sample(name, args.steps, min(args.warmup, 1), budget_s=150.0)
    line = {"metric": cfg["metric"], "value": round(value, 4), "unit": UNIT, "n_gpus": args.gpus, "steps": steps,
            "warmup": min(args.warmup, 1), "ms_per_step": round(1000 / value, 3),
            "higher_is_better": True, "scaling": cfg["scaling"], "vs_baseline": None, "dtype": "int64",
            "data": "synthetic", "impl": "reference",
            "config": {"workload": cfg["workload"], "streams": cfg["streams"], "prompt": cfg["prompt"],
                       "words": cfg["words"]},
            "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------------------------------------
# our arm: decode configs
# ---------------------------------------------------------------------------------------------------------------------
def _dist(local_rank, world):
    if world <= 1:
        return None
    import datetime

    import torch.distributed as dist
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))
    return dist


def _parity(name, words, lo, hi, rank, world, dist):
    """The first job's words of this rank's streams against the oracle's digests (tests/golden): every word of every
    stream the digest holds. Summed over ranks."""
    import numpy as np
    import torch
    gold = os.path.join(ROOT, "tests", "golden", f"digests_{name}.npz")
    checked, equal = 0, 1
    if name == "c1":
        with open(os.path.join(ROOT, "tests", "golden", "gpt2_seed0.json")) as f:
            want = np.asarray([json.load(f)["c1"]["tokens"]])
        src = "the reference's own C1 words (tests/golden/gpt2_seed0.json)"
    else:
        want = np.load(gold)["tokens"]
        src = f"the oracle's whole-job digests (tests/golden/digests_{name}.npz)"
    if lo < len(want):                       # rows of this rank that the single-GPU job holds
        hi2 = min(hi, len(want))
        got = words[: hi2 - lo]
        checked = got.size
        equal = int(np.array_equal(got, want[lo:hi2]))
    if dist:
        t = torch.tensor([checked, 1 - equal], dtype=torch.int64, device="cuda")
        dist.all_reduce(t)
        checked, equal = int(t[0]), int(t[1] == 0)
    return {"all_equal": bool(equal), "words_checked": checked, "against": src}


def run_decode(args, name):
    import numpy as np
    import torch

    cfg = DECODE[name]
    rank, world, local_rank = env_rank()
    alone = bool(args.rank_of) and world == 1
    if alone:                                # one rank of an N-GPU strong-scaling run, alone on this GPU
        world, rank = (int(x) for x in args.rank_of.split(":"))
    torch.cuda.set_device(local_rank)
    dist = None if alone else _dist(local_rank, world)

    def barrier():
        if dist:
            dist.barrier(device_ids=[local_rank])

    from streaming_machine_b200 import convert, engine
    from streaming_machine_b200.shard import max_over_ranks, partition, stream_ids
    load = convert.load_pythia if cfg["model"] == "pythia" else convert.load_gpt2
    if rank == 0:                            # one process writes the converted-weights cache, the others read it
        M = load(0)
        barrier()
    else:
        barrier()
        M = load(0)
    V, P, words = VOCAB[cfg["model"]], cfg["prompt"], cfg["words"]
    if cfg["scaling"] == "strong":
        lo, hi = partition(cfg["streams"], rank, world)
        ids = np.random.default_rng(cfg["seed"]).integers(0, V, (cfg["streams"], P))[lo:hi]
        total_streams = cfg["streams"]
    else:
        lo, hi = rank * cfg["streams"], (rank + 1) * cfg["streams"]
        ids = stream_ids(cfg["seed"], cfg["streams"], P, rank, world, V)
        total_streams = cfg["streams"] * world
    B = len(ids)
    cycle = words - 1
    eng = engine.Engine(M, device=local_rank, n_streams=B, max_ctx=P + words)
    lens = torch.full((B,), P, dtype=torch.int32, device="cuda")
    buf = torch.empty(B * cycle, dtype=torch.int32, device="cuda")

    # ---- one full job, untimed: its words against the oracle's ----
    first = eng.prefill(ids)
    first_t = torch.as_tensor(first, device="cuda")
    eng.generate_device(B, cycle, buf.view(B, cycle))
    job_words = np.concatenate([first[:, None], buf.view(B, cycle).cpu().numpy()], 1)
    parity = _parity(name, job_words, lo, hi, rank, world, dist)

    K, W = args.steps, args.warmup
    start = 0 if K % cycle == 0 else (cycle - K % cycle) // 2      # the timed window, centred on the cycle
    positions = [(start + t) % cycle for t in range(K)]            # decode step index within the cycle
    keys = sum(P + 1 + c for c in positions)                       # keys attended per stream over the K steps

    class Cur:
        pos = 0

    def run(n, host=False, tok=None):
        """n decode steps from the cursor, rewinding to the prompt at the end of a cycle."""
        while n > 0:
            seg = min(n, cycle - Cur.pos)
            if host:
                for _ in range(seg):
                    tok = eng.step_host(tok)
            else:
                eng.generate_device(B, seg, buf[:B * seg].view(B, seg))
            Cur.pos += seg
            n -= seg
            if Cur.pos == cycle:
                eng.rewind(lens, first_t)
                Cur.pos = 0
                if host:
                    tok = first.astype(np.int32)
        return tok

    def position_at(p, host=False):
        """rewind to the prompt, W warm-up steps, then on to step p of the cycle (all untimed)"""
        eng.rewind(lens, first_t)
        Cur.pos = 0
        tok = first.astype(np.int32)
        tok = run(W, host, tok)
        tok = run((p - Cur.pos) % cycle, host, tok)
        return tok

    if args.quick:                           # profiling aid: W + K steps from the job's start, one short JSON line
        position_at(W % cycle)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        run(K)
        torch.cuda.synchronize()
        if rank == 0:
            print(json.dumps({"quick": True, "config": name, "steps": K,
                              "ms_per_step": round(1000 * (time.perf_counter() - t0) / K, 4)}))
        eng.close()
        if dist:
            dist.destroy_process_group()
        return

    # ---- pass 1: the device-timed value ----
    position_at(start)
    torch.cuda.synchronize()
    eng.profile(0)
    barrier()
    torch.cuda.synchronize()
    clk_proc, clk_path = clocks_start(local_rank)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    run(K)
    ev1.record()
    ev1.synchronize()
    clocks = clocks_stop(clk_proc, clk_path)
    barrier()
    launches, _ = eng.profile_read()
    t_ms = max_over_ranks(ev0.elapsed_time(ev1), dist, device="cuda")
    value = total_streams * K / (t_ms / 1000.0)

    # ---- pass 2: the same window with in-kernel stamps (graph + programmatic launches kept) ----
    position_at(start)
    torch.cuda.synchronize()
    eng.profile(2)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    run(K)
    e1.record()
    e1.synchronize()
    n_st, by = eng.profile_read()
    eng.profile(0)
    stamped_ms = e0.elapsed_time(e1)

    # ---- pass 3: end to end through the C ABI with host buffers ----
    tok = position_at(start, host=True)
    torch.cuda.synchronize()
    barrier()
    h0, h1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    h0.record()
    run(K, host=True, tok=tok)
    h1.record()
    h1.synchronize()
    barrier()
    e2e_ms = max_over_ranks(h0.elapsed_time(h1), dist, device="cuda")
    e2e = {"value": round(total_streams * K / (e2e_ms / 1000.0), 2), "unit": UNIT,
           "h2d_bytes_per_step": 4 * B, "d2h_bytes_per_step": 4 * B}

    pk, peak_kind = peaks()
    peak = float(pk["hbm_gbs"])
    wbytes = WEIGHT_BYTES[cfg["model"]]
    bank_n, bank_ms = by["bank"]
    att_n, att_ms = by["attend"]
    bank_gbs = wbytes * K / (bank_ms / 1000.0) / 1e9 if bank_ms > 0 else None
    kv_bytes = B * KV_BYTES_PER_KEY * keys
    att_gbs = kv_bytes / (att_ms / 1000.0) / 1e9 if att_ms > 0 else None
    step_bytes = (wbytes * K + kv_bytes) / K
    roofline = {"bound": "hbm", "achieved": round(bank_gbs, 1) if bank_gbs else None, "peak": peak, "unit": "GB/s",
                "frac": round(bank_gbs / peak, 4) if bank_gbs else None,
                "traffic": BANK_TRAFFIC.get(name) if world == 1 or cfg["scaling"] == "weak" else None,
                "traffic_source": BANK_TRAFFIC_SOURCE if name in BANK_TRAFFIC else None,
                "kernel": "bank product (48 layer banks + the head per step)",
                "algorithmic_bytes_per_launch": round(wbytes / BANK_LAUNCHES),
                "avg_launch_us": round(1000 * bank_ms / max(bank_n, 1), 3),
                "bank_ms_per_step": round(bank_ms / K, 4),
                "timing": "in-kernel stamps (b2_profile mode 2) in a second pass over the same steps, same CUDA graph "
                          "and programmatic launches: a launch lasts from the start of its dependent work to the next "
                          "stamped launch's",
                "ms_per_step_stamped_pass": round(stamped_ms / K, 4),
                "peak_kind": peak_kind + " (MEASURED_PEAKS.json hbm_gbs, a copy kernel's read + write rate)"}
    line = {"metric": cfg["metric"], "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": K,
            "warmup": W, "ms_per_step": round(t_ms / K, 4), "higher_is_better": True,
            "scaling": cfg["scaling"], "vs_baseline": None, "dtype": "int64", "data": "synthetic",
            "value_per_gpu": round(value / world, 2),
            "config": {"workload": cfg["workload"], "streams_per_gpu": B, "streams_total": total_streams,
                       "prompt": P, "words": words,
                       "window": f"decode steps {positions[0]}..{positions[-1]} of the {cycle}-step job"
                                 + (" (whole cycles)" if K % cycle == 0 else " (centred on the job)")
                                 + f", {keys / K:.1f} keys attended per stream per step",
                       "parallelism": f"stream sharding over {world} GPU(s), no collective",
                       "l2": "no flush: 247 MB of weights streamed per step exceed the 126 MB L2"},
            "roofline": roofline,
            "roofline_attend": {"bound": "hbm", "achieved": round(att_gbs, 1) if att_gbs else None, "peak": peak,
                                "unit": "GB/s", "frac": round(att_gbs / peak, 4) if att_gbs else None,
                                "avg_launch_us": round(1000 * att_ms / max(att_n, 1), 3),
                                "algorithmic_bytes": "keys, values and exponents the steps attend"},
            "step_hbm_frac": round(step_bytes / (t_ms / K / 1000.0) / 1e9 / peak, 4),
            "step_algorithmic_bytes": int(step_bytes),
            "e2e": e2e, "clocks": clocks, "gpu_launches": int(launches),
            "kernel_ms_per_step": {k: round(v[1] / K, 4) for k, v in by.items()},
            "parity": parity}
    if rank == 0 and world == 1 and not args.no_cpu:
        cv, cores, sample, _ = cpu_sample(name, 2, 0, budget_s=30.0)
        line["cpu_baseline"] = {"value": round(cv, 4), "unit": UNIT, "cores": cores, "kind": "port", "sample": sample}
    if alone:
        line["n_gpus"] = 1
        line["rank_of"] = {"world": world, "rank": rank,
                           "note": "this rank's shard alone on one GPU; value = all streams x K / this rank's time, the "
                                   "N-GPU aggregate if every rank took as long"}
    eng.close()
    if rank == 0 or alone:
        print(json.dumps(line), flush=True)
    if dist:
        dist.destroy_process_group()


# ---------------------------------------------------------------------------------------------------------------------
# C4: the prompt pass (int8 tensor-pipe bound)
# ---------------------------------------------------------------------------------------------------------------------
C4_B, C4_P, C4_SEED = 32, 512, 3
C4_MACS_PER_ROW = 84_934_656            # int16 multiply-adds of the 48 layer banks per position


def run_c4(args):
    import numpy as np
    import torch

    rank, world, local_rank = env_rank()
    torch.cuda.set_device(local_rank)
    dist = _dist(local_rank, world)
    from streaming_machine_b200 import convert, engine
    from streaming_machine_b200.shard import max_over_ranks, stream_ids
    M = convert.load_gpt2(0)
    V = VOCAB["gpt2"]
    eng = engine.Engine(M, device=local_rank, n_streams=C4_B, max_ctx=C4_P)
    ids = stream_ids(C4_SEED, C4_B, C4_P, rank, world, V)
    ids_t = torch.as_tensor(ids.astype(np.int32).ravel(), device="cuda")
    lens_t = torch.full((C4_B,), C4_P, dtype=torch.int32, device="cuda")
    nxt = torch.empty(C4_B, dtype=torch.int32, device="cuda")

    def one():
        eng._call("b2_prefill", eng.h, ids_t.data_ptr(), lens_t.data_ptr(), C4_B, nxt.data_ptr(), None, eng._stream())

    for _ in range(max(args.warmup, 1)):
        one()
    parity = _parity("c4", nxt.cpu().numpy()[:, None], rank * C4_B, (rank + 1) * C4_B, rank, world, dist)
    torch.cuda.synchronize()
    eng.profile(0)
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
    # end to end: host ids in, the next words back (Engine.prefill: pageable host buffers)
    torch.cuda.synchronize()
    h0, h1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    h0.record()
    for _ in range(args.steps):
        eng.prefill(ids)
    h1.record()
    h1.synchronize()
    e2e_ms = max_over_ranks(h0.elapsed_time(h1), dist, device="cuda")
    # in-kernel stamps over one pass: the bank products' time
    eng.profile(2)
    one()
    torch.cuda.synchronize()
    _, by = eng.profile_read()
    eng.profile(0)
    bank_ms = by["bank"][1]
    ops = C4_B * C4_P * C4_MACS_PER_ROW * 4 * 2 + C4_B * 768 * V * 4 * 2      # int8 ops: 4 per int16 MAC, x2
    pk, peak_kind = peaks()
    peak = 2.0 * float(pk["bf16_tflops"])
    achieved = ops / (bank_ms / 1000.0) / 1e12
    line = {"metric": "prompt-pass tokens/sec/GPU (C4, bit-exact vs base2.py); % int8 tensor roofline",
            "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(t_ms / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int64", "data": "synthetic",
            "value_per_gpu": round(value / world, 1),
            "config": {"workload": "C4: GPT-2 124M base2 prompt pass, 32 streams x 512 ids per GPU (seed 3)",
                       "l2": "no flush: each pass streams 2 x 247 MB of weight planes and ~1 GB of activations"},
            "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": peak, "unit": "TOPS (int8)",
                         "frac": round(achieved / peak, 4), "traffic": None,
                         "kernel": "bank products (k_bank_tiles), int8 ops per pass / their stamped time",
                         "peak_kind": "2 x measured dense bf16 (int8's nominal rate is twice bf16's; no measured "
                                      "int8 peak is given)",
                         "bank_ms_per_pass": round(bank_ms, 3)},
            "e2e": {"value": round(tokens / (e2e_ms / 1000.0), 1), "unit": "tokens/s",
                    "h2d_bytes_per_step": 4 * C4_B * C4_P + 4 * C4_B, "d2h_bytes_per_step": 4 * C4_B},
            "clocks": clocks, "gpu_launches": int(launches),
            "kernel_ms_per_step": {k: round(v[1], 4) for k, v in by.items()},
            "parity": parity}
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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=127)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline leg")
    ap.add_argument("--config", choices=("c1", "c2", "c3", "c4", "c5"), default="c2",
                    help="c2 (default): the metric's batch-64 decode; c1/c3/c5 the other decode configs; c4 the "
                         "prompt pass")
    ap.add_argument("--quick", action="store_true", help="profiling aid: --warmup and --steps decode steps only")
    ap.add_argument("--rank-of", default="", metavar="N:R",
                    help="profiling aid (c5): rank R's shard of an N-GPU run, timed alone on this GPU with the same "
                         "procedure (the ranks share nothing inside the timed region); its line is that rank's")
    args = ap.parse_args()
    if args.rank_of and (args.config != "c5" or len(args.rank_of.split(":")) != 2):
        ap.error("--rank-of N:R applies to the strong-scaling config c5")
    if args.warmup < 3 and not args.quick and args.impl == "ours":
        ap.error("--warmup must be at least 3")
    if args.impl == "reference":
        run_reference(args)
    elif args.config == "c4":
        run_c4(args)
    else:
        run_decode(args, args.config)


if __name__ == "__main__":
    main()
