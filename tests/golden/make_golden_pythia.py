"""Golden vectors for the Pythia-160M variant (config 5), from the reference's own foundation0/pythia_base2.py.

Runs ONLY where a checkout of the reference exists (first argument, or B2_REFERENCE). In a temporary directory
holding copies of the reference's two Pythia-160M config.json files, it execs `foundation0/pythia_convert.py` with
`safetensors.safe_open` patched to serve `streaming_machine_b200.convert.pythia_seeded_state(0)` as both the start
and the finished checkpoint, then execs `foundation0/pythia_base2.py` (size=160m, not as __main__) from the same
directory, and records:

  pythia_seed0.json       digests of the reference converter's arrays, mismatches against ours, words, logit digests
  pythia_micro.npz        turn (rotary), gauge, power past 2^45 (exact big-int path), attention on a short sequence
  pythia_layer0.npz       one layer branch by branch on a 6-id prompt

    python tests/golden/make_golden_pythia.py <reference checkout>
"""
import hashlib
import json
import os
import shutil
import sys
import tempfile
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
from streaming_machine_b200 import convert  # noqa: E402

V = 50304


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(np.asarray(a, dtype=np.int64)).tobytes()).hexdigest()


def load_reference(ref, sd, work, argv=()):
    import safetensors

    class _File:
        def get_tensor(self, name):
            return np.asarray(sd[name])

    saved = safetensors.safe_open
    sargv, cwd = sys.argv, os.getcwd()
    src0 = os.path.join(ref, "foundation0")
    for step in ("step143000", "step0"):
        os.makedirs(os.path.join(work, "models", f"pythia-160m-{step}"), exist_ok=True)
        shutil.copy(os.path.join(src0, "models", f"pythia-160m-{step}", "config.json"),
                    os.path.join(work, "models", f"pythia-160m-{step}", "config.json"))
    try:
        safetensors.safe_open = lambda path, fw, *a, **k: _File()
        os.chdir(work)
        if not os.path.exists(os.path.join(work, "base2_pythia-160m.npz")):
            sys.argv = ["pythia_convert.py", "size=160m"]
            exec(compile(open(os.path.join(src0, "pythia_convert.py")).read(), "pythia_convert.py", "exec"),
                 {"__name__": "pythia_convert", "__file__": os.path.join(work, "pythia_convert.py")})
        sys.argv = ["pythia_base2.py", "size=160m", *argv]
        ns = {"__name__": "pythia_base2", "__file__": os.path.join(work, "pythia_base2.py")}
        exec(compile(open(os.path.join(src0, "pythia_base2.py")).read(), "pythia_base2.py", "exec"), ns)
        return ns
    finally:
        safetensors.safe_open = saved
        sys.argv = sargv
        os.chdir(cwd)


def main():
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("B2_REFERENCE", "")
    if not ref or not os.path.isdir(ref):
        sys.exit("usage: give the reference checkout's path (first argument or B2_REFERENCE)")
    t0 = time.time()
    sd = convert.pythia_seeded_state(0)
    mine = convert.convert_pythia(sd)
    work = tempfile.mkdtemp(prefix="b2gold_pythia_")
    J = load_reference(ref, sd, work)
    M = J["M"]
    print(f"converted + loaded {time.time() - t0:.0f}s", flush=True)
    out = {"seed": 0, "reference_files": ["foundation0/pythia_convert.py", "foundation0/pythia_base2.py"]}
    ref_arrays = {k: M[k] for k in M.files}
    out["reference_digests"] = {k: hashlib.sha256(np.ascontiguousarray(v).tobytes()).hexdigest()
                                for k, v in sorted(ref_arrays.items())}
    diff = {}
    for k, v in ref_arrays.items():
        m = mine.get(k)
        if m is None or m.shape != v.shape:
            diff[k] = "missing or shape"
        else:
            nd = int((m.astype(np.int64) != v.astype(np.int64)).sum())
            if nd:
                diff[k] = nd
    extra = sorted(set(mine) - set(ref_arrays))
    out["converter_mismatches"], out["converter_extra_keys"] = diff, extra
    print("converter mismatches vs reference:", diff or "none", "extra:", extra, flush=True)

    # ---------------- micro (pythia_base2.py:61-149) ----------------
    rng = np.random.default_rng(99)
    mic = {}
    X = rng.integers(-(1 << 30), 1 << 30, size=(40, 64), dtype=np.int64)
    pos = rng.integers(0, 2048, size=40)
    mic["turn_x"], mic["turn_pos"], mic["turn_y"] = X, pos, J["turn"](X, pos)
    R = rng.integers(-(1 << 22), 1 << 22, size=(8, 768), dtype=np.int64)
    R[1, 3] = (1 << 22) - 1
    mic["gauge_x"], mic["gauge_y"] = R, J["gauge"](R, "ln1.3")
    PX = rng.integers(-(1 << 60), 1 << 60, size=(4, 64), dtype=np.int64)          # past 2^45: the exact path
    PF = rng.integers(-60 * 65536, 20 * 65536, size=(4, 64), dtype=np.int64)
    mic["power_x"], mic["power_f"] = PX, PF
    try:
        mic["power_y"] = J["power"](PX, PF)
    except OverflowError:
        PF = rng.integers(-60 * 65536, -20 * 65536, size=(4, 64), dtype=np.int64)
        mic["power_f"], mic["power_y"] = PF, J["power"](PX, PF)
    np.savez_compressed(os.path.join(HERE, "pythia_micro.npz"), **mic)

    # ---------------- one layer, branch by branch (pythia_base2.py:151-157) ----------------
    ids6 = np.random.default_rng(7).integers(0, V, 6)
    R0 = J["rshift"](M["embed.w"][ids6].astype(np.int64), -(M["embed.e"][ids6][:, None] + 16))
    G1 = J["gauge"](R0, "ln1.0")
    QKV = J["plain"](G1, "qkv.0")
    ATT = J["attention"](QKV)
    At = J["plain"](ATT, "proj.0")
    G2 = J["gauge"](R0, "ln2.0")
    H = J["plain"](G2, "fc.0")
    HE = J["edge"](H)
    Mo = J["plain"](HE, "mproj.0")
    np.savez_compressed(os.path.join(HERE, "pythia_layer0.npz"), ids=ids6, R0=R0, G1=G1, QKV=QKV, ATT=ATT, At=At,
                        G2=G2, H=H, HE=HE, Mo=Mo, R1=R0 + At + Mo)
    print(f"layer0 {time.time() - t0:.0f}s", flush=True)

    # ---------------- C5: [512, 64] prompts (seed 4) ----------------
    ids5 = np.random.default_rng(4).integers(0, V, (512, 64))
    out["c5"] = {}
    for s in (0, 1, 511):
        words, lg = J["forward"](ids5[s].tolist(), last=4)
        got = []
        for _ in range(4):
            got.append(J["forward"](ids5[s].tolist() + got)[0][0])
        _, lg_next = J["forward"](ids5[s].tolist() + got[:-1], last=4)
        out["c5"][str(s)] = dict(prompt_last4_words=[int(w) for w in words], prompt_last4_sha=[sha(r) for r in lg],
                                 greedy=[int(w) for w in got], greedy_logits_sha=[sha(r) for r in lg_next])
        print(f"c5 stream {s}: {got} {time.time() - t0:.0f}s", flush=True)
    with open(os.path.join(HERE, "pythia_seed0.json"), "w") as f:
        json.dump(out, f, indent=1)
    print(f"done {time.time() - t0:.0f}s")


if __name__ == "__main__":
    main()
