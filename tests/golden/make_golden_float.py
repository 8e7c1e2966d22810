"""Golden vectors for the float stage switches (base2.py `gauge=/edge=/arrival= float`, base2.py:66-69, 79-80,
89-92, 110-113; pythia_base2.py `gauge=/turn=/edge=/arrival= float`, :102-104, 118-120, 130-133, 144-146).

Runs ONLY where a checkout of the reference exists (first argument, or B2_REFERENCE). Loads the reference
machines exactly as make_golden.py and make_golden_pythia.py do, once per switch setting, and records what each
switched stage gives on the inputs of the integer layer-0 fixtures, plus a few greedy words with the switches on:

  gpt2_float.npz     gauged_bank (qkv.0, fc.0) with gauge=float, edge with edge=float, attention with arrival=float,
                     4 greedy words of C1's prompt for each switch alone and all three together
  pythia_float.npz   gauge (ln1.0, ln1.3), turn, edge, attention with their switch; 3 greedy words of C5 stream 0's
                     first 16 ids for each switch alone and all four together

    python tests/golden/make_golden_float.py <reference checkout>
"""
import os
import sys
import tempfile
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import make_golden as g2  # noqa: E402
import make_golden_pythia as gp  # noqa: E402
from streaming_machine_b200 import convert  # noqa: E402


def gpt2(ref, t0):
    sd = convert.gpt2_seeded_state(0)
    work = tempfile.mkdtemp(prefix="b2gold_float_")
    L0 = np.load(os.path.join(HERE, "gpt2_layer0.npz"))
    ids1 = [int(i) for i in np.random.default_rng(0).integers(0, g2.V, 8)]
    out = {}
    for tag, argv in (("g", ["gauge=float"]), ("e", ["edge=float"]), ("a", ["arrival=float"]),
                      ("all", ["gauge=float", "edge=float", "arrival=float"])):
        J = g2.load_reference(ref, sd, work, argv)
        if tag == "g":
            out["qkv_g"] = J["gauged_bank"](L0["R0"], "qkv.0")
            out["fc_g"] = J["gauged_bank"](L0["R1"], "fc.0")
        if tag == "e":
            out["hidE_e"] = J["edge"](L0["hid"])
        if tag == "a":
            out["att_a"] = J["attention"](L0["qkv"])
        got = []
        for _ in range(4):
            got.append(int(J["forward"](ids1 + got)))
        out["words_" + tag] = np.array(got)
        print(f"gpt2 {tag}: {got} {time.time() - t0:.0f}s", flush=True)
    out["ids"] = np.array(ids1)
    np.savez_compressed(os.path.join(HERE, "gpt2_float.npz"), **out)


def pythia(ref, t0):
    sd = convert.pythia_seeded_state(0)
    work = tempfile.mkdtemp(prefix="b2gold_pfloat_")
    L0 = np.load(os.path.join(HERE, "pythia_layer0.npz"))
    mic = np.load(os.path.join(HERE, "pythia_micro.npz"))
    ids = [int(i) for i in np.random.default_rng(4).integers(0, gp.V, (512, 64))[0][:16]]
    out = {}
    for tag, argv in (("g", ["gauge=float"]), ("t", ["turn=float"]), ("e", ["edge=float"]), ("a", ["arrival=float"]),
                      ("all", ["gauge=float", "turn=float", "edge=float", "arrival=float"])):
        J = gp.load_reference(ref, sd, work, argv)
        if tag == "g":
            out["G1_g"] = J["gauge"](L0["R0"], "ln1.0")
            out["gauge_y_g"] = J["gauge"](mic["gauge_x"], "ln1.3")
        if tag == "t":
            out["turn_y_t"] = J["turn"](mic["turn_x"], mic["turn_pos"])
        if tag == "e":
            out["HE_e"] = J["edge"](L0["H"])
        if tag == "a":
            out["ATT_a"] = J["attention"](L0["QKV"])
        got = []
        for _ in range(3):
            got.append(int(J["forward"](ids + got)[0][0]))
        out["words_" + tag] = np.array(got)
        print(f"pythia {tag}: {got} {time.time() - t0:.0f}s", flush=True)
    out["ids"] = np.array(ids)
    np.savez_compressed(os.path.join(HERE, "pythia_float.npz"), **out)


def main():
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("B2_REFERENCE", "")
    if not ref or not os.path.isdir(ref):
        sys.exit("usage: give the reference checkout's path (first argument or B2_REFERENCE)")
    t0 = time.time()
    gpt2(ref, t0)
    pythia(ref, t0)
    print(f"done {time.time() - t0:.0f}s")


if __name__ == "__main__":
    main()
