"""Generate the whole-job digests of the BASELINE configs from the CPU oracle (test infrastructure).

For every stream of a config: the greedy words and, at every generated position, the 64-bit digest of the int64
scores the word was raced on (`oracle.logit_hash`: the sum of score x key modulo 2^64). The oracle itself is pinned
to the reference's base2.py / pythia_base2.py by the golden vectors beside this file (tests/test_oracle_golden.py,
tests/test_oracle_pythia.py), so equal digests at every position mean equal integers with the reference machine.

    C2  GPT-2, 64 streams x 32-id prompts (seed 1), 128 words          -> digests_c2.npz
    C3  GPT-2, 16 streams x 960-id prompts (seed 2), 64 words           -> digests_c3.npz
    C4  GPT-2, 32 streams x 512-id prompts (seed 3), the word after     -> digests_c4.npz
    C5  Pythia-160M, 512 streams x 64-id prompts (seed 4), 128 words    -> digests_c5.npz

The prompts are numpy default_rng(seed).integers(0, vocab, (streams, prompt)). Runs on the CPU (all cores; C5 is
the long one, several minutes on 8 cores):

    python tests/golden/make_digests.py [c2 c3 c4 c5]
"""
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

CONFIGS = {
    # name: (model, seed, streams, prompt, words)
    "c2": ("gpt2", 1, 64, 32, 128),
    "c3": ("gpt2", 2, 16, 960, 64),
    "c4": ("gpt2", 3, 32, 512, 1),
    "c5": ("pythia", 4, 512, 64, 128),
}


def prompts(name: str) -> np.ndarray:
    model, seed, B, P, _ = CONFIGS[name]
    V = 50257 if model == "gpt2" else 50304
    return np.random.default_rng(seed).integers(0, V, (B, P))


def main(names):
    from oracle.oracle import Oracle, PythiaOracle
    from streaming_machine_b200 import convert
    orc = {}
    for name in names:
        model, seed, B, P, n = CONFIGS[name]
        if model not in orc:
            orc[model] = Oracle(convert.load_gpt2(0)) if model == "gpt2" else PythiaOracle(convert.load_pythia(0))
        ids = prompts(name)
        t0 = time.time()
        tok, hs = orc[model].generate_digest(ids, n)
        np.savez_compressed(os.path.join(HERE, f"digests_{name}.npz"), tokens=tok.astype(np.int32), hashes=hs,
                            seed=seed, streams=B, prompt=P, words=n)
        print(f"{name}: {B} streams x {n} words in {time.time() - t0:.1f} s", flush=True)


if __name__ == "__main__":
    main(sys.argv[1:] or list(CONFIGS))
