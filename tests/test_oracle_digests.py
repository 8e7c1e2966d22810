"""The whole-job digests (tests/golden/digests_*.npz, from the CPU oracle) against the reference's own outputs: every
word the reference machine produced for the same seeded prompts (tests/golden/gpt2_seed0.json and pythia_seed0.json,
made by running base2.py and pythia_base2.py), and the digest function itself against the oracle's scores."""
import numpy as np
import pytest

from conftest import gload


def test_digest_shapes():
    for name, (B, n) in {"c2": (64, 128), "c3": (16, 64), "c4": (32, 1), "c5": (512, 128)}.items():
        d = gload(f"digests_{name}.npz")
        assert d["tokens"].shape == (B, n) and d["hashes"].shape == (B, n) and d["hashes"].dtype == np.uint64
        assert (int(d["streams"]), int(d["words"])) == (B, n)


def test_digests_hold_the_reference_words(golden, pgold):
    c2 = gload("digests_c2.npz")["tokens"]
    for s, g in golden["c2"].items():
        assert c2[int(s), :len(g["tokens"])].tolist() == g["tokens"]
    # the word after C3's 960-id and C4's 512-id prompt of stream 0 (the reference's last-position race)
    assert int(gload("digests_c3.npz")["tokens"][0, 0]) == golden["c3"]["next"][-1]
    assert int(gload("digests_c4.npz")["tokens"][0, 0]) == golden["c4"]["next"][-1]
    c5 = gload("digests_c5.npz")["tokens"]
    for s, g in pgold["c5"].items():
        assert c5[int(s), :len(g["greedy"])].tolist() == g["greedy"]


def test_digest_function_on_oracle_scores(orc):
    """Two C2 streams, four words: the stored digests are logit_hash of the oracle's score rows."""
    from oracle.oracle import logit_hash
    d = gload("digests_c2.npz")
    ids = np.random.default_rng(1).integers(0, 50257, (64, 32))[[0, 63]]
    tok, lg = orc.generate(ids, 4, logits=True)
    assert np.array_equal(tok, d["tokens"][[0, 63], :4])
    assert np.array_equal(logit_hash(lg), d["hashes"][[0, 63], :4])
    # one score changed by one changes the digest
    lg[0, 0, 123] += 1
    assert logit_hash(lg)[0, 0] != d["hashes"][0, 0]
