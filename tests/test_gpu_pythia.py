"""Parity of the CUDA engine's Pythia-160M path (through the C ABI) with the reference's foundation0/pythia_base2.py:
bit-exact integers. Expected values come from the reference itself (tests/golden/pythia_*) and, at sizes the golden
vectors do not cover, from the Pythia CPU oracle, pinned to those vectors by test_oracle_pythia.py."""
import hashlib

import numpy as np
import pytest

from conftest import gload, with_streams

pytestmark = pytest.mark.gpu
V = 50304


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(np.asarray(a, dtype=np.int64)).tobytes()).hexdigest()


def test_pythia_layer0_pieces(pythia_engine):
    """The norm (b2_gauge) and each bank alone (b2_bank modes 2, 3) on the golden layer-0 inputs."""
    L = gload("pythia_layer0.npz")
    e = with_streams(pythia_engine, 1, 128)
    assert np.array_equal(e.gauge("ln1.0", L["R0"]), L["G1"])
    assert np.array_equal(e.gauge("ln2.0", L["R0"]), L["G2"])
    assert np.array_equal(e.bank("qkv.0", L["G1"], 2), L["QKV"])
    assert np.array_equal(e.bank("proj.0", L["ATT"], 2), L["At"])
    assert np.array_equal(e.bank("fc.0", L["G2"], 2), L["H"])
    assert np.array_equal(e.bank("fc.0", L["G2"], 3), L["HE"])
    assert np.array_equal(e.bank("mproj.0", L["HE"], 2), L["Mo"])
    g = gload("pythia_micro.npz")
    assert np.array_equal(e.gauge("ln1.3", g["gauge_x"]), g["gauge_y"])


def test_pythia_c5_golden_streams(pythia_engine, pgold):
    """C5's prompts (seed 4, [512, 64]): streams 0, 1, 511 of the reference's own run. The last four prompt positions'
    scores (four prompts cut at 61..64 ids, one stream each) and four greedy words with every score they raced on."""
    ids = np.random.default_rng(4).integers(0, V, (512, 64))
    e = with_streams(pythia_engine, 4, 128)
    for s, want in pgold["c5"].items():
        p = ids[int(s)]
        words, lg = e.prefill([p[:n] for n in (61, 62, 63, 64)], logits=True)
        assert [int(w) for w in words] == want["prompt_last4_words"]
        assert [sha(r) for r in lg] == want["prompt_last4_sha"]
        first, lg0 = e.prefill([p], logits=True)
        toks, lgs = [int(first[0])], [lg0[0]]
        for _ in range(3):
            o, lgn = e.step(n=1, logits=True)
            toks.append(int(o[0]))
            lgs.append(lgn[0])
        assert toks == want["greedy"]
        assert [sha(r) for r in lgs] == want["greedy_logits_sha"]


@pytest.mark.parametrize("n_streams,prompt,words", [(1, 16, 6), (2, 16, 6), (8, 16, 6), (64, 64, 3)])
def test_pythia_batch_vs_oracle(pythia_engine, porc, n_streams, prompt, words):
    """Many streams at once (64 x 64 prompt rows take the tensor-core banks): every word and every score row equal
    the oracle's."""
    ids = np.random.default_rng(40 + n_streams).integers(0, V, (n_streams, prompt))
    e = with_streams(pythia_engine, n_streams, 128)
    first, lg0 = e.prefill(ids, logits=True)
    toks, lgs = [first], [lg0]
    for _ in range(words - 1):
        o, lg = e.step(logits=True)
        toks.append(o)
        lgs.append(lg)
    want_tok, want_lg = porc.generate(ids, words, logits=True)
    assert np.array_equal(np.stack(toks, 1), want_tok)
    assert np.array_equal(np.stack(lgs, 1), want_lg)


def test_pythia_generate_device_matches_steps(pythia_engine, porc):
    """b2_generate (words fed back on the device, the step replayed from a CUDA graph) gives the oracle's words."""
    ids = np.random.default_rng(77).integers(0, V, (16, 24))
    e = with_streams(pythia_engine, 16, 128)
    got = e.generate(ids, 8)
    assert np.array_equal(got, porc.generate(ids, 8))
