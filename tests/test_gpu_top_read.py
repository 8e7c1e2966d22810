"""The exact collapsing top read (the reference's top=fr, base2_stream_fr2.swift:23-38: coarse scores from the high
byte plane, bounds from the input's positive and negative sums, low bytes only for the words that can still win)
against the plain race over every score: the same words, ties included (to the lowest index)."""
import numpy as np
import pytest

from conftest import gload, with_streams

pytestmark = pytest.mark.gpu
V = 50257


def _words(e, ids, n):
    return e.generate(ids, n)      # b2_generate: no scores stored, so the collapsing read takes the decode steps


def test_c1_words(gpu_engine, golden):
    g = gload("gpt2_logits_c1.npz")
    e = with_streams(gpu_engine, 4, 64)
    e.set_top_read(True)
    try:
        assert _words(e, [g["ids"]], 16)[0].tolist() == golden["c1"]["tokens"]
    finally:
        e.set_top_read(False)


@pytest.mark.parametrize("n", [1, 3, 4, 5])
def test_batches_vs_oracle(gpu_engine, orc, n):
    """Up to 4 streams take the collapsing read, 5 fall back to the plain one: all equal the oracle's words."""
    ids = np.random.default_rng(40 + n).integers(0, V, (n, 12))
    e = with_streams(gpu_engine, 8, 64)
    e.set_top_read(True)
    try:
        got = _words(e, ids, 6)
    finally:
        e.set_top_read(False)
    assert np.array_equal(got, orc.generate(ids, 6))


def test_ties_to_the_lowest_index(M):
    """Head columns in equal pairs (2i, 2i + 1): every race is a tie, and the collapsing read keeps the lower word."""
    from oracle.oracle import Oracle
    from streaming_machine_b200 import engine
    M2 = dict(M)
    w, e_, b = M["head.w"].copy(), M["head.e"].copy(), M["head.b"].copy()
    j = np.arange(V // 2) * 2
    w[:, j + 1], e_[j + 1], b[j + 1] = w[:, j], e_[j], b[j]
    M2["head.w"], M2["head.e"], M2["head.b"] = w, e_, b
    ids = np.random.default_rng(41).integers(0, V, (4, 10))
    e = engine.Engine(M2, n_streams=4, max_ctx=32)
    try:
        e.set_top_read(True)
        got = _words(e, ids, 5)
    finally:
        e.close()
    want = Oracle(M2).generate(ids, 5)
    assert np.array_equal(got, want)
    assert (got[got < 2 * (V // 2)] % 2 == 0).all()


def test_pythia_words(pythia_engine, porc):
    ids = np.random.default_rng(42).integers(0, 50304, (3, 9))
    e = with_streams(pythia_engine, 4, 32)
    e.set_top_read(True)
    try:
        got = _words(e, ids, 5)
    finally:
        e.set_top_read(False)
    assert np.array_equal(got, porc.generate(ids, 5))
