"""The one-kernel decode step (b2_mega.cu, B2_MEGA=1) against the oracle and the per-launch path: bit-exact."""
import os

import numpy as np
import pytest

from conftest import gload, with_streams

pytestmark = pytest.mark.gpu
V = 50257


@pytest.fixture(scope="module")
def mega_engine(M):
    from streaming_machine_b200 import engine
    old = os.environ.get("B2_MEGA")
    os.environ["B2_MEGA"] = "1"
    try:
        e = engine.Engine(M, n_streams=64, max_ctx=160)
    finally:
        if old is None:
            del os.environ["B2_MEGA"]
        else:
            os.environ["B2_MEGA"] = old
    yield e
    e.close()


def _run(e, ids, words):
    first, lg0 = e.prefill(ids, logits=True)
    toks, lgs = [first], [lg0]
    for _ in range(words - 1):
        o, lg = e.step(n=len(ids), logits=True)
        toks.append(o)
        lgs.append(lg)
    return np.stack(toks, 1), np.stack(lgs, 1)


def test_mega_c1_logits(mega_engine, golden):
    g = gload("gpt2_logits_c1.npz")
    tok, lg = _run(mega_engine, [g["ids"]], 16)
    assert tok[0].tolist() == golden["c1"]["tokens"]
    assert np.array_equal(lg[0], g["logits"])


@pytest.mark.parametrize("n", [64, 37, 5])
def test_mega_batch_vs_oracle(mega_engine, orc, n):
    ids = np.random.default_rng(1 + n).integers(0, V, (n, 32))
    tok, lg = _run(mega_engine, ids, 4)
    want_tok, want_lg = orc.generate(ids, 4, logits=True)
    assert np.array_equal(tok, want_tok)
    assert np.array_equal(lg, want_lg)


def test_mega_c2_words_vs_launches(mega_engine, gpu_engine, orc, golden):
    """C2's 64 streams, 128 words with the steps replayed from a CUDA graph: every word equals the per-launch path's,
    the golden streams equal base2.py's, and three streams equal the oracle over all 128 words."""
    ids = np.random.default_rng(1).integers(0, V, (64, 32))
    words = mega_engine.generate(ids, 128)
    mega_engine.sync()
    ref = with_streams(gpu_engine, 64, 160).generate(ids, 128)
    assert np.array_equal(words, ref)
    for s, g in golden["c2"].items():
        assert words[int(s), :len(g["tokens"])].tolist() == g["tokens"]
    pick = [0, 31, 63]
    assert np.array_equal(words[pick], orc.generate(ids[pick], 128))
