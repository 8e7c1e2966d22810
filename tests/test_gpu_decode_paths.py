"""The decode step's alternative paths against each other and the oracle: rows quantised inside the bank kernels (the
default, producers publishing each row's OR; at <= 2 streams the CUDA-core GEMV banks and GEMV head) and a quantisation kernel before
every bank (B2_WQ=0); stream counts that fill one or two 32-row halves partly; words with and without the logits
stored (the head's folded race)."""
import os

import numpy as np
import pytest

from conftest import with_streams

pytestmark = pytest.mark.gpu
V = 50257


@pytest.fixture(scope="module")
def wq0_engine(M):
    from streaming_machine_b200 import engine
    old = os.environ.get("B2_WQ")
    os.environ["B2_WQ"] = "0"
    try:
        e = engine.Engine(M, n_streams=64, max_ctx=160)
    finally:
        if old is None:
            del os.environ["B2_WQ"]
        else:
            os.environ["B2_WQ"] = old
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


@pytest.mark.parametrize("n", [1, 2, 3, 31, 33])
def test_default_decode_vs_oracle(gpu_engine, orc, n):
    """Every logit of 4 words: one and two streams (the CUDA-core GEMV banks and head), three, just under / over one 32-row half
    (64 streams: test_gpu_parity)."""
    e = with_streams(gpu_engine, 64, 160)
    ids = np.random.default_rng(100 + n).integers(0, V, (n, 32))
    tok, lg = _run(e, ids, 4)
    want_tok, want_lg = orc.generate(ids, 4, logits=True)
    assert np.array_equal(tok, want_tok)
    assert np.array_equal(lg, want_lg)


def test_quant_kernel_path_vs_oracle(wq0_engine, orc):
    ids = np.random.default_rng(7).integers(0, V, (37, 32))
    tok, lg = _run(wq0_engine, ids, 4)
    want_tok, want_lg = orc.generate(ids, 4, logits=True)
    assert np.array_equal(tok, want_tok)
    assert np.array_equal(lg, want_lg)


def test_paths_agree_on_c2(wq0_engine, gpu_engine, golden):
    """C2's 64 streams, 128 words from the CUDA graph with no logits stored: both paths give the same words, and the
    golden streams are base2.py's."""
    ids = np.random.default_rng(1).integers(0, V, (64, 32))
    a = with_streams(gpu_engine, 64, 160).generate(ids, 128)
    b = wq0_engine.generate(ids, 128)
    assert np.array_equal(a, b)
    for s, g in golden["c2"].items():
        assert a[int(s), :len(g["tokens"])].tolist() == g["tokens"]
