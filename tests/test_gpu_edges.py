"""Edge cases of the reference's arithmetic and of the engine's device checks, through the C ABI.

* race ties (base2.py:34-40: the first of equal largest scores wins; base2_stream.swift:139-142: ties to the lower
  index): heads whose columns come in identical pairs, so words are decided by ties, inside one 32-column group of
  the head's epilogue race or across groups;
* a value-store entry beyond int32 (base2.py:98 reads v at full width; the device store holds int32, so such a value
  is a device-checked error, B2_ERR_VALUE, in the prompt pass and in a decode step);
* a bounded device wait that runs out (b2_check_wait with a short "wait_ns"): B2_ERR_DEVICE, and the handle still
  works afterwards;
* decode steps whose stream count moves across the 32-row halves on one handle (33, then 20, then 33 streams): the
  quantising bank kernels' CTA split and arrival counters stay consistent;
* decode-step bank inputs with +32768 entries (base2.py:24-27 rounds a row's largest value up to 2^15; the byte
  planes carry it as 32512 and the pile adds 256 w back), met by the in-kernel quantisation's +32768 lists.
"""
import numpy as np
import pytest

from conftest import with_streams

pytestmark = pytest.mark.gpu
V = 50257


def _tied(M, pairs):
    """M with head columns j2 := j1 for every (j1, j2) in pairs (same weights, exponent and bias: equal scores)."""
    M2 = dict(M)
    w, e, b = M["head.w"].copy(), M["head.e"].copy(), M["head.b"].copy()
    j1, j2 = np.asarray(pairs).T
    w[:, j2], e[j2], b[j2] = w[:, j1], e[j1], b[j1]
    M2["head.w"], M2["head.e"], M2["head.b"] = w, e, b
    return M2


def _words_and_scores(e, ids, words):
    first, lg0 = e.prefill(ids, logits=True)
    toks, lgs = [first], [lg0]
    for _ in range(words - 1):
        o, lg = e.step(n=len(ids), logits=True)
        toks.append(o)
        lgs.append(lg)
    return np.stack(toks, 1), np.stack(lgs, 1)


@pytest.mark.parametrize("kind", ["within_group", "across_groups"])
def test_race_ties_go_to_the_lowest_index(M, kind):
    from oracle.oracle import Oracle
    from streaming_machine_b200 import engine
    if kind == "within_group":   # columns 2i, 2i + 1 equal: both in one 32-column group, 2i must win
        pairs = [(2 * i, 2 * i + 1) for i in range(V // 2)]
    else:                        # column j + 25000 equals j: different groups, the lower column must win
        pairs = [(j, j + 25000) for j in range(25000)]
    M2 = _tied(M, pairs)
    ids = np.random.default_rng(21).integers(0, V, (8, 16))
    e = engine.Engine(M2, n_streams=8, max_ctx=32)
    try:
        tok, lg = _words_and_scores(e, ids, 4)
        tok_graph = e.generate(ids, 4)          # the head's folded race (no scores stored)
    finally:
        e.close()
    want_tok, want_lg = Oracle(M2).generate(ids, 4, logits=True)
    assert np.array_equal(lg, want_lg)
    assert np.array_equal(tok, want_tok)
    assert np.array_equal(tok_graph, want_tok)
    # every race won by a paired column was a tie, and the lower column took it
    paired = np.zeros(V, bool)
    paired[np.asarray(pairs).ravel()] = True
    best = lg.max(axis=-1)
    n_ties = 0
    for s in range(tok.shape[0]):
        for t in range(tok.shape[1]):
            tied = np.flatnonzero(lg[s, t] == best[s, t])
            assert tok[s, t] == tied[0]
            if paired[tok[s, t]]:
                assert len(tied) >= 2
                n_ties += 1
    assert n_ties >= tok.size - 2
    if kind == "within_group":
        assert (tok[tok < 2 * (V // 2)] % 2 == 0).all()
    else:
        assert ((tok < 25000) | (tok >= 50000)).all()


def test_value_store_overflow_is_an_error(M):
    """qkv.0's value columns pushed past int32: the prompt pass and a decode step report B2_ERR_VALUE."""
    from streaming_machine_b200 import engine
    M2 = dict(M)
    b = M["qkv.0.b"].copy()
    b[1536:2304] += np.int64(1) << 34
    M2["qkv.0.b"] = b
    ids = np.random.default_rng(22).integers(0, V, (4, 8))
    e = engine.Engine(M2, n_streams=4, max_ctx=32)
    try:
        with pytest.raises(engine.B2Error) as ex:
            e.prefill(ids)
        assert ex.value.code == 5 and "int32" in str(ex.value)
        with pytest.raises(engine.B2Error) as ex:
            e.step(n=4)
        assert ex.value.code == 5
    finally:
        e.close()


def test_bounded_wait_gives_up_and_the_handle_recovers(gpu_engine, orc):
    from streaming_machine_b200 import engine
    e = with_streams(gpu_engine, 4, 64)
    e.set_wait_limit(2_000_000)                       # 2 ms
    try:
        with pytest.raises(engine.B2Error) as ex:
            e.check_wait()
        assert ex.value.code == 7 and "gave up" in str(ex.value)
    finally:
        e.set_wait_limit(0)
    ids = np.random.default_rng(23).integers(0, V, (4, 8))
    assert np.array_equal(e.generate(ids, 3), orc.generate(ids, 3))


def test_stream_count_across_row_halves(gpu_engine, orc):
    """One handle: 3 steps of 33 streams, 2 of the first 20, 2 more of all 33. Each stream's words depend only on
    its own prefix, so streams 0-19 have 8 words and 20-32 have 6, each equal to the oracle's."""
    ids = np.random.default_rng(24).integers(0, V, (33, 16))
    e = with_streams(gpu_engine, 64, 64)
    got = [[int(w)] for w in e.prefill(ids)]
    for n, k in ((33, 3), (20, 2), (33, 2)):
        for _ in range(k):
            o = e.step(n=n)
            for s in range(n):
                got[s].append(int(o[s]))
    assert np.array_equal(np.asarray(got[:20]), orc.generate(ids[:20], 8))
    assert np.array_equal(np.asarray(got[20:]), orc.generate(ids[20:], 6))


@pytest.mark.parametrize("n_streams", [40, 2])
def test_plus_32768_inputs_in_decode_banks(M, n_streams):
    """Residual columns held at 2^20 - 1 through every layer (their embedding columns set, wpe's zeroed, and the proj
    and mproj output columns zeroed), so that to16 rounds them to +32768 in every qkv and fc input row (the row's
    largest value: every other |value| stays below 2^20). The columns fall in different CTAs' shares of the row and on
    both sides of the qkv bank's K split; 40 streams fill one row half and part of the next, 2 streams run the
    CUDA-core GEMV banks."""
    from oracle.oracle import Oracle
    from streaming_machine_b200 import engine
    cols = [5, 200, 383, 384, 700]
    M2 = dict(M)
    wte, wpe = M["wte"].copy(), M["wpe"].copy()
    wte[:, cols] = (1 << 20) - 1
    wpe[:, cols] = 0
    M2["wte"], M2["wpe"] = wte, wpe
    for l in range(12):
        for b in ("proj", "mproj"):
            w, bb = M[f"{b}.{l}.w"].copy(), M[f"{b}.{l}.b"].copy()
            w[:, cols] = 0
            bb[cols] = 0
            M2[f"{b}.{l}.w"], M2[f"{b}.{l}.b"] = w, bb
    ids = np.random.default_rng(25).integers(0, V, (n_streams, 8))
    # every embedded row (any word, any position) has these columns as its largest values: layer 0's qkv inputs
    # reach +32768 there in every decode step
    assert np.abs(np.delete(wte, cols, 1)).max() + np.abs(np.delete(wpe, cols, 1)).max() < (1 << 20) - 1
    e = engine.Engine(M2, n_streams=n_streams, max_ctx=32)
    try:
        tok, lg = _words_and_scores(e, ids, 4)
        tok_graph = e.generate(ids, 4)
    finally:
        e.close()
    want_tok, want_lg = Oracle(M2).generate(ids, 4, logits=True)
    assert np.array_equal(lg, want_lg)
    assert np.array_equal(tok, want_tok)
    assert np.array_equal(tok_graph, want_tok)


def test_stored_layer0_entry_rows(M, orc):
    """Layer 0's qkv bank of a decode step from stored rows (entry_tables: Tw = wte . W, Tp = wpe . W, the reference's
    stored layer-0 entry): every word and score row equal to the oracle's at 1 stream (the CUDA-core banks) and 40
    streams (the tensor-core banks), and C2's 64 streams over 24 words."""
    from streaming_machine_b200 import engine
    e = engine.Engine(M, n_streams=1, max_ctx=160)
    try:
        e.set_entry_tables(True)
        for n in (1, 40):
            e.alloc_streams(n, 64)
            ids = np.random.default_rng(26 + n).integers(0, V, (n, 16))
            tok, lg = _words_and_scores(e, ids, 4)
            want_tok, want_lg = orc.generate(ids, 4, logits=True)
            assert np.array_equal(lg, want_lg)
            assert np.array_equal(tok, want_tok)
        e.alloc_streams(64, 160)
        ids = np.random.default_rng(1).integers(0, V, (64, 32))
        got = e.generate(ids, 24)
        assert np.array_equal(got, orc.generate(ids, 24))
    finally:
        e.close()
