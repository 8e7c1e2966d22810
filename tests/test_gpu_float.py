"""The float stage switches on the device (gauge=/edge=/arrival= float, base2.py:66-69, 79-80, 89-92, 110-113;
Pythia's gauge=/turn=/edge=/arrival= float, pythia_base2.py:102-104, 118-120, 130-133, 144-146) against the oracle
with the same switches (itself pinned to the reference's float outputs by test_oracle_float.py) and the reference's
own greedy words.

Tolerance: the gauge and the turn are correctly rounded IEEE-754 operations in the reference's order on both sides:
every logit integer equal. The bends and the arrival call the device's tanh/pow/erf/exp, which can differ from the C
library's in the last place; a rounding moved by one then travels through the later layers. There the words must
equal the oracle's and the reference's, and every logit must be within 2^-10 of the largest |logit| of its row of
the oracle's."""
import numpy as np
import pytest

from conftest import gload

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _engine(M, flags, n_streams, max_ctx):
    from streaming_machine_b200 import engine
    kw = {k: "float" for k, bit in (("gauge", 1), ("edge", 2), ("arrival", 4), ("turn", 8)) if flags & bit}
    return engine.Engine(M, n_streams=n_streams, max_ctx=max_ctx, **kw)


def _run(e, ids, words):
    first, lg0 = e.prefill(ids, logits=True)
    toks, lgs = [first], [lg0]
    for _ in range(words - 1):
        o, lg = e.step(logits=True)
        toks.append(o)
        lgs.append(lg)
    return np.stack(toks, 1), np.stack(lgs, 1)


def _check(tok, lg, want_tok, want_lg, exact):
    assert np.array_equal(tok, want_tok)
    if exact:
        assert np.array_equal(lg, want_lg)
    else:
        scale = np.abs(want_lg).max(axis=-1, keepdims=True).astype(np.float64)
        assert (np.abs(lg - want_lg) <= scale / 1024).all()


@pytest.mark.parametrize("flags", [O.GAUGE_FLOAT, O.EDGE_FLOAT, O.ARRIVAL_FLOAT,
                                   O.GAUGE_FLOAT | O.EDGE_FLOAT | O.ARRIVAL_FLOAT])
def test_gpt2_float_switches(M, orc, flags):
    G = gload("gpt2_float.npz")
    tag = {1: "g", 2: "e", 4: "a", 7: "all"}[flags]
    ids = np.random.default_rng(50 + flags).integers(0, 50257, (8, 12))
    e = _engine(M, flags, 8, 64)
    try:
        # the reference's own words on C1's prompt
        assert e.generate([G["ids"]], 4)[0].tolist() == G["words_" + tag].tolist()
        tok, lg = _run(e, ids, 4)
        orc.set_flags(flags)
        want_tok, want_lg = orc.generate(ids, 4, logits=True)
        _check(tok, lg, want_tok, want_lg, exact=flags == O.GAUGE_FLOAT)
        if flags == O.GAUGE_FLOAT:
            L0 = gload("gpt2_layer0.npz")
            assert np.array_equal(e.bank("qkv.0", L0["R0"], 0), G["qkv_g"])
            assert np.array_equal(e.bank("fc.0", L0["R1"], 0), G["fc_g"])
    finally:
        orc.set_flags(0)
        e.close()


@pytest.mark.parametrize("flags", [O.GAUGE_FLOAT, O.TURN_FLOAT, O.EDGE_FLOAT, O.ARRIVAL_FLOAT, 15])
def test_pythia_float_switches(PM, porc, flags):
    P = gload("pythia_float.npz")
    tag = {1: "g", 8: "t", 2: "e", 4: "a", 15: "all"}[flags]
    ids = np.random.default_rng(60 + flags).integers(0, 50304, (8, 12))
    e = _engine(PM, flags, 8, 64)
    try:
        assert e.generate([P["ids"]], 3)[0].tolist() == P["words_" + tag].tolist()
        tok, lg = _run(e, ids, 3)
        porc.set_flags(flags)
        want_tok, want_lg = porc.generate(ids, 3, logits=True)
        _check(tok, lg, want_tok, want_lg, exact=flags in (O.GAUGE_FLOAT, O.TURN_FLOAT))
        if flags == O.GAUGE_FLOAT:
            L0 = gload("pythia_layer0.npz")
            assert np.array_equal(e.gauge("ln1.0", L0["R0"]), P["G1_g"])
    finally:
        porc.set_flags(0)
        e.close()
