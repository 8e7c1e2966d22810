"""Pin the oracle's float stage switches (gauge=/edge=/arrival= float, base2.py:66-69, 79-80, 89-92, 110-113;
Pythia's gauge=/turn=/edge=/arrival= float, pythia_base2.py:102-104, 118-120, 130-133, 144-146) to the reference's
own outputs (tests/golden/make_golden_float.py).

Tolerance: the gauge, the turn and Pythia's erf bend are IEEE-754 adds, multiplies, divides, sqrt, cos, sin and erf
in the reference's order (numpy's pairwise sums for the means): bit-exact. GPT-2's tanh bend and both float arrivals
go through numpy's own tanh/exp/pow and a BLAS matmul whose rounding is the library's: each integer within 1 of the
reference's, differing at no more than 1 in 1,000 places (on these fixtures they are equal)."""
import numpy as np
import pytest

from conftest import gload

from oracle import oracle as O


def close(a, b, frac=1e-3):
    d = np.abs(np.asarray(a, np.int64) - np.asarray(b, np.int64))
    return d.max(initial=0) <= 1 and (d > 0).mean() <= frac


def test_pairwise_sum_is_numpys():
    rng = np.random.default_rng(3)
    for n in (1, 5, 8, 9, 64, 127, 128, 129, 768, 1000, 3072):
        x = rng.standard_normal(n) * np.exp(rng.standard_normal(n) * 4)
        assert O.pairwise_sum(x) == np.sum(x)


def test_gpt2_float_stages(M, orc):
    G, L0 = gload("gpt2_float.npz"), gload("gpt2_layer0.npz")
    try:
        orc.set_flags(O.GAUGE_FLOAT)
        assert np.array_equal(orc.gauged_bank(L0["R0"], "qkv.0"), G["qkv_g"])
        assert np.array_equal(orc.gauged_bank(L0["R1"], "fc.0"), G["fc_g"])
        assert close(O.edge_float(L0["hid"]), G["hidE_e"])
        orc.set_flags(O.ARRIVAL_FLOAT)
        assert close(orc.attention(L0["qkv"]), G["att_a"])
        for tag, fl in (("g", 1), ("e", 2), ("a", 4), ("all", 7)):
            orc.set_flags(fl)
            assert orc.generate(G["ids"][None, :], 4)[0].tolist() == G["words_" + tag].tolist(), tag
    finally:
        orc.set_flags(0)


def test_pythia_float_stages(porc):
    P, L0, mic = gload("pythia_float.npz"), gload("pythia_layer0.npz"), gload("pythia_micro.npz")
    try:
        porc.set_flags(O.GAUGE_FLOAT)
        assert np.array_equal(porc.gauge(L0["R0"], "ln1.0"), P["G1_g"])
        assert np.array_equal(porc.gauge(mic["gauge_x"], "ln1.3"), P["gauge_y_g"])
        porc.set_flags(O.TURN_FLOAT)
        assert np.array_equal(porc.turn(mic["turn_x"], mic["turn_pos"]), P["turn_y_t"])
        assert np.array_equal(O.edge_float(L0["H"], erf_form=True), P["HE_e"])
        porc.set_flags(O.ARRIVAL_FLOAT)
        assert close(porc.attention(L0["QKV"]), P["ATT_a"])
        for tag, fl in (("g", 1), ("t", 8), ("e", 2), ("a", 4), ("all", 15)):
            porc.set_flags(fl)
            assert porc.generate(P["ids"][None, :], 3)[0].tolist() == P["words_" + tag].tolist(), tag
    finally:
        porc.set_flags(0)
