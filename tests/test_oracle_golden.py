"""Pin the CPU oracle (oracle/base2_oracle.c) to the reference machine.

Every expected value here came from the reference's own base2.py run in the build container
(tests/golden/make_golden.py); the oracle must reproduce them bit for bit.
"""
import hashlib

import numpy as np
import pytest

from conftest import gload
from oracle import oracle as O


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(np.asarray(a, dtype=np.int64)).tobytes()).hexdigest()


# ---- element functions (base2.py:18-60) ------------------------------------------------------------------------------
def test_rshift():
    g = gload("gpt2_micro.npz")
    assert np.array_equal(O.rshift(g["rshift_x"], g["rshift_s"]), g["rshift_y"])


def test_to16_incl_plus_32768():
    g = gload("gpt2_micro.npz")
    x16, e = O.to16(g["to16_x"], -16)
    assert np.array_equal(x16, g["to16_y"]) and np.array_equal(e, g["to16_e"])
    assert x16.max() == 32768            # the 17-bit case the device layout must carry


def test_gauge_log(orc):
    g = gload("gpt2_micro.npz")
    x16, ex, LS = orc.gauge_log(g["gauge_x"])
    assert np.array_equal(x16, g["gauge_x16"]) and np.array_equal(ex, g["gauge_ex"]) and np.array_equal(LS, g["gauge_LS"])


def test_log2fix(orc):
    g = gload("gpt2_micro.npz")
    assert np.array_equal(orc.log2fix(g["log2fix_x"]), g["log2fix_y"])


def test_power_wraps_like_numpy(orc):
    g = gload("gpt2_micro.npz")
    assert np.array_equal(orc.power(g["power_x"], g["power_f"]), g["power_y"])


def test_edge(orc):
    g = gload("gpt2_micro.npz")
    assert np.array_equal(orc.edge(g["edge_x"]), g["edge_y"])


def test_race_ties_lowest_index():
    g = gload("gpt2_micro.npz")
    assert [O.race(r) for r in g["race_x"]] == g["race_y"].tolist()
    assert g["race_y"][0] == 0 and g["race_y"][1] == 3


# ---- one layer, bank by bank (base2.py:62-100) -------------------------------------------------------------------------
def test_layer0_banks(orc):
    L = gload("gpt2_layer0.npz")
    assert np.array_equal(orc.gauged_bank(L["R0"], "qkv.0"), L["qkv"])
    assert np.array_equal(orc.attention(L["qkv"]), L["att"])
    assert np.array_equal(L["R0"] + orc.plain_bank(L["att"], "proj.0"), L["R1"])
    assert np.array_equal(orc.gauged_bank(L["R1"], "fc.0"), L["hid"])
    assert np.array_equal(orc.edge(L["hid"]), L["hidE"])
    assert np.array_equal(L["R1"] + orc.plain_bank(L["hidE"], "mproj.0"), L["R2"])


# ---- whole machine ---------------------------------------------------------------------------------------------------
def test_c1_tokens_and_logits(orc, golden):
    g = gload("gpt2_logits_c1.npz")
    tok, lg = orc.generate(g["ids"][None, :], 16, logits=True)
    assert tok[0].tolist() == golden["c1"]["tokens"] == g["tokens"].tolist()
    assert np.array_equal(lg[0], g["logits"])


def test_c1_recompute_equals_cached(orc, golden):
    """base2.py recomputes the prefix every word; the cached machine must give the same words."""
    ids = golden["c1"]["ids"]
    assert orc.greedy_recompute(ids, 3).tolist() == golden["c1"]["tokens"][:3]


def test_c2_streams(orc, golden):
    ids = np.random.default_rng(1).integers(0, 50257, (64, 32))
    for s, want in golden["c2"].items():
        tok, lg = orc.generate(ids[int(s)][None, :], 4, logits=True)
        assert tok[0].tolist() == want["tokens"]
        assert [sha(r) for r in lg[0]] == want["logits_sha"]


@pytest.mark.slow
def test_c4_prompt_pass(orc, golden):
    ids = np.random.default_rng(3).integers(0, 50257, (32, 512))[0]
    lg = orc.scores(ids, 508, 512)
    assert [sha(r) for r in lg] == golden["c4"]["logits_sha"]
    assert [O.race(r) for r in lg] == golden["c4"]["next"]


@pytest.mark.slow
def test_c3_long_context(orc, golden):
    """P=960: the attention output's X*EXP2 wraps mod 2^64 in base2.py; the oracle must wrap the same way."""
    if "c3" not in golden:
        pytest.skip("golden C3 not generated")
    ids = np.random.default_rng(2).integers(0, 50257, (16, 960))[0]
    lg = orc.scores(ids, 956, 960)
    assert [sha(r) for r in lg] == golden["c3"]["logits_sha"]
    assert [O.race(r) for r in lg] == golden["c3"]["next"]
