"""Pin the Pythia-160M oracle to the reference's own foundation0/pythia_base2.py (vectors from
tests/golden/make_golden_pythia.py) and our converter to the reference's pythia_convert.py."""
import hashlib

import numpy as np
import pytest

from conftest import gload

V = 50304


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(np.asarray(a, dtype=np.int64)).tobytes()).hexdigest()


def test_pythia_converter_matches_reference(PM, pgold):
    assert pgold["converter_mismatches"] == {} and pgold["converter_extra_keys"] == []
    ref = pgold["reference_digests"]
    assert set(ref) == set(PM)
    assert [k for k in ref if hashlib.sha256(np.ascontiguousarray(PM[k]).tobytes()).hexdigest() != ref[k]] == []


def test_pythia_micro(porc):
    g = gload("pythia_micro.npz")
    assert np.array_equal(porc.turn(g["turn_x"], g["turn_pos"]), g["turn_y"])
    assert np.array_equal(porc.gauge(g["gauge_x"], "ln1.3"), g["gauge_y"])
    assert np.array_equal(porc.power(g["power_x"], g["power_f"]), g["power_y"])     # the exact (big-int) path


def test_pythia_layer0(porc):
    L = gload("pythia_layer0.npz")
    assert np.array_equal(porc.gauge(L["R0"], "ln1.0"), L["G1"])
    assert np.array_equal(porc.plain(L["G1"], "qkv.0"), L["QKV"])
    assert np.array_equal(porc.attention(L["QKV"]), L["ATT"])
    assert np.array_equal(porc.plain(L["ATT"], "proj.0"), L["At"])
    assert np.array_equal(porc.gauge(L["R0"], "ln2.0"), L["G2"])
    assert np.array_equal(porc.plain(L["G2"], "fc.0"), L["H"])
    assert np.array_equal(porc.plain(L["HE"], "mproj.0"), L["Mo"])


def test_pythia_c5_streams(porc, pgold):
    ids = np.random.default_rng(4).integers(0, V, (512, 64))
    for s, want in pgold["c5"].items():
        lg = porc.scores(ids[int(s)], 60, 64)
        assert [sha(r) for r in lg] == want["prompt_last4_sha"]
        tok, lgs = porc.generate(ids[int(s)][None, :], 4, logits=True)
        assert tok[0].tolist() == want["greedy"]
        assert [sha(r) for r in lgs[0]] == want["greedy_logits_sha"]
