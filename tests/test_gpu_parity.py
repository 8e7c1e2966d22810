"""Parity of the CUDA engine (through the C ABI) with the reference machine: bit-exact integers everywhere.

Expected values come from the reference's own base2.py (tests/golden) and, at sizes golden vectors do not cover,
from the CPU oracle (oracle/), itself pinned to those vectors by test_oracle_golden.py.
"""
import hashlib

import numpy as np
import pytest

from conftest import gload, with_streams

pytestmark = pytest.mark.gpu
V = 50257


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(np.asarray(a, dtype=np.int64)).tobytes()).hexdigest()


def test_banks_layer0(gpu_engine):
    """Each bank alone (base2.py:62-83) on the golden layer-0 inputs."""
    L = gload("gpt2_layer0.npz")
    e = with_streams(gpu_engine, 1, 64)
    assert np.array_equal(e.bank("qkv.0", L["R0"], 0), L["qkv"])
    assert np.array_equal(e.bank("fc.0", L["R1"], 1), L["hidE"])
    assert np.array_equal(L["R0"] + e.bank("proj.0", L["att"], 2), L["R1"])
    assert np.array_equal(L["R1"] + e.bank("mproj.0", L["hidE"], 2), L["R2"])


def test_bank_head_many_rows(gpu_engine, orc):
    """The head bank over 64 rows of a real residual stream, against the oracle."""
    rng = np.random.default_rng(5)
    R = (rng.standard_normal((64, 768)) * 2 ** 18).astype(np.int64)
    e = with_streams(gpu_engine, 64, 64)
    assert np.array_equal(e.bank("head", R, 0), orc.gauged_bank(R, "head"))


def test_c1_tokens_and_logits(gpu_engine, golden):
    """C1: 8 ids (seed 0), 16 greedy words; every logit integer equals base2.py's."""
    g = gload("gpt2_logits_c1.npz")
    e = with_streams(gpu_engine, 1, 64)
    first, lg0 = e.prefill([g["ids"]], logits=True)
    toks, lgs = [int(first[0])], [lg0[0]]
    for _ in range(15):
        o, lg = e.step(n=1, logits=True)
        toks.append(int(o[0]))
        lgs.append(lg[0])
    assert toks == golden["c1"]["tokens"]
    assert np.array_equal(np.stack(lgs), g["logits"])


def test_c2_batch64_logits_vs_oracle(gpu_engine, orc, golden):
    """C2's 64 streams (seed 1): 4 words each, all 64 x 4 logit rows equal the oracle's; golden streams equal base2.py."""
    ids = np.random.default_rng(1).integers(0, V, (64, 32))
    e = with_streams(gpu_engine, 64, 160)
    first, lg0 = e.prefill(ids, logits=True)
    toks, lgs = [first], [lg0]
    for _ in range(3):
        o, lg = e.step(logits=True)
        toks.append(o)
        lgs.append(lg)
    toks = np.stack(toks, 1)
    lgs = np.stack(lgs, 1)
    want_tok, want_lg = orc.generate(ids, 4, logits=True)
    assert np.array_equal(toks, want_tok)
    assert np.array_equal(lgs, want_lg)
    for s, want in golden["c2"].items():
        assert toks[int(s)].tolist() == want["tokens"]
        assert [sha(r) for r in lgs[int(s)]] == want["logits_sha"]


def test_c2_full_generation(gpu_engine, orc):
    """C2 in full: 64 streams x 128 greedy words (KV to 160); sampled streams checked word for word."""
    ids = np.random.default_rng(1).integers(0, V, (64, 32))
    e = with_streams(gpu_engine, 64, 160)
    toks = e.generate(ids, 128)
    assert toks.shape == (64, 128)
    sample = [0, 21, 63]
    want = orc.generate(ids[sample], 128)
    assert np.array_equal(toks[sample], want)


def test_device_feedback_equals_host_feedback(gpu_engine):
    """b2_generate's on-device feedback and b2_step_host's host round trip give the same words."""
    ids = np.random.default_rng(11).integers(0, V, (8, 12))
    e = with_streams(gpu_engine, 8, 64)
    a = e.generate(ids, 6)
    first = e.prefill(ids)
    got = [first]
    for _ in range(5):
        got.append(e.step_host(got[-1]))
    assert np.array_equal(a, np.stack(got, 1))


def test_rewind_replays_identically(gpu_engine):
    ids = np.random.default_rng(12).integers(0, V, (4, 10))
    e = with_streams(gpu_engine, 4, 64)
    first = e.prefill(ids)
    a = e.generate_device(4, 5).cpu().numpy()
    e.rewind([10] * 4, first)
    b = e.generate_device(4, 5).cpu().numpy()
    assert np.array_equal(a, b)


def test_ragged_prompts(gpu_engine, orc):
    rng = np.random.default_rng(13)
    prompts = [rng.integers(0, V, n) for n in (1, 5, 17, 2)]
    e = with_streams(gpu_engine, 4, 64)
    got = e.prefill(prompts)
    want = [orc.forward(p) for p in prompts]
    assert got.tolist() == want


def test_c4_prompt_pass(gpu_engine, orc, golden):
    """C4: 32 x 512-id prompt pass (seed 3); stream 0's last logits equal base2.py's, streams 1, 31 the oracle's."""
    ids = np.random.default_rng(3).integers(0, V, (32, 512))
    e = with_streams(gpu_engine, 32, 512)
    nxt, lg = e.prefill(ids, logits=True)
    assert sha(lg[0]) == golden["c4"]["logits_sha"][-1]
    assert int(nxt[0]) == golden["c4"]["next"][-1]
    for s in (1, 31):
        assert np.array_equal(lg[s], orc.scores(ids[s], 511, 512)[0])


def test_c3_long_context(gpu_engine, orc, golden):
    """C3: 960-id prompt (seed 2), then greedy to the 1024-position limit; power()'s int64 wrap must match."""
    ids = np.random.default_rng(2).integers(0, V, (16, 960))[:2]
    e = with_streams(gpu_engine, 2, 1024)
    nxt, lg = e.prefill(ids, logits=True)
    assert sha(lg[0]) == golden["c3"]["logits_sha"][-1]
    assert int(nxt[0]) == golden["c3"]["next"][-1]
    rest = e.generate_device(2, 63).cpu().numpy()
    toks = np.concatenate([nxt[:, None], rest], 1)
    assert np.array_equal(toks[1], orc.generate(ids[1:2], 64)[0])


def test_context_overflow_is_reported(gpu_engine):
    from streaming_machine_b200.engine import B2Error
    ids = np.random.default_rng(14).integers(0, V, (1, 8))
    e = with_streams(gpu_engine, 1, 8)
    e.prefill(ids)
    with pytest.raises(B2Error) as ei:
        e.step()
    assert ei.value.code == 4
    e.sync()


def test_bad_token_is_reported(gpu_engine):
    from streaming_machine_b200.engine import B2Error
    e = with_streams(gpu_engine, 1, 16)
    e.prefill([[1, 2, 3]])
    with pytest.raises(B2Error) as ei:
        e.step([V + 5])
    assert ei.value.code == 7
    e.sync()


def test_launch_count_and_profile(gpu_engine):
    ids = np.random.default_rng(15).integers(0, V, (4, 6))
    e = with_streams(gpu_engine, 4, 16)
    e.prefill(ids)
    e.profile(True)
    e.generate_device(4, 2)
    n, by = e.profile_read()
    e.profile(False)
    assert n == sum(c for c, _ in by.values()) and n >= 2 * 60
    assert by["bank"][0] == 2 * 49 and by["bank"][1] > 0
