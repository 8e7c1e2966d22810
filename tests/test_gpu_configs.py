"""Whole-job parity on the BASELINE configs: every stream, every generated word, and the digest of every score row the
word was raced on, against the oracle's (tests/golden/digests_*.npz, written by tests/golden/make_digests.py from the
CPU oracle, which test_oracle_golden.py and test_oracle_pythia.py pin to the reference's base2.py and
pythia_base2.py). A digest is the sum of score x key modulo 2^64 over the vocabulary with odd keys
(oracle.logit_hash), so any single differing score changes it.

Each decode config runs twice on the device: once with the scores stored every step (digests checked), once as the
benchmark runs it (b2_generate: the step's CUDA graph, the race folded into the head's epilogue, no scores stored;
words checked).
"""
import numpy as np
import pytest

from conftest import gload, with_streams

pytestmark = pytest.mark.gpu


def _prompts(d, vocab):
    return np.random.default_rng(int(d["seed"])).integers(0, vocab, (int(d["streams"]), int(d["prompt"])))


class Digest:
    def __init__(self, e):
        from oracle.oracle import logit_hash_keys
        self.keys = e.torch.from_numpy(logit_hash_keys(e.V).view(np.int64)).to(e.device)

    def __call__(self, lg):
        # int64 products and sums wrap modulo 2^64 on the device as in the oracle's uint64 arithmetic
        return (lg * self.keys).sum(dim=-1)


def _job(e, ids, words, dg):
    torch = e.torch
    first, lg = e.prefill_device(ids, logits=True)
    toks, hs = [first], [dg(lg)]
    for _ in range(words - 1):
        o, lg = e.step_device(n=len(ids), logits=True)
        toks.append(o)
        hs.append(dg(lg))
    tok = torch.stack(toks, 1).cpu().numpy()
    h = torch.stack(hs, 1).cpu().numpy().view(np.uint64)
    return tok, h


def _first_diff(a, b):
    bad = np.argwhere(a != b)
    return None if len(bad) == 0 else tuple(int(x) for x in bad[0])


def _check_config(e, name, vocab):
    d = gload(f"digests_{name}.npz")
    ids = _prompts(d, vocab)
    words = int(d["words"])
    e = with_streams(e, len(ids), ids.shape[1] + words)
    tok, h = _job(e, ids, words, Digest(e))
    assert _first_diff(tok, d["tokens"]) is None, f"{name}: first differing (stream, word) {_first_diff(tok, d['tokens'])}"
    assert _first_diff(h, d["hashes"]) is None, f"{name}: first differing score digest {_first_diff(h, d['hashes'])}"
    if words > 1:
        g = e.generate(ids, words)
        assert _first_diff(g, d["tokens"]) is None, f"{name} (graph, no scores): {_first_diff(g, d['tokens'])}"


def test_c2_every_stream_every_word(gpu_engine):
    """C2: 64 streams x 32-id prompts (seed 1), 128 words, key/value store to 160 positions."""
    _check_config(gpu_engine, "c2", 50257)


def test_c3_every_stream_every_word(gpu_engine):
    """C3: 16 streams x 960-id prompts (seed 2), 64 words: the store fills all 1,024 positions and power()'s
    int64 product wraps (base2.py:53)."""
    _check_config(gpu_engine, "c3", 50257)


def test_c4_prompt_pass_every_stream(gpu_engine):
    """C4: 32 streams x 512-id prompts (seed 3), the prompt pass: each stream's next word and last-position scores."""
    _check_config(gpu_engine, "c4", 50257)


def test_c5_every_stream_every_word(pythia_engine):
    """C5 (Pythia-160M): 512 streams x 64-id prompts (seed 4), 128 words, on one GPU."""
    _check_config(pythia_engine, "c5", 50304)


@pytest.mark.parametrize("world", [2, 8])
def test_c5_partitioned_shards(pythia_engine, world):
    """C5 split by stream as `bench.py --config c5 --gpus N` splits it: rank r takes streams [r 512/N, (r+1) 512/N).
    The first and last shard of N = 2 and 8 run here (on one GPU, in turn), each at its own, smaller batch, and give
    the single-GPU job's words for their streams."""
    from streaming_machine_b200.shard import partition
    d = gload("digests_c5.npz")
    ids = _prompts(d, 50304)
    words = int(d["words"])
    for rank in (0, world - 1):
        lo, hi = partition(len(ids), rank, world)
        e = with_streams(pythia_engine, hi - lo, ids.shape[1] + words)
        g = e.generate(ids[lo:hi], words)
        assert _first_diff(g, d["tokens"][lo:hi]) is None, (world, rank, _first_diff(g, d["tokens"][lo:hi]))
