"""The tensor-core bank product (hi/lo int8 planes on tcgen05) against the oracle's exact int64 product.

Row counts cover one row, a partial tile, exactly one 64-row tile (split-K path), 65 rows (two tiles, 128-row
tiles), several tiles, and inputs that round to +32768 (17-bit activations, the correction list) and -32768.
"""
import numpy as np
import pytest

from conftest import with_streams

pytestmark = pytest.mark.gpu


def rows_with_extremes(rng, rows, n):
    X = (rng.standard_normal((rows, n)) * 2 ** 16).astype(np.int64)
    X = np.clip(X, -(2 ** 19), 2 ** 19)
    k = max(1, rows // 3)
    X[:k, 5] = 2 ** 20 - 1            # top bit 20 -> shift 5 -> +32768
    X[:k, n - 3] = 2 ** 20 - 1        # two of them in a row
    X[k:2 * k, 9] = -(2 ** 20 - 1)    # -> -32768
    return X


@pytest.mark.parametrize("rows", [1, 7, 64, 65, 200, 777])
@pytest.mark.parametrize("bank,mode", [("qkv.3", 0), ("fc.5", 1), ("proj.2", 2), ("mproj.7", 2)])
def test_bank_vs_oracle(gpu_engine, orc, bank, mode, rows):
    e = with_streams(gpu_engine, 1, 64)
    nin = orc.M[bank + ".w"].shape[0]
    X = rows_with_extremes(np.random.default_rng(rows * 31 + nin), rows, nin)
    got = e.bank(bank, X, mode)
    if mode == 0:
        want = orc.gauged_bank(X, bank)
    elif mode == 1:
        want = orc.edge(orc.gauged_bank(X, bank))
    else:
        want = orc.plain_bank(X, bank)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("rows", [1, 64, 130])
def test_head_vs_oracle(gpu_engine, orc, rows):
    e = with_streams(gpu_engine, 1, 64)
    X = rows_with_extremes(np.random.default_rng(rows), rows, 768)
    assert np.array_equal(e.bank("head", X, 0), orc.gauged_bank(X, "head"))


def test_repeat_is_deterministic(gpu_engine):
    """Split-K partial piles are summed across a cluster: the integers must not change between calls."""
    e = with_streams(gpu_engine, 1, 64)
    X = rows_with_extremes(np.random.default_rng(3), 64, 3072)
    a = e.bank("mproj.0", X, 2)
    b = e.bank("mproj.0", X, 2)
    assert np.array_equal(a, b)


def test_all_saturated_row(gpu_engine, orc):
    """A row whose every entry rounds to +32768 (the correction touches all 768 weights of every column)."""
    e = with_streams(gpu_engine, 1, 64)
    X = np.full((3, 768), 2 ** 20 - 1, dtype=np.int64)
    X[1] = -(2 ** 20 - 1)
    X[2, ::2] = 2 ** 20 - 1
    X[2, 1::2] = 5
    for bank, mode in (("qkv.0", 0), ("proj.0", 2)):
        assert np.array_equal(e.bank(bank, X, mode), orc.gauged_bank(X, bank) if mode == 0 else orc.plain_bank(X, bank))
