"""b2_bank_noalloc (allocates nothing; its rows go to a fixed scratch area inside the library) against b2_bank.

Every bank mode, two calls in a row on the same scratch, bit-exact (integer results: the tolerance is zero). The
file name sorts last so that the test runs after every other GPU test as well as alone."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CASES = [("qkv.0", 0, 5), ("fc.3", 1, 64), ("mproj.7", 2, 33), ("proj.2", 3, 200), ("head", 0, 7)]


def _noalloc(e, name, X, out, mode):
    from streaming_machine_b200 import engine
    return engine.lib().b2_bank_noalloc(e.h, name.encode(), X.data_ptr(), X.shape[0], out.data_ptr(), mode,
                                        e._stream())


def _err(e):
    from streaming_machine_b200 import engine
    return engine.lib().b2_last_error(e.h).decode()


@pytest.mark.parametrize("name,mode,rows", CASES)
def test_noalloc_matches_bank_twice(gpu_engine, name, mode, rows):
    e, torch = gpu_engine, gpu_engine.torch
    nin = 3072 if name.startswith("mproj") else 768
    rng = np.random.default_rng(rows)
    Xs = [(rng.standard_normal((rows, nin)) * 2.0 ** (18 + k)).astype(np.int64) for k in range(2)]
    want = [e.bank(name, X, mode) for X in Xs]
    Xd = [torch.as_tensor(X).to(e.device) for X in Xs]
    outs = [torch.full(w.shape, -1, dtype=torch.int64, device=e.device) for w in want]
    for rnd in range(2):
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info(e.device)[0]
        for X, o in zip(Xd, outs):                      # two calls in a row, the second reusing the scratch
            assert _noalloc(e, name, X, o, mode) == 0, _err(e)
        e.sync()
        if rnd == 1:                                    # the first round may load code; the second allocates nothing
            assert torch.cuda.mem_get_info(e.device)[0] == free0
        for o, w in zip(outs, want):
            assert np.array_equal(o.cpu().numpy(), w)
        for o in outs:
            o.fill_(-1)


def test_noalloc_rejects_oversize(gpu_engine):
    """rows x (4 nin + 12) bytes past the fixed area: B2_ERR_ARG with the sizes in the message, nothing launched."""
    e, torch = gpu_engine, gpu_engine.torch
    X = torch.zeros((1400, 768), dtype=torch.int64, device=e.device)
    out = torch.zeros((1400, 768), dtype=torch.int64, device=e.device)
    assert _noalloc(e, "proj.0", X, out, 2) == 1
    assert "scratch" in _err(e) and "1400 rows" in _err(e)
    assert int(out.abs().sum()) == 0
