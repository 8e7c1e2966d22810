"""The device layouts on disk (streaming_machine_b200/layout.py): the reference's base2_gpu/ files (base2_gpu.py:9-17)
written from the converter and read back to the same arrays, and the tensor-core layout computed on the host, whose
byte planes give back every weight (w = 256 wh + wl + 128) and whose corrections are the weights' sums."""
import json
import os

import numpy as np
import pytest


def test_gpu_dir_round_trip(M, tmp_path):
    from streaming_machine_b200 import layout
    layout.write_gpu_dir(M, str(tmp_path))
    man = json.load(open(os.path.join(tmp_path, "manifest.json")))
    assert len(man["banks"]) == 49 and man["arrival_len"] == len(M["arrival"])
    assert man["banks"][0] == {"name": "qkv.0", "nin": 768, "nout": 2304}
    R = layout.read_gpu_dir(str(tmp_path))
    for k, v in M.items():
        if k in R:
            assert np.array_equal(np.asarray(R[k]).reshape(np.shape(v)), np.asarray(v)), k
    assert set(k for k in M if k.split(".")[-1] in ("w", "e", "b") or k in layout.GPT2_TABLES) <= set(R)


def test_gpu_dir_rejects_bad_shapes(M, tmp_path):
    from streaming_machine_b200 import layout
    layout.write_gpu_dir(M, str(tmp_path))
    with open(os.path.join(tmp_path, "proj.3.wc"), "ab") as f:
        f.write(b"\0\0")
    with pytest.raises(ValueError):
        layout.read_gpu_dir(str(tmp_path))


def test_tc_layout_identity():
    from streaming_machine_b200 import layout
    rng = np.random.default_rng(8)
    w = rng.integers(-32767, 32768, (256, 200)).astype(np.int16)
    w[0, :3] = (-32767, 32767, 0)
    t = layout.tc_layout(w)
    assert t["wh"].shape == (256, 256) and t["cckb"].shape == (2, 256)
    back = 256 * t["wh"].astype(np.int64) + t["wl"].astype(np.int64) + 128
    assert np.array_equal(back[:200].T, w.astype(np.int64)) and (back[200:] == 0).all()
    assert np.array_equal(t["cc"][:200], 128 * w.astype(np.int64).sum(0) - 16384 * 256)
    assert np.array_equal(t["cckb"].sum(0)[:200], t["cc"][:200])
    assert (t["cc"][200:] == 0).all() and (t["cckb"][:, 200:] == 0).all()


def test_tc_layout_files_checked_against_weights(M, tmp_path):
    from streaming_machine_b200 import layout
    small = {k: v for k, v in M.items()}
    layout.write_tc_layout(small, str(tmp_path))
    got = layout.read_tc_layout(str(tmp_path), small)
    ref = layout.tc_layout(M["proj.5.w"])
    assert all(np.array_equal(got["proj.5"][k], ref[k]) for k in ref)
    other = dict(small)
    w = M["fc.2.w"].copy()
    w[0, 0] ^= 1
    other["fc.2.w"] = w
    with pytest.raises(ValueError):
        layout.read_tc_layout(str(tmp_path), other)
