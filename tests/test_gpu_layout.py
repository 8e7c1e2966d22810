"""Layouts on the device: the tensor-core planes and corrections b2_finalize builds equal the ones computed on the host
(streaming_machine_b200/layout.py), and an engine made from the reference's device files (base2_gpu/, base2_gpu.py:9-17)
plus an uploaded tensor-core layout runs the reference's C1 words and scores."""
import numpy as np
import pytest

from conftest import gload

pytestmark = pytest.mark.gpu


def test_device_layout_equals_host_layout(gpu_engine, M):
    from streaming_machine_b200 import layout
    for name in ("qkv.0", "proj.7", "fc.11", "mproj.3", "head"):
        dev = gpu_engine.bank_layout(name)
        host = layout.tc_layout(M[name + ".w"])
        for k in ("wh", "wl", "cc", "cckb"):
            assert np.array_equal(dev[k], host[k]), (name, k)


def test_engine_from_reference_files_and_uploaded_layout(M, golden, tmp_path):
    from streaming_machine_b200 import engine, layout
    layout.write_gpu_dir(M, str(tmp_path))
    layout.write_tc_layout(M, str(tmp_path))
    R = layout.read_gpu_dir(str(tmp_path))
    e = engine.Engine(R, n_streams=1, max_ctx=32, layout=layout.read_tc_layout(str(tmp_path), R))
    try:
        g = gload("gpt2_logits_c1.npz")
        first, lg0 = e.prefill([g["ids"]], logits=True)
        toks, lgs = [int(first[0])], [lg0[0]]
        for _ in range(15):
            o, lg = e.step(n=1, logits=True)
            toks.append(int(o[0]))
            lgs.append(lg[0])
        assert toks == golden["c1"]["tokens"]
        assert np.array_equal(np.stack(lgs), g["logits"])
        assert np.array_equal(e.bank_layout("fc.4")["cckb"], layout.tc_layout(R["fc.4.w"])["cckb"])
    finally:
        e.close()
