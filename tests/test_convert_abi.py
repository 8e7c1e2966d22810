"""CPU checks of the conversion, the C ABI's exports and the host logic (no GPU work)."""
import ctypes
import hashlib
import os
import re

import numpy as np
import pytest

from conftest import ROOT


def _digest(v):
    v = np.asarray(v)
    if v.dtype == np.int16:
        return hashlib.sha256(np.ascontiguousarray(v).tobytes()).hexdigest()
    return hashlib.sha256(np.ascontiguousarray(v.astype(np.int64)).tobytes()).hexdigest()


def test_converter_matches_reference_converter(M, golden):
    """Our restated base2_convert.py gives the reference converter's arrays bit for bit (seed 0)."""
    assert golden["converter_mismatches"] == {}
    ref = golden["reference_digests"]
    assert set(ref) == set(M)
    bad = [k for k in ref if _digest(M[k]) != ref[k]]
    assert bad == []


def test_tables_shape(M):
    assert len(M["arrival"]) == 17745 and M["arrival"][0] == 1 << 24
    assert M["phi"].max() == 65536 and M["exp2"].min() == 65536 and M["exp2"].max() == 131071
    assert all(abs(int(M[f"{b}.0.w"].astype(np.int64).__abs__().max())) <= 32767 for b in ("qkv", "proj", "fc", "mproj"))


def _declared():
    src = open(os.path.join(ROOT, "include", "base2.h")).read()
    return sorted(set(re.findall(r"\b(b2_[a-z_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    from streaming_machine_b200 import build, engine
    lib = ctypes.CDLL(build.build())
    names = _declared()
    assert set(names) == set(engine.EXPORTS)
    for n in names:
        assert hasattr(lib, n), n
    assert lib.b2_abi_version() == 1


def test_library_is_sm100a():
    """The shared library carries sm_100a code (nvcc -gencode arch=compute_100a,code=sm_100a)."""
    from streaming_machine_b200 import build
    assert "arch=compute_100a,code=sm_100a" in " ".join(build.ARCH)
    assert os.path.getsize(build.build()) > 100_000


def test_errors_without_gpu_are_loud():
    """No CPU fallback: building an engine without a CUDA device raises."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from streaming_machine_b200 import engine
    with pytest.raises(RuntimeError):
        engine.Engine({"wte": np.zeros((1, 768))})


def test_create_rejects_bad_config():
    """b2_create validates its config on the host before touching a device."""
    from streaming_machine_b200 import engine
    L = engine.lib()
    cfg = engine.Config(0, 12, 770, 12, 3072, 50257, 1024)      # d_model not 64 x heads
    h = ctypes.c_void_p()
    assert L.b2_create(ctypes.byref(cfg), 0, 0, ctypes.byref(h)) == 1 and not h.value
    cfg = engine.Config(0, 12, 768, 12, 3072, 50257, 1024)
    assert L.b2_create(ctypes.byref(cfg), 0, 8, ctypes.byref(h)) == 1   # turn=float is Pythia's switch only
    cfg = engine.Config(2, 12, 768, 12, 3072, 50257, 1024)
    assert L.b2_create(ctypes.byref(cfg), 0, 0, ctypes.byref(h)) == 1   # unknown model kind
