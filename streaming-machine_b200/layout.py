"""Device layouts on disk: the reference's GPU file layout, and the engine's tensor-core layout computed ahead of time.

The reference lays the converted machine out for its GPU engine with base2_gpu.py (reference base2_gpu.py:9-17): a
directory with, per bank, `<name>.wc` (int16 [nin][nout], input-major), `<name>.e` (int32 [nout]) and `<name>.b`
(int64 [nout]); the tables `wte, wpe, phi, arrival, log2, exp2` as int64 `<key>.bin`; and `manifest.json` with the
banks' names and shapes, `log2_768`, `eps40` and `arrival_len`.

    from streaming_machine_b200 import convert, layout, engine
    layout.write_gpu_dir(convert.load_gpt2(0), "base2_gpu")          # the reference's files, from our converter
    M = layout.read_gpu_dir("base2_gpu")                              # the reference's files -> the npz keys
    layout.write_tc_layout(M, "base2_gpu")                            # + the tensor-core planes, once
    eng = engine.Engine(M, layout=layout.read_tc_layout("base2_gpu", M))   # finalize uploads them, builds nothing

The tensor-core layout of a bank (what b2_finalize otherwise builds on the device) is a function of its int16 weights
alone: the byte planes wh = w >> 8 and wl = (w & 255) - 128, K-major [nout_pad][nin] with nout_pad = nout rounded up
to 128 (padded outputs have w = 0), and the column corrections 128 sum_i w[i][j] - 16384 nin, whole and per
128-input block (include/base2.h, b2_set_bank_layout). Its files, `<name>.wh`, `<name>.wl` (int8), `<name>.cc`,
`<name>.cckb` (int64), sit beside the reference's, listed in `tc_layout.json` with a sha256 of the bank's weights so
a layout is never paired with other weights.
"""
from __future__ import annotations

import hashlib
import json
import os

import numpy as np

GPT2_TABLES = ("wte", "wpe", "phi", "arrival", "log2", "exp2")


def bank_names(n_layer: int = 12):
    return [f"{b}.{l}" for l in range(n_layer) for b in ("qkv", "proj", "fc", "mproj")] + ["head"]


def _n_layer(M) -> int:
    return sum(1 for k in M if k.startswith("qkv.") and k.endswith(".w"))


# ---------------------------------------------------------------------------------------------------------------------
# the reference's layout (base2_gpu.py)
# ---------------------------------------------------------------------------------------------------------------------
def write_gpu_dir(M: dict, out: str) -> str:
    """GPT-2 arrays (keys of base2_gpt2.npz) in the reference's base2_gpu/ layout (base2_gpu.py:9-17)."""
    os.makedirs(out, exist_ok=True)
    man = []
    for name in bank_names(_n_layer(M)):
        w = np.ascontiguousarray(M[name + ".w"])
        nin, nout = w.shape
        w.astype(np.int16).tofile(os.path.join(out, f"{name}.wc"))
        np.asarray(M[name + ".e"]).astype(np.int32).tofile(os.path.join(out, f"{name}.e"))
        np.asarray(M[name + ".b"]).astype(np.int64).tofile(os.path.join(out, f"{name}.b"))
        man.append(dict(name=name, nin=int(nin), nout=int(nout)))
    for k in GPT2_TABLES:
        np.asarray(M[k]).astype(np.int64).tofile(os.path.join(out, f"{k}.bin"))
    with open(os.path.join(out, "manifest.json"), "w") as f:
        json.dump(dict(banks=man, log2_768=int(np.asarray(M["log2_768"]).reshape(-1)[0]),
                       eps40=int(np.asarray(M["eps40"]).reshape(-1)[0]), arrival_len=int(len(M["arrival"]))), f)
    return out


def read_gpu_dir(path: str, d_model: int | None = None) -> dict:
    """The reference's base2_gpu/ directory back as the converter's npz keys (what engine.Engine takes). The tables are
    flat int64 files; wte and wpe are reshaped by the model width (the qkv banks' input count unless given)."""
    with open(os.path.join(path, "manifest.json")) as f:
        man = json.load(f)
    M = {}
    for b in man["banks"]:
        name, nin, nout = b["name"], int(b["nin"]), int(b["nout"])
        w = np.fromfile(os.path.join(path, f"{name}.wc"), dtype=np.int16)
        if w.size != nin * nout:
            raise ValueError(f"{name}.wc holds {w.size} values, the manifest says {nin} x {nout}")
        M[name + ".w"] = w.reshape(nin, nout)
        M[name + ".e"] = np.fromfile(os.path.join(path, f"{name}.e"), dtype=np.int32).astype(np.int64)
        M[name + ".b"] = np.fromfile(os.path.join(path, f"{name}.b"), dtype=np.int64)
        if len(M[name + ".e"]) != nout or len(M[name + ".b"]) != nout:
            raise ValueError(f"{name}: exponents or biases do not match {nout} outputs")
    d = d_model or M["qkv.0.w"].shape[0]
    for k in GPT2_TABLES:
        t = np.fromfile(os.path.join(path, f"{k}.bin"), dtype=np.int64)
        M[k] = t.reshape(-1, d) if k in ("wte", "wpe") else t
    if len(M["arrival"]) != int(man["arrival_len"]):
        raise ValueError("arrival.bin does not match the manifest's arrival_len")
    M["log2_768"] = np.int64(man["log2_768"])
    M["eps40"] = np.int64(man["eps40"])
    return M


# ---------------------------------------------------------------------------------------------------------------------
# the tensor-core layout, computed on the host
# ---------------------------------------------------------------------------------------------------------------------
def tc_layout(w) -> dict:
    """One bank's tensor-core layout from its int16 weights [nin][nout] (exactly what b2_finalize builds)."""
    w = np.ascontiguousarray(w, dtype=np.int16)
    nin, nout = w.shape
    if nin % 128:
        raise ValueError("the tensor-core layout needs a multiple of 128 inputs")
    pad = (nout + 127) // 128 * 128
    wt = np.zeros((pad, nin), np.int16)
    wt[:nout] = w.T
    wh = (wt >> 8).astype(np.int8)
    wl = ((wt & 255) - 128).astype(np.int8)
    w64 = w.astype(np.int64)
    cc = np.zeros(pad, np.int64)
    cc[:nout] = 128 * w64.sum(0) - 16384 * nin
    cckb = np.zeros((nin // 128, pad), np.int64)
    cckb[:, :nout] = 128 * w64.reshape(nin // 128, 128, nout).sum(1) - 16384 * 128
    return dict(wh=wh, wl=wl, cc=cc, cckb=cckb)


def _wdigest(w) -> str:
    return hashlib.sha256(np.ascontiguousarray(w, dtype=np.int16).tobytes()).hexdigest()


def write_tc_layout(M: dict, out: str) -> str:
    """Every bank's tensor-core layout into `out` (beside the reference's files), with tc_layout.json."""
    os.makedirs(out, exist_ok=True)
    index = {}
    for name in bank_names(_n_layer(M)):
        t = tc_layout(M[name + ".w"])
        for k, ext in (("wh", "wh"), ("wl", "wl"), ("cc", "cc"), ("cckb", "cckb")):
            t[k].tofile(os.path.join(out, f"{name}.{ext}"))
        nin, nout = M[name + ".w"].shape
        index[name] = dict(nin=int(nin), nout=int(nout), nout_pad=int(t["wh"].shape[0]), w_sha256=_wdigest(M[name + ".w"]))
    with open(os.path.join(out, "tc_layout.json"), "w") as f:
        json.dump(index, f, indent=1)
    return out


def read_tc_layout(path: str, M: dict) -> dict:
    """The tensor-core layout files of `path` for the banks of M: {bank: {wh, wl, cc, cckb}}. A bank whose weights do
    not match the layout's sha256 is an error (ValueError)."""
    with open(os.path.join(path, "tc_layout.json")) as f:
        index = json.load(f)
    out = {}
    for name in bank_names(_n_layer(M)):
        ent = index.get(name)
        if ent is None:
            raise ValueError(f"no tensor-core layout for {name}")
        if ent["w_sha256"] != _wdigest(M[name + ".w"]):
            raise ValueError(f"{name}: the layout was made from other weights")
        nin, pad = int(ent["nin"]), int(ent["nout_pad"])
        out[name] = dict(
            wh=np.fromfile(os.path.join(path, f"{name}.wh"), dtype=np.int8).reshape(pad, nin),
            wl=np.fromfile(os.path.join(path, f"{name}.wl"), dtype=np.int8).reshape(pad, nin),
            cc=np.fromfile(os.path.join(path, f"{name}.cc"), dtype=np.int64),
            cckb=np.fromfile(os.path.join(path, f"{name}.cckb"), dtype=np.int64).reshape(nin // 128, pad))
    return out
