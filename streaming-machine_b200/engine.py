"""Host side of the CUDA engine: the reference machine's interface (base2.py) over the C ABI of libbase2cuda.so.

    from streaming_machine_b200 import convert, engine
    M = convert.load_gpt2(seed=0)                     # arrays keyed like base2_gpt2.npz (or base2_pythia-160m.npz)
    eng = engine.Engine(M, n_streams=64, max_ctx=160)
    first = eng.prefill(prompts)                      # the race's word after each prompt  (base2_stream.swift:274-275)
    nxt = eng.step()                                  # one new position per stream        (base2_stream.swift:276-280)
    eng.forward(ids)                                  # base2.py:102-114: the word after ids

PyTorch supplies device memory and the CUDA stream only; every computation runs in the library's sm_100a kernels.
There is no CPU path: without a CUDA device or without the library the constructor raises.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import build as _build

B2_GPT2, B2_PYTHIA = 0, 1
B2_GAUGE_FLOAT, B2_EDGE_FLOAT, B2_ARRIVAL_FLOAT, B2_TURN_FLOAT = 1, 2, 4, 8
STATUS = {0: "OK", 1: "ERR_ARG", 2: "ERR_CUDA", 3: "ERR_NOMEM", 4: "ERR_CTX", 5: "ERR_VALUE", 6: "ERR_STATE",
          7: "ERR_DEVICE"}

# every symbol include/base2.h declares
EXPORTS = ("b2_create", "b2_set_bank", "b2_set_array", "b2_set_scalar", "b2_finalize", "b2_alloc_streams",
           "b2_prefill", "b2_step", "b2_generate", "b2_step_host", "b2_bank", "b2_gauge", "b2_bank_noalloc",
           "b2_rewind", "b2_profile", "b2_profile_read", "b2_sync", "b2_check_wait", "b2_set_bank_layout",
           "b2_get_bank_layout", "b2_last_error", "b2_destroy", "b2_abi_version")
PROF_CLASSES = ("bank", "attend", "quant", "heads", "race", "other")


class B2Error(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{STATUS.get(code, code)}: {msg}")
        self.code = code


class Config(ctypes.Structure):
    _fields_ = [(k, ctypes.c_int32) for k in ("kind", "n_layer", "d_model", "n_head", "d_ff", "vocab", "n_ctx")]


_lib = None


def lib():
    """Load (building first if stale) libbase2cuda.so and declare its signatures."""
    global _lib
    if _lib is None:
        L = ctypes.CDLL(_build.build())
        vp, i32, i64, cp = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_char_p
        L.b2_create.argtypes = [ctypes.POINTER(Config), ctypes.c_int, ctypes.c_int, ctypes.POINTER(vp)]
        L.b2_set_bank.argtypes = [vp, cp, vp, vp, vp, i32, i32]
        L.b2_set_array.argtypes = [vp, cp, vp, i64]
        L.b2_set_scalar.argtypes = [vp, cp, i64]
        L.b2_finalize.argtypes = [vp]
        L.b2_alloc_streams.argtypes = [vp, i32, i32]
        L.b2_prefill.argtypes = [vp, vp, vp, i32, vp, vp, vp]
        L.b2_step.argtypes = [vp, vp, i32, vp, vp, vp]
        L.b2_generate.argtypes = [vp, i32, i32, vp, vp]
        L.b2_step_host.argtypes = [vp, vp, i32, vp]
        L.b2_bank.argtypes = [vp, cp, vp, i32, vp, i32, vp]
        L.b2_gauge.argtypes = [vp, cp, vp, i32, vp, vp]
        L.b2_bank_noalloc.argtypes = [vp, cp, vp, i32, vp, i32, vp]
        L.b2_rewind.argtypes = [vp, i32, vp, vp, vp]
        L.b2_profile.argtypes = [vp, ctypes.c_int]
        L.b2_profile_read.argtypes = [vp, vp, vp, vp]
        L.b2_sync.argtypes = [vp]
        L.b2_check_wait.argtypes = [vp, vp]
        L.b2_set_bank_layout.argtypes = [vp, cp, vp, vp, vp, vp]
        L.b2_get_bank_layout.argtypes = [vp, cp, vp, vp, vp, vp]
        L.b2_last_error.argtypes = [vp]
        L.b2_last_error.restype = cp
        L.b2_destroy.argtypes = [vp]
        L.b2_destroy.restype = None
        for f in EXPORTS:
            if f not in ("b2_last_error", "b2_destroy"):
                getattr(L, f).restype = ctypes.c_int
        _lib = L
    return _lib


def _torch():
    import torch
    if not torch.cuda.is_available():
        raise RuntimeError("the base2 CUDA engine needs a CUDA device (there is no CPU path)")
    return torch


def _scalar(M, k) -> int:
    return int(np.asarray(M[k]).reshape(-1)[0])


class Engine:
    """The integer GPT-2 machine (base2.py) or its Pythia variant (foundation0/pythia_base2.py, chosen when M holds
    Pythia's "embed.w") on one GPU, with `n_streams` independent streams of up to `max_ctx` positions."""

    def __init__(self, M: dict, device: int = 0, n_streams: int = 1, max_ctx: int = 1024,
                 gauge: str = "int", edge: str = "int", arrival: str = "int", turn: str = "int", layout: dict | None = None):
        """gauge=/edge=/arrival= "float" (and Pythia's turn=) put that stage back to float64, as the reference's
        switches do (base2.py:10-11, pythia_base2.py:20). layout: the banks' tensor-core layouts computed ahead of time
        ({bank: {wh, wl, cc, cckb}}, streaming_machine_b200.layout.read_tc_layout), uploaded instead of built."""
        torch = _torch()
        self.torch = torch
        self.device = torch.device("cuda", device)
        flags = (B2_GAUGE_FLOAT if gauge == "float" else 0) | (B2_EDGE_FLOAT if edge == "float" else 0) | \
                (B2_ARRIVAL_FLOAT if arrival == "float" else 0) | (B2_TURN_FLOAT if turn == "float" else 0)
        self.flags = flags
        self.pythia = "embed.w" in M
        n_layer = sum(1 for k in M if k.startswith("qkv.") and k.endswith(".w"))
        if self.pythia:
            d = int(M["embed.w"].shape[1])
            if _scalar(M, "hs") != 64 or _scalar(M, "heads") * 64 != d:
                raise ValueError("the engine takes heads of 64 dims")
            self.cfg = Config(B2_PYTHIA, n_layer, d, d // 64, int(M["fc.0.w"].shape[1]), int(M["head.w"].shape[1]),
                              int(M["cos"].shape[0]))
        else:
            d = int(M["wte"].shape[1])
            self.cfg = Config(B2_GPT2, n_layer, d, d // 64, int(M["fc.0.w"].shape[1]), int(M["head.w"].shape[1]),
                              int(M["wpe"].shape[0]))
        self.V = self.cfg.vocab
        L = lib()
        h = ctypes.c_void_p()
        self._check(L.b2_create(ctypes.byref(self.cfg), device, flags, ctypes.byref(h)), None)
        self.h = h
        for name in [f"{b}.{l}" for l in range(n_layer) for b in ("qkv", "proj", "fc", "mproj")] + ["head"]:
            w = np.ascontiguousarray(M[name + ".w"], dtype=np.int16)
            e = np.ascontiguousarray(M[name + ".e"], dtype=np.int64)
            b = np.ascontiguousarray(M[name + ".b"], dtype=np.int64) if name + ".b" in M else None   # Pythia's head
            self._call("b2_set_bank", h, name.encode(), w.ctypes.data, e.ctypes.data,
                       b.ctypes.data if b is not None else None, w.shape[0], w.shape[1])
            if layout is not None:
                t = layout[name]
                arrs = [np.ascontiguousarray(t[k], dtype=dt) for k, dt in
                        (("wh", np.int8), ("wl", np.int8), ("cc", np.int64), ("cckb", np.int64))]
                self._call("b2_set_bank_layout", h, name.encode(), *[a.ctypes.data for a in arrs])
        if self.pythia:
            norms = [f"ln{i}.{l}" for l in range(n_layer) for i in (1, 2)] + ["lnf"]
            arrays = ["embed.w", "embed.e", "cos", "sin", "phi", "arrival", "log2", "exp2"] + \
                     [f"{n}.{p}" for n in norms for p in ("g", "b")]
            scalars = ["eps40", "half_log2_hs", "rot"] + [f"{n}.ge" for n in norms]
        else:
            arrays = ["wte", "wpe", "phi", "arrival", "log2", "exp2"]
            scalars = ["log2_768", "eps40"]
        for k in arrays:
            a = np.ascontiguousarray(M[k], dtype=np.int64)
            self._call("b2_set_array", h, k.encode(), a.ctypes.data, a.size)
        for k in scalars:
            self._call("b2_set_scalar", h, k.encode(), _scalar(M, k))
        self._call("b2_finalize", h)
        self.n_streams, self.max_ctx = 0, 0
        self.alloc_streams(n_streams, max_ctx)

    # ---- plumbing ---------------------------------------------------------------------------------------------
    def _check(self, rc: int, h):
        if rc:
            msg = lib().b2_last_error(h).decode() if h else "b2_create failed"
            raise B2Error(rc, msg)

    def _call(self, fn: str, *args):
        self._check(getattr(lib(), fn)(*args), self.h)

    def _stream(self):
        return ctypes.c_void_p(self.torch.cuda.current_stream(self.device).cuda_stream)

    def _i32(self, a):
        return self.torch.as_tensor(np.ascontiguousarray(a, dtype=np.int32)).to(self.device)

    def close(self):
        if getattr(self, "h", None):
            lib().b2_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- streams ----------------------------------------------------------------------------------------------
    def alloc_streams(self, n_streams: int, max_ctx: int):
        self._call("b2_alloc_streams", self.h, n_streams, max_ctx)
        self.n_streams, self.max_ctx = n_streams, max_ctx

    def prefill(self, prompts, logits: bool = False):
        """Prompt pass for streams 0..len(prompts)-1; returns the race's word after each prompt (and the scores)."""
        prompts = [list(map(int, p)) for p in prompts]
        n = len(prompts)
        ids = self._i32(np.concatenate([np.asarray(p, np.int32) for p in prompts]))
        lens = self._i32([len(p) for p in prompts])
        nxt = self.torch.empty(n, dtype=self.torch.int32, device=self.device)
        lg = self.torch.empty((n, self.V), dtype=self.torch.int64, device=self.device) if logits else None
        self._call("b2_prefill", self.h, ids.data_ptr(), lens.data_ptr(), n, nxt.data_ptr(),
                   lg.data_ptr() if logits else None, self._stream())
        out = nxt.cpu().numpy()
        return (out, lg.cpu().numpy()) if logits else out

    def step(self, tokens=None, n: int | None = None, logits: bool = False):
        """One new position per stream; tokens=None feeds back each stream's last word on the device."""
        n = n if n is not None else (len(tokens) if tokens is not None else self.n_streams)
        tin = self._i32(tokens) if tokens is not None else None
        out = self.torch.empty(n, dtype=self.torch.int32, device=self.device)
        lg = self.torch.empty((n, self.V), dtype=self.torch.int64, device=self.device) if logits else None
        self._call("b2_step", self.h, tin.data_ptr() if tin is not None else None, n, out.data_ptr(),
                   lg.data_ptr() if logits else None, self._stream())
        self._call("b2_sync", self.h)
        o = out.cpu().numpy()
        return (o, lg.cpu().numpy()) if logits else o

    def prefill_device(self, prompts, logits: bool = False):
        """prefill() with the words (and scores) left on the device as torch tensors."""
        prompts = [list(map(int, p)) for p in prompts]
        n = len(prompts)
        ids = self._i32(np.concatenate([np.asarray(p, np.int32) for p in prompts]))
        lens = self._i32([len(p) for p in prompts])
        nxt = self.torch.empty(n, dtype=self.torch.int32, device=self.device)
        lg = self.torch.empty((n, self.V), dtype=self.torch.int64, device=self.device) if logits else None
        self._call("b2_prefill", self.h, ids.data_ptr(), lens.data_ptr(), n, nxt.data_ptr(),
                   lg.data_ptr() if logits else None, self._stream())
        return nxt, lg

    def step_device(self, n: int | None = None, logits: bool = False):
        """One new position for streams 0..n-1 with each stream's last word fed back on the device; the words (and
        scores) as torch tensors on the device, nothing copied to the host."""
        n = n if n is not None else self.n_streams
        out = self.torch.empty(n, dtype=self.torch.int32, device=self.device)
        lg = self.torch.empty((n, self.V), dtype=self.torch.int64, device=self.device) if logits else None
        self._call("b2_step", self.h, None, n, out.data_ptr(), lg.data_ptr() if logits else None, self._stream())
        return out, lg

    def generate_device(self, n: int, n_steps: int, out=None):
        """n_steps decode steps with on-device feedback; returns the [n, n_steps] int32 device tensor."""
        out = out if out is not None else self.torch.empty((n, n_steps), dtype=self.torch.int32, device=self.device)
        self._call("b2_generate", self.h, n, n_steps, out.data_ptr(), self._stream())
        return out

    def generate(self, prompts, n_new: int):
        """Greedy words for each prompt (base2.py:122-123): [len(prompts), n_new]."""
        first = self.prefill(prompts)
        if n_new <= 1:
            return first[:, None][:, :n_new]
        rest = self.generate_device(len(prompts), n_new - 1)
        self._call("b2_sync", self.h)
        return np.concatenate([first[:, None], rest.cpu().numpy()], axis=1)

    def step_host(self, tokens):
        """b2_step_host: host buffers in and out (the end-to-end path)."""
        tin = np.ascontiguousarray(tokens, dtype=np.int32)
        out = np.empty_like(tin)
        self._call("b2_step_host", self.h, tin.ctypes.data, len(tin), out.ctypes.data)
        return out

    def forward(self, ids) -> int:
        """base2.py:102-114: the word after ids (uses stream slot 0)."""
        return int(self.prefill([ids])[0])

    def bank(self, name: str, X, mode: int = 0):
        """One bank on rows X (base2.py:62-76): mode 0 gauged, 1 gauged + edge, 2 plain, 3 plain + edge
        (Pythia's fc, pythia_base2.py:166)."""
        X = self.torch.as_tensor(np.ascontiguousarray(X, dtype=np.int64)).to(self.device)
        nout = {"qkv": 3, "proj": 1, "fc": 4, "mproj": 1}.get(name.split(".")[0], None)
        nout = self.V if name == "head" else nout * self.cfg.d_model
        out = self.torch.empty((X.shape[0], nout), dtype=self.torch.int64, device=self.device)
        self._call("b2_bank", self.h, name.encode(), X.data_ptr(), X.shape[0], out.data_ptr(), mode, self._stream())
        self._call("b2_sync", self.h)
        return out.cpu().numpy()

    def gauge(self, name: str, X):
        """Pythia's layer norm on rows X (pythia_base2.py:100-110): name "ln1.<l>", "ln2.<l>" or "lnf"."""
        X = self.torch.as_tensor(np.ascontiguousarray(X, dtype=np.int64)).to(self.device)
        out = self.torch.empty_like(X)
        self._call("b2_gauge", self.h, name.encode(), X.data_ptr(), X.shape[0], out.data_ptr(), self._stream())
        self._call("b2_sync", self.h)
        return out.cpu().numpy()

    def rewind(self, lens, last_tok):
        """Truncate streams back to `lens` positions, `last_tok` fed next (device tensors or arrays)."""
        lens = lens if hasattr(lens, "data_ptr") else self._i32(lens)
        last_tok = last_tok if hasattr(last_tok, "data_ptr") else self._i32(last_tok)
        self._call("b2_rewind", self.h, int(lens.numel()), lens.data_ptr(), last_tok.data_ptr(), self._stream())

    def profile(self, timing: bool):
        self._call("b2_profile", self.h, int(timing))

    def profile_read(self):
        """(total launches, {class: (launches, ms)}) since the last profile() reset."""
        n = np.zeros(1, np.int64)
        cnt = np.zeros(len(PROF_CLASSES), np.int64)
        ms = np.zeros(len(PROF_CLASSES), np.float64)
        self._call("b2_profile_read", self.h, n.ctypes.data, cnt.ctypes.data, ms.ctypes.data)
        return int(n[0]), {k: (int(c), float(t)) for k, c, t in zip(PROF_CLASSES, cnt, ms)}

    def sync(self):
        self._call("b2_sync", self.h)

    def bank_layout(self, name: str) -> dict:
        """The tensor-core layout the device holds for a bank (as streaming_machine_b200.layout.tc_layout gives it)."""
        nin, nout = (self.cfg.d_ff, self.cfg.d_model) if name.startswith("mproj") else (self.cfg.d_model, None)
        nout = nout or ({"qkv": 3 * self.cfg.d_model, "proj": self.cfg.d_model, "fc": self.cfg.d_ff}.get(
            name.split(".")[0]) if name != "head" else self.V)
        pad = (nout + 127) // 128 * 128
        out = dict(wh=np.empty((pad, nin), np.int8), wl=np.empty((pad, nin), np.int8), cc=np.empty(pad, np.int64),
                   cckb=np.empty((nin // 128, pad), np.int64))
        self._call("b2_get_bank_layout", self.h, name.encode(), *[out[k].ctypes.data for k in ("wh", "wl", "cc", "cckb")])
        return out

    def set_top_read(self, collapsing: bool):
        """The reference's top=fr (True) / top=plain (False) switch: decode steps of up to 4 streams that store no
        scores pick their word by the exact collapsing read."""
        self._call("b2_set_scalar", self.h, b"top_read", int(bool(collapsing)))

    def set_entry_tables(self, on: bool):
        """GPT-2: layer 0's qkv bank of every decode step from stored rows (wte . W and wpe . W, the reference's stored
        layer-0 entry), built at the next alloc_streams; refused when an embedded value can reach 2^15."""
        self._call("b2_set_scalar", self.h, b"entry_tables", int(bool(on)))

    def set_wait_limit(self, ns: int):
        """How long a device-side wait may take before the kernel gives up and the call reports B2_ERR_DEVICE
        (0 = the default, 0.5 s)."""
        self._call("b2_set_scalar", self.h, b"wait_ns", int(ns))

    def check_wait(self):
        """Run the bounded-wait self-check (a wait nothing satisfies): raises B2Error(ERR_DEVICE) once it gives up."""
        self._call("b2_check_wait", self.h, self._stream())
