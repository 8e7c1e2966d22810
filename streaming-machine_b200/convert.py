"""Seeded weights and the fp32 -> base-2 conversion for the integer GPT-2 machine.

The conversion is the only place a float exists. It restates `base2_convert.py` (reference `base2_convert.py:18-61`):

  * layer norm's DC block, gain and offset are folded into the bank that follows it
    (`W' = C diag(g) W`, `b' = offset @ W + b`, reference `base2_convert.py:31-41`);
  * every bank is 16-bit whole numbers with one power of two per column, the smallest that holds the column's
    largest value, rounded half-to-even (`cols16`, reference `base2_convert.py:20-26`);
  * biases, the token table and the position table are whole numbers at the stream's scale 2^-16
    (`stream`, reference `base2_convert.py:28`);
  * the head is `C diag(g_f) wte^T` with the final offset as a standing amount per word
    (reference `base2_convert.py:43-45`);
  * the tables: PHI (the bend's share, erf form), ARRIVAL (e^-d at score scale 2^-10, 2^24, until it rounds to 0),
    LOG2 and EXP2 of a 16-digit fine part, log2(768) and eps*768^2*2^40 (reference `base2_convert.py:49-61`).

One deliberate difference in HOW (not what) is computed: the DC block `C @ X` is evaluated as `X - mean(X)` with
the column mean taken by an exactly rounded sum (`math.fsum`), instead of a BLAS float64 matmul against
`eye(n) - 1/n`. BLAS results depend on the CPU's kernel choice; this form gives the same bits on every machine.
The quantised outputs are checked against the reference converter's on the seeded weights (tests/golden).

Seeded weights (no checkpoint is available offline): every >=2-D parameter of GPT-2 124M is
`float32(standard_normal) * float32(0.02)` drawn from `numpy.random.default_rng(seed)` in the fixed order
wte, wpe, then per layer c_attn, attn.c_proj, c_fc, mlp.c_proj (each in HF's Conv1D [in, out] layout);
every layer-norm gain is 1, every layer-norm offset and linear bias is 0.
"""
from __future__ import annotations

import hashlib
import math
import os

import numpy as np

ES = 16          # the stream's scale is 2^-ES
SC = 10          # attention scores live on a scale of 2^-SC

GPT2 = dict(n_layer=12, d=768, n_head=12, d_head=64, d_ff=3072, vocab=50257, n_ctx=1024)

BANKS = ("qkv", "proj", "fc", "mproj")


def bank_names(n_layer: int = 12):
    """Bank keys in the order the machine meets them (reference `base2_gpu.py:9`)."""
    return [f"{b}.{l}" for l in range(n_layer) for b in BANKS] + ["head"]


# ----------------------------------------------------------------------------------------------------------------
# seeded fp32 weights
# ----------------------------------------------------------------------------------------------------------------
def gpt2_seeded_state(seed: int = 0, cfg: dict = GPT2) -> dict:
    """HF-named fp32 state dict of a seeded random-init GPT-2 (see module docstring for the recipe)."""
    rng = np.random.default_rng(seed)
    d, F, V, T = cfg["d"], cfg["d_ff"], cfg["vocab"], cfg["n_ctx"]
    s = np.float32(0.02)

    def normal(shape):
        return rng.standard_normal(shape, dtype=np.float32) * s

    sd = {"transformer.wte.weight": normal((V, d)), "transformer.wpe.weight": normal((T, d))}
    for l in range(cfg["n_layer"]):
        p = f"transformer.h.{l}."
        sd[p + "attn.c_attn.weight"] = normal((d, 3 * d))
        sd[p + "attn.c_proj.weight"] = normal((d, d))
        sd[p + "mlp.c_fc.weight"] = normal((d, F))
        sd[p + "mlp.c_proj.weight"] = normal((F, d))
        sd[p + "attn.c_attn.bias"] = np.zeros(3 * d, np.float32)
        sd[p + "attn.c_proj.bias"] = np.zeros(d, np.float32)
        sd[p + "mlp.c_fc.bias"] = np.zeros(F, np.float32)
        sd[p + "mlp.c_proj.bias"] = np.zeros(d, np.float32)
        for ln in ("ln_1", "ln_2"):
            sd[p + ln + ".weight"] = np.ones(d, np.float32)
            sd[p + ln + ".bias"] = np.zeros(d, np.float32)
    sd["transformer.ln_f.weight"] = np.ones(d, np.float32)
    sd["transformer.ln_f.bias"] = np.zeros(d, np.float32)
    return sd


# ----------------------------------------------------------------------------------------------------------------
# conversion (reference base2_convert.py:18-61)
# ----------------------------------------------------------------------------------------------------------------
def cols16(W: np.ndarray):
    """16-bit whole numbers, one power of two per column (reference `base2_convert.py:20-26`)."""
    mx = np.maximum(np.abs(W).max(0), 1e-30)
    e = np.ceil(np.log2(mx / 32767)).astype(np.int64)
    q = np.round(W / 2.0 ** e).astype(np.int64)
    if np.abs(q).max() > 32767:
        raise ValueError("cols16: a weight does not fit 16 bits")
    return q.astype(np.int16), e


def stream(v: np.ndarray) -> np.ndarray:
    """Whole numbers at the stream's scale 2^-16 (reference `base2_convert.py:28`)."""
    return np.round(np.asarray(v, dtype=np.float64) * 2.0 ** ES).astype(np.int64)


def block_dc(X: np.ndarray) -> np.ndarray:
    """`(I - 1/n) @ X` for X [n, m]: each column minus its mean, the mean from an exactly rounded sum."""
    X = np.asarray(X, dtype=np.float64)
    n = X.shape[0]
    XT = np.ascontiguousarray(X.T)
    mean = np.fromiter((math.fsum(col) for col in XT), dtype=np.float64, count=XT.shape[0]) / n
    return X - mean[None, :]


def tables() -> dict:
    """The machine's tables (reference `base2_convert.py:48-61`)."""
    out = {}
    out["phi"] = np.array([round(0.5 * (1 + math.erf(((i - 32768) / 4096) / math.sqrt(2))) * 65536)
                           for i in range(65536)], dtype=np.int64)
    arr, d = [], 0
    while True:
        a = round(math.exp(-d / 2 ** SC) * 2 ** 24)
        if a == 0:
            break
        arr.append(a)
        d += 1
    out["arrival"] = np.array(arr, dtype=np.int64)
    out["log2"] = np.array([round(math.log2(1 + m / 65536) * 65536) for m in range(65536)], dtype=np.int64)
    out["exp2"] = np.array([round(2 ** (f / 65536) * 65536) for f in range(65536)], dtype=np.int64)
    out["log2_768"] = np.array(round(math.log2(768) * 65536))
    out["eps40"] = np.array(round(1e-5 * 768 * 768 * 2 ** 40))
    return out


def convert_gpt2(sd: dict, n_layer: int = 12) -> dict:
    """fp32 GPT-2 state dict -> the base-2 machine's arrays, keyed like `base2_gpt2.npz`."""
    f64 = {k: np.asarray(v, dtype=np.float64) for k, v in sd.items()}
    out = {}
    for k in range(n_layer):
        p = f"transformer.h.{k}."
        g1, b1, g2, b2 = f64[p + "ln_1.weight"], f64[p + "ln_1.bias"], f64[p + "ln_2.weight"], f64[p + "ln_2.bias"]
        Wq, bq = f64[p + "attn.c_attn.weight"], f64[p + "attn.c_attn.bias"]
        Wf, bf = f64[p + "mlp.c_fc.weight"], f64[p + "mlp.c_fc.bias"]
        for name, W, b in (("qkv", block_dc(g1[:, None] * Wq), b1 @ Wq + bq),
                           ("proj", f64[p + "attn.c_proj.weight"], f64[p + "attn.c_proj.bias"]),
                           ("fc", block_dc(g2[:, None] * Wf), b2 @ Wf + bf),
                           ("mproj", f64[p + "mlp.c_proj.weight"], f64[p + "mlp.c_proj.bias"])):
            out[f"{name}.{k}.w"], out[f"{name}.{k}.e"] = cols16(W)
            out[f"{name}.{k}.b"] = stream(b)
    wte = f64["transformer.wte.weight"]
    gf, bfin = f64["transformer.ln_f.weight"], f64["transformer.ln_f.bias"]
    out["head.w"], out["head.e"] = cols16(block_dc(gf[:, None] * wte.T))
    out["head.b"] = stream(bfin @ wte.T)
    out["wte"], out["wpe"] = stream(wte), stream(f64["transformer.wpe.weight"])
    out.update(tables())
    return out


def digest(arrays: dict) -> dict:
    """sha256 of every array's bytes (int arrays as little-endian int64/int16 as stored)."""
    return {k: hashlib.sha256(np.ascontiguousarray(v).tobytes()).hexdigest() for k, v in sorted(arrays.items())}


def cache_dir() -> str:
    d = os.environ.get("B2_CACHE", os.path.join(os.path.expanduser("~"), ".cache", "base2_b200"))
    os.makedirs(d, exist_ok=True)
    return d


def load_gpt2(seed: int = 0, cache: bool = True) -> dict:
    """The converted seeded GPT-2 machine, cached as an .npz (the conversion takes a few seconds)."""
    path = os.path.join(cache_dir(), f"base2_gpt2_seed{seed}.npz")
    if cache and os.path.exists(path):
        with np.load(path) as z:
            return {k: z[k] for k in z.files}
    out = convert_gpt2(gpt2_seeded_state(seed))
    if cache:
        tmp = path + f".tmp{os.getpid()}.npz"
        np.savez(tmp, **out)
        os.replace(tmp, path)
    return out


# ================================================================================================================
# Pythia-160M (reference foundation0/pythia_convert.py, foundation0/pythia_base2.py)
# ================================================================================================================
PYTHIA160M = dict(n_layer=12, d=768, n_head=12, d_head=64, d_ff=3072, vocab=50304, n_ctx=2048, rotary_pct=0.25,
                  rotary_base=10000, eps=1e-5)


def pythia_seeded_state(seed: int = 0, cfg: dict = PYTHIA160M) -> dict:
    """Safetensors-named fp32 state of a seeded random-init Pythia-160M: embed_in, embed_out, then per layer
    query_key_value, dense, dense_h_to_4h, dense_4h_to_h (torch Linear [out, in]), each
    float32(standard_normal) * float32(0.02) from numpy default_rng(seed) in that order; layer-norm gains 1,
    offsets and biases 0. The same state serves as the reference's "start" and "finished" checkpoints."""
    rng = np.random.default_rng(seed)
    d, F, V = cfg["d"], cfg["d_ff"], cfg["vocab"]
    s = np.float32(0.02)

    def normal(shape):
        return rng.standard_normal(shape, dtype=np.float32) * s

    sd = {"gpt_neox.embed_in.weight": normal((V, d)), "embed_out.weight": normal((V, d))}
    for l in range(cfg["n_layer"]):
        p = f"gpt_neox.layers.{l}."
        sd[p + "attention.query_key_value.weight"] = normal((3 * d, d))
        sd[p + "attention.dense.weight"] = normal((d, d))
        sd[p + "mlp.dense_h_to_4h.weight"] = normal((F, d))
        sd[p + "mlp.dense_4h_to_h.weight"] = normal((d, F))
        sd[p + "attention.query_key_value.bias"] = np.zeros(3 * d, np.float32)
        sd[p + "attention.dense.bias"] = np.zeros(d, np.float32)
        sd[p + "mlp.dense_h_to_4h.bias"] = np.zeros(F, np.float32)
        sd[p + "mlp.dense_4h_to_h.bias"] = np.zeros(d, np.float32)
        for ln in ("input_layernorm", "post_attention_layernorm"):
            sd[p + ln + ".weight"] = np.ones(d, np.float32)
            sd[p + ln + ".bias"] = np.zeros(d, np.float32)
    sd["gpt_neox.final_layer_norm.weight"] = np.ones(d, np.float32)
    sd["gpt_neox.final_layer_norm.bias"] = np.zeros(d, np.float32)
    return sd


def shared16(Wf: np.ndarray, Ws: np.ndarray, axis: int):
    """16-bit whole numbers with one power of two per neuron along `axis`, shared by the finished and start weights
    (reference pythia_convert.py:50-60)."""
    mf, ms = np.abs(Wf).max(axis), np.abs(Ws).max(axis)
    e = np.ceil(np.log2(np.maximum(np.maximum(mf, ms), 1e-30) / 32767)).astype(np.int64)
    sh = np.expand_dims(e, axis)
    qf, qs = np.round(Wf / 2.0 ** sh).astype(np.int64), np.round(Ws / 2.0 ** sh).astype(np.int64)
    if np.abs(qf).max() > 32767 or np.abs(qs).max() > 32767:
        raise ValueError("shared16: a weight does not fit 16 bits")
    return qf.astype(np.int16), qs.astype(np.int16), e


def convert_pythia(finished: dict, start: dict | None = None, cfg: dict = PYTHIA160M) -> dict:
    """Pythia state(s) -> the base-2 machine's arrays, keyed like base2_pythia-160m.npz (pythia_convert.py:64-110)."""
    start = finished if start is None else start

    def get(sd, k):
        return np.asarray(sd[("gpt_neox." + k) if not k.startswith("embed_out") else k], dtype=np.float64)

    out = {}

    def plate(name, key, bias=True):
        Wf, Ws = get(finished, key + ".weight").T, get(start, key + ".weight").T
        out[name + ".w"], out[name + ".s"], out[name + ".e"] = shared16(Wf, Ws, 0)
        if bias:
            out[name + ".b"], out[name + ".bs"] = stream(get(finished, key + ".bias")), stream(get(start, key + ".bias"))

    def norm(name, key):
        gf, gs = get(finished, key + ".weight"), get(start, key + ".weight")
        ge = int(np.ceil(np.log2(max(np.abs(gf).max(), np.abs(gs).max()) / 32767)))
        out[name + ".g"] = np.round(gf / 2.0 ** ge).astype(np.int64)
        out[name + ".gs"] = np.round(gs / 2.0 ** ge).astype(np.int64)
        out[name + ".ge"] = np.array(ge)
        out[name + ".b"], out[name + ".bs"] = stream(get(finished, key + ".bias")), stream(get(start, key + ".bias"))

    L, d, NH = cfg["n_layer"], cfg["d"], cfg["n_head"]
    HS = d // NH
    ROT = int(HS * cfg["rotary_pct"])
    for l in range(L):
        p = f"layers.{l}."
        norm(f"ln1.{l}", p + "input_layernorm")
        norm(f"ln2.{l}", p + "post_attention_layernorm")
        plate(f"qkv.{l}", p + "attention.query_key_value")
        plate(f"proj.{l}", p + "attention.dense")
        plate(f"fc.{l}", p + "mlp.dense_h_to_4h")
        plate(f"mproj.{l}", p + "mlp.dense_4h_to_h")
    norm("lnf", "final_layer_norm")
    plate("head", "embed_out", bias=False)
    out["embed.w"], out["embed.s"], out["embed.e"] = shared16(get(finished, "embed_in.weight"),
                                                              get(start, "embed_in.weight"), 1)
    t = tables()
    for k in ("phi", "arrival", "log2", "exp2"):
        out[k] = t[k]
    inv = float(cfg["rotary_base"]) ** (-np.arange(0, ROT, 2) / ROT)
    ang = np.arange(cfg["n_ctx"])[:, None] * inv[None, :]
    out["cos"] = np.array([[round(math.cos(x) * 2 ** 30) for x in row] for row in ang], dtype=np.int64)
    out["sin"] = np.array([[round(math.sin(x) * 2 ** 30) for x in row] for row in ang], dtype=np.int64)
    out["eps40"] = np.array(round(cfg["eps"] * d * d * 2 ** 40))
    out["half_log2_hs"] = np.array(round(math.log2(HS) / 2 * 65536))
    for k, v in dict(d=d, L=L, heads=NH, hs=HS, rot=ROT, vocab=cfg["vocab"]).items():
        out[k] = np.array(v)
    return out


def load_pythia(seed: int = 0, cache: bool = True) -> dict:
    """The converted seeded Pythia-160M machine, cached as an .npz."""
    path = os.path.join(cache_dir(), f"base2_pythia160m_seed{seed}.npz")
    if cache and os.path.exists(path):
        with np.load(path) as z:
            return {k: z[k] for k in z.files}
    out = convert_pythia(pythia_seeded_state(seed))
    if cache:
        tmp = path + f".tmp{os.getpid()}.npz"
        np.savez(tmp, **out)
        os.replace(tmp, path)
    return out
