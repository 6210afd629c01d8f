"""ctypes bindings of the CPU oracle (oracle/liboracle.so) — TEST INFRASTRUCTURE ONLY.

Imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline and
reference legs, as the checker and the timed CPU restatement of tendo's path.
The tendo_b200 library never imports this module.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

_f32p = ctypes.POINTER(ctypes.c_float)
_i8p = ctypes.POINTER(ctypes.c_int8)
_i64p = ctypes.POINTER(ctypes.c_int64)
_i64 = ctypes.c_int64


class Config(ctypes.Structure):
    """or_config: the llama.Config fields the path uses (models/llama/config.go:5-21)."""

    _fields_ = [
        ("vocab", ctypes.c_int),
        ("dim", ctypes.c_int),
        ("layers", ctypes.c_int),
        ("heads", ctypes.c_int),
        ("kv_heads", ctypes.c_int),
        ("hidden", ctypes.c_int),
        ("max_seq", ctypes.c_int),
        ("rope_base", ctypes.c_float),
        ("eps", ctypes.c_float),
    ]


def build() -> str:
    """Compile the oracle with its Makefile (a no-op when up to date)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        L.or_set_threads.argtypes = [ctypes.c_int]
        L.or_get_threads.restype = ctypes.c_int
        L.or_quantize.argtypes = [_f32p, _i64, _i64, _i64, _f32p, _i8p, _f32p]
        L.or_dequantize.argtypes = [_i8p, _f32p, _i64, _i64, _i64, _f32p]
        L.or_dequant_matmul.argtypes = [_f32p, _i8p, _f32p, _i64, _i64, _i64, _i64, _f32p]
        L.or_matmul_nt.argtypes = [_f32p, _f32p, _i64, _i64, _i64, _f32p]
        L.or_matmul_nn.argtypes = [_f32p, _f32p, _i64, _i64, _i64, _f32p]
        L.or_rmsnorm.argtypes = [_f32p, _f32p, _i64, _i64, ctypes.c_float, _f32p]
        L.or_silu.argtypes = [_f32p, _i64, _f32p]
        L.or_softmax.argtypes = [_f32p, _i64, _i64, _f32p]
        L.or_rope_tables.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_float, _f32p, _f32p]
        L.or_rope_apply.argtypes = [_f32p, _i64, _i64, _i64, _i64, _f32p, _f32p, _i64]
        L.or_argmax.argtypes = [_f32p, _i64]
        L.or_argmax.restype = _i64
        L.or_embedding.argtypes = [_f32p, _i64, _i64, _i64p, _i64, _f32p]
        L.or_embedding.restype = ctypes.c_int
        L.or_synth_normal.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, _i64, ctypes.c_double,
                                      _f32p]
        L.or_synth_tokens.argtypes = [ctypes.c_uint64, _i64, _i64, _i64p]
        L.or_synth_uniform.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, _i64, _f32p]
        L.or_model_create.argtypes = [ctypes.POINTER(Config), ctypes.c_int, ctypes.c_uint64, ctypes.c_int]
        L.or_model_create.restype = ctypes.c_void_p
        L.or_model_create_grouped.argtypes = [ctypes.POINTER(Config), ctypes.c_int, ctypes.c_uint64, ctypes.c_int,
                                              _i64]
        L.or_model_create_grouped.restype = ctypes.c_void_p
        L.or_model_free.argtypes = [ctypes.c_void_p]
        L.or_model_q.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int]
        L.or_model_q.restype = _i8p
        L.or_model_scale.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int]
        L.or_model_scale.restype = _f32p
        L.or_model_norm.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int]
        L.or_model_norm.restype = _f32p
        L.or_model_embed.argtypes = [ctypes.c_void_p]
        L.or_model_embed.restype = _f32p
        L.or_model_lm_head.argtypes = [ctypes.c_void_p]
        L.or_model_lm_head.restype = _f32p
        L.or_model_kcache.argtypes = [ctypes.c_void_p, ctypes.c_int]
        L.or_model_kcache.restype = _f32p
        L.or_model_vcache.argtypes = [ctypes.c_void_p, ctypes.c_int]
        L.or_model_vcache.restype = _f32p
        L.or_model_reset.argtypes = [ctypes.c_void_p]
        L.or_model_set_pos.argtypes = [ctypes.c_void_p, _i64]
        L.or_model_set_kv_bf16.argtypes = [ctypes.c_void_p, ctypes.c_int]
        L.or_round_bf16.argtypes = [ctypes.c_float]
        L.or_round_bf16.restype = ctypes.c_float
        L.or_model_pos.argtypes = [ctypes.c_void_p]
        L.or_model_pos.restype = _i64
        L.or_model_forward.argtypes = [ctypes.c_void_p, _i64p, _i64, _f32p, _f32p, _f32p]
        L.or_model_forward.restype = ctypes.c_int
        L.or_model_generate_greedy.argtypes = [ctypes.c_void_p, _i64p, _i64, _i64, _i64p, _f32p]
        L.or_model_generate_greedy.restype = ctypes.c_int
        L.or_model_decode_step.argtypes = [ctypes.c_void_p, _i64p, _i64p]
        L.or_model_decode_step.restype = ctypes.c_int
        _lib = L
    return _lib


def _p(a: np.ndarray, t):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(t)


def f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def set_threads(n: int) -> None:
    lib().or_set_threads(int(n))


def get_threads() -> int:
    return int(lib().or_get_threads())


def quantize(w: np.ndarray, group: int = 0):
    """(q_f32, q_i8, scale) of nn.Quantize (nn/quantize.go:42-187)."""
    w = f32(w)
    N, K = w.shape
    ng = 1 if group == 0 else K // group
    qf = np.empty((N, K), np.float32)
    qi = np.empty((N, K), np.int8)
    s = np.empty((N, ng) if group else (N,), np.float32)
    lib().or_quantize(_p(w, _f32p), N, K, group, _p(qf, _f32p), _p(qi, _i8p), _p(s, _f32p))
    return qf, qi, s


def dequantize(q: np.ndarray, scale: np.ndarray, group: int = 0) -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.int8)
    scale = f32(scale)
    N, K = q.shape
    w = np.empty((N, K), np.float32)
    lib().or_dequantize(_p(q, _i8p), _p(scale, _f32p), N, K, group, _p(w, _f32p))
    return w


def dequant_matmul(x: np.ndarray, q: np.ndarray, scale: np.ndarray, group: int = 0) -> np.ndarray:
    x = f32(x)
    q = np.ascontiguousarray(q, dtype=np.int8)
    scale = f32(scale)
    M, K = x.shape
    N = q.shape[0]
    y = np.empty((M, N), np.float32)
    lib().or_dequant_matmul(_p(x, _f32p), _p(q, _i8p), _p(scale, _f32p), M, N, K, group, _p(y, _f32p))
    return y


def matmul_nt(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    a, b = f32(a), f32(b)
    y = np.empty((a.shape[0], b.shape[0]), np.float32)
    lib().or_matmul_nt(_p(a, _f32p), _p(b, _f32p), a.shape[0], b.shape[0], a.shape[1], _p(y, _f32p))
    return y


def matmul_nn(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    a, b = f32(a), f32(b)
    y = np.empty((a.shape[0], b.shape[1]), np.float32)
    lib().or_matmul_nn(_p(a, _f32p), _p(b, _f32p), a.shape[0], b.shape[1], a.shape[1], _p(y, _f32p))
    return y


def rmsnorm(x: np.ndarray, w, eps: float) -> np.ndarray:
    x = f32(x)
    d = x.shape[-1]
    out = np.empty_like(x)
    wp = None if w is None else _p(f32(w), _f32p)
    lib().or_rmsnorm(_p(x, _f32p), wp, x.size // d, d, eps, _p(out, _f32p))
    return out


def silu(x: np.ndarray) -> np.ndarray:
    x = f32(x)
    out = np.empty_like(x)
    lib().or_silu(_p(x, _f32p), x.size, _p(out, _f32p))
    return out


def softmax(x: np.ndarray) -> np.ndarray:
    x = f32(x)
    out = np.empty_like(x)
    cols = x.shape[-1]
    lib().or_softmax(_p(x, _f32p), x.size // cols, cols, _p(out, _f32p))
    return out


def rope_tables(dim: int, max_seq: int, base: float):
    c = np.empty((max_seq, dim // 2), np.float32)
    s = np.empty((max_seq, dim // 2), np.float32)
    lib().or_rope_tables(dim, max_seq, base, _p(c, _f32p), _p(s, _f32p))
    return c, s


def rope_apply(x: np.ndarray, cos_t, sin_t, pos_offset: int) -> np.ndarray:
    """x: [B, H, S, D]; returns the rotated copy."""
    x = f32(x).copy()
    B, H, S, D = x.shape
    lib().or_rope_apply(_p(x, _f32p), B, H, S, D, _p(f32(cos_t), _f32p), _p(f32(sin_t), _f32p), pos_offset)
    return x


def argmax(v: np.ndarray) -> int:
    v = f32(v)
    return int(lib().or_argmax(_p(v, _f32p), v.size))


def synth_normal(seed: int, stream: int, n: int, std: float, offset: int = 0) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().or_synth_normal(seed, stream, offset, n, std, _p(out, _f32p))
    return out


def synth_tokens(seed: int, n: int, vocab: int) -> np.ndarray:
    out = np.empty(n, np.int64)
    lib().or_synth_tokens(seed, n, vocab, _p(out, _i64p))
    return out


STREAM_EMBED = 0x7FFF0001
STREAM_LMHEAD = 0x7FFF0002
STREAM_PROMPT = 0x7FFF0003
STREAM_X = 0x7FFF0004
STREAM_W = 0x7FFF0005


class Model:
    """Quantized Llama oracle (models/llama/quantized.go) for B lockstep sequences;
    with ``group`` > 0 every Linear is quantized per group of that many input
    columns (QuantizeModel(m, groupSize), models/llama/quantized.go:52-73)."""

    MATS = ("q", "k", "v", "o", "gate", "up", "down")

    def __init__(self, cfg: dict, batch: int = 1, seed: int = 0, generate: bool = True, group: int = 0):
        self.cfg = dict(cfg)
        c = Config(
            cfg["vocab"], cfg["dim"], cfg["layers"], cfg["heads"], cfg["kv_heads"], cfg["hidden"],
            cfg["max_seq"], cfg["rope_base"], cfg["eps"],
        )
        self._c = c
        self.B = batch
        self.group = group
        self.h = lib().or_model_create_grouped(ctypes.byref(c), batch, seed, 1 if generate else 0, group)
        if not self.h:
            raise MemoryError("or_model_create failed")

    def close(self):
        if self.h:
            lib().or_model_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def shape(self, mat: int):
        c = self.cfg
        d, D = c["dim"], c["dim"] // c["heads"]
        hq, hkv, F = c["heads"] * D, c["kv_heads"] * D, c["hidden"]
        return [(hq, d), (hkv, d), (hkv, d), (d, hq), (F, d), (F, d), (d, F)][mat]

    def q(self, layer: int, mat: int) -> np.ndarray:
        N, K = self.shape(mat)
        return np.ctypeslib.as_array(lib().or_model_q(self.h, layer, mat), shape=(N, K))

    def scale(self, layer: int, mat: int) -> np.ndarray:
        N, K = self.shape(mat)
        shape = (N, K // self.group) if self.group else (N,)
        return np.ctypeslib.as_array(lib().or_model_scale(self.h, layer, mat), shape=shape)

    def embed(self) -> np.ndarray:
        c = self.cfg
        return np.ctypeslib.as_array(lib().or_model_embed(self.h), shape=(c["vocab"], c["dim"]))

    def lm_head(self) -> np.ndarray:
        c = self.cfg
        return np.ctypeslib.as_array(lib().or_model_lm_head(self.h), shape=(c["vocab"], c["dim"]))

    def norm(self, layer: int, which: int) -> np.ndarray:
        return np.ctypeslib.as_array(lib().or_model_norm(self.h, layer, which), shape=(self.cfg["dim"],))

    def kcache(self, layer: int) -> np.ndarray:
        c = self.cfg
        D = c["dim"] // c["heads"]
        return np.ctypeslib.as_array(
            lib().or_model_kcache(self.h, layer), shape=(self.B, c["kv_heads"], c["max_seq"], D))

    def vcache(self, layer: int) -> np.ndarray:
        c = self.cfg
        D = c["dim"] // c["heads"]
        return np.ctypeslib.as_array(
            lib().or_model_vcache(self.h, layer), shape=(self.B, c["kv_heads"], c["max_seq"], D))

    def reset(self):
        lib().or_model_reset(self.h)

    def set_pos(self, pos: int):
        lib().or_model_set_pos(self.h, pos)

    def set_kv_bf16(self, on: bool = True):
        """K and V rounded to bf16 as they are appended (a bf16 KV cache)."""
        lib().or_model_set_kv_bf16(self.h, 1 if on else 0)

    @property
    def pos(self) -> int:
        return int(lib().or_model_pos(self.h))

    def forward(self, tokens: np.ndarray, want_logits=True, want_hidden=False):
        tokens = np.ascontiguousarray(tokens, dtype=np.int64).reshape(self.B, -1)
        S = tokens.shape[1]
        c = self.cfg
        logits = np.empty((self.B, S, c["vocab"]), np.float32) if want_logits else None
        last = np.empty((self.B, c["vocab"]), np.float32)
        hidden = np.empty((c["layers"] + 1, self.B, S, c["dim"]), np.float32) if want_hidden else None
        rc = lib().or_model_forward(
            self.h, _p(tokens, _i64p), S, None if logits is None else _p(logits, _f32p), _p(last, _f32p),
            None if hidden is None else _p(hidden, _f32p))
        if rc != 0:
            raise ValueError("or_model_forward failed (bad token id or cache overflow)")
        return logits, last, hidden

    def generate_greedy(self, prompt: np.ndarray, n_new: int):
        prompt = np.ascontiguousarray(prompt, dtype=np.int64).reshape(self.B, -1)
        toks = np.empty((self.B, n_new), np.int64)
        margins = np.empty((self.B, n_new), np.float32)
        rc = lib().or_model_generate_greedy(
            self.h, _p(prompt, _i64p), prompt.shape[1], n_new, _p(toks, _i64p), _p(margins, _f32p))
        if rc != 0:
            raise ValueError("or_model_generate_greedy failed")
        return toks, margins

    def decode_step(self, tokens: np.ndarray) -> np.ndarray:
        tokens = np.ascontiguousarray(tokens, dtype=np.int64).reshape(self.B)
        nxt = np.empty(self.B, np.int64)
        rc = lib().or_model_decode_step(self.h, _p(tokens, _i64p), _p(nxt, _i64p))
        if rc != 0:
            raise ValueError("or_model_decode_step failed")
        return nxt


# The workload configurations (synthetic weights, stated seeds).
TINY = dict(vocab=32000, dim=512, layers=8, heads=8, kv_heads=8, hidden=1408, max_seq=2048,
            rope_base=10000.0, eps=1e-5)
LLAMA7B = dict(vocab=32000, dim=4096, layers=32, heads=32, kv_heads=32, hidden=11008, max_seq=2048,
               rope_base=10000.0, eps=1e-6)


# ---------------------------------------------------------------------------
# Sampler.Sample (models/sampling.go:47-70, :99-161), restated with float32
# scalars for every operation, loops in the reference's order.  The uniform
# draw r (the reference's rng.Float32()) is an argument.
# ---------------------------------------------------------------------------
def _softmax_ref(x):
    """models/sampling.go:140-161: max from x[0], float32(exp(float64(v - max))),
    fp32 sum in index order, division."""
    import math

    f32 = np.float32
    m = x[0]
    for v in x[1:]:
        if v > m:
            m = v
    e = [f32(math.exp(float(f32(v - m)))) if np.isfinite(f32(v - m)) else f32(0.0 if f32(v - m) < 0 else np.nan)
         for v in x]
    s = f32(0.0)
    for p in e:
        s = f32(s + p)
    return [f32(p / s) for p in e]


def sample(logits, temperature=1.0, top_k=0, top_p=0.0, r=0.5):
    f32 = np.float32
    x = [f32(v) for v in np.asarray(logits, np.float32)]
    V = len(x)
    T = f32(temperature)
    if T != f32(1.0) and T > 0:
        x = [f32(v / T) for v in x]
    if 0 < top_k < V:
        thr = sorted(x, reverse=True)[top_k - 1]  # findKthLargest: the k-th largest value
        x = [f32(-np.inf) if v < thr else v for v in x]
    if 0 < top_p < 1.0:
        probs = _softmax_ref(x)
        order = sorted(range(V), key=lambda i: (-probs[i], i))  # stable insertion sort, descending
        cs, cut = f32(0.0), 0
        for n, i in enumerate(order):
            cs = f32(cs + probs[i])
            if cs >= f32(top_p):
                cut = n + 1
                break
        for i in order[cut:]:
            x[i] = f32(-np.inf)
    if all(v == -np.inf for v in x):
        return V - 1
    probs = _softmax_ref(x)
    cs = f32(0.0)
    r = f32(r)
    for i, p in enumerate(probs):
        cs = f32(cs + p)
        if r < cs:
            return i
    return V - 1


STREAM_SAMPLE = 0x7FFF0006


def synth_uniform(seed: int, stream: int, n: int, offset: int = 0) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().or_synth_uniform(seed, stream, offset, n, _p(out, _f32p))
    return out


def generate_sample(model, prompt, n_new, temperature, top_k, top_p, seed):
    """QuantizedModel.Generate with the Sampler (models/llama/quantized.go:422-477,
    models/sampling.go:47-70): forward the prompt, then per step sample every
    row's last logits with the uniform draw (seed, step * B + row) and feed the
    tokens back."""
    prompt = np.ascontiguousarray(prompt, dtype=np.int64).reshape(model.B, -1)
    B = model.B
    _, last, _ = model.forward(prompt, want_logits=False)
    out = np.empty((B, n_new), np.int64)
    for j in range(n_new):
        u = synth_uniform(seed, STREAM_SAMPLE, B, offset=j * B)
        toks = np.array([sample(last[b], temperature, top_k, top_p, float(u[b])) for b in range(B)], np.int64)
        out[:, j] = toks
        if j + 1 < n_new:
            _, last, _ = model.forward(toks[:, None], want_logits=False)
    return out
