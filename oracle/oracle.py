"""ctypes front end of the CPU oracle (oracle/enx_oracle.cpp).  TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import this module, and
only as the checker.  The product library never loads it.

Build: `make -C oracle` (also done by `build()` below and by __graft_entry__.build()).
"""

from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path
from typing import Dict, Optional, Sequence

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "libenx_oracle.so"

_lib = None


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        _lib = C.CDLL(str(LIB_PATH))
        _declare(_lib)
    return _lib


P = C.c_void_p
I64 = C.c_int64


class SampleDims(C.Structure):
    _fields_ = [("vocab", C.c_uint32), ("history_length", C.c_uint32), ("temperature", C.c_float),
                ("top_p", C.c_float), ("repetition_penalty", C.c_float), ("random", C.c_float),
                ("pad0", C.c_uint32), ("pad1", C.c_uint32)]


class SampleTrace(C.Structure):
    _fields_ = [("top1_gap", C.c_double), ("max_prob", C.c_double), ("sum", C.c_double),
                ("min_mass_margin", C.c_double), ("threshold", C.c_double), ("kept", C.c_double),
                ("target", C.c_double), ("cross_margin", C.c_double), ("prev_margin", C.c_double),
                ("kept_count", C.c_uint32), ("fallback", C.c_uint32)]

    def as_dict(self) -> Dict[str, float]:
        return {name: getattr(self, name) for name, _ in self._fields_}


class Config(C.Structure):
    _fields_ = [("layers", C.c_uint32), ("hidden", C.c_uint32), ("heads", C.c_uint32),
                ("kv_heads", C.c_uint32), ("head_dim", C.c_uint32), ("intermediate", C.c_uint32),
                ("vocab", C.c_uint32), ("rms_norm_eps", C.c_float), ("rope_theta", C.c_float)]


class QTensor(C.Structure):
    _fields_ = [("packed", P), ("scales", P), ("zeros", P), ("bits", C.c_int32), ("rows", C.c_int32),
                ("cols", C.c_int32)]


class Layer(C.Structure):
    _fields_ = [("input_norm", P), ("post_norm", P), ("q", QTensor), ("k", QTensor), ("v", QTensor),
                ("o", QTensor), ("gate", QTensor), ("up", QTensor), ("down", QTensor), ("q_bias", P),
                ("k_bias", P), ("v_bias", P)]


class Weights(C.Structure):
    _fields_ = [("embed", QTensor), ("final_norm", P), ("layers", C.POINTER(Layer))]


def _declare(L):
    L.orc_mulberry32_next.restype = C.c_double
    L.orc_mulberry32_next.argtypes = [C.POINTER(C.c_uint32)]
    L.orc_mulberry32_fill.argtypes = [C.c_uint32, I64, P]
    L.orc_dequant.argtypes = [C.c_int, P, P, P, I64, I64, I64, P]
    L.orc_linear_q.argtypes = [C.c_int, P, P, P, P, P, I64, I64, I64, I64, I64, I64, P]
    L.orc_linear_f32.argtypes = [P, P, P, I64, I64, I64, P]
    L.orc_rmsnorm.argtypes = [P, P, I64, I64, C.c_float, P]
    L.orc_rope.argtypes = [P, I64, I64, I64, C.c_double, I64, P]
    L.orc_rope_table.argtypes = [I64, I64, C.c_double, P, P]
    L.orc_silu_mul.argtypes = [P, P, I64, P]
    L.orc_add.argtypes = [P, P, I64, P]
    L.orc_embed_q.argtypes = [C.c_int, P, I64, P, P, P, I64, I64, P]
    L.orc_argmax.restype = C.c_uint32
    L.orc_argmax.argtypes = [P, I64]
    L.orc_attention_f16.argtypes = [P, P, P, I64, I64, I64, I64, I64, P]
    L.orc_cache_pack.argtypes = [P, I64, I64, I64, P]
    L.orc_f32_to_f16.argtypes = [P, I64, P]
    L.orc_f16_to_f32.argtypes = [P, I64, P]
    L.orc_sample.restype = C.c_uint32
    L.orc_sample.argtypes = [P, P, C.POINTER(SampleDims), C.POINTER(SampleTrace)]
    L.orc_set_threads.argtypes = [C.c_int]
    L.orc_max_threads.restype = C.c_int
    L.orc_model_create.restype = P
    L.orc_model_create.argtypes = [C.POINTER(Config), C.POINTER(Weights), I64]
    L.orc_model_destroy.argtypes = [P]
    L.orc_model_fork.restype = P
    L.orc_model_fork.argtypes = [P]
    L.orc_model_reset.argtypes = [P]
    L.orc_model_filled.restype = I64
    L.orc_model_filled.argtypes = [P]
    L.orc_prefill.restype = C.c_int
    L.orc_prefill.argtypes = [P, P, I64, I64, P]
    L.orc_decode.restype = C.c_int
    L.orc_decode.argtypes = [P, C.c_uint32, P, P]
    L.orc_model_kv.argtypes = [P, C.c_uint32, P, P]
    L.orc_nll.restype = C.c_double
    L.orc_nll.argtypes = [P, I64, C.c_uint32]


def _p(a: Optional[np.ndarray]):
    return None if a is None else a.ctypes.data


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def set_threads(n: int) -> None:
    lib().orc_set_threads(int(n))


def max_threads() -> int:
    return int(lib().orc_max_threads())


# --- primitive ops ---------------------------------------------------------------------------


class Mulberry32:
    """The session RNG (src/runtime/session.ts:75-83)."""

    def __init__(self, seed: int):
        self.state = C.c_uint32(seed & 0xFFFFFFFF)

    def __call__(self) -> float:
        return float(lib().orc_mulberry32_next(C.byref(self.state)))


def mulberry32(seed: int, n: int) -> np.ndarray:
    out = np.empty(n, dtype=np.float64)
    lib().orc_mulberry32_fill(seed & 0xFFFFFFFF, n, _p(out))
    return out


def random_floats(count: int, seed: int = 1) -> np.ndarray:
    """randomFloats of test/reference/rng.ts:13-18: mulberry32 - 0.5, stored as float32."""
    return (mulberry32(seed, count) - 0.5).astype(np.float32)


def dequant(t) -> np.ndarray:
    out = np.empty((t.rows, t.cols), dtype=np.float32)
    lib().orc_dequant(t.bits, _p(t.packed), _p(t.scales), _p(t.zeros), t.rows, t.cols, 64, _p(out))
    return out


def linear_q(t, x: np.ndarray, bias: Optional[np.ndarray] = None, out_stride: Optional[int] = None,
             out_offset: int = 0, out: Optional[np.ndarray] = None) -> np.ndarray:
    x = _c(x, np.float32).reshape(-1, t.cols)
    m = x.shape[0]
    stride = t.rows if out_stride is None else out_stride
    if out is None:
        out = np.zeros(m * stride + out_offset if m > 0 else 0, dtype=np.float32)
    b = None if bias is None else _c(bias, np.float32)
    lib().orc_linear_q(t.bits, _p(x), _p(t.packed), _p(t.scales), _p(t.zeros), _p(b), m, t.cols, t.rows, 64,
                       stride, out_offset, _p(out))
    return out


def linear_f32(x, w, bias=None):
    x = _c(x, np.float32)
    w = _c(w, np.float32)
    n, k = w.shape
    m = x.size // k
    out = np.empty((m, n), dtype=np.float32)
    b = None if bias is None else _c(bias, np.float32)
    lib().orc_linear_f32(_p(x), _p(w), _p(b), m, k, n, _p(out))
    return out


def rmsnorm(x, w, eps=1e-6):
    x = _c(x, np.float32)
    w = _c(w, np.float32)
    f = w.shape[0]
    out = np.empty_like(x)
    lib().orc_rmsnorm(_p(x), _p(w), x.size // f, f, eps, _p(out))
    return out


def rope(x, heads, head_dim, theta=1e6, pos_offset=0):
    x = _c(x, np.float32)
    seq = x.size // (heads * head_dim)
    out = np.empty_like(x)
    lib().orc_rope(_p(x), seq, heads, head_dim, float(theta), pos_offset, _p(out))
    return out


def rope_table(max_pos, head_dim, theta=1e6):
    c = np.empty((max_pos, head_dim // 2), dtype=np.float32)
    s = np.empty_like(c)
    lib().orc_rope_table(max_pos, head_dim, float(theta), _p(c), _p(s))
    return c, s


def silu_mul(g, u):
    g = _c(g, np.float32)
    u = _c(u, np.float32)
    out = np.empty_like(g)
    lib().orc_silu_mul(_p(g), _p(u), g.size, _p(out))
    return out


def add(a, b):
    a = _c(a, np.float32)
    b = _c(b, np.float32)
    out = np.empty_like(a)
    lib().orc_add(_p(a), _p(b), a.size, _p(out))
    return out


def embed_q(t, ids) -> np.ndarray:
    ids = _c(ids, np.uint32)
    out = np.empty((ids.size, t.cols), dtype=np.float32)
    lib().orc_embed_q(t.bits, _p(ids), ids.size, _p(t.packed), _p(t.scales), _p(t.zeros), t.cols, 64, _p(out))
    return out


def argmax(x) -> int:
    x = _c(x, np.float32)
    return int(lib().orc_argmax(_p(x), x.size))


def f32_to_f16_bits(x) -> np.ndarray:
    x = _c(x, np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().orc_f32_to_f16(_p(x), x.size, _p(out))
    return out


def attention_f16(q, kcache_bits, vcache_bits, begin, heads, kv_heads, head_dim):
    """Causal GQA attention of q [queries, heads*hd] over f16 caches [pos][kv*hd] (uint16 bits)."""
    q = _c(q, np.float32)
    queries = q.size // (heads * head_dim)
    out = np.empty((queries, heads * head_dim), dtype=np.float32)
    lib().orc_attention_f16(_p(q), _p(_c(kcache_bits, np.uint16)), _p(_c(vcache_bits, np.uint16)),
                            queries, begin, heads, kv_heads, head_dim, _p(out))
    return out


def nll(logits: np.ndarray, target: int) -> float:
    """-log softmax(logits)[target] (the perplexity harness's per-position term)."""
    lg = _c(logits, np.float32)
    return float(lib().orc_nll(_p(lg), lg.size, int(target)))


def sample(logits: np.ndarray, history: Sequence[int], temperature: float, top_p: float,
           repetition_penalty: float, random: float, trace: bool = False):
    """Runs the sampler IN PLACE on `logits` (float32, modified by the penalty) and returns the id
    (and the margin trace when asked)."""
    assert logits.dtype == np.float32 and logits.flags.c_contiguous
    hist = _c(history, np.uint32)
    d = SampleDims(logits.size, hist.size, temperature, top_p, repetition_penalty, random, 0, 0)
    tr = SampleTrace()
    tok = int(lib().orc_sample(_p(logits), _p(hist) if hist.size else None, C.byref(d), C.byref(tr)))
    return (tok, tr.as_dict()) if trace else tok


# --- whole model -----------------------------------------------------------------------------


def _qt(t) -> QTensor:
    return QTensor(t.packed.ctypes.data, t.scales.ctypes.data, t.zeros.ctypes.data, t.bits, t.rows, t.cols)


class OracleModel:
    """Qwen2 decoder over an `EnargeiaFile`, with an f16 KV cache of `max_context` positions."""

    def __init__(self, f, cfg, max_context: int):
        self.f = f
        self.cfg = cfg
        self.max_context = max_context
        # keep contiguous copies alive: the C side holds raw pointers
        self._keep = []

        def q(name):
            t = f.quant(name)
            for a in (t.packed, t.scales, t.zeros):
                self._keep.append(a)
            return _qt(t)

        def v(name):
            a = _c(f.f32(name), np.float32)
            self._keep.append(a)
            return a.ctypes.data

        layers = (Layer * cfg.layers)()
        for l in range(cfg.layers):
            p = f"model.layers.{l}."
            layers[l] = Layer(v(p + "input_layernorm.weight"), v(p + "post_attention_layernorm.weight"),
                              q(p + "self_attn.q_proj.weight"), q(p + "self_attn.k_proj.weight"),
                              q(p + "self_attn.v_proj.weight"), q(p + "self_attn.o_proj.weight"),
                              q(p + "mlp.gate_proj.weight"), q(p + "mlp.up_proj.weight"),
                              q(p + "mlp.down_proj.weight"), v(p + "self_attn.q_proj.bias"),
                              v(p + "self_attn.k_proj.bias"), v(p + "self_attn.v_proj.bias"))
        self._layers = layers
        w = Weights(q("model.embed_tokens.weight"), v("model.norm.weight"), layers)
        c = Config(cfg.layers, cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.intermediate, cfg.vocab,
                   cfg.rms_norm_eps, cfg.rope_theta)
        self._h = lib().orc_model_create(C.byref(c), C.byref(w), max_context)

    def fork(self) -> "OracleModel":
        """An independent copy of this model's state (same weights, same cache and fill)."""
        other = OracleModel.__new__(OracleModel)
        other.f, other.cfg, other.max_context = self.f, self.cfg, self.max_context
        other._keep, other._layers = self._keep, self._layers
        other._h = lib().orc_model_fork(self._h)
        return other

    def __del__(self):
        h = getattr(self, "_h", None)
        if h and lib is not None:  # at interpreter shutdown the module's globals may already be gone
            lib().orc_model_destroy(h)
            self._h = None

    @property
    def filled(self) -> int:
        return int(lib().orc_model_filled(self._h))

    def reset(self) -> None:
        lib().orc_model_reset(self._h)

    def prefill(self, ids: Sequence[int], chunk: int = 256) -> np.ndarray:
        ids = _c(ids, np.uint32)
        logits = np.empty(self.cfg.vocab, dtype=np.float32)
        if lib().orc_prefill(self._h, _p(ids), ids.size, chunk, _p(logits)) != 0:
            raise RangeError(f"prompt of {ids.size} exceeds the remaining context")
        return logits

    def decode(self, token: int, want_normed: bool = False):
        logits = np.empty(self.cfg.vocab, dtype=np.float32)
        normed = np.empty(self.cfg.hidden, dtype=np.float32) if want_normed else None
        if lib().orc_decode(self._h, int(token), _p(logits), _p(normed)) != 0:
            raise RangeError("context exhausted")
        return (logits, normed) if want_normed else logits

    def kv(self, layer: int):
        per = self.max_context * self.cfg.kv_heads * self.cfg.head_dim
        k = np.empty(per, dtype=np.uint16)
        v = np.empty(per, dtype=np.uint16)
        lib().orc_model_kv(self._h, layer, _p(k), _p(v))
        return k, v


class RangeError(ValueError):
    pass


class OracleSession:
    """`Session.generate` of src/runtime/session.ts:416-495 over the oracle model.

    Prefill, sample the first token from the prefill logits, then decode with the fed token in the
    history; one mulberry32 draw per sampled token.
    """

    def __init__(self, model: OracleModel, temperature=0.0, top_p=1.0, repetition_penalty=1.0, seed=0x5EED):
        self.model = model
        self.params = (temperature, top_p, repetition_penalty)
        self.random = Mulberry32(seed)
        self.tokens = []
        self.traces = []

    def _sample(self, logits):
        t, p, rp = self.params
        r = np.float32(self.random())
        tok, tr = sample(logits, self.tokens, t, p, rp, float(r), trace=True)
        self.traces.append(tr)
        return tok

    def generate(self, prompt, max_tokens, stop_tokens=(), chunk=256):
        stop = set(stop_tokens)
        logits = self.model.prefill(prompt, chunk)
        self.tokens = list(prompt)
        nxt = self._sample(logits)
        produced = [nxt]
        self.tokens.append(nxt)
        i = 1
        while i < max_tokens and nxt not in stop:
            if self.model.filled >= self.model.max_context:
                break
            logits = self.model.decode(nxt)
            nxt = self._sample(logits)
            produced.append(nxt)
            self.tokens.append(nxt)
            i += 1
        return produced
