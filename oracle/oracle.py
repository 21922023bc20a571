"""ctypes binding of the CPU oracle (oracle/liboracle.so).

TEST INFRASTRUCTURE: only tests/, __graft_entry__.smoke() and bench.py's CPU
legs import this module.  The product path (static-lm_b200) never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

Q4_DTYPE = np.dtype([("d", "<u2"), ("qs", "u1", (16,))])  # BlockQ4_0, 18 B
Q8_DTYPE = np.dtype([("d", "<u2"), ("qs", "i1", (32,))])  # BlockQ8_0, 34 B
assert Q4_DTYPE.itemsize == 18 and Q8_DTYPE.itemsize == 34

MODE_X86 = 0
MODE_SCALAR = 1

_F = C.POINTER(C.c_float)
_V = C.c_void_p
_I32P = C.POINTER(C.c_int32)


class Config(C.Structure):
    _fields_ = [("dim", C.c_int32), ("hidden_dim", C.c_int32), ("num_heads", C.c_int32),
                ("num_kv_heads", C.c_int32), ("max_seq_len", C.c_int32), ("rms_eps", C.c_float)]


class LayerWeights(C.Structure):
    _fields_ = [("rms_att_weight", _V), ("wq", _V), ("wk", _V), ("wv", _V), ("wo", _V),
                ("rms_ffn_weight", _V), ("w_gate", _V), ("w_up", _V), ("w_down", _V)]


class ModelWeights(C.Structure):
    _fields_ = [("token_embd", _V), ("layers", C.POINTER(LayerWeights)), ("num_layers", C.c_int32),
                ("output_norm", _V), ("lm_head", _V), ("vocab_size", C.c_int32)]


def build():
    subprocess.run(["make", "-s", "-C", HERE, "CC=gcc"], check=True)


def _load():
    if not os.path.exists(LIB_PATH):
        build()
    lib = C.CDLL(LIB_PATH)
    sig = {
        "orc_f32_to_f16": (C.c_uint16, [C.c_float]),
        "orc_f16_to_f32": (C.c_float, [C.c_uint16]),
        "orc_quantize_row_q4_0": (None, [_V, _V, C.c_size_t]),
        "orc_dequantize_row_q4_0": (None, [_V, _V, C.c_size_t]),
        "orc_quantize_row_q8_0": (None, [_V, _V, C.c_size_t]),
        "orc_dequantize_row_q8_0": (None, [_V, _V, C.c_size_t]),
        "orc_vec_dot_scalar": (C.c_float, [_V, _V, C.c_size_t]),
        "orc_vec_dot_x86": (C.c_float, [_V, _V, C.c_size_t]),
        "orc_vec_dot_avx2": (C.c_float, [_V, _V, C.c_size_t]),
        "orc_host_has_avx2": (C.c_int, []),
        "orc_gemm_q4_0": (None, [_V, _V, _V, C.c_size_t, C.c_size_t, C.c_size_t, C.c_int, C.c_int]),
        "orc_gemm_q4_0_f32": (None, [_V, _V, _V, _V, C.c_size_t, C.c_size_t, C.c_size_t, C.c_int,
                                     C.c_int]),
        "orc_default_pool_threads": (C.c_int, []),
        "orc_exp_poly": (C.c_float, [C.c_float]),
        "orc_softmax": (None, [_V, _V, C.c_size_t, C.c_int]),
        "orc_rmsnorm": (None, [_V, _V, _V, C.c_size_t, C.c_float, C.c_int]),
        "orc_swiglu": (None, [_V, _V, _V, C.c_size_t, C.c_int]),
        "orc_residual_add": (None, [_V, _V, _V, C.c_size_t]),
        "orc_l2_norm": (None, [_V, _V, C.c_size_t, C.c_float]),
        "orc_rope_tables": (None, [C.c_int32, C.c_int32, _V, _V]),
        "orc_apply_rope_cached": (None, [_V, C.c_size_t, _V, _V, C.c_int32]),
        "orc_apply_rope_in_place": (None, [_V, C.c_size_t, C.c_int32, C.c_int32]),
        "orc_attention": (None, [_V, _V, _V, _V, _V, C.POINTER(Config), C.c_int32, C.c_int]),
        "orc_sample_argmax": (C.c_int32, [_V, C.c_size_t]),
        "orc_model_new": (_V, [C.POINTER(Config), C.c_int32, C.c_int32, C.c_int, C.c_int]),
        "orc_model_free": (None, [_V]),
        "orc_model_set_weights": (C.c_int, [_V, C.POINTER(ModelWeights)]),
        "orc_forward_token": (C.c_int32, [_V, C.c_int32, C.c_int32]),
        "orc_prefill_tokens": (C.c_int32, [_V, _I32P, C.c_int32, C.c_int32]),
        "orc_generate": (C.c_int32, [_V, _I32P, C.c_int32, _I32P, C.c_int32, C.c_int32]),
        "orc_embed_tokens": (None, [_V, _I32P, C.c_int32, _F]),
        "orc_layer_forward_token": (None, [_V, C.c_int32, C.c_int32]),
        "orc_model_x": (_F, [_V]),
        "orc_model_xb": (_F, [_V]),
        "orc_model_logits": (_F, [_V]),
        "orc_model_k_cache": (_F, [_V, C.c_int32]),
        "orc_model_v_cache": (_F, [_V, C.c_int32]),
        "orc_model_rope_cos": (_F, [_V]),
        "orc_model_rope_sin": (_F, [_V]),
        "orc_xorshift_f32": (None, [_V, C.c_size_t, C.c_uint32, C.c_float]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


# ---------------------------------------------------------------- blocks / kernels

def f32_to_f16(x: float) -> int:
    return int(lib.orc_f32_to_f16(float(x)))


def f16_to_f32(h: int) -> float:
    return float(lib.orc_f16_to_f32(int(h)))


def quantize_q4_0(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros(x.size // 32, dtype=Q4_DTYPE)
    lib.orc_quantize_row_q4_0(ptr(x), ptr(out), x.size)
    return out


def dequantize_q4_0(b: np.ndarray) -> np.ndarray:
    out = np.zeros(b.size * 32, dtype=np.float32)
    lib.orc_dequantize_row_q4_0(ptr(np.ascontiguousarray(b)), ptr(out), out.size)
    return out


def quantize_q8_0(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros(x.size // 32, dtype=Q8_DTYPE)
    lib.orc_quantize_row_q8_0(ptr(x), ptr(out), x.size)
    return out


def dequantize_q8_0(b: np.ndarray) -> np.ndarray:
    out = np.zeros(b.size * 32, dtype=np.float32)
    lib.orc_dequantize_row_q8_0(ptr(np.ascontiguousarray(b)), ptr(out), out.size)
    return out


def vec_dot(w: np.ndarray, a: np.ndarray, kind: str = "x86") -> float:
    fn = {"x86": lib.orc_vec_dot_x86, "scalar": lib.orc_vec_dot_scalar,
          "avx2": lib.orc_vec_dot_avx2}[kind]
    assert w.size == a.size
    return float(fn(ptr(np.ascontiguousarray(w)), ptr(np.ascontiguousarray(a)), w.size))


def gemm_q8(w: np.ndarray, xq: np.ndarray, batch: int, rows: int, cols: int,
            mode: int = MODE_X86, threads: int = 1) -> np.ndarray:
    out = np.zeros(batch * rows, dtype=np.float32)
    lib.orc_gemm_q4_0(ptr(np.ascontiguousarray(w)), ptr(np.ascontiguousarray(xq)), ptr(out),
                      batch, rows, cols, mode, threads)
    return out


def gemm_f32(w: np.ndarray, x: np.ndarray, batch: int, rows: int, cols: int,
             mode: int = MODE_X86, threads: int = 1) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    q8 = np.zeros(batch * cols // 32, dtype=Q8_DTYPE)
    out = np.zeros(batch * rows, dtype=np.float32)
    lib.orc_gemm_q4_0_f32(ptr(np.ascontiguousarray(w)), ptr(x), ptr(q8), ptr(out), batch, rows,
                          cols, mode, threads)
    return out


# ---------------------------------------------------------------- vector ops

def exp_poly(x: float) -> float:
    return float(lib.orc_exp_poly(float(x)))


def softmax(x: np.ndarray, mode: int = MODE_X86) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros_like(x)
    lib.orc_softmax(ptr(x), ptr(out), x.size, mode)
    return out


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float, mode: int = MODE_X86) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    out = np.zeros_like(x)
    lib.orc_rmsnorm(ptr(x), ptr(w), ptr(out), x.size, eps, mode)
    return out


def swiglu(g: np.ndarray, u: np.ndarray, mode: int = MODE_X86) -> np.ndarray:
    g = np.ascontiguousarray(g, dtype=np.float32)
    u = np.ascontiguousarray(u, dtype=np.float32)
    out = np.zeros_like(g)
    lib.orc_swiglu(ptr(g), ptr(u), ptr(out), g.size, mode)
    return out


def residual_add(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    out = np.zeros_like(a)
    lib.orc_residual_add(ptr(a), ptr(b), ptr(out), a.size)
    return out


def l2_norm(x: np.ndarray, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros_like(x)
    lib.orc_l2_norm(ptr(x), ptr(out), x.size, eps)
    return out


def rope_tables(max_seq: int, head_dim: int):
    c = np.zeros(max_seq * (head_dim // 2), dtype=np.float32)
    s = np.zeros_like(c)
    lib.orc_rope_tables(max_seq, head_dim, ptr(c), ptr(s))
    return c, s


def apply_rope_cached(vec: np.ndarray, cos_row: np.ndarray, sin_row: np.ndarray, head_dim: int):
    v = np.ascontiguousarray(vec, dtype=np.float32).copy()
    lib.orc_apply_rope_cached(ptr(v), v.size, ptr(np.ascontiguousarray(cos_row)),
                              ptr(np.ascontiguousarray(sin_row)), head_dim)
    return v


def apply_rope_in_place(vec: np.ndarray, pos: int, head_dim: int):
    v = np.ascontiguousarray(vec, dtype=np.float32).copy()
    lib.orc_apply_rope_in_place(ptr(v), v.size, pos, head_dim)
    return v


def attention(q, k_cache, v_cache, cfg: Config, pos: int, mode: int = MODE_X86):
    att = np.zeros(cfg.num_heads * cfg.max_seq_len, dtype=np.float32)
    out = np.zeros(cfg.dim, dtype=np.float32)
    lib.orc_attention(ptr(np.ascontiguousarray(q, dtype=np.float32)),
                      ptr(np.ascontiguousarray(k_cache, dtype=np.float32)),
                      ptr(np.ascontiguousarray(v_cache, dtype=np.float32)), ptr(att), ptr(out),
                      C.byref(cfg), pos, mode)
    return out, att


def argmax(logits: np.ndarray) -> int:
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    return int(lib.orc_sample_argmax(ptr(logits), logits.size))


# ---------------------------------------------------------------- synthetic inputs

def xorshift_f32(n: int, seed: int, scale: float = 1.0) -> np.ndarray:
    out = np.zeros(n, dtype=np.float32)
    lib.orc_xorshift_f32(ptr(out), n, seed & 0xFFFFFFFF, scale)
    return out


# ---------------------------------------------------------------- model

class Model:
    """One sequence of the reference's TransformerModel on the CPU oracle."""

    LAYER_KEYS = ["rms_att_weight", "wq", "wk", "wv", "wo", "rms_ffn_weight", "w_gate", "w_up",
                  "w_down"]

    def __init__(self, cfg, weights, mode: int = MODE_X86, threads: int = 1):
        """cfg: any object with the TransformerConfig fields; weights: any
        object with token_embd, layers (dicts keyed like TransformerWeights),
        output_norm, lm_head (None = tied) and vocab, as host arrays."""
        cfg = Config(cfg.dim, cfg.hidden_dim, cfg.num_heads, cfg.num_kv_heads, cfg.max_seq_len,
                     cfg.rms_eps)
        self.cfg = cfg
        self.weights = weights
        nl = len(weights.layers)
        self.h = lib.orc_model_new(C.byref(cfg), nl, weights.vocab, mode, threads)
        self._layers = (LayerWeights * nl)()
        for l, lw in enumerate(weights.layers):
            self._layers[l] = LayerWeights(*[ptr(lw[k]) for k in self.LAYER_KEYS])
        lm = weights.lm_head if weights.lm_head is not None else weights.token_embd
        self._mw = ModelWeights(ptr(weights.token_embd), self._layers, nl,
                                ptr(weights.output_norm), ptr(lm), weights.vocab)
        rc = lib.orc_model_set_weights(self.h, C.byref(self._mw))
        assert rc == 0

    def close(self):
        if self.h:
            lib.orc_model_free(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def _view(self, p, n):
        return np.ctypeslib.as_array(p, shape=(n,))

    @property
    def kv_dim(self):
        return self.cfg.dim // self.cfg.num_heads * self.cfg.num_kv_heads

    def x(self):
        return self._view(lib.orc_model_x(self.h), self.cfg.dim)

    def xb(self):
        return self._view(lib.orc_model_xb(self.h), self.cfg.dim)

    def logits(self):
        return self._view(lib.orc_model_logits(self.h), self.weights.vocab)

    def k_cache(self, layer):
        return self._view(lib.orc_model_k_cache(self.h, layer), self.cfg.max_seq_len * self.kv_dim)

    def v_cache(self, layer):
        return self._view(lib.orc_model_v_cache(self.h, layer), self.cfg.max_seq_len * self.kv_dim)

    def forward_token(self, token: int, pos: int) -> int:
        return int(lib.orc_forward_token(self.h, token, pos))

    def layer_forward_token(self, layer: int, pos: int):
        lib.orc_layer_forward_token(self.h, layer, pos)

    def prefill_tokens(self, tokens, start_pos: int = 0) -> int:
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        return int(lib.orc_prefill_tokens(self.h, t.ctypes.data_as(_I32P), t.size, start_pos))

    def generate(self, prompt, n_out: int, eos: int = -1):
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(n_out, dtype=np.int32)
        n = lib.orc_generate(self.h, p.ctypes.data_as(_I32P), p.size, out.ctypes.data_as(_I32P),
                             n_out, eos)
        return out[:n].tolist()

    def embed_tokens(self, tokens):
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        out = np.zeros(self.cfg.dim, dtype=np.float32)
        lib.orc_embed_tokens(self.h, t.ctypes.data_as(_I32P), t.size,
                             out.ctypes.data_as(_F))
        return out


class XorshiftWeights:
    def __init__(self, token_embd, layers, output_norm, lm_head, vocab):
        self.token_embd, self.layers, self.output_norm = token_embd, layers, output_norm
        self.lm_head, self.vocab = lm_head, vocab


def xorshift_model(cfg, num_layers: int, vocab: int, scale: float = 0.25,
                   seeds=None) -> XorshiftWeights:
    """The reference's unit-test model recipe (transformer.rs:971-976 and
    :1269-1300): xorshift32 values times `scale`, quantized to Q4_0."""
    d, h = cfg.dim, cfg.hidden_dim
    kvd = d // cfg.num_heads * cfg.num_kv_heads
    sd = seeds or {}

    def qm(rows, cols, seed):
        return quantize_q4_0(xorshift_f32(rows * cols, seed, scale))

    layer = {
        "rms_att_weight": xorshift_f32(d, sd.get("rms_att", 0x1001), scale),
        "wq": qm(d, d, sd.get("wq", 0x2001)),
        "wk": qm(kvd, d, sd.get("wk", 0x2002)),
        "wv": qm(kvd, d, sd.get("wv", 0x2003)),
        "wo": qm(d, d, sd.get("wo", 0x2004)),
        "rms_ffn_weight": xorshift_f32(d, sd.get("rms_ffn", 0x1002), scale),
        "w_gate": qm(h, d, sd.get("w_gate", 0x3001)),
        "w_up": qm(h, d, sd.get("w_up", 0x3002)),
        "w_down": qm(d, h, sd.get("w_down", 0x3003)),
    }
    return XorshiftWeights(qm(vocab, d, sd.get("token_embd", 0x0100)), [layer] * num_layers,
                           np.ones(d, dtype=np.float32), qm(vocab, d, sd.get("lm_head", 0x0200)),
                           vocab)
