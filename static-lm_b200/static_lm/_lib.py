"""ctypes binding of libslm_b200.so (the C ABI declared in include/slm_b200.h).

The library is the product: there is no Python or CPU fallback.  Loading it
fails loudly when the shared object is missing; calls fail loudly (SlmError)
when it reports an error.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(os.path.dirname(HERE), "libslm_b200.so")

SLM_OK = 0
STATUS_NAMES = {1: "INVALID_ARG", 2: "OUT_OF_BOUNDS", 3: "OVERLAP", 4: "SHAPE", 5: "CAPACITY",
                6: "CUDA", 7: "DEVICE_INPUT", 8: "TIMEOUT"}


class SlmError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{STATUS_NAMES.get(code, code)}: {msg}")
        self.code = code


class Config(C.Structure):
    """slm_config == TransformerConfig (transformer.rs:8-16)."""
    _fields_ = [("dim", C.c_uint32), ("hidden_dim", C.c_uint32), ("num_heads", C.c_uint32),
                ("num_kv_heads", C.c_uint32), ("max_seq_len", C.c_uint32), ("rms_eps", C.c_float)]


class Slice(C.Structure):
    """slm_slice == ArenaSlice (arena.rs:11-14), f32 units."""
    _fields_ = [("offset", C.c_uint64), ("len", C.c_uint64)]

    def __repr__(self):
        return f"Slice(offset={self.offset}, len={self.len})"

    def subslice(self, rel: int, n: int) -> "Slice":
        if rel + n > self.len:
            raise SlmError(2, "ArenaSlice::subslice out of bounds")
        return Slice(self.offset + rel, n)


class LayerWeights(C.Structure):
    _fields_ = [("rms_att_weight", C.c_void_p), ("wq", C.c_void_p), ("wk", C.c_void_p),
                ("wv", C.c_void_p), ("wo", C.c_void_p), ("rms_ffn_weight", C.c_void_p),
                ("w_gate", C.c_void_p), ("w_up", C.c_void_p), ("w_down", C.c_void_p)]


class ModelWeights(C.Structure):
    _fields_ = [("token_embd", C.c_void_p), ("layers", C.POINTER(LayerWeights)),
                ("num_layers", C.c_uint32), ("output_norm", C.c_void_p), ("lm_head", C.c_void_p),
                ("vocab_size", C.c_uint32)]


_V = C.c_void_p
_U64 = C.c_uint64
_U32 = C.c_uint32
_I32P = C.POINTER(C.c_int32)
_U32P = C.POINTER(C.c_uint32)

# name -> (restype, argtypes, checked)
SIGNATURES = {
    "slm_last_error": (C.c_char_p, [], False),
    "slm_version": (C.c_char_p, [], False),
    "slm_arena_create": (C.c_int, [C.c_int, _U64, C.POINTER(_V)], True),
    "slm_arena_destroy": (None, [_V], False),
    "slm_arena_alloc_slice": (C.c_int, [_V, _U64, C.POINTER(Slice)], True),
    "slm_arena_alloc_q8_scratch": (C.c_int, [_V, _U64, C.POINTER(Slice)], True),
    "slm_arena_reset": (None, [_V], False),
    "slm_arena_capacity": (_U64, [_V], False),
    "slm_arena_used": (_U64, [_V], False),
    "slm_arena_device_ptr": (_V, [_V, Slice], False),
    "slm_arena_write": (C.c_int, [_V, Slice, _V, _U64], True),
    "slm_arena_read": (C.c_int, [_V, Slice, _V, _U64], True),
    "slm_qmatrix_upload": (C.c_int, [C.c_int, _V, _U64, _U64, C.POINTER(_V)], True),
    "slm_qmatrix_download": (C.c_int, [_V, _V], True),
    "slm_qmatrix_destroy": (None, [_V], False),
    "slm_gemv_q4_0_arena": (C.c_int, [_V, _V, Slice, Slice, Slice, _U64, _U64, _V], True),
    "slm_gemm_q4_0_arena": (C.c_int, [_V, _V, Slice, Slice, Slice, _U64, _U64, _U64, _V], True),
    "slm_gemm_q4_0": (C.c_int, [_V, _V, _V, _U64, _U64, _U64, _V, _U64, _V], True),
    "slm_gemm_q4_0_scratch_bytes": (_U64, [_U64, _U64], False),
    "slm_gemm_q4_0_tensor_cores": (C.c_int, [_V, _V, _V, _U64, _U64, _U64, _V, _U64, _V], True),
    "slm_gemm_q4_0_f32_noalloc": (C.c_int, [_V, _V, _V, _U64, _U64, _U64, _V], True),
    "slm_quantize_row_q8_0": (C.c_int, [_V, _V, _U64, _V], True),
    "slm_selftest_bounded_wait": (C.c_int, [C.c_int, _U64], False),
    "slm_exec_rmsnorm": (C.c_int, [C.POINTER(_V), _V, _U64, C.c_float, _V], True),
    "slm_exec_softmax": (C.c_int, [C.POINTER(_V), _V, _U64, _V], True),
    "slm_exec_swiglu": (C.c_int, [C.POINTER(_V), _V, _U64, _V], True),
    "slm_exec_residual_add": (C.c_int, [C.POINTER(_V), _V, _U64, _V], True),
    "slm_exec_l2_norm": (C.c_int, [C.POINTER(_V), _V, _U64, C.c_float, _V], True),
    "slm_jit_compile": (C.c_int, [C.c_int, _U64, C.c_float, _V, C.POINTER(_V)], True),
    "slm_rope_tables": (C.c_int, [_U32, _U32, _V, _V], True),
    "slm_apply_rope_cached": (C.c_int, [_V, _U64, _V, _V, _U32, _V], True),
    "slm_causal_attention": (C.c_int, [_V, _V, _V, _V, _V, C.POINTER(Config), _U32, _V], True),
    "slm_causal_attention_rows": (C.c_int, [_V, _V, _V, _V, _V, C.POINTER(Config), _U32, _U32, C.c_int, _V],
                                  True),
    "slm_sample_argmax": (C.c_int, [_V, _U64, _V, _V], True),
    "slm_model_create": (C.c_int, [C.c_int, C.POINTER(Config), C.POINTER(ModelWeights), _U32, _U32,
                                   C.POINTER(_V)], True),
    "slm_model_destroy": (None, [_V], False),
    "slm_model_stream": (_V, [_V], False),
    "slm_model_device_bytes": (_U64, [_V], False),
    "slm_model_forward_token": (C.c_int, [_V, _U32, C.c_int32, _U32, _I32P], True),
    "slm_model_prefill_tokens": (C.c_int, [_V, _U32, _I32P, _U32, _U32, _I32P], True),
    "slm_model_prefill_batch": (C.c_int, [_V, _U32, _U32P, _I32P, _U32, _I32P], True),
    "slm_nccl_unique_id": (C.c_int, [_V, _U64], True),
    "slm_model_attach_shard": (C.c_int, [_V, _V, _U64, C.c_int, C.c_int], True),
    "slm_model_set_comm_timeout": (C.c_int, [_V, _U32], True),
    "slm_model_set_prefill_mode": (C.c_int, [_V, C.c_int], True),
    "slm_model_set_decode_mode": (C.c_int, [_V, C.c_int], True),
    "slm_shard_units": (_U32, [_U32, _U32, _U32, _U32, _U32P, _U32], False),
    "slm_model_generate": (C.c_int, [_V, _U32, _I32P, _U32, _I32P, _U32, C.c_int32, _U32P], True),
    "slm_model_embed_tokens": (C.c_int, [_V, _U32, _I32P, _U32, C.POINTER(C.c_float)], True),
    "slm_model_decode_batch": (C.c_int, [_V, _U32, _U32P, _I32P, _U32P, _I32P], True),
    "slm_model_decode_steps_device": (C.c_int, [_V, _U32, _V, _V, _V, _U32, _V, _U32], True),
    "slm_model_kv_write": (C.c_int, [_V, _U32, _U32, _U32, _U32, _U32, _V], True),
    "slm_model_kv_read": (C.c_int, [_V, _U32, _U32, _U32, _U32, _U32, _V], True),
    "slm_model_read_logits": (C.c_int, [_V, _U32, _V], True),
    "slm_model_read_hidden": (C.c_int, [_V, _U32, _V], True),
    "slm_model_kv_write_device": (C.c_int, [_V, _U32, _U32, _U32, _U32, _U32, _V], True),
    "slm_model_profile_decode": (C.c_int, [_V, _U32, _V, _V, _V, _U32, _U32,
                                           C.POINTER(C.c_float)], True),
    "slm_model_launches_per_decode_step": (_U32, [_V, _U32], False),
}

# JitKernelFn (src/jit/engine.rs:15) as returned by slm_jit_compile
JIT_KERNEL_FN = C.CFUNCTYPE(None, C.POINTER(C.c_void_p), C.c_void_p, C.c_size_t)
JIT_OPS = {"rmsnorm": 0, "softmax": 1, "swiglu": 2, "residual_add": 3, "l2_norm": 4}

PHASES = ["embed", "rmsnorm_q8", "qkv_gemv_rope", "attn_scores", "attn_softmax", "attn_pv",
          "quantize_q8", "wo_gemv_residual", "gate_up_gemv_swiglu", "down_gemv_residual",
          "lm_head_gemv", "argmax", "advance", "attn_fused"]


class _Lib:
    def __init__(self, path: str = LIB_PATH):
        if not os.path.exists(path):
            raise ImportError(
                f"{path} is missing: build it with `python static-lm_b200/build.py` "
                "(there is no CPU fallback)")
        self.path = path
        self.dll = C.CDLL(path)
        for name, (res, args, checked) in SIGNATURES.items():
            fn = getattr(self.dll, name)
            fn.restype = res
            fn.argtypes = args
            setattr(self, name, self._checked(name, fn) if checked else fn)

    def _checked(self, name, fn):
        def call(*args):
            rc = fn(*args)
            if rc != SLM_OK:
                msg = self.dll.slm_last_error().decode(errors="replace")
                raise SlmError(rc, f"{name}: {msg}")
            return rc
        call.__name__ = name
        return call


_instance = None


def lib() -> _Lib:
    global _instance
    if _instance is None:
        _instance = _Lib()
    return _instance
