"""The C ABI without a GPU: libslm_b200.so loads, exports every function
include/slm_b200.h declares, and its host-only entry points and argument
checks behave like the reference (errors instead of panics)."""
import ctypes as C
import os
import re

import numpy as np
import pytest

import oracle as O
import static_lm as S
from static_lm._lib import SIGNATURES, Config, SlmError, lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "slm_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(slm_\w+)\s*\(", text)))


def test_header_declares_the_binding_and_library_exports_all():
    names = declared_functions()
    assert len(names) >= 40
    assert set(names) == set(SIGNATURES), set(names) ^ set(SIGNATURES)
    dll = C.CDLL(lib().path)
    for n in names:
        assert hasattr(dll, n), n


def test_version_and_last_error():
    assert b"sm_100a" in lib().slm_version()
    with pytest.raises(SlmError) as e:
        lib().slm_arena_create(0, 16, None)
    assert e.value.code == 1
    assert b"null" in lib().slm_last_error()


def test_rope_tables_match_oracle_bit_exact():
    for T, hd in ((512, 64), (256, 48), (64, 128), (8, 16)):
        c, s = S.rope_tables(T, hd)
        oc, os_ = O.rope_tables(T, hd)
        assert np.array_equal(c, oc) and np.array_equal(s, os_)


def test_host_side_argument_checks_without_gpu():
    # checks that fail before any CUDA call
    w = np.zeros(18, np.uint8)
    h = C.c_void_p()
    with pytest.raises(SlmError) as e:
        lib().slm_qmatrix_upload(0, w.ctypes.data, 1, 33, C.byref(h))
    assert e.value.code == 4
    with pytest.raises(SlmError) as e:
        lib().slm_quantize_row_q8_0(None, None, 33, None)
    assert e.value.code == 4
    bad = Config(100, 128, 4, 4, 16, 1e-5)  # dim % 32
    with pytest.raises(SlmError) as e:
        lib().slm_causal_attention(None, None, None, None, None, C.byref(bad), 0, None)
    assert e.value.code == 4
    gqa_bad = Config(128, 128, 8, 3, 16, 1e-5)  # heads % kv_heads
    with pytest.raises(SlmError) as e:
        lib().slm_model_create(0, C.byref(gqa_bad), None, 1, 1, C.byref(h))
    assert e.value.code == 4
    with pytest.raises(SlmError) as e:
        lib().slm_rope_tables(4, 7, None, None)
    assert e.value.code in (1, 4)


def test_product_path_has_no_oracle_dependency():
    """Nothing in the product package or the library names the oracle."""
    pkg = os.path.join(ROOT, "static-lm_b200")
    for dirpath, _, files in os.walk(pkg):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".h", ".cpp")):
                text = open(os.path.join(dirpath, f)).read()
                assert "import oracle" not in text and "liboracle" not in text, f
    syms = open(lib().path, "rb").read()
    assert b"orc_" not in syms


def test_jit_compile_caches_like_the_engine_without_gpu():
    """slm_jit_compile hands out JitKernelFn pointers (engine.rs:15, 66-72):
    the same graph (operator, n, eps, stream) gives the same pointer, another
    graph another pointer; unknown operators are rejected.  No GPU work."""
    from static_lm._lib import JIT_OPS

    def comp(op, n=0, eps=0.0, stream=None):
        fp = C.c_void_p()
        lib().slm_jit_compile(JIT_OPS[op], n, eps, stream, C.byref(fp))
        return fp.value

    a = comp("rmsnorm", 576, 1e-5)
    assert a and comp("rmsnorm", 576, 1e-5) == a
    assert comp("rmsnorm", 576, 1e-6) != a
    assert comp("rmsnorm", 288, 1e-5) not in (a, None)
    s = comp("softmax")
    assert s not in (a, None) and comp("softmax", 7, 0.5) == s  # constants softmax ignores
    with pytest.raises(SlmError) as e:
        comp("rmsnorm", 0, 1e-5)
    assert e.value.code == 1
    fp = C.c_void_p()
    with pytest.raises(SlmError):
        lib().slm_jit_compile(9, 0, 0.0, None, C.byref(fp))
