"""Operator-level parity of the sm_100a kernels with the CPU oracle, through
the C ABI.  Every comparison is bit-exact: Q8_0 bytes, int dot sums, and the
f32 results of the reference's operation order."""
import ctypes as C

import numpy as np
import pytest

import oracle as O
import static_lm as S
from static_lm import synth
from static_lm._lib import JIT_KERNEL_FN, JIT_OPS, Config, SlmError, lib

pytestmark = pytest.mark.gpu


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    t.device  # noqa
    import torch
    torch.cuda.synchronize()
    return t.cpu().numpy()


def rand_f32(n, seed, scale=1.0):
    return (np.random.default_rng(seed).standard_normal(n) * scale).astype(np.float32)


def tricky_f32(n, seed):
    """Values that stress Q8 rounding: exact ties, zeros, tiny and huge blocks."""
    x = rand_f32(n, seed)
    nb = n // 32
    for b in range(nb):
        kind = b % 6
        blk = x[b * 32:(b + 1) * 32]
        if kind == 1:
            blk[:] = 0.0
        elif kind == 2:  # amax 127 -> id 1: x.5 ties
            blk[:] = (np.arange(32, dtype=np.float32) - 16) + np.float32(0.5)
            blk[0] = 127.0
        elif kind == 3:
            blk *= np.float32(1e-30)
        elif kind == 4:
            blk *= np.float32(3e4)
        elif kind == 5:
            blk[:] = np.float32(-1.0)
    return x


def test_quantize_row_q8_0_bit_exact(cuda):
    for n, seed in ((32, 1), (576, 2), (1536, 3), (32 * 1000, 4)):
        x = tricky_f32(n, seed)
        xd = dev(cuda, x)
        out = cuda.zeros(n // 32 * 34, dtype=cuda.uint8, device="cuda")
        lib().slm_quantize_row_q8_0(xd.data_ptr(), out.data_ptr(), n, None)
        assert np.array_equal(host(out), O.quantize_q8_0(x).view(np.uint8))


def one_block_q4(d, byte):
    b = np.zeros(18, np.uint8)
    b[0:2] = np.array([d], np.float16).view(np.uint8)
    b[2:] = byte
    return b


def one_block_q8(d, val):
    b = np.zeros(34, np.uint8)
    b[0:2] = np.array([d], np.float16).view(np.uint8)
    b[2:] = np.array([val], np.int8).view(np.uint8)
    return b


def test_gemm_q4_0_known_answers(cuda):
    """kernels.rs:640-649 through the pre-quantized entry point."""
    for wb, ab, want in ((0x00, -127, 32512.0), (0xFF, 127, 28448.0), (0x00, -128, 32512.0)):
        w = S.QMatrix(one_block_q4(1.0, wb), 1, 32)
        xq = dev(cuda, one_block_q8(1.0, ab))
        out = cuda.zeros(1, dtype=cuda.float32, device="cuda")
        scratch = cuda.zeros(256, dtype=cuda.uint8, device="cuda")
        lib().slm_gemm_q4_0(w.h, xq.data_ptr(), out.data_ptr(), 1, 1, 32, scratch.data_ptr(), 256,
                            None)
        assert host(out)[0] == want


GEMM_SHAPES = [  # (batch, rows, cols)
    (1, 1, 32), (1, 576, 576), (1, 960, 576), (3, 100, 64), (2, 33, 96), (4, 3072, 576),
    (5, 576, 1536), (64, 1536, 576), (64, 576, 1536), (8, 4096, 4096), (1, 14336, 4096),
    (1, 32000, 288), (7, 49152, 576),
    # batch 1 of wide matrices: the block-split GEMV (64+ blocks a row), ragged
    # row tiles and a last round of one block (65 and 129 blocks)
    (1, 4096, 4096), (1, 100, 2048), (1, 576, 2080), (1, 33, 4128),
    # prefill-sized batches: the GEMM shape (4 activation rows per warp), ragged edges
    (1024, 576, 576), (1037, 300, 64), (1100, 960, 576), (2048, 576, 1536),
]


@pytest.mark.parametrize("batch,rows,cols", GEMM_SHAPES)
def test_gemm_q4_0_arena_bit_exact(cuda, batch, rows, cols):
    w = synth.synth_q4(rows, cols, rows * 7 + cols)
    x = rand_f32(batch * cols, batch + rows)
    ref = O.gemm_f32(w, x, batch, rows, cols, O.MODE_X86, threads=4)
    qm = S.QMatrix(w, rows, cols)
    nb = batch * cols // 32
    ar = S.Arena(batch * cols + batch * rows + nb * 17 + 256)
    s_in, s_q8, s_out = ar.alloc_slice(batch * cols), ar.alloc_q8_scratch(nb), ar.alloc_slice(batch * rows)
    ar.write(s_in, x)
    if batch == 1:
        S.gemv_q4_0_arena(ar, qm, s_in, s_q8, s_out, rows, cols)
    else:
        S.gemm_q4_0_arena(ar, qm, s_in, s_q8, s_out, batch, rows, cols)
    got = ar.read(s_out)
    assert np.array_equal(got, ref), np.abs(got - ref).max()


def test_gemm_q4_0_prequantized_matches_oracle(cuda):
    batch, rows, cols = 6, 300, 512
    w = synth.synth_q4(rows, cols, 99)
    xq = O.quantize_q8_0(tricky_f32(batch * cols, 5))
    raw = xq.view(np.uint8).copy()
    raw[2] = 0x80  # a -128 activation: the SIMD path clamps it (kernels.rs:189-191)
    ref = O.gemm_q8(w, raw.view(O.Q8_DTYPE), batch, rows, cols, O.MODE_X86)
    qm = S.QMatrix(w, rows, cols)
    need = int(lib().slm_gemm_q4_0_scratch_bytes(batch, cols))
    scratch = cuda.zeros(need, dtype=cuda.uint8, device="cuda")
    xd = dev(cuda, raw)
    out = cuda.zeros(batch * rows, dtype=cuda.float32, device="cuda")
    lib().slm_gemm_q4_0(qm.h, xd.data_ptr(), out.data_ptr(), batch, rows, cols, scratch.data_ptr(),
                        need, None)
    assert np.array_equal(host(out), ref)


def test_qmatrix_roundtrip_byte_exact(cuda):
    for rows, cols in ((1, 32), (33, 64), (960, 576), (49152, 576)):
        w = synth.synth_q4(rows, cols, rows + cols)
        assert np.array_equal(S.QMatrix(w, rows, cols).download(), w)


def test_arena_slice_checks(cuda):
    ar = S.Arena(4096)
    a = ar.alloc_slice(100)
    assert a.offset == 0 and a.len == 100
    b = ar.alloc_slice(10)
    assert b.offset == 112  # 64-byte alignment (arena.rs:96-110)
    q8 = ar.alloc_q8_scratch(2)
    w = S.QMatrix(synth.synth_q4(10, 64, 1), 10, 64)
    with pytest.raises(SlmError) as e:
        S.gemv_q4_0_arena(ar, w, a.subslice(0, 64), q8, a.subslice(50, 10), 10, 64)
    assert e.value.code == 3  # OVERLAP
    with pytest.raises(SlmError) as e:
        S.gemv_q4_0_arena(ar, w, a.subslice(0, 64), ar.alloc_q8_scratch(1), b, 10, 64)
    assert e.value.code == 5  # CAPACITY
    with pytest.raises(SlmError) as e:
        ar.alloc_slice(1 << 20)
    assert e.value.code == 5
    with pytest.raises(SlmError) as e:
        S.gemv_q4_0_arena(ar, w, a.subslice(0, 64), q8, b, 11, 64)
    assert e.value.code == 4  # SHAPE


def exec_op(cuda, name, inputs, n, *extra, out_len=None):
    ins = [dev(cuda, a) for a in inputs]
    out = cuda.full(((out_len or n) + 4,), -999.0, dtype=cuda.float32, device="cuda")
    arr = (C.c_void_p * len(ins))(*[t.data_ptr() for t in ins])
    getattr(lib(), name)(C.cast(arr, C.POINTER(C.c_void_p)), out.data_ptr(), n, *extra, None)
    h = host(out)
    assert np.all(h[n:] == -999.0), "wrote past len"
    return h[:n]


LENS = [1, 2, 3, 5, 7, 15, 33, 256, 576, 1024, 2049, 4099]


@pytest.mark.parametrize("n", LENS)
def test_jit_ops_bit_exact(cuda, n):
    a = rand_f32(n, n, 2.0)
    b = rand_f32(n, n + 1, 2.0)
    assert np.array_equal(exec_op(cuda, "slm_exec_softmax", [a], n), O.softmax(a))
    assert np.array_equal(exec_op(cuda, "slm_exec_rmsnorm", [a, b], n, C.c_float(1e-5)),
                          O.rmsnorm(a, b, 1e-5))
    assert np.array_equal(exec_op(cuda, "slm_exec_swiglu", [a, b], n), O.swiglu(a, b))
    assert np.array_equal(exec_op(cuda, "slm_exec_residual_add", [a, b], n), O.residual_add(a, b))
    assert np.array_equal(exec_op(cuda, "slm_exec_l2_norm", [a], n, C.c_float(1e-5)),
                          O.l2_norm(a, 1e-5))


def jit_call(cuda, op, inputs, n, graph_n=0, eps=0.0):
    """Compile `op` to a JitKernelFn pointer and call it exactly as the
    reference's JitEngine::exec_* do: (host array of input pointers, output
    pointer, len) (engine.rs:153-206)."""
    fp = C.c_void_p()
    lib().slm_jit_compile(JIT_OPS[op], graph_n, eps, None, C.byref(fp))
    fn = JIT_KERNEL_FN(fp.value)
    ins = [dev(cuda, a) for a in inputs]
    out = cuda.full((n + 4,), -999.0, dtype=cuda.float32, device="cuda")
    arr = (C.c_void_p * len(ins))(*[t.data_ptr() for t in ins])
    fn(C.cast(arr, C.POINTER(C.c_void_p)), out.data_ptr(), n)
    h = host(out)
    assert np.all(h[n:] == -999.0), "wrote past len"
    return h[:n]


@pytest.mark.parametrize("n", [1, 7, 33, 576, 2049])
def test_jit_kernel_fn_entry_points_bit_exact(cuda, n):
    a = rand_f32(n, n + 7, 2.0)
    b = rand_f32(n, n + 8, 2.0)
    assert np.array_equal(jit_call(cuda, "softmax", [a], n), O.softmax(a))
    assert np.array_equal(jit_call(cuda, "rmsnorm", [a, b], n, n, 1e-5), O.rmsnorm(a, b, 1e-5))
    assert np.array_equal(jit_call(cuda, "swiglu", [a, b], n), O.swiglu(a, b))
    assert np.array_equal(jit_call(cuda, "residual_add", [a, b], n), O.residual_add(a, b))
    assert np.array_equal(jit_call(cuda, "l2_norm", [a], n, 0, 1e-5), O.l2_norm(a, 1e-5))


def test_jit_rmsnorm_uses_the_graph_n(cuda):
    """FuseGraph::rmsnorm(n, eps) bakes 1/n in (graph.rs:147): run on len != n
    it scales the sum of squares by 1/n, not 1/len."""
    n, graph_n = 64, 96
    a, b = rand_f32(n, 1, 2.0), rand_f32(n, 2, 2.0)
    got = jit_call(cuda, "rmsnorm", [a, b], n, graph_n, 1e-5)
    s = O.rmsnorm(np.concatenate([a, np.zeros(graph_n - n, np.float32)]),
                  np.concatenate([b, np.zeros(graph_n - n, np.float32)]), 1e-5)[:n]
    assert np.array_equal(got, s)


def test_softmax_in_place_and_extremes(cuda):
    x = np.float32([-1e30, 0.0, 1e4, 88.0, -88.0, 3.0, 3.0, -0.0, 0.5])
    t = dev(cuda, x)
    arr = (C.c_void_p * 1)(t.data_ptr())
    lib().slm_exec_softmax(C.cast(arr, C.POINTER(C.c_void_p)), t.data_ptr(), x.size, None)
    assert np.array_equal(host(t), O.softmax(x))


def test_rope_cached_bit_exact(cuda):
    hd, T = 64, 64
    c, s = O.rope_tables(T, hd)
    for pos in (0, 1, 17, 63):
        v = rand_f32(576, pos)
        t = dev(cuda, v)
        cd, sd = dev(cuda, c[pos * 32:(pos + 1) * 32]), dev(cuda, s[pos * 32:(pos + 1) * 32])
        lib().slm_apply_rope_cached(t.data_ptr(), 576, cd.data_ptr(), sd.data_ptr(), hd, None)
        assert np.array_equal(host(t), O.apply_rope_cached(v, c[pos * 32:(pos + 1) * 32],
                                                           s[pos * 32:(pos + 1) * 32], hd))


ATT_CFGS = [  # dim, heads, kv_heads, max_seq
    (64, 4, 4, 512), (128, 8, 2, 512), (288, 6, 6, 512), (576, 9, 3, 2112), (4096, 32, 8, 2112),
]


@pytest.mark.parametrize("dim,heads,kvh,T", ATT_CFGS)
def test_attention_bit_exact(cuda, dim, heads, kvh, T):
    cfg_o = O.Config(dim, 4 * dim, heads, kvh, T, 1e-5)
    cfg_s = Config(dim, 4 * dim, heads, kvh, T, 1e-5)
    kvd = dim // heads * kvh
    k = rand_f32(T * kvd, 1)
    v = rand_f32(T * kvd, 2)
    kd, vd = dev(cuda, k), dev(cuda, v)
    for pos in (0, 1, 5, 127, 128, 300, T - 1):
        q = rand_f32(dim, pos + 3)
        ref_out, ref_att = O.attention(q, k, v, cfg_o, pos)
        qd = dev(cuda, q)
        att = cuda.zeros(heads * T, dtype=cuda.float32, device="cuda")
        out = cuda.zeros(dim, dtype=cuda.float32, device="cuda")
        lib().slm_causal_attention(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), att.data_ptr(),
                                   out.data_ptr(), C.byref(cfg_s), pos, None)
        got = host(out)
        assert np.array_equal(got, ref_out), (pos, np.abs(got - ref_out).max())
        ga = host(att).reshape(heads, T)[:, :pos + 1]
        assert np.array_equal(ga, ref_att.reshape(heads, T)[:, :pos + 1])


def test_argmax_first_max(cuda):
    cases = [np.float32([1, 3, 3, 2]), np.float32([-np.inf, -np.inf]),
             np.float32([np.nan, 5.0, 1.0]), np.float32([0.0, np.nan, 1.0]),
             np.concatenate([np.zeros(5000, np.float32), np.float32([7]), np.zeros(40000, np.float32),
                             np.float32([7])])]
    for x in cases:
        t = dev(cuda, x)
        o = cuda.zeros(1, dtype=cuda.int32, device="cuda")
        lib().slm_sample_argmax(t.data_ptr(), x.size, o.data_ptr(), None)
        assert int(host(o)[0]) == O.argmax(x)
