"""Pins the CPU oracle's quantizers and vec-dot against the reference's own
known answers and error bounds (src/quant/blocks.rs:137-220,
src/quant/kernels.rs:417-650)."""
import numpy as np
import pytest

import oracle as O


def q4_block(d: float, byte: int):
    b = np.zeros(1, O.Q4_DTYPE)
    b["d"] = O.f32_to_f16(d)
    b["qs"] = byte
    return b


def q8_block(d: float, val: int):
    b = np.zeros(1, O.Q8_DTYPE)
    b["d"] = O.f32_to_f16(d)
    b["qs"] = val
    return b


def test_block_sizes():
    assert O.Q4_DTYPE.itemsize == 18 and O.Q8_DTYPE.itemsize == 34


def test_f16_conversion_matches_ieee_rne():
    # numpy's float16 cast is IEEE round-to-nearest-even, like half 2.7.1
    rng = np.random.default_rng(1)
    xs = np.concatenate([rng.standard_normal(20000).astype(np.float32) * s
                         for s in (1e-8, 1e-6, 1e-4, 0.01, 1, 100, 1e4, 7e4)])
    xs = np.concatenate([xs, np.float32([0.0, -0.0, 65504, 65520, 65536, 6e-8, 3e-8, 2.98e-8])])
    for x in xs:
        assert O.f32_to_f16(float(x)) == int(np.float16(x).view(np.uint16)), x
    for h in range(0, 65536, 7):
        f = np.uint16(h).view(np.float16).astype(np.float32)
        got = O.f16_to_f32(h)
        assert (np.isnan(f) and np.isnan(got)) or got == f


def test_vec_dot_known_answers_kernels_rs_640_649():
    wmin, wmax = q4_block(1.0, 0x00), q4_block(1.0, 0xFF)
    amin, amax, a128 = q8_block(1.0, -127), q8_block(1.0, 127), q8_block(1.0, -128)
    for kind in ("x86", "avx2", "scalar"):
        assert O.vec_dot(wmin, amin, kind) == 32512.0
        assert O.vec_dot(wmax, amax, kind) == 28448.0
    # the SIMD path clamps -128 to -127 before the sign trick (kernels.rs:189-191)
    assert O.vec_dot(wmin, a128, "x86") == 32512.0
    assert O.vec_dot(wmin, a128, "avx2") == 32512.0


@pytest.mark.parametrize("nb", [1, 3, 7, 17])
def test_vec_dot_odd_block_counts(nb):
    n = nb * 32
    w = O.quantize_q4_0(O.xorshift_f32(n, 0x1000 + nb))
    a = O.quantize_q8_0(O.xorshift_f32(n, 0x2000 + nb))
    s, v = O.vec_dot(w, a, "scalar"), O.vec_dot(w, a, "x86")
    assert abs(s - v) < 1e-5
    assert O.vec_dot(w, a, "avx2") == v  # intrinsics == lane emulation, bit for bit


def test_vec_dot_simd_matches_scalar():
    n = 1024
    w = O.quantize_q4_0(O.xorshift_f32(n, 0x11223344))
    a = O.quantize_q8_0(O.xorshift_f32(n, 0x55667788))
    assert abs(O.vec_dot(w, a, "scalar") - O.vec_dot(w, a, "x86")) < 1e-5


def test_vec_dot_scalar_vs_f32_reference():
    n = 4096
    wf = O.xorshift_f32(n, 0xCAFEBABE) + np.float32(0.5)
    af = O.xorshift_f32(n, 0xDEADBEEF) + np.float32(0.5)
    ref = np.float32(0)
    for i in range(n):
        ref = np.float32(ref + wf[i] * af[i])
    q = O.vec_dot(O.quantize_q4_0(wf), O.quantize_q8_0(af), "scalar")
    assert abs(ref - q) / abs(ref) < 1e-2


def test_avx2_intrinsics_bit_exact_many():
    rng = np.random.default_rng(7)
    for nb in (1, 2, 5, 18, 48, 128, 448):
        for _ in range(5):
            w = O.quantize_q4_0(rng.standard_normal(nb * 32).astype(np.float32))
            a = O.quantize_q8_0(rng.standard_normal(nb * 32).astype(np.float32))
            assert O.vec_dot(w, a, "avx2") == O.vec_dot(w, a, "x86")


def test_gemv_against_naive_f32_and_parallel():
    rows, cols = 512, 4096
    wf = O.xorshift_f32(rows * cols, 0x99AABBCC) + np.float32(0.5)
    xf = O.xorshift_f32(cols, 0xDDEEFF11) + np.float32(0.5)
    wq, xq = O.quantize_q4_0(wf), O.quantize_q8_0(xf)
    par = O.gemm_q8(wq, xq, 1, rows, cols, O.MODE_X86, threads=4)
    ser = O.gemm_q8(wq, xq, 1, rows, cols, O.MODE_X86, threads=1)
    assert np.array_equal(par, ser)  # the pool changes who computes a row, not its value
    nb = cols // 32
    ref = wf.reshape(rows, cols).astype(np.float64) @ xf.astype(np.float64)
    rel = np.abs(ref - par) / np.abs(ref)
    assert rel.max() < 1.5e-2 and rel.mean() < 1e-2
    for r in range(0, rows, 37):
        s = O.vec_dot(wq[r * nb:(r + 1) * nb], xq, "scalar")
        assert abs(s - par[r]) / max(abs(s), 1.0) < 1e-5


def test_gemm_batch_matches_per_row_gemv():
    batch, rows, cols = 4, 32, 256
    wq = O.quantize_q4_0(O.xorshift_f32(rows * cols, 0xABCD1234) + np.float32(0.5))
    xf = O.xorshift_f32(batch * cols, 0x5678EF90) + np.float32(0.5)
    out = O.gemm_f32(wq, xf, batch, rows, cols)
    nb = cols // 32
    for b in range(batch):
        xq = O.quantize_q8_0(xf[b * cols:(b + 1) * cols])
        for r in range(rows):
            assert out[b * rows + r] == O.vec_dot(wq[r * nb:(r + 1) * nb], xq, "x86")
            assert abs(out[b * rows + r] - O.vec_dot(wq[r * nb:(r + 1) * nb], xq, "scalar")) < 1e-4


def test_q4_roundtrip_error_blocks_rs_154():
    x = O.xorshift_f32(256, 0x12345678)
    r = O.dequantize_q4_0(O.quantize_q4_0(x))
    assert np.abs(x - r).max() <= 0.0725


def test_q8_roundtrip_error_blocks_rs_173():
    x = O.xorshift_f32(256, 0x87654321)
    r = O.dequantize_q8_0(O.quantize_q8_0(x))
    assert np.abs(x - r).max() <= 0.005


def test_quantize_zero_and_negative_extremes_blocks_rs_191():
    z = np.zeros(64, np.float32)
    q4, q8 = O.quantize_q4_0(z), O.quantize_q8_0(z)
    assert O.f16_to_f32(int(q4["d"][0])) == 0.0 and O.f16_to_f32(int(q8["d"][0])) == 0.0
    assert np.all(O.dequantize_q4_0(q4) == 0) and np.all(O.dequantize_q8_0(q8) == 0)
    neg = -(np.arange(32, dtype=np.float32) + 1) * 10
    r = O.dequantize_q4_0(O.quantize_q4_0(neg))
    assert np.abs(neg - r).max() <= 20.5


def test_q8_rounding_is_half_away_from_zero():
    # amax = 127 -> id = 1: values x.5 must round away from zero (f32::round)
    x = np.zeros(32, np.float32)
    x[0] = 127.0
    x[1:9] = [0.5, -0.5, 1.5, -1.5, 2.5, -2.5, 126.5, -126.5]
    q = O.quantize_q8_0(x)["qs"][0]
    assert list(q[:9]) == [127, 1, -1, 2, -2, 3, -3, 127, -127]
