"""The allocation-free GEMM entry point (static device scratch) through the C
ABI, against the CPU oracle's gemm_q4_0 and against the arena entry point.
Collected last on purpose: it must pass alone in a fresh process and after
every other test, since all calls share one static buffer that keeps the
previous call's contents."""
import numpy as np
import pytest

import oracle as O
import static_lm as S
from static_lm import synth
from static_lm._lib import SlmError, lib

pytestmark = pytest.mark.gpu

NOALLOC_SCRATCH_BYTES = 4 << 20  # SLM_NOALLOC_SCRATCH_BYTES
Q8X_BLOCK_BYTES = 68             # one 32-element block in the scratch


def _arena_gemm(qm, x, batch, rows, cols):
    nb = batch * cols // 32
    ar = S.Arena(batch * cols + batch * rows + nb * 17 + 256)
    s_in, s_q8, s_out = ar.alloc_slice(batch * cols), ar.alloc_q8_scratch(nb), ar.alloc_slice(batch * rows)
    ar.write(s_in, x)
    S.gemm_q4_0_arena(ar, qm, s_in, s_q8, s_out, batch, rows, cols)
    return ar.read(s_out)


def _noalloc_gemm(torch, qm, x, batch, rows, cols):
    xd = torch.from_numpy(x).cuda()
    out = torch.full((batch * rows,), float("nan"), dtype=torch.float32, device="cuda")
    lib().slm_gemm_q4_0_f32_noalloc(qm.h, xd.data_ptr(), out.data_ptr(), batch, rows, cols, None)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def test_noalloc_gemm_matches_oracle_and_arena_gemm_on_consecutive_calls(cuda):
    # calls in a row with different inputs and sizes: a later call must not
    # see anything of an earlier call's scratch contents
    for batch, rows, cols, seed in ((64, 960, 576, 1), (3, 300, 1536, 2), (64, 960, 576, 3)):
        w = synth.synth_q4(rows, cols, seed)
        qm = S.QMatrix(w, rows, cols)
        x = (np.random.default_rng(seed).standard_normal(batch * cols)).astype(np.float32)
        got = _noalloc_gemm(cuda, qm, x, batch, rows, cols)
        want = O.gemm_f32(w, x, batch, rows, cols, O.MODE_X86, 4)
        assert np.array_equal(got, want), (batch, rows, cols, np.abs(got - want).max())
        assert np.array_equal(got, _arena_gemm(qm, x, batch, rows, cols))


def test_noalloc_gemm_rejects_sizes_beyond_the_static_scratch(cuda):
    rows, cols = 32, 1536
    w = synth.synth_q4(rows, cols, 4)
    qm = S.QMatrix(w, rows, cols)
    fit = NOALLOC_SCRATCH_BYTES // Q8X_BLOCK_BYTES * 32 // cols  # the largest batch that fits
    batch = fit + 1
    x = cuda.zeros(batch * cols, dtype=cuda.float32, device="cuda")
    out = cuda.zeros(batch * rows, dtype=cuda.float32, device="cuda")
    with pytest.raises(SlmError) as e:
        lib().slm_gemm_q4_0_f32_noalloc(qm.h, x.data_ptr(), out.data_ptr(), batch, rows, cols, None)
    assert "static buffer" in str(e.value)
    # the largest size that fits runs and fills the buffer to its last block:
    # its output is checked, so an off-by-one at the buffer's end would show
    xf = (np.random.default_rng(5).standard_normal(fit * cols)).astype(np.float32)
    got = _noalloc_gemm(cuda, qm, xf, fit, rows, cols)
    assert np.array_equal(got, O.gemm_f32(w, xf, fit, rows, cols, O.MODE_X86, 4))
