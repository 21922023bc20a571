"""Tensor-core Q4_0 x Q8_0 GEMM (slm_gemm_q4_0_tensor_cores, tcgen05
kind::i8): not bit-exact by design.  Each 32-element block's int8 dot product
is exact on the tensor cores; the f32 combination over blocks,
out += (dw * da) * isum, differs from the reference's eight AVX2 lane sums per
block (src/quant/kernels.rs:163-212) by rounding only.  Checked against the
CPU oracle's gemm_q4_0 (the reference's arithmetic) at a relative bound
derived from f32 rounding over nb blocks, on shapes with ragged row tiles,
ragged activation tiles and K not a multiple of the 128-element staging
group."""
import numpy as np
import pytest

import oracle as O
import static_lm as S
from static_lm import synth
from static_lm._lib import lib

pytestmark = pytest.mark.gpu

# (rows, cols, batch): config-3 QKV / Wo / down shapes at prefill batches, a
# row count that is not a multiple of 128, K = 18 and 48 blocks (groups of 4
# with a ragged last group), the Llama-3-8B Wq shape
CASES = [(960, 576, 300), (576, 1536, 513), (200, 576, 128), (4096, 4096, 256), (576, 576, 1000)]


def _q8_blocks(x):
    return O.quantize_q8_0(x)


@pytest.mark.parametrize("rows,cols,batch", CASES)
def test_tensor_core_gemm_against_oracle(cuda, rows, cols, batch):
    w = synth.synth_q4(rows, cols, rows + cols)
    qm = S.QMatrix(w, rows, cols)
    x = np.random.default_rng(batch).standard_normal(batch * cols).astype(np.float32)
    xq = _q8_blocks(x)
    want = O.gemm_q8(w, xq, batch, rows, cols, O.MODE_X86, 8)
    xd = cuda.from_numpy(xq.view(np.uint8).copy()).cuda()
    nbytes = int(lib().slm_gemm_q4_0_scratch_bytes(batch, cols))
    scratch = cuda.empty(nbytes // 4 + 4, dtype=cuda.float32, device="cuda")
    out_tc = cuda.full((batch * rows,), float("nan"), dtype=cuda.float32, device="cuda")
    out_ex = cuda.full((batch * rows,), float("nan"), dtype=cuda.float32, device="cuda")
    lib().slm_gemm_q4_0_tensor_cores(qm.h, xd.data_ptr(), out_tc.data_ptr(), batch, rows, cols,
                                     scratch.data_ptr(), nbytes, None)
    lib().slm_gemm_q4_0(qm.h, xd.data_ptr(), out_ex.data_ptr(), batch, rows, cols, scratch.data_ptr(),
                        nbytes, None)
    cuda.cuda.synchronize()
    tc, ex = out_tc.cpu().numpy(), out_ex.cpu().numpy()
    assert np.array_equal(ex, want)  # the exact path stays bit-exact
    # f32 rounding of the nb block terms of each chain (the reference's and
    # this one), partial sums up to a few times the final magnitude
    nb = cols // 32
    bound = 16.0 * (nb + 8) * np.finfo(np.float32).eps * np.abs(want).max()
    err = np.abs(tc - want)
    assert np.all(np.isfinite(tc))
    assert float(err.max()) <= bound, (float(err.max()), bound)
    assert np.all(err <= 1e-3 * np.abs(want) + 1e-4 * np.abs(want).max())
