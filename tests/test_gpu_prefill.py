"""Batched prefill (slm_model_prefill_batch) against per-sequence prefill, and
its KV-head-sharded form on two GPUs against one GPU.  Bit-exact: the batched
and sharded forms run the same per-(row, head) chains; the all-gather only
moves bytes."""
import os

import numpy as np
import pytest

import static_lm as S
from static_lm import synth

pytestmark = pytest.mark.gpu


def _prompts(vocab, nseq, n, seed):
    return np.random.default_rng(seed).integers(0, vocab, (nseq, n)).astype(np.int32)


# (cfg3, 3 x 400): the batch of 1200 rows takes the GEMM shape of the
# projections (4 activation rows per warp, separate RMSNorm launch) while the
# 400-row prompts take the GEMV shape, so equality also pins GEMM == GEMV
@pytest.mark.parametrize("name,layers,nseq,n", [("cfg1", None, 3, 20), ("cfg2", 2, 2, 24),
                                                ("cfg3", 2, 2, 40), ("cfg3", 2, 3, 400)])
def test_prefill_batch_matches_per_sequence_prefill(cuda, name, layers, nseq, n):
    cfg, nl, vocab = synth.config(name)
    w = synth.synth_model(cfg, layers or nl, vocab, seed=21)
    prompts = _prompts(vocab, nseq, n, 3)
    batch = S.Model(cfg, w, max_sequences=nseq, max_rows=nseq * n)
    got = batch.prefill_batch(prompts)
    one = S.Model(cfg, w, max_sequences=nseq, max_rows=n)
    for s in range(nseq):
        assert one.prefill_tokens(prompts[s], seq=s) == got[s]
        want = one.logits(0)
        assert np.array_equal(batch.logits(s), want), s
    # decode continues from the batched prefill's KV exactly as from the sequential one
    nxt_b = batch.decode_batch(list(range(nseq)), list(got), [n] * nseq)
    for s in range(nseq):
        one.prefill_tokens(prompts[s], seq=s)
    nxt_o = one.decode_batch(list(range(nseq)), list(got), [n] * nseq)
    assert list(nxt_b) == list(nxt_o)


SH = ("cfg3", 2, 4, 48)  # name, layers, sequences, tokens: 12 (sequence, KV head) units


def _sharded_rank(rank, world, q_in, q_out, tensor_cores=False):
    import torch
    try:
        torch.cuda.set_device(rank)
        name, layers, nseq, n = SH
        cfg, _, vocab = synth.config(name)
        w = synth.synth_model(cfg, layers, vocab, seed=22)
        m = S.Model(cfg, w, max_sequences=nseq, max_rows=nseq * n, device=rank)
        m.set_prefill_mode(tensor_cores)
        if rank == 0:
            uid = S.nccl_unique_id()
            for _ in range(world - 1):
                q_in.put(uid)
        else:
            uid = q_in.get(timeout=120)
        m.attach_shard(uid, world, rank)
        nxt = m.prefill_batch(_prompts(vocab, nseq, n, 4))
        q_out.put((rank, list(nxt), [m.logits(s) for s in range(nseq)]))
        m.close()
    except Exception as e:
        q_out.put((rank, repr(e), None))
        raise


@pytest.mark.parametrize("tensor_cores", [False, True])
def test_sharded_prefill_on_two_gpus_matches_one_gpu(cuda, tensor_cores):
    """Either arithmetic mode: a (sequence, KV head) unit is computed by the
    same kernel whichever rank owns it, so two GPUs match one bit for bit."""
    if cuda.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    world = 2
    ctx = mp.get_context("spawn")
    q_in, q_out = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_sharded_rank, args=(r, world, q_in, q_out, tensor_cores))
             for r in range(world)]
    for p in procs:
        p.start()
    try:
        res = sorted(q_out.get(timeout=300) for _ in range(world))
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for rank, nxt, logits in res:
        assert logits is not None, (rank, nxt)
    name, layers, nseq, n = SH
    cfg, _, vocab = synth.config(name)
    w = synth.synth_model(cfg, layers, vocab, seed=22)
    ref = S.Model(cfg, w, max_sequences=nseq, max_rows=nseq * n)
    ref.set_prefill_mode(tensor_cores)
    want = list(ref.prefill_batch(_prompts(vocab, nseq, n, 4)))
    for rank, nxt, logits in res:
        assert nxt == want, rank
        for s in range(nseq):
            assert np.array_equal(logits[s], ref.logits(s)), (rank, s)


def test_tiled_prefill_matches_oracle_and_rowwise_kernels(cuda):
    """GQA (kv_mul 3, head_dim 64): a 150-token prompt (several 128-key and
    64-key tiles, a partial 16-row query tile), then 37 more tokens from
    start_pos 150; logits equal the oracle's and the per-row kernels'."""
    import oracle as O
    cfg, _, vocab = synth.config("cfg3", max_seq_len=256)
    w = synth.synth_model(cfg, 2, vocab, seed=23)
    toks = _prompts(vocab, 1, 187, 6)[0]
    tiled = S.Model(cfg, w, max_sequences=1, max_rows=160)
    os.environ["SLM_PREFILL_ROWWISE"] = "1"
    try:
        rowwise = S.Model(cfg, w, max_sequences=1, max_rows=160)
    finally:
        del os.environ["SLM_PREFILL_ROWWISE"]
    o = O.Model(cfg, w, threads=4)
    for lo, hi in ((0, 150), (150, 187)):
        want = o.prefill_tokens(list(toks[lo:hi]), lo)
        for m in (tiled, rowwise):
            assert m.prefill_tokens(toks[lo:hi], start_pos=lo) == want
            assert np.array_equal(m.logits(0), o.logits())
