"""Failure paths in forms that fault, trap or hang no GPU.

- A device wait that cannot complete: the library's bounded mbarrier wait
  (the one every TMA pipeline uses) given a short limit on a barrier that
  nothing arrives on; the kernel gives up, sets the error flag and returns,
  and the host reports SLM_ERR_DEVICE_INPUT.  The context stays usable.
- A rank that never joins: rank 0 of a two-rank shard group set up alone;
  the non-blocking communicator set-up runs into the model's communicator
  timeout, is aborted and reported as SLM_ERR_TIMEOUT, and the model keeps
  working (it computes unsharded after attaching as a group of one).
The reference aborts on any fault (Cargo.toml:21); these are the error returns
that replace its panics on this path.
"""
import os

import numpy as np
import pytest

import static_lm as S
from static_lm import synth
from static_lm._lib import SlmError, lib

pytestmark = pytest.mark.gpu

SLM_ERR_DEVICE_INPUT, SLM_ERR_TIMEOUT = 7, 8


def test_bounded_device_wait_gives_up_and_reports(cuda):
    # 2e7 cycles is about 10 ms at the B200's clocks
    rc = lib().slm_selftest_bounded_wait(0, 20_000_000)
    assert rc == SLM_ERR_DEVICE_INPUT, lib().slm_last_error()
    assert b"timed out" in lib().slm_last_error()
    # the context is intact: the model path still runs and matches the oracle
    import oracle as O
    cfg, _, vocab = synth.config("cfg1")
    w = synth.synth_model(cfg, 1, vocab, seed=31)
    m = S.Model(cfg, w, max_sequences=1, max_rows=8)
    o = O.Model(cfg, w)
    assert m.prefill_tokens([3, 5, 7], seq=0) == o.prefill_tokens([3, 5, 7], 0)
    m.close()


def _lonely_rank(q):
    import torch
    try:
        torch.cuda.set_device(0)
        cfg, _, vocab = synth.config("cfg1")
        w = synth.synth_model(cfg, 1, vocab, seed=32)
        m = S.Model(cfg, w, max_sequences=2, max_rows=32)
        m.set_comm_timeout(3000)
        import time
        t0 = time.time()
        code = None
        try:
            m.attach_shard(S.nccl_unique_id(), 2, 0)  # rank 1 never joins
        except SlmError as e:
            code = e.code
        waited = time.time() - t0
        # the model still works, as a group of one
        m.attach_shard(b"", 1, 0)
        nxt = m.prefill_batch(np.array([[1, 2, 3, 4]] * 2, dtype=np.int32))
        q.put((code, waited, list(nxt)))
        m.close()
    except Exception as e:  # reported to the parent, which fails the test
        q.put((repr(e), None, None))


def test_attach_shard_times_out_when_a_rank_never_joins(cuda):
    import torch.multiprocessing as mp
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_lonely_rank, args=(q,))
    p.start()
    try:
        code, waited, nxt = q.get(timeout=240)
    finally:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert code == SLM_ERR_TIMEOUT, code
    assert 2.5 < waited < 60, waited
    assert nxt is not None and len(nxt) == 2
