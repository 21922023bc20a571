"""Multi-rank host logic of the sequence-sharded decode (bench.py), on CPU
with `gloo` ranks: the shards partition the batch, the job time is the max
over ranks, and decoding each rank's shard on its own gives exactly the
tokens of decoding the whole batch in one process (sequences are
independent, so the sharded path needs no data-path collective)."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

import bench
import oracle as O
from static_lm import synth

GLOBAL = 6
STEPS = 3


def _decode(cfg, w, vocab, gseqs):
    """Greedy decode of the given global sequences, one oracle model each."""
    out = {}
    for g in gseqs:
        m = O.Model(cfg, w, threads=1)
        prompt = [int((g * 31 + i * 7 + 1) % vocab) for i in range(3 + g % 3)]
        tok = m.prefill_tokens(prompt)
        toks = [tok]
        pos = len(prompt)
        for _ in range(STEPS - 1):
            tok = m.forward_token(tok, pos)
            pos += 1
            toks.append(tok)
        out[g] = toks
        m.close()
    return out


def _rank(rank, world, port, q):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg, layers, vocab = synth.config("cfg1")
        w = synth.synth_model(cfg, layers, vocab, seed=3)
        mine = bench.shard_sequences(GLOBAL, world, rank)
        toks = _decode(cfg, w, vocab, mine)
        slowest = bench.max_over_ranks(torch, float(rank + 1), world)
        gathered = [None] * world
        dist.all_gather_object(gathered, {"seqs": mine, "toks": toks, "max": slowest})
        if rank == 0:
            q.put(gathered)
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shards_partition_the_batch():
    for world in (1, 2, 3, 6):
        shards = [bench.shard_sequences(GLOBAL, world, r) for r in range(world)]
        flat = [g for sh in shards for g in sh]
        assert sorted(flat) == list(range(GLOBAL)) and len(set(flat)) == GLOBAL
        assert len({len(sh) for sh in shards}) == 1
    with pytest.raises(SystemExit):
        bench.shard_sequences(GLOBAL, 4, 0)


def test_weak_and_strong_batches():
    """Weak scaling (the bench's default) gives every rank its own batch of
    64 sequences, strong scaling splits the 64 over the ranks; either way the
    shards are disjoint and cover the job's batch."""
    for world in (1, 2, 4, 8):
        for scaling, per in (("weak", 64), ("strong", 64 // world)):
            gb = bench.global_batch(world, scaling)
            shards = [bench.shard_sequences(gb, world, r) for r in range(world)]
            assert all(len(sh) == per for sh in shards)
            flat = sorted(g for sh in shards for g in sh)
            assert flat == list(range(gb))
            cfgd = bench.workload(world, scaling)
            assert cfgd["global_batch"] == gb and cfgd["rows_per_gpu"] == per


def test_two_gloo_ranks_decode_their_shards_like_one_process():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    gathered = q.get(timeout=240)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(g["max"] == float(world) for g in gathered)
    sharded = {}
    for g in gathered:
        sharded.update(g["toks"])
    cfg, layers, vocab = synth.config("cfg1")
    w = synth.synth_model(cfg, layers, vocab, seed=3)
    whole = _decode(cfg, w, vocab, list(range(GLOBAL)))
    assert sharded == whole


# ---- KV-head-sharded batched prefill: the exchange layout -----------------

NSEQ, NTOK = 4, 6
SH_CFG = (128, 256, 4, 2, 16, 1e-5)  # dim, hidden, heads, kv heads, max_seq, eps


def _full_attention():
    """Attention outputs [NSEQ*NTOK][dim] of seeded q/K/V, every (row, head)."""
    cfg = O.Config(*SH_CFG)
    dim, heads, kvh = SH_CFG[0], SH_CFG[2], SH_CFG[3]
    kvd = dim // heads * kvh
    rng = np.random.default_rng(9)
    out = np.zeros((NSEQ * NTOK, dim), np.float32)
    for s in range(NSEQ):
        k = rng.standard_normal(SH_CFG[4] * kvd).astype(np.float32)
        v = rng.standard_normal(SH_CFG[4] * kvd).astype(np.float32)
        for t in range(NTOK):
            q = rng.standard_normal(dim).astype(np.float32)
            out[s * NTOK + t] = O.attention(q, k, v, cfg, t)[0]
    return out


def _unit_block(out, u):
    """Rows and dims of unit u = sequence * kv_heads + KV head."""
    dim, heads, kvh = SH_CFG[0], SH_CFG[2], SH_CFG[3]
    kd = dim // heads * (heads // kvh)
    s, g = divmod(u, kvh)
    return out[s * NTOK:(s + 1) * NTOK, g * kd:(g + 1) * kd]


def _shard_rank(rank, world, port, q):
    import torch
    import torch.distributed as dist
    import static_lm as S
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        full = _full_attention()
        units = S.shard_units(NSEQ, SH_CFG[3], world, rank)
        # this rank's attention outputs, packed [unit][row][kd] as the library sends them
        send = torch.from_numpy(np.stack([_unit_block(full, u) for u in units]).copy())
        recv = torch.empty((world * send.shape[0],) + tuple(send.shape[1:]), dtype=send.dtype)
        dist.all_gather_into_tensor(recv, send)
        # unpack with the all-gather order: rank r's i-th unit is i*world + r
        got = np.zeros_like(full)
        for r in range(world):
            for i, u in enumerate(S.shard_units(NSEQ, SH_CFG[3], world, r)):
                _unit_block(got, u)[:] = recv[r * len(units) + i].numpy()
        q.put((rank, bool(np.array_equal(got, full)), units))
    except Exception as e:  # report instead of leaving the parent waiting
        q.put((rank, False, repr(e)))
        raise
    finally:
        dist.destroy_process_group()


def test_shard_units_partition_the_units():
    import static_lm as S
    for world in (1, 2, 4, 8):
        parts = [S.shard_units(NSEQ, SH_CFG[3], world, r) for r in range(world)]
        flat = sorted(u for p in parts for u in p)
        assert flat == list(range(NSEQ * SH_CFG[3]))
        assert len({len(p) for p in parts}) == 1
    assert S.shard_units(3, 3, 2, 0) == []  # 9 units do not divide over 2 ranks


def test_two_gloo_ranks_assemble_the_sharded_attention():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_shard_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(ok for _, ok, _ in res), res
    assert sorted(u for _, _, units in res for u in units) == list(range(NSEQ * SH_CFG[3]))
