"""Model-level parity: prefill, decode, batched decode over independent
sequences, device-resident multi-step decode and embeddings on the GPU against
the CPU oracle -- bit-exact logits and KV caches, identical greedy tokens."""
import os

import numpy as np
import pytest

import oracle as O
import static_lm as S
from static_lm import synth
from static_lm._lib import Config, SlmError

pytestmark = pytest.mark.gpu


def small_cfg():
    return Config(64, 128, 4, 2, 16, 1e-5)


def small_weights():
    cfg = small_cfg()
    return cfg, O.xorshift_model(cfg, 2, 128, 0.25, dict(token_embd=0x0100, lm_head=0x0200))


def test_prefill_and_generate_reference_test_model(cuda):
    """transformer.rs:1268-1358 model: prefill then decode, every step exact."""
    cfg, w = small_weights()
    g = S.Model(cfg, w, max_sequences=1, max_rows=16)
    o = O.Model(cfg, w)
    prompt = [1, 7, 19, 42]
    assert g.prefill_tokens(prompt) == o.prefill_tokens(prompt)
    assert np.array_equal(g.logits(0), o.logits())
    for l in range(2):
        assert np.array_equal(g.kv_read(0, l, 0, 0, 4), o.k_cache(l)[:4 * g.kv_dim])
        assert np.array_equal(g.kv_read(0, l, 1, 0, 4), o.v_cache(l)[:4 * g.kv_dim])
    tok = o.forward_token(5, 4)
    assert g.forward_token(5, 4) == tok
    assert np.array_equal(g.logits(0), o.logits())
    assert np.array_equal(g.hidden(0), o.x())


def test_generate_matches_sequential_and_oracle(cuda):
    cfg, w = small_weights()
    g = S.Model(cfg, w, max_sequences=1, max_rows=16)
    prompt = [3, 1, 4, 1, 5]
    want = O.Model(cfg, w).generate(prompt, 11)
    assert g.generate(prompt, 11) == want
    assert len(want) == 11  # runs to max_seq_len


def test_cfg1_generate_identical_tokens(cuda):
    cfg, layers, vocab = synth.config("cfg1")
    w = synth.synth_model(cfg, layers, vocab, seed=1)
    g = S.Model(cfg, w, max_sequences=1, max_rows=64)
    o = O.Model(cfg, w)
    prompt = list(range(1, 17))
    assert g.generate(prompt, 64) == o.generate(prompt, 64)
    assert np.array_equal(g.logits(0), o.logits())


def test_cfg2_batched_decode_of_independent_sequences(cuda):
    cfg, layers, vocab = synth.config("cfg2")
    w = synth.synth_model(cfg, layers, vocab, seed=2)
    B, steps = 4, 6
    g = S.Model(cfg, w, max_sequences=B, max_rows=32)
    prompts = [list(np.random.default_rng(s).integers(0, vocab, 8 + s)) for s in range(B)]
    toks, pos = [], []
    oracles = []
    for s, p in enumerate(prompts):
        o = O.Model(cfg, w, threads=4)
        t = o.prefill_tokens(p)
        assert g.prefill_tokens(p, seq=s) == t
        oracles.append(o)
        toks.append(t)
        pos.append(len(p))
    for _ in range(steps):
        nxt = g.decode_batch(list(range(B)), toks, pos)
        want = [oracles[s].forward_token(toks[s], pos[s]) for s in range(B)]
        assert list(nxt) == want
        for s in range(B):
            assert np.array_equal(g.logits(s), oracles[s].logits())
        toks = list(nxt)
        pos = [p + 1 for p in pos]


def test_batched_decode_rows_in_any_sequence_order(cuda):
    cfg, w = small_weights()
    g = S.Model(cfg, w, max_sequences=3, max_rows=16)
    os_ = [O.Model(cfg, w) for _ in range(3)]
    for s in range(3):
        assert g.prefill_tokens([s + 1, 2 * s + 3], seq=s) == os_[s].prefill_tokens([s + 1, 2 * s + 3])
    nxt = g.decode_batch([2, 0, 1], [9, 8, 7], [2, 2, 2])
    assert list(nxt) == [os_[2].forward_token(9, 2), os_[0].forward_token(8, 2),
                         os_[1].forward_token(7, 2)]


def test_decode_steps_device_matches_host_loop(cuda):
    torch = cuda
    cfg, layers, vocab = synth.config("cfg1")
    w = synth.synth_model(cfg, layers, vocab, seed=3)
    B, steps = 5, 12
    a = S.Model(cfg, w, max_sequences=B, max_rows=32)
    b = S.Model(cfg, w, max_sequences=B, max_rows=32)
    toks, pos = [], []
    for s in range(B):
        p = list(range(s + 1, s + 9))
        t1, t2 = a.prefill_tokens(p, seq=s), b.prefill_tokens(p, seq=s)
        assert t1 == t2
        toks.append(t1)
        pos.append(len(p))
    host_out = []
    t, ps = list(toks), list(pos)
    for _ in range(steps):
        t = list(a.decode_batch(list(range(B)), t, ps))
        ps = [p + 1 for p in ps]
        host_out.append(t)
    seqs = torch.arange(B, dtype=torch.int32, device="cuda")
    td = torch.tensor(toks, dtype=torch.int32, device="cuda")
    pd = torch.tensor(pos, dtype=torch.int32, device="cuda")
    out = torch.zeros(steps * B, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()  # the model stream does not order against torch's stream
    b.decode_steps_device(B, seqs.data_ptr(), td.data_ptr(), pd.data_ptr(), steps, out.data_ptr(),
                          max(pos))
    torch.cuda.synchronize()
    assert out.cpu().numpy().reshape(steps, B).tolist() == host_out
    assert pd.cpu().tolist() == [p + steps for p in pos]


def test_two_stream_decode_matches_one_stream(cuda):
    cfg, layers, vocab = synth.config("cfg1")
    w = synth.synth_model(cfg, layers, vocab, seed=6)
    B = 20
    os.environ["SLM_DECODE_ONE_STREAM"] = "1"
    try:
        one = S.Model(cfg, w, max_sequences=B, max_rows=B)
    finally:
        del os.environ["SLM_DECODE_ONE_STREAM"]
    os.environ["SLM_DECODE_PARTS"] = "2"
    try:
        two = S.Model(cfg, w, max_sequences=B, max_rows=B)
    finally:
        del os.environ["SLM_DECODE_PARTS"]
    assert two.launches_per_decode_step(B) > one.launches_per_decode_step(B)
    toks = [(s * 37 + 1) % vocab for s in range(B)]
    pos = [0] * B
    for _ in range(3):
        a = one.decode_batch(list(range(B)), toks, pos)
        b = two.decode_batch(list(range(B)), toks, pos)
        assert list(a) == list(b)
        for r in (0, B // 2, B - 1):
            assert np.array_equal(one.logits(r), two.logits(r))
        toks, pos = list(a), [p + 1 for p in pos]


def test_graphs_and_eager_agree(cuda):
    cfg, w = small_weights()
    os.environ["SLM_DISABLE_GRAPHS"] = "1"
    try:
        e = S.Model(cfg, w, max_sequences=2, max_rows=16)
    finally:
        del os.environ["SLM_DISABLE_GRAPHS"]
    g = S.Model(cfg, w, max_sequences=2, max_rows=16)
    for m in (e, g):
        m.prefill_tokens([1, 2, 3], seq=0)
        m.prefill_tokens([4, 5], seq=1)
    t1 = e.decode_batch([0, 1], [6, 7], [3, 2])
    t2 = g.decode_batch([0, 1], [6, 7], [3, 2])
    assert list(t1) == list(t2)
    assert np.array_equal(e.logits(1), g.logits(1))


def test_fused_and_three_pass_attention_agree(cuda):
    cfg, layers, vocab = synth.config("cfg2")
    w = synth.synth_model(cfg, layers, vocab, seed=5)
    os.environ["SLM_ATTENTION_3PASS"] = "1"
    try:
        three = S.Model(cfg, w, max_sequences=2, max_rows=32)
    finally:
        del os.environ["SLM_ATTENTION_3PASS"]
    fused = S.Model(cfg, w, max_sequences=2, max_rows=32)
    for m in (three, fused):
        m.prefill_tokens(list(range(3, 30)), seq=0)
        m.prefill_tokens([5, 6, 7], seq=1)
    a = three.decode_batch([0, 1], [9, 10], [27, 3])
    b = fused.decode_batch([0, 1], [9, 10], [27, 3])
    assert list(a) == list(b)
    for r in range(2):
        assert np.array_equal(three.logits(r), fused.logits(r))
    assert fused.launches_per_decode_step(2) < three.launches_per_decode_step(2)


def test_norm_fused_into_gemv_matches_separate_rmsnorm(cuda):
    cfg, layers, vocab = synth.config("cfg2")
    w = synth.synth_model(cfg, layers, vocab, seed=8)
    os.environ["SLM_UNFUSED_NORM"] = "1"
    try:
        sep = S.Model(cfg, w, max_sequences=3, max_rows=32)
    finally:
        del os.environ["SLM_UNFUSED_NORM"]
    fus = S.Model(cfg, w, max_sequences=3, max_rows=32)
    assert fus.launches_per_decode_step(3) < sep.launches_per_decode_step(3)
    for m in (sep, fus):
        m.prefill_tokens(list(range(1, 20)), seq=0)
        m.prefill_tokens([4, 5, 6], seq=1)
        m.prefill_tokens([7], seq=2)
    toks, pos = [11, 12, 13], [19, 3, 1]
    for _ in range(3):
        a = sep.decode_batch([0, 1, 2], toks, pos)
        b = fus.decode_batch([0, 1, 2], toks, pos)
        assert list(a) == list(b)
        for r in range(3):
            assert np.array_equal(sep.logits(r), fus.logits(r))
        toks, pos = list(a), [p + 1 for p in pos]


def test_cfg3_shape_prefilled_kv_decode(cuda):
    """SmolLM2-135M shape, KV rows 0..2047 from seeded N(0,1), two sequences,
    two decode steps at positions 2048 and 2049: logits bit-exact."""
    cfg, layers, vocab = synth.config("cfg3", max_seq_len=2048 + 8)
    w = synth.synth_model(cfg, layers, vocab, seed=4)
    B, L = 2, 2048
    g = S.Model(cfg, w, max_sequences=B, max_rows=B)
    kvd = g.kv_dim
    oracles = []
    for s in range(B):
        o = O.Model(cfg, w, threads=4)
        for l in range(layers):
            for which in (0, 1):
                data = synth.normal_f32(L * kvd, 1000 + s * 100 + l * 2 + which)
                g.kv_write(s, l, which, 0, data)
                (o.k_cache(l) if which == 0 else o.v_cache(l))[:L * kvd] = data
        oracles.append(o)
    toks, pos = [11, 22], [L, L]
    for _ in range(2):
        nxt = g.decode_batch([0, 1], toks, pos)
        want = [oracles[s].forward_token(toks[s], pos[s]) for s in range(B)]
        assert list(nxt) == want
        for s in range(B):
            assert np.array_equal(g.logits(s), oracles[s].logits())
        toks, pos = list(nxt), [p + 1 for p in pos]


def test_embed_tokens_bit_exact(cuda):
    cfg, w = small_weights()
    g = S.Model(cfg, w, max_sequences=1, max_rows=16)
    o = O.Model(cfg, w)
    for toks in ([1, 2, 3, 4], [10, 20, 30, 40, 50], [7]):
        assert np.array_equal(g.embed_tokens(toks), o.embed_tokens(toks))


def test_model_errors(cuda):
    cfg, w = small_weights()
    g = S.Model(cfg, w, max_sequences=2, max_rows=16)
    with pytest.raises(SlmError) as e:
        g.forward_token(128, 0)
    assert e.value.code == 2
    with pytest.raises(SlmError) as e:
        g.forward_token(1, 16)
    assert e.value.code == 2
    with pytest.raises(SlmError) as e:
        g.decode_batch([0, 0], [1, 2], [0, 0])
    assert e.value.code == 1
    with pytest.raises(SlmError) as e:
        g.prefill_tokens(list(range(10)), start_pos=10)
    assert e.value.code == 2
    with pytest.raises(SlmError):
        g.prefill_tokens([])
    # the model still works after rejected calls
    assert g.forward_token(1, 0) == O.Model(cfg, w).forward_token(1, 0)


@pytest.mark.parametrize("unfused", [False, True])
def test_wide_model_batch1_generate_matches_oracle(cuda, unfused):
    """dim 2048, hidden 2048 (64 blocks a row): batch-1 decode steps take the
    block-split GEMV for Wo, down and lm_head, and, with the RMSNorm as its own
    launch (SLM_UNFUSED_NORM=1), also for QKV and gate/up; tokens and logits
    equal the oracle's."""
    cfg = Config(2048, 2048, 16, 4, 64, 1e-5)
    w = synth.synth_model(cfg, 1, 1024, seed=31)
    if unfused:
        os.environ["SLM_UNFUSED_NORM"] = "1"
    try:
        g = S.Model(cfg, w, max_sequences=1, max_rows=8)
    finally:
        os.environ.pop("SLM_UNFUSED_NORM", None)
    o = O.Model(cfg, w)
    prompt = [3, 17, 255, 1000]
    assert g.generate(prompt, 6) == o.generate(prompt, 6)
    assert np.array_equal(g.logits(0), o.logits())
    o.close()
    g.close()
