"""Speculative decoding: the n-gram draft source (the cases of
Tests/NovaMLXEngineTests/NGramSpeculatorTests.swift, on the CPU) and the
batched verify (nmx_spec_verify, on the GPU): under the prefix rule a verify
of the model's own greedy continuation accepts every draft and continues
exactly as plain greedy decoding does; wrong drafts are rejected at the
first mismatch; the n-gram rule follows FusedBatchScheduler.swift:1247-1300
as written."""
import threading

import numpy as np
import pytest


@pytest.fixture(scope="module")
def nmx():
    from novamlx_b200 import nmx as mod
    return mod


# ----------------------------------------------------------------- CPU

def test_speculate_empty_when_cache_empty(nmx):
    spec = nmx.NGramSpeculator(3, 3, 1)
    assert spec.speculate([1, 2, 3]) == []


def test_speculate_empty_when_context_too_short(nmx):
    spec = nmx.NGramSpeculator(4, 3, 1)
    spec.record_tokens([1, 2, 3, 4, 5])
    assert spec.speculate([1, 2]) == []


def test_record_and_speculate_basic_hit(nmx):
    spec = nmx.NGramSpeculator(2, 3, 1)
    spec.record_tokens([1, 2, 3, 4, 5])  # [1,2]->3, [2,3]->4, [3,4]->5
    assert spec.speculate([10, 3, 4]) == [5]


def test_min_hits_filters_low_confidence(nmx):
    spec = nmx.NGramSpeculator(2, 3, 2)
    spec.record_tokens([1, 2, 3])
    assert spec.speculate([1, 2]) == []
    spec.record_tokens([1, 2, 3])
    assert spec.speculate([1, 2]) == [3]


def test_max_draft_limits_output(nmx):
    spec = nmx.NGramSpeculator(1, 2, 1)
    for i in range(10, 20):
        spec.record_tokens([1, i])
    r = spec.speculate([1])
    assert len(r) <= 2 and len(r) > 0


def test_speculate_with_internal_buffer(nmx):
    spec = nmx.NGramSpeculator(2, 3, 1)
    for t in [1, 2, 3, 4, 5]:
        spec.record_token(t)
    spec.speculate()
    spec.record_token(6)
    spec.record_token(7)
    assert spec.speculate() == []  # [6,7] has no continuation yet
    assert spec.speculate([4, 5]) == [6]


def test_eviction_when_cache_full(nmx):
    spec = nmx.NGramSpeculator(1, 1, 1, max_cache_size=4)
    for i in range(10):
        spec.record_tokens([100, i])
    assert spec.stats["cache_size"] <= 4


def test_stats_reporting(nmx):
    spec = nmx.NGramSpeculator(2, 3, 1)
    spec.record_tokens([1, 2, 3, 4, 5])
    st = spec.stats
    assert st["cache_size"] > 0 and st["total_hits"] > 0 and st["buffer_size"] > 0


def test_decoder_tracks_acceptance(nmx):
    spec = nmx.NGramSpeculator(2, 3, 1)
    for t in [1, 2, 3, 4]:
        spec.record_token(t)
    spec.record_accepted([5, 6, 7], 2)
    assert abs(spec.stats["acceptance_rate"] - 2.0 / 3.0) < 0.01


def test_decoder_acceptance_zero_without_speculation(nmx):
    assert nmx.NGramSpeculator().stats["acceptance_rate"] == 0


def test_decoder_speculate_delegates(nmx):
    spec = nmx.NGramSpeculator(2, 3, 1)
    for t in [1, 2, 3]:
        spec.record_token(t)
    assert spec.speculate([1, 2]) == [3]


def test_buffer_is_bounded(nmx):
    spec = nmx.NGramSpeculator(4, 5, 1)
    spec.record_tokens(list(range(100)))
    assert spec.stats["buffer_size"] == 4 + 5 + 10


def test_continuations_are_distinct_and_ordered(nmx):
    """record(tokens:) walks the new tokens newest first: 7->4, 7->3, 7->1,
    then the list is full (max_draft 3) and 7->2 is dropped"""
    spec = nmx.NGramSpeculator(1, 3, 1)
    spec.record_tokens([7, 1, 7, 2, 7, 1, 7, 3, 7, 4])
    assert spec.speculate([7]) == [4, 3, 1]
    one = nmx.NGramSpeculator(1, 3, 1)  # record(token:) walks oldest first
    for t in [7, 1, 7, 2, 7, 1, 7, 3, 7, 4]:
        one.record_token(t)
    assert one.speculate([7]) == [1, 2, 3]


def test_concurrent_record_and_speculate(nmx):
    spec = nmx.NGramSpeculator(2, 3, 1)
    for i in range(50):
        spec.record_tokens([i, i + 1, i + 2])

    def rec():
        for i in range(100, 120):
            spec.record_tokens([i, i + 1, i + 2])

    def spc():
        for _ in range(50):
            spec.speculate([1, 2])

    ts = [threading.Thread(target=f) for _ in range(10) for f in (rec, spc)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    assert spec.stats["cache_size"] > 0


# ----------------------------------------------------------------- GPU

def _model(nmx):
    from oracle import oracle as O
    d = dict(vocab=1024, hidden=512, n_layers=2, n_heads=8, n_kv_heads=2, head_dim=64, ffn=1024,
             rope_theta=500000.0, rope_factor=8.0, rope_low_freq_factor=1.0, rope_high_freq_factor=4.0,
             rope_original_max_pos=64, rms_eps=1e-5)
    tensors = O.random_tensors(O.TinyCfg(**d), seed=2, std=0.05)
    ctx = nmx.Context(0)
    m = nmx.Model(ctx, nmx.ModelConfig(**d, max_batch=8, max_tokens=512))
    for k, v in tensors.items():
        m.load_tensor(k, v.view(np.float16) if v.dtype == np.uint16 else v)
    return ctx, m


def _greedy(nmx, m, pool, prompt, table, n):
    """prefill + n greedy steps through nmx_forward: the ids and the last position"""
    ids = [int(m.forward(pool, [dict(tokens=prompt, start_pos=0, block_table=table)])[0])]
    pos = len(prompt)
    for _ in range(n - 1):
        ids.append(int(m.forward(pool, [dict(tokens=[ids[-1]], start_pos=pos, block_table=table)])[0]))
        pos += 1
    return ids


@pytest.mark.gpu
def test_verify_prefix_rule_accepts_greedy_continuation(nmx):
    ctx, m = _model(nmx)
    pool = nmx.KVPool(m, 64)
    rng = np.random.default_rng(21)
    B, D = 4, 4
    prompts = [rng.integers(0, 1024, n) for n in (20, 33, 7, 50)]
    tables = [np.arange(12 * i + 1, 12 * i + 13, dtype=np.int32) for i in range(B)]
    ref = [_greedy(nmx, m, pool, p, t, D + 3) for p, t in zip(prompts, tables)]
    # re-prefill, then verify the true continuation: all D drafts accepted
    first = [int(m.forward(pool, [dict(tokens=p, start_pos=0, block_table=t)])[0]) for p, t in zip(prompts, tables)]
    assert first == [r[0] for r in ref]
    seqs = [dict(last_token=r[0], drafts=r[1:1 + D], start_pos=len(p), block_table=t)
            for r, p, t in zip(ref, prompts, tables)]
    out = nmx.spec_verify(m, pool, seqs, nmx.VERIFY_PREFIX)
    for (toks, acc), r in zip(out, ref):
        assert acc == D
        assert toks == r[1:2 + D]  # D accepted drafts + the bonus id
    # the pages now hold the accepted positions: continuing equals greedy
    for (toks, acc), r, p, t in zip(out, ref, prompts, tables):
        nxt = int(m.forward(pool, [dict(tokens=[toks[-1]], start_pos=len(p) + 1 + acc, block_table=t)])[0])
        assert nxt == r[2 + D]


@pytest.mark.gpu
def test_verify_prefix_rule_rejects_at_first_mismatch(nmx):
    ctx, m = _model(nmx)
    pool = nmx.KVPool(m, 64)
    rng = np.random.default_rng(22)
    prompt = rng.integers(0, 1024, 30)
    table = np.arange(1, 13, dtype=np.int32)
    ref = _greedy(nmx, m, pool, prompt, table, 8)
    for k in range(0, 4):  # the first k drafts right, the next wrong
        m.forward(pool, [dict(tokens=prompt, start_pos=0, block_table=table)])
        drafts = list(ref[1:1 + k]) + [(ref[1 + k] + 1) % 1024] + list(ref[2 + k:5])
        (toks, acc), = nmx.spec_verify(m, pool, [dict(last_token=ref[0], drafts=drafts, start_pos=len(prompt),
                                                      block_table=table)], nmx.VERIFY_PREFIX)
        assert acc == k
        assert toks == ref[1:2 + k]  # k accepted + the model's own id at the mismatch
        # continuing from the kept positions equals greedy decoding
        nxt = int(m.forward(pool, [dict(tokens=[toks[-1]], start_pos=len(prompt) + 1 + acc, block_table=table)])[0])
        assert nxt == ref[2 + k]


@pytest.mark.gpu
def test_verify_ngram_rule_as_written(nmx):
    """FusedBatchScheduler's rule: tokens g0, g1, ... up to the first p >= 1
    with g_p != drafts[p-1]; the per-position greedy ids g come from the
    same forward (checked against a teacher-forced forward of the block)."""
    ctx, m = _model(nmx)
    pool = nmx.KVPool(m, 64)
    rng = np.random.default_rng(23)
    prompt = rng.integers(0, 1024, 25)
    table = np.arange(1, 13, dtype=np.int32)
    first = int(m.forward(pool, [dict(tokens=prompt, start_pos=0, block_table=table)])[0])
    for drafts in ([5, 6, 7], [], [first, first, first]):
        block = [first] + drafts
        g = m.forward(pool, [dict(tokens=block, start_pos=len(prompt), block_table=table)], nmx.OUT_ARGMAX_ALL)
        exp, acc = [int(g[0])], 0
        for p in range(1, len(block)):
            exp.append(int(g[p]))
            if int(g[p]) != drafts[p - 1]:
                break
            acc += 1
        (toks, a), = nmx.spec_verify(m, pool, [dict(last_token=first, drafts=drafts, start_pos=len(prompt),
                                                    block_table=table)], nmx.VERIFY_NGRAM)
        assert toks == exp and a == acc
