"""Continuous batching: the budget arithmetic of MemoryBudgetTracker
(Sources/NovaMLXEngine/MemoryBudgetTracker.swift:40-130, cases of
Tests/NovaMLXEngineTests/MemoryBudgetTrackerTests.swift) on the CPU, and the
engine-step scheduler (nmx_sched_*, FusedBatchScheduler's loop) on the GPU:
every request's ids are checked step by step against the oracle forward
teacher-forced on them, shared prompt prefixes are computed once, and
sequences preempted on page exhaustion can be submitted again."""
import numpy as np
import pytest


@pytest.fixture(scope="module")
def nmx():
    from novamlx_b200 import nmx as mod
    return mod


# ----------------------------------------------------------------- CPU

def test_budget_can_admit_when_available(nmx):
    b = nmx.MemoryBudget(1_000_000_000)
    assert b.can_admit(1000, 256)


def test_budget_cannot_admit_when_exceeded(nmx):
    b = nmx.MemoryBudget(1_000_000)
    b.reserve(1, 3600, 256)  # 921,600 bytes
    assert not b.can_admit(3600, 256)


def test_budget_release_frees(nmx):
    b = nmx.MemoryBudget(1_000_000)
    b.reserve(7, 3000, 256)
    b.release(7)
    assert b.can_admit(3000, 256)
    assert b.available == 1_000_000


def test_budget_headroom(nmx):
    b = nmx.MemoryBudget(1_000_000)
    assert not b.can_admit(3700, 256)  # 947,200 bytes > 90% of 1 MB
    assert b.can_admit(3515, 256)      # 899,840 bytes <= 900,000
    assert not b.can_admit(3516, 256)
    z = nmx.MemoryBudget(1_000_000, headroom_percent=0)
    assert z.can_admit(3906, 256) and not z.can_admit(3907, 256)


def test_budget_multiple_sequences(nmx):
    b = nmx.MemoryBudget(10_000_000)
    b.reserve(1, 2500, 256)
    b.reserve(2, 2500, 256)
    assert b.available == 10_000_000 - 2 * 640_000
    assert b.can_admit(2500, 256)
    b.release(1)
    assert b.available == 10_000_000 - 640_000
    b.release(1)  # unknown sequence: no change
    assert b.available == 10_000_000 - 640_000


def test_budget_weights_count_against_limit(nmx):
    b = nmx.MemoryBudget(10_000_000)
    b.add_weights(9_000_000)
    assert b.available == 1_000_000
    assert not b.can_admit(4000, 256)
    b.add_weights(2_000_000)
    assert b.available == 0  # saturates, never wraps


# ----------------------------------------------------------------- GPU

def _model(nmx, max_batch=8, max_tokens=512, seed=1):
    from oracle import oracle as O
    d = dict(vocab=1024, hidden=512, n_layers=2, n_heads=8, n_kv_heads=2, head_dim=64, ffn=1024,
             rope_theta=500000.0, rope_factor=8.0, rope_low_freq_factor=1.0, rope_high_freq_factor=4.0,
             rope_original_max_pos=64, rms_eps=1e-5)
    tensors = O.random_tensors(O.TinyCfg(**d), seed=seed, std=0.05)
    ctx = nmx.Context(0)
    m = nmx.Model(ctx, nmx.ModelConfig(**d, max_batch=max_batch, max_tokens=max_tokens))
    for k, v in tensors.items():
        m.load_tensor(k, v.view(np.float16) if v.dtype == np.uint16 else v)
    return ctx, m, O.OracleModel(O.TinyCfg(**d), tensors)


def _run(sched, ids, max_steps=2000):
    from novamlx_b200 import nmx
    for _ in range(max_steps):
        states = [sched.poll(r)[1] for r in ids]
        if all(s in (nmx.REQ_DONE, nmx.REQ_PREEMPTED) for s in states):
            return
        sched.step()
    raise AssertionError("scheduler did not drain")


def _check_against_oracle(m, om, prompt, out):
    """Teacher-force the scheduler's ids through the oracle and through a
    batch-1 GPU forward of the same model: the GPU logits are within the bars
    at every step, and each id is the oracle's argmax wherever that is
    determined. The scheduler computed its ids inside batches (other rows,
    other summation orders), so the band is twice the batch-1 error measured
    at that step. Returns the number of determined ids."""
    from novamlx_b200 import nmx
    from parity import check_id, check_logits
    n = len(prompt) + len(out) + 16
    pool = nmx.KVPool(m, (n + 15) // 16)
    table = np.arange((n + 15) // 16, dtype=np.int32)
    cache = om.new_cache(n)
    r = om.forward(cache, prompt, 0)
    g = m.forward(pool, [dict(tokens=prompt, start_pos=0, block_table=table)], nmx.OUT_LOGITS_LAST)
    determined = 0
    pos = len(prompt)
    for tok in out:
        determined += int(check_id(int(tok), r, 2.0 * check_logits(g, r)))
        r = om.forward(cache, [int(tok)], pos)
        g = m.forward(pool, [dict(tokens=[int(tok)], start_pos=pos, block_table=table)], nmx.OUT_LOGITS_LAST)
        pos += 1
    pool.close()
    return determined


@pytest.mark.gpu
def test_scheduler_matches_oracle_with_shared_prefix(nmx):
    ctx, m, om = _model(nmx)
    pool = nmx.KVPool(m, 128)
    # a budget well above the pool's: optimalConcurrency (4096-token
    # sequences in 90% of the budget) would otherwise allow one sequence
    sched = nmx.Scheduler(m, pool, max_batch=4, max_step_tokens=160, prefill_chunk=32, model_name="tiny",
                          kv_budget_bytes=1 << 30)
    rng = np.random.default_rng(11)
    prefix = rng.integers(0, 1024, 48)
    prompts = [np.concatenate([prefix, rng.integers(0, 1024, n)]) for n in (5, 19, 40)]
    prompts += [rng.integers(0, 1024, n) for n in (1, 17, 70, 33)]
    max_new = [8, 12, 5, 9, 7, 10, 6]
    ids = [sched.submit(p, n) for p, n in zip(prompts, max_new)]
    _run(sched, ids)
    st = sched.stats()
    for rid, p, n in zip(ids, prompts, max_new):
        out, state = sched.poll(rid)
        assert state == nmx.REQ_DONE and len(out) == n
        _check_against_oracle(m, om, p, out)
    # the 48-token prefix (three full pages) was computed once and reused twice
    assert st["prefix_hit_tokens"] == 2 * 48
    assert st["finished"] == len(ids) and st["running"] == 0 and st["waiting"] == 0
    assert st["blocks_in_use"] == 0 and st["preemptions"] == 0
    assert st["generated"] == sum(max_new)
    # never more than max_batch sequences or max_step_tokens tokens in one step
    assert st["tokens_in_steps"] <= st["steps"] * 160
    sched.close()


@pytest.mark.gpu
def test_scheduler_shares_prefix_pages_while_running(nmx):
    """Sequences sharing a prompt prefix hold the same pages: distinct pages
    in use stay below the pages their tables name."""
    ctx, m, om = _model(nmx)
    pool = nmx.KVPool(m, 128)
    sched = nmx.Scheduler(m, pool, max_batch=8, max_step_tokens=256, prefill_chunk=128, kv_budget_bytes=1 << 30)
    rng = np.random.default_rng(12)
    prefix = rng.integers(0, 1024, 64)
    prompts = [np.concatenate([prefix, rng.integers(0, 1024, 3 + i)]) for i in range(4)]
    ids = [sched.submit(p, 16) for p in prompts]
    seen_sharing = False
    for _ in range(200):
        sched.step()
        st = sched.stats()
        if st["running"] == 4:
            assert st["blocks_in_use"] < st["logical_blocks"]
            seen_sharing = True
        if all(sched.poll(r)[1] == nmx.REQ_DONE for r in ids):
            break
    assert seen_sharing
    for rid, p in zip(ids, prompts):
        out, _ = sched.poll(rid)
        assert len(out) == 16
        _check_against_oracle(m, om, p, out)
    sched.close()


@pytest.mark.gpu
def test_scheduler_preempts_newest_on_page_exhaustion(nmx):
    """A pool of 11 usable pages and a budget that admits more than it holds:
    the newest sequence is preempted, the others finish, and a preempted
    request submitted again finishes too."""
    ctx, m, om = _model(nmx)
    pool = nmx.KVPool(m, 12)
    sched = nmx.Scheduler(m, pool, max_batch=4, max_step_tokens=256, prefill_chunk=64,
                          kv_budget_bytes=1 << 40)
    rng = np.random.default_rng(13)
    prompts = [rng.integers(0, 1024, 40) for _ in range(4)]
    ids = [sched.submit(p, 24) for p in prompts]
    _run(sched, ids)
    states = [sched.poll(r)[1] for r in ids]
    assert nmx.REQ_PREEMPTED in states and nmx.REQ_DONE in states
    assert sched.stats()["preemptions"] == states.count(nmx.REQ_PREEMPTED)
    # the newest sequences were the ones to go
    first_preempted = states.index(nmx.REQ_PREEMPTED)
    assert all(s == nmx.REQ_PREEMPTED for s in states[first_preempted:])
    for rid, p, s in zip(ids, prompts, states):
        if s == nmx.REQ_DONE:
            out, _ = sched.poll(rid)
            assert len(out) == 24
            _check_against_oracle(m, om, p, out)
    again = [sched.submit(p, 24) for p, s in zip(prompts, states) if s == nmx.REQ_PREEMPTED]
    _run(sched, again)
    for rid in again:
        out, s = sched.poll(rid)
        assert s == nmx.REQ_DONE and len(out) == 24
    assert sched.stats()["blocks_in_use"] == 0
    sched.close()


@pytest.mark.gpu
@pytest.mark.parametrize("seqs_of_4096", [2.5, 0.05])
def test_scheduler_concurrency_follows_budget(nmx, seqs_of_4096):
    """optimalConcurrency: as many 4096-token sequences as fit 90% of the
    available KV budget, at least one."""
    ctx, m, om = _model(nmx)
    pool = nmx.KVPool(m, 128)
    bpt = m.kv_bytes_per_token
    budget = int(seqs_of_4096 * 4096 * bpt / 0.9)
    sched = nmx.Scheduler(m, pool, max_batch=8, max_step_tokens=256, kv_budget_bytes=budget)
    rng = np.random.default_rng(14)
    ids = [sched.submit(rng.integers(0, 1024, 30), 10) for _ in range(5)]
    peak = 0
    for _ in range(500):
        sched.step()
        peak = max(peak, sched.stats()["running"])
        if all(sched.poll(r)[1] == nmx.REQ_DONE for r in ids):
            break
    assert peak == max(1, int(seqs_of_4096))
    assert all(len(sched.poll(r)[0]) == 10 for r in ids)
    assert sched.stats()["kv_available_bytes"] == budget
    sched.close()
