"""Sampling beyond greedy on the device (nmx_op_sample) against
CompiledSampler's rules (Sources/NovaMLXEngine/CompiledSampler.swift:17-49)
restated in numpy: temperature 0 is argmax; the categorical draw follows
softmax(logSoftmax(l) / T) (checked by frequencies over many rows); top-p
keeps exactly the reference's nucleus (ascending sort, inclusive cumulative
probability > 1 - p); logprobs match logSoftmax (computeRawLogprobs,
FusedBatchScheduler.swift:900-941)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def env():
    import torch
    from novamlx_b200 import nmx
    return torch, nmx, nmx.Context(0)


def log_softmax(l):
    l = l.astype(np.float64)
    m = l.max(axis=-1, keepdims=True)
    return l - m - np.log(np.exp(l - m).sum(axis=-1, keepdims=True))


def nucleus_ref(l, p):
    """CompiledSampler's top-p filter as MLX ops: the kept mask"""
    lp = log_softmax(l)
    idx = np.argsort(lp, kind="stable")
    cum = np.cumsum(np.exp(lp[idx]))
    keep = np.zeros(lp.shape, bool)
    keep[idx[cum > 1 - p]] = True
    return keep


@pytest.mark.parametrize("dtype", ["f16", "f32"])
def test_temperature_zero_is_argmax(env, dtype):
    torch, nmx, ctx = env
    rng = np.random.default_rng(0)
    l = rng.standard_normal((7, 1000)).astype(np.float32)
    t = torch.from_numpy(l).cuda()
    if dtype == "f16":
        t = t.half()
    ids, lp, _, _ = ctx.sample(t, 0.0)
    ref = t.float().cpu().numpy()
    assert np.array_equal(ids.cpu().numpy(), ref.argmax(axis=1))
    assert np.allclose(lp.cpu().numpy(), log_softmax(ref)[np.arange(7), ref.argmax(axis=1)], atol=1e-4)


def test_draws_are_reproducible(env):
    torch, nmx, ctx = env
    t = torch.randn(64, 5000, device="cuda")
    a = ctx.sample(t, 0.8, 0.9, seed=7, counter=3)[0].cpu().numpy()
    b = ctx.sample(t, 0.8, 0.9, seed=7, counter=3)[0].cpu().numpy()
    c = ctx.sample(t, 0.8, 0.9, seed=7, counter=4)[0].cpu().numpy()
    assert np.array_equal(a, b)
    assert (a != c).mean() > 0.5


@pytest.mark.parametrize("T", [0.7, 1.0, 1.6])
def test_categorical_frequencies(env, T):
    torch, nmx, ctx = env
    l = np.array([2.0, 1.0, 0.5, 0.0, -1.0, -2.0, 0.3, 1.5], np.float32)
    n = 20000
    t = torch.from_numpy(np.tile(l, (n, 1))).cuda()
    ids = ctx.sample(t, T, 1.0, seed=11, counter=0)[0].cpu().numpy()
    freq = np.bincount(ids, minlength=8) / n
    p = np.exp(log_softmax(l) / T)
    p /= p.sum()
    sigma = np.sqrt(p * (1 - p) / n)
    assert np.all(np.abs(freq - p) <= 5 * sigma + 1e-4), (freq, p)


@pytest.mark.parametrize("top_p", [0.3, 0.6, 0.9, 0.95])
def test_top_p_nucleus(env, top_p):
    torch, nmx, ctx = env
    l = np.array([2.0, 1.0, 0.5, 0.0, -1.0, -2.0, 0.3, 1.5, -0.5, 0.9], np.float32)
    keep = nucleus_ref(l, top_p)
    n = 20000
    t = torch.from_numpy(np.tile(l, (n, 1))).cuda()
    T = 0.9
    ids = ctx.sample(t, T, top_p, seed=5, counter=1)[0].cpu().numpy()
    freq = np.bincount(ids, minlength=len(l)) / n
    assert np.all(freq[~keep] == 0), (freq, keep)
    p = np.where(keep, np.exp(log_softmax(l) / T), 0.0)
    p /= p.sum()
    sigma = np.sqrt(p * (1 - p) / n)
    assert np.all(np.abs(freq - p) <= 5 * sigma + 1e-4), (freq, p)


def test_top_p_large_vocab_matches_nucleus(env):
    """the nucleus boundary by binary search equals the sort-based rule on a
    realistic vocabulary (rows of random logits, various p)"""
    torch, nmx, ctx = env
    rng = np.random.default_rng(3)
    l = (rng.standard_normal((6, 32000)) * 3).astype(np.float32)
    t = torch.from_numpy(l).cuda()
    for p in (0.5, 0.8, 0.95):
        keeps = [nucleus_ref(row, p) for row in l]
        # many draws per row through distinct counters: every id drawn is kept
        for c in range(40):
            ids = ctx.sample(t, 1.0, p, seed=1, counter=c)[0].cpu().numpy()
            assert all(keeps[r][ids[r]] for r in range(6))


def test_logprobs_top_k(env):
    torch, nmx, ctx = env
    rng = np.random.default_rng(4)
    l = rng.standard_normal((5, 3000)).astype(np.float32)
    t = torch.from_numpy(l).cuda()
    ids, lp, tid, tlp = ctx.sample(t, 1.0, 1.0, seed=2, counter=0, top_k=5)
    ref = log_softmax(l)
    ids = ids.cpu().numpy()
    assert np.allclose(lp.cpu().numpy(), ref[np.arange(5), ids], atol=1e-4)
    order = np.argsort(-ref, axis=1, kind="stable")[:, :5]
    assert np.array_equal(tid.cpu().numpy(), order)
    assert np.allclose(tlp.cpu().numpy(), np.take_along_axis(ref, order, axis=1), atol=1e-4)
