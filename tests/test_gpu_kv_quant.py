"""Quantized KV pages (the kvBits path; the reference turns on mlx-swift-lm's
quantized KV cache in TurboQuantService.applyToGenerateParameters,
Sources/NovaMLXEngine/TurboQuantCache.swift:78-104): K/V rows are
quantized MLX-affine on append (4 or 8 bits, groups of 32 or 64 along
head_dim) and attention reads the dequantized values. The model's prefill,
teacher-forced decode steps and device greedy loop over such pages are
checked against the oracle with the same quantize-on-append rule (bars and
the id rule: tests/parity.py), and the quantizer itself bit for bit.

Where the GPU's and the oracle's f16 k or v differ by one ulp on a rounding
boundary, the two quantizers pick neighbouring codes and that cached value
moves by a whole step (a fifteenth of its group's range at 4-bit), so an
end-to-end comparison of two independently quantized caches drifts further
than the f16 bars. The quantizer is checked exact on identical input
(test_append_quantizer_bit_exact), and the attention kernels are checked
with the oracle's cache synced from the GPU's own pages before each
compared step, under the standard bars."""
import numpy as np
import pytest

from oracle import oracle as O
from parity import check_id, check_logits

pytestmark = pytest.mark.gpu


def _cfgs():
    llama = dict(vocab=1024, hidden=512, n_layers=2, n_heads=8, n_kv_heads=2, head_dim=64, ffn=1024,
                 rope_theta=500000.0, rope_factor=8.0, rope_low_freq_factor=1.0, rope_high_freq_factor=4.0,
                 rope_original_max_pos=64, rms_eps=1e-5)
    qwen = dict(vocab=1024, hidden=512, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=128, ffn=1536,
                qkv_bias=True, rope_theta=1e6, rms_eps=1e-6)
    return {"llama": llama, "qwen": qwen}


@pytest.fixture(scope="module")
def ctx():
    from novamlx_b200 import nmx
    return nmx.Context(0)


def _build(ctx, name, kv_bits, gs):
    from novamlx_b200 import nmx
    d = _cfgs()[name]
    tensors = O.random_tensors(O.TinyCfg(**d), seed=2, std=0.05)
    m = nmx.Model(ctx, nmx.ModelConfig(**d, max_batch=4, max_tokens=512))
    for k, v in tensors.items():
        m.load_tensor(k, v.view(np.float16) if v.dtype == np.uint16 else v)
    om = O.OracleModel(O.TinyCfg(**d, kv_bits=kv_bits, kv_group_size=gs), tensors)
    return m, om, d


def _records(raw, Hkv, D, bits, gs):
    """Split raw page records [n, Hkv * rec] into codes [n, Hkv, 16, D*bits/32]
    u32, scales and biases [n, Hkv, 16, D/gs] f16 bits."""
    n = raw.shape[0]
    rb, ng = D * bits // 8, D // gs
    rec = 16 * (rb + 2 * ng * 2)
    r = raw.reshape(n, Hkv, rec)
    codes = r[:, :, :16 * rb].copy().view(np.uint32).reshape(n, Hkv, 16, rb // 4)
    sc = r[:, :, 16 * rb:16 * rb + 32 * ng].copy().view(np.uint16).reshape(n, Hkv, 16, ng)
    bi = r[:, :, 16 * rb + 32 * ng:].copy().view(np.uint16).reshape(n, Hkv, 16, ng)
    return codes, sc, bi


@pytest.mark.parametrize("name", ["llama", "qwen"])
@pytest.mark.parametrize("kv_bits,gs", [(4, 64), (8, 32)])
def test_append_quantizer_bit_exact(ctx, name, kv_bits, gs):
    """The same prefill and decode step into an f16 pool and a quantized
    pool: layer 0's K and V rows (which depend on nothing the KV format
    changes) quantized on the CPU by the workload's rule equal the GPU's
    codes, scales and biases bit for bit — the prefill append and the
    decode kernel's append of the new token."""
    from novamlx_b200 import nmx
    m, _, d = _build(ctx, name, kv_bits, gs)
    D, Hkv = d["head_dim"], d["n_kv_heads"]
    pf = nmx.KVPool(m, 16)
    pq = nmx.KVPool(m, 16, kv_bits=kv_bits, kv_group_size=gs)
    rng = np.random.default_rng(99)
    prompt = rng.integers(0, d["vocab"], 37)
    table = np.array([5, 2, 9, 11], np.int32)
    for pool in (pf, pq):
        m.forward(pool, [dict(tokens=prompt, start_pos=0, block_table=table)])
        m.forward(pool, [dict(tokens=[7], start_pos=37, block_table=table)])  # the fused decode append
    n_tok = 38
    fb = pf.read_blocks(table)       # [4, L, 2, Hkv, 16, D] f16 bits
    qb = pq.read_blocks(table)       # [4, L, 2, Hkv * rec] bytes
    for kind in (0, 1):
        rows = O.f16bits_to_f32(fb[:, 0, kind])          # [4, Hkv, 16, D]
        codes, sc, bi = _records(qb[:, 0, kind], Hkv, D, kv_bits, gs)
        flat = rows.transpose(0, 2, 1, 3).reshape(-1, Hkv, D)[:n_tok]  # [tok, Hkv, D]
        wq, s, b = O.quantize(flat.reshape(-1, D), kv_bits, gs)
        gc = codes.transpose(0, 2, 1, 3).reshape(-1, Hkv, D * kv_bits // 32)[:n_tok].reshape(-1, D * kv_bits // 32)
        gs_ = sc.transpose(0, 2, 1, 3).reshape(-1, Hkv, D // gs)[:n_tok].reshape(-1, D // gs)
        gb = bi.transpose(0, 2, 1, 3).reshape(-1, Hkv, D // gs)[:n_tok].reshape(-1, D // gs)
        assert np.array_equal(gc, wq), kind
        assert np.array_equal(gs_, s), kind
        assert np.array_equal(gb, b), kind


def _dequant_records(raw, Hkv, D, bits, gs):
    """Raw page records [Hkv * rec] of one block -> f16 bits [Hkv, 16, D]
    (w = q * s + b with the f16 scale and bias, rounded once to f16)."""
    codes, sc, bi = _records(raw[None], Hkv, D, bits, gs)
    codes, sc, bi = codes[0], sc[0], bi[0]          # [Hkv, 16, words], [Hkv, 16, ng]
    per = 32 // bits
    q = np.stack([(codes >> (bits * j)) & ((1 << bits) - 1) for j in range(per)], axis=-1)
    q = q.reshape(Hkv, 16, D).astype(np.float32)
    s = np.repeat(sc.view(np.float16).astype(np.float32), gs, axis=-1)
    b = np.repeat(bi.view(np.float16).astype(np.float32), gs, axis=-1)
    return (q * s + b).astype(np.float16).view(np.uint16)


def _sync_cache(pool, table, n_tok, cache, d, bits, gs):
    """The oracle's cache rows 0..n_tok-1 of every layer := the GPU's pages,
    dequantized, so the next oracle step reads exactly what the kernels read."""
    kc, vc, _ = cache
    raw = pool.read_blocks(table)                     # [nb, L, 2, Hkv * rec]
    for blk in range((n_tok + 15) // 16):
        for layer in range(d["n_layers"]):
            for kind, dst in ((0, kc), (1, vc)):
                rows = _dequant_records(raw[blk, layer, kind], d["n_kv_heads"], d["head_dim"], bits, gs)
                t0, t1 = blk * 16, min(n_tok, blk * 16 + 16)
                dst[layer, :, t0:t1] = rows[:, :t1 - t0]


@pytest.mark.parametrize("name", ["llama", "qwen"])
@pytest.mark.parametrize("kv_bits,gs", [(4, 64), (4, 32), (8, 64), (8, 32)])
def test_quantized_pages_match_oracle(ctx, name, kv_bits, gs):
    """Prefill in two chunks and teacher-forced decode steps over quantized
    pages. Before each compared step the oracle's cache is synced from the
    GPU's own pages, so the prefill-chunk and decode attention kernels are
    compared on the same dequantized keys and values; only the step's own
    new rows are quantized independently on each side."""
    from novamlx_b200 import nmx
    m, om, d = _build(ctx, name, kv_bits, gs)
    pool = nmx.KVPool(m, 64, kv_bits=kv_bits, kv_group_size=gs)
    D = d["head_dim"]
    assert pool.bytes_per_token == d["n_layers"] * 2 * d["n_kv_heads"] * (D * kv_bits // 8 + 2 * (D // gs) * 2)
    rng = np.random.default_rng(kv_bits * 10 + gs)
    prompt = rng.integers(0, d["vocab"], 45)
    table = rng.permutation(64)[:8].astype(np.int32)
    cache = om.new_cache(128)
    # chunk A on the GPU, then a 4-token chunk B on both over the GPU's
    # chunk-A pages (the prefill kernel over quantized pages; only chunk B's
    # own rows are quantized independently on each side)
    m.forward(pool, [dict(tokens=prompt[:41], start_pos=0, block_table=table)])
    _sync_cache(pool, table, 41, cache, d, kv_bits, gs)
    got = m.forward(pool, [dict(tokens=prompt[41:], start_pos=41, block_table=table)], nmx.OUT_LOGITS_ALL)
    ref = om.forward(cache, prompt[41:], 41, all_logits=True)
    err = check_logits(got, ref)
    pos = len(prompt)
    for _ in range(5):  # teacher-forced decode steps: the fused append quantizes the new token
        tok = int(rng.integers(0, d["vocab"]))
        _sync_cache(pool, table, pos, cache, d, kv_bits, gs)
        g = m.forward(pool, [dict(tokens=[tok], start_pos=pos, block_table=table)], nmx.OUT_LOGITS_LAST)
        r = om.forward(cache, [tok], pos)
        err = max(err, check_logits(g, r))
        ids = m.forward(pool, [dict(tokens=[tok], start_pos=pos, block_table=table)], nmx.OUT_ARGMAX_LAST)
        assert ids[0] == int(np.argmax(g[0]))
        check_id(ids[0], r, err)
        pos += 1


def test_quantized_pages_close_to_f16(ctx):
    """End to end without syncing: the 8-bit model stays within the f16
    bars of the oracle's own quantized run (codes can flip only by one 8-bit
    step), and 4-bit stays close in direction."""
    from novamlx_b200 import nmx
    for kv_bits, cos_min in ((8, 0.999), (4, 0.99)):
        m, om, d = _build(ctx, "qwen", kv_bits, 64)
        pool = nmx.KVPool(m, 16, kv_bits=kv_bits)
        prompt = np.random.default_rng(3).integers(0, d["vocab"], 40)
        g = m.forward(pool, [dict(tokens=prompt, start_pos=0, block_table=np.arange(4, dtype=np.int32))],
                      nmx.OUT_LOGITS_ALL)
        r = om.forward(om.new_cache(64), prompt, 0, all_logits=True)
        for gi, ri in zip(g, r):
            assert O.cosine(gi, ri) >= cos_min, (kv_bits, O.cosine(gi, ri))


@pytest.mark.parametrize("kv_bits", [4, 8])
def test_quantized_pages_greedy_loop(ctx, kv_bits):
    """The device greedy loop over quantized pages, a batch of three ragged
    sequences, equals the host loop through nmx_forward and the oracle."""
    from novamlx_b200 import nmx
    m, om, d = _build(ctx, "llama", kv_bits, 64)
    pool = nmx.KVPool(m, 80, kv_bits=kv_bits)
    rng = np.random.default_rng(17 + kv_bits)
    lens = [20, 33, 7]
    prompts = [rng.integers(0, d["vocab"], n) for n in lens]
    tables = rng.permutation(80)[:12].astype(np.int32).reshape(3, 4)
    first = m.forward(pool, [dict(tokens=p, start_pos=0, block_table=t) for p, t in zip(prompts, tables)])
    S = 8
    dev = m.decode_greedy(pool, first, lens, tables, S)
    m.forward(pool, [dict(tokens=p, start_pos=0, block_table=t) for p, t in zip(prompts, tables)])
    caches = [om.new_cache(64) for _ in lens]
    for i in range(3):
        om.forward(caches[i], prompts[i], 0)
    cur = first.copy()
    for s in range(S):
        for i in range(3):
            _sync_cache(pool, tables[i], lens[i] + s, caches[i], d, kv_bits, 64)
        g = m.forward(pool, [dict(tokens=[int(cur[i])], start_pos=lens[i] + s, block_table=tables[i])
                             for i in range(3)], nmx.OUT_LOGITS_LAST)
        for i in range(3):
            assert dev[s, i] == int(np.argmax(g[i]))
            r = om.forward(caches[i], [int(cur[i])], lens[i] + s)
            check_id(dev[s, i], r, check_logits(g[i], r))
        cur = dev[s].copy()


def test_quantized_pool_rejects_bad_formats(ctx):
    from novamlx_b200 import nmx
    m, _, _ = _build(ctx, "llama", 4, 64)
    for bits, gs in ((3, 64), (4, 128), (2, 32)):
        with pytest.raises(nmx.NmxError) as e:
            nmx.KVPool(m, 8, kv_bits=bits, kv_group_size=gs)
        assert e.value.status == nmx.NMX_ERR_UNSUPPORTED


def test_pool_destroyed_and_recreated_between_decodes(ctx):
    """A decode graph captured over a pool is dropped with the pool: a new
    pool (which may get the old one's host address) decodes over its own
    pages, equal to a pool created while it is alive."""
    from novamlx_b200 import nmx
    m, _, d = _build(ctx, "qwen", 4, 64)
    prompt = np.random.default_rng(8).integers(0, d["vocab"], 20)
    table = np.arange(4, dtype=np.int32)

    def run(pool):
        first = m.forward(pool, [dict(tokens=prompt, start_pos=0, block_table=table)])
        return m.decode_greedy(pool, first, [20], table[None], 6)

    p1 = nmx.KVPool(m, 8)
    run(p1)
    p1.close()
    p2 = nmx.KVPool(m, 8, kv_bits=4)
    ids2 = run(p2)
    p3 = nmx.KVPool(m, 8, kv_bits=4)
    ids3 = run(p3)
    assert np.array_equal(ids2, ids3)
