"""Quantized KV pages (the kvBits path; the reference turns on mlx-swift-lm's
quantized KV cache in TurboQuantService.applyToGenerateParameters,
Sources/NovaMLXEngine/TurboQuantCache.swift:78-104): K/V rows are
quantized MLX-affine on append (4 or 8 bits, groups of 32 or 64 along
head_dim) and attention reads the dequantized values. The model's prefill,
teacher-forced decode steps and device greedy loop over such pages are
checked against the oracle with the same quantize-on-append rule (bars and
the id rule: tests/parity.py), and the quantizer itself bit for bit.

With 4-bit pages the model-level max error bar is 6e-2 instead of 2e-2:
where the GPU's and the oracle's f16 k or v differ by one ulp on a rounding
boundary, the two quantizers pick neighbouring codes and that cached value
moves by a whole 4-bit step (a fifteenth of its group's range). The
quantizer is exact on identical input (test_append_quantizer_bit_exact).
8-bit pages keep the 2e-2 bar."""
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


@pytest.mark.parametrize("name", ["llama", "qwen"])
@pytest.mark.parametrize("kv_bits,gs", [(4, 64), (4, 32), (8, 64), (8, 32)])
def test_quantized_pages_match_oracle(ctx, name, kv_bits, gs):
    from novamlx_b200 import nmx
    m, om, d = _build(ctx, name, kv_bits, gs)
    pool = nmx.KVPool(m, 64, kv_bits=kv_bits, kv_group_size=gs)
    D = d["head_dim"]
    assert pool.bytes_per_token == d["n_layers"] * 2 * d["n_kv_heads"] * (D * kv_bits // 8 + 2 * (D // gs) * 2)
    rng = np.random.default_rng(kv_bits * 10 + gs)
    prompt = rng.integers(0, d["vocab"], 45)
    table = rng.permutation(64)[:8].astype(np.int32)
    rel = 6e-2 if kv_bits == 4 else 2e-2
    got = m.forward(pool, [dict(tokens=prompt, start_pos=0, block_table=table)], nmx.OUT_LOGITS_ALL)
    cache = om.new_cache(128)
    ref = om.forward(cache, prompt, 0, all_logits=True)
    err = check_logits(got, ref, rel)
    pos = len(prompt)
    for _ in range(5):  # teacher-forced decode steps: the fused append quantizes the new token
        tok = int(rng.integers(0, d["vocab"]))
        g = m.forward(pool, [dict(tokens=[tok], start_pos=pos, block_table=table)], nmx.OUT_LOGITS_LAST)
        r = om.forward(cache, [tok], pos)
        err = max(err, check_logits(g, r, rel))
        ids = m.forward(pool, [dict(tokens=[tok], start_pos=pos, block_table=table)], nmx.OUT_ARGMAX_LAST)
        assert ids[0] == int(np.argmax(g[0]))
        check_id(ids[0], r, err)
        pos += 1


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
        g = m.forward(pool, [dict(tokens=[int(cur[i])], start_pos=lens[i] + s, block_table=tables[i])
                             for i in range(3)], nmx.OUT_LOGITS_LAST)
        for i in range(3):
            assert dev[s, i] == int(np.argmax(g[i]))
            r = om.forward(caches[i], [int(cur[i])], lens[i] + s)
            check_id(dev[s, i], r, check_logits(g[i], r, 6e-2 if kv_bits == 4 else 2e-2))
        cur = dev[s].copy()


def test_quantized_pool_rejects_bad_formats(ctx):
    from novamlx_b200 import nmx
    m, _, _ = _build(ctx, "llama", 4, 64)
    for bits, gs in ((3, 64), (4, 128), (2, 32)):
        with pytest.raises(nmx.NmxError) as e:
            nmx.KVPool(m, 8, kv_bits=bits, kv_group_size=gs)
        assert e.value.status == nmx.NMX_ERR_UNSUPPORTED


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
