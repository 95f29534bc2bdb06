"""CPU tests of the oracle: pinned to the known-answer vectors and
cross-checked against the independent numpy restatement."""
import json
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O
import oracle_np as NP

KAT = json.loads((Path(__file__).parent / "golden" / "kat.json").read_text())


@pytest.mark.parametrize("case", KAT["nibble"], ids=lambda c: f"{c['bits']}b-{c['word']:#x}")
def test_nibble_order(case):
    bits = case["bits"]
    wq = np.array([[case["word"]]], dtype=np.uint32)
    q = O.unpack(wq, 32 // bits, bits)
    assert q[0].tolist() == case["values"]
    assert NP.unpack(wq, 32 // bits, bits)[0].tolist() == case["values"]


@pytest.mark.parametrize("i", range(len(KAT["quantize"])))
def test_quantize_kat(i):
    case = KAT["quantize"][i]
    w = np.array([case["w"]], dtype=np.float32)
    wq, s, b = O.quantize(w, case["bits"], case["group"])
    assert O.unpack(wq, w.shape[1], case["bits"])[0].tolist() == case["q"]
    exp_s = case["scale_f16"] if isinstance(case["scale_f16"], list) else [case["scale_f16"]]
    exp_b = case["bias_f16"] if isinstance(case["bias_f16"], list) else [case["bias_f16"]]
    assert s[0].tolist() == exp_s
    assert b[0].tolist() == exp_b


def test_qmatmul_kat():
    k = KAT["qmatmul"]
    w = np.tile(np.array(k["w_row"], np.float32), (k["rows"], 1))
    wq, s, b = O.quantize(w, k["bits"], k["group"])
    x = O.f32_to_f16bits(np.array([k["x"]], np.float32))
    y = O.f16bits_to_f32(O.qmatmul(x, wq, s, b, k["bits"], k["group"]))
    assert np.all(y == k["y"])


def test_f16_conversions_exhaustive():
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    finite = (bits & 0x7C00) != 0x7C00
    ref = bits.view(np.float16).astype(np.float32)
    got = np.array([O.lib.oracle_h2f(int(h)) for h in bits[::97]], dtype=np.float32)
    assert np.array_equal(got[finite[::97]], ref[::97][finite[::97]])
    # float → f16 round to nearest even agrees with numpy
    rng = np.random.default_rng(1)
    xs = np.concatenate([rng.standard_normal(2000).astype(np.float32) * 10,
                         rng.standard_normal(500).astype(np.float32) * 1e-6,
                         np.array([65504.0, 65520.0, 1e-8, -0.0, 2.0 ** -24, 2.0 ** -25, 3 * 2.0 ** -26],
                                  np.float32)])
    ours = np.array([O.lib.oracle_f2h(float(x)) for x in xs], dtype=np.uint16)
    assert np.array_equal(ours, xs.astype(np.float16).view(np.uint16))


@pytest.mark.parametrize("bits,gs", [(4, 64), (4, 32), (4, 128), (8, 64), (8, 32)])
def test_quantize_matches_numpy(bits, gs):
    rng = np.random.default_rng(bits * 1000 + gs)
    w = rng.standard_normal((48, 256), dtype=np.float32) * 0.02
    w[3, :gs] = 0.5  # constant group
    a = O.quantize(w, bits, gs)
    b = NP.quantize(w, bits, gs)
    for x, y in zip(a, b):
        assert np.array_equal(x, y)
    wd = O.dequantize(*a, bits=bits, group_size=gs)
    assert np.allclose(wd, NP.dequantize(*a, bits=bits, gs=gs), rtol=0, atol=1e-7)
    # dequantisation error bounded by half a step (+ f16 rounding of scale/bias)
    step = np.repeat(O.f16bits_to_f32(a[1]), gs, axis=1)
    assert np.all(np.abs(wd - w) <= 0.5 * step + 2e-3 * np.abs(w) + 1e-4)


@pytest.mark.parametrize("bits,gs,M", [(4, 64, 4), (8, 64, 3), (4, 32, 1), (4, 128, 7)])
def test_qmatmul_matches_numpy(bits, gs, M):
    rng = np.random.default_rng(7)
    K, N = 512, 96
    w = rng.standard_normal((N, K), dtype=np.float32) * 0.02
    wq, s, b = O.quantize(w, bits, gs)
    x = O.f32_to_f16bits(rng.standard_normal((M, K), dtype=np.float32))
    y = O.f16bits_to_f32(O.qmatmul(x, wq, s, b, bits, gs))
    r = O.f16bits_to_f32(NP.qmatmul(x, wq, s, b, bits, gs))
    assert O.max_rel_err(y, r) < 2e-3


def test_attention_matches_numpy():
    rng = np.random.default_rng(3)
    T, S, Hq, Hkv, D = 5, 37, 8, 2, 64
    q = O.f32_to_f16bits(rng.standard_normal((T, Hq, D), dtype=np.float32))
    k = O.f32_to_f16bits(rng.standard_normal((S, Hkv, D), dtype=np.float32))
    v = O.f32_to_f16bits(rng.standard_normal((S, Hkv, D), dtype=np.float32))
    a = O.f16bits_to_f32(O.attention(q, k, v, Hq, Hkv, D, S - T, D ** -0.5))
    b = O.f16bits_to_f32(NP.attention(q, k, v, Hq, Hkv, D, S - T, D ** -0.5))
    assert O.max_rel_err(a, b) < 2e-3


def test_quantized_sdpa_equals_dequantized_attention():
    """The reference kernel's math (quantized K/V, L=1) equals plain attention
    over the dequantized K/V."""
    rng = np.random.default_rng(11)
    B, Hq, Hkv, N, D, gs, bits = 2, 4, 2, 23, 64, 32, 4
    q = O.f32_to_f16bits(rng.standard_normal((B * Hq, 1, D), dtype=np.float32))
    kf = rng.standard_normal((B * Hkv * N, D), dtype=np.float32)
    vf = rng.standard_normal((B * Hkv * N, D), dtype=np.float32)
    kw, ks, kb = O.quantize(kf, bits, gs)
    vw, vs, vb = O.quantize(vf, bits, gs)
    sh = lambda a: a.reshape(B * Hkv, N, -1)
    out = O.quantized_sdpa(q, sh(kw), sh(ks), sh(kb), sh(vw), sh(vs), sh(vb), Hq // Hkv, D ** -0.5, gs, bits)
    kd = O.dequantize(kw, ks, kb, bits, gs).reshape(B, Hkv, N, D)
    vd = O.dequantize(vw, vs, vb, bits, gs).reshape(B, Hkv, N, D)
    for bb in range(B):
        qb = q.reshape(B, Hq, D)[bb][None]
        kk = O.f32_to_f16bits(kd[bb].transpose(1, 0, 2))
        vv = O.f32_to_f16bits(vd[bb].transpose(1, 0, 2))
        ref = O.f16bits_to_f32(O.attention(qb, kk, vv, Hq, Hkv, D, N - 1, D ** -0.5))[0]
        got = O.f16bits_to_f32(out.reshape(B, Hq, D)[bb])
        assert O.max_rel_err(got, ref) < 5e-3


def test_argmax_ties_lowest_index():
    x = np.array([[1.0, 3.0, 3.0, -1.0], [np.nan, 2.0, 2.0, 2.0]], np.float32)
    assert O.argmax(x).tolist() == [1, 1]


def test_penalized_argmax():
    x = np.array([[5.0, 4.9, 1.0, 0.0]], np.float32)
    # id 0 appears twice → 5.0 - 2·0.1 = 4.8 < 4.9
    assert O.penalized_argmax(x, [[0, 0, 3]], [3], 0.1).tolist() == [1]
    assert O.penalized_argmax(x, [[0, 0, 3]], [0], 0.1).tolist() == [0]


def test_rope_frequencies_llama3():
    f = O.rope_inv_freq(128, 500000.0, 8.0, 1.0, 4.0, 8192)
    base = 1.0 / (500000.0 ** (np.arange(0, 128, 2) / 128.0))
    wl = 2 * np.pi / base
    assert np.allclose(f[wl < 8192 / 4], base[wl < 8192 / 4], rtol=1e-6)
    assert np.allclose(f[wl > 8192], base[wl > 8192] / 8.0, rtol=1e-6)


def test_tiny_model_prefix_equals_full():
    """Prefill of a prompt equals prefill of its prefix followed by the rest
    (the contract the prefix cache relies on)."""
    cfg = O.TinyCfg(vocab=256, hidden=128, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=32, ffn=256,
                    rope_theta=10000.0)
    m = O.OracleModel(cfg, O.random_tensors(cfg, seed=5))
    toks = np.random.default_rng(0).integers(0, 256, 40)
    c1 = m.new_cache(64)
    full = m.forward(c1, toks, 0)
    c2 = m.new_cache(64)
    m.forward(c2, toks[:32], 0)
    rest = m.forward(c2, toks[32:], 32)
    assert np.array_equal(full, rest)
    assert np.array_equal(c1[0][:, :, :40], c2[0][:, :, :40])


def test_quantized_kv_cache_oracle():
    """The oracle's quantized KV cache (quantize on append, read the
    dequantized values): 8-bit stays close to the f16 cache, 4-bit further
    away but still close, and the cached rows are exactly representable by
    their group's codes (at most 2^bits distinct values per group)."""
    d = dict(vocab=256, hidden=128, n_layers=1, n_heads=4, n_kv_heads=2, head_dim=64, ffn=256, rope_theta=1e4)
    t = O.random_tensors(O.TinyCfg(**d), seed=4, std=0.05)
    prompt = np.arange(1, 40) % 256
    ref = O.OracleModel(O.TinyCfg(**d), t).forward(O.OracleModel(O.TinyCfg(**d), t).new_cache(64), prompt, 0)
    cos = {}
    for bits in (8, 4):
        om = O.OracleModel(O.TinyCfg(**d, kv_bits=bits, kv_group_size=32), t)
        cache = om.new_cache(64)
        out = om.forward(cache, prompt, 0)
        cos[bits] = O.cosine(out, ref)
        kc = O.f16bits_to_f32(cache[0][0, :, :len(prompt)])  # [Hkv, T, D]
        for row in kc.reshape(-1, 32):
            assert len(np.unique(row)) <= 2 ** bits
    assert cos[8] > 0.9999 and cos[4] > 0.99 and cos[8] >= cos[4]
