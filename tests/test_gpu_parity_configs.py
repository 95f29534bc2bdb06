"""Parity on the benchmarked configurations themselves, against the CPU oracle.

* the Llama-3.1-8B architecture at full depth (32 layers, 8B widths, vocab
  128256): prefill, teacher-forced decode steps and the device greedy loop
  the benchmark times, logits and ids checked at every step;
* one block each of the Qwen2.5-32B shape (hidden 5120, 40/8 heads, qkv
  bias, RoPE 1e6: GQA 5) and the Llama-3.3-70B shape (hidden 8192, 64/8
  heads: GQA 8);
* the paged decode attention op at the GQA ratios of those models and of
  their tensor-parallel shards (40/8, 5/1 and 8/1 per rank at TP8, 64/8);
* prefills of 2048 and 8192 tokens, in one forward and in 512-token chunks
  (the scheduler's prefill step), checked through the last logits and the
  K/V every position wrote into the second layer's pages.

Weights are random-init on the GPU (nmx_model_init_random, N(0, 0.02)
quantized 4-bit g64) and read back through nmx_model_get_tensor, so the
oracle runs on exactly the packed bytes the kernels read. Bars and the id
rule: tests/parity.py.
"""
import numpy as np
import pytest

from oracle import oracle as O
from parity import check_id, check_logits

pytestmark = pytest.mark.gpu

_LIN = {"q": "self_attn.q_proj", "k": "self_attn.k_proj", "v": "self_attn.v_proj", "o": "self_attn.o_proj",
        "g": "mlp.gate_proj", "u": "mlp.up_proj", "d": "mlp.down_proj"}


@pytest.fixture(scope="module")
def nmx():
    from novamlx_b200 import nmx as mod
    return mod


@pytest.fixture(scope="module")
def ctx(nmx):
    return nmx.Context(0)


def oracle_cfg(cfg):
    return O.TinyCfg(vocab=cfg.vocab, hidden=cfg.hidden, n_layers=cfg.n_layers, n_heads=cfg.n_heads,
                     n_kv_heads=cfg.n_kv_heads, head_dim=cfg.head_dim, ffn=cfg.ffn, bits=cfg.bits,
                     group_size=cfg.group_size, qkv_bias=cfg.qkv_bias, rms_eps=cfg.rms_eps,
                     rope_theta=cfg.rope_theta, rope_factor=cfg.rope_factor,
                     rope_low_freq_factor=cfg.rope_low_freq_factor,
                     rope_high_freq_factor=cfg.rope_high_freq_factor,
                     rope_original_max_pos=cfg.rope_original_max_pos)


def gpu_tensors(m, cfg) -> dict:
    """MLX-named host copies of every tensor of a GPU model (linears
    unpacked from the decode records back to the MLX layout)."""
    H, F, V = cfg.hidden, cfg.ffn, cfg.vocab
    Nq, Nkv = cfg.n_heads * cfg.head_dim, cfg.n_kv_heads * cfg.head_dim
    per_word, gs = 32 // cfg.bits, cfg.group_size
    t = {}

    def lin(name, N, K):
        t[f"{name}.weight"] = m.get_tensor(f"{name}.weight", (N, K // per_word), np.uint32)
        t[f"{name}.scales"] = m.get_tensor(f"{name}.scales", (N, K // gs), np.uint16)
        t[f"{name}.biases"] = m.get_tensor(f"{name}.biases", (N, K // gs), np.uint16)

    t["model.embed_tokens.weight"] = m.get_tensor("model.embed_tokens.weight", (V, H), np.uint16)
    t["model.norm.weight"] = m.get_tensor("model.norm.weight", (H,), np.uint16)
    lin("lm_head", V, H)
    for i in range(cfg.n_layers):
        p = f"model.layers.{i}"
        for nm in ("input_layernorm", "post_attention_layernorm"):
            t[f"{p}.{nm}.weight"] = m.get_tensor(f"{p}.{nm}.weight", (H,), np.uint16)
        for short, N, K in (("q", Nq, H), ("k", Nkv, H), ("v", Nkv, H), ("o", H, Nq), ("g", F, H), ("u", F, H),
                            ("d", H, F)):
            lin(f"{p}.{_LIN[short]}", N, K)
        if cfg.qkv_bias:
            for short, N in (("q", Nq), ("k", Nkv), ("v", Nkv)):
                t[f"{p}.{_LIN[short]}.bias"] = m.get_tensor(f"{p}.{_LIN[short]}.bias", (N,), np.uint16)
    return t


def run_decode_parity(nmx, m, om, cfg, prompt_len, tf_steps, greedy_steps, seed, ctx_blocks=16):
    """Prefill, teacher-forced decode steps, then the device greedy loop from
    the prompt's end; logits and ids checked at every step. Returns
    (determined ids, ids checked)."""
    rng = np.random.default_rng(seed)
    prompt = rng.integers(0, cfg.vocab, prompt_len)
    table = rng.permutation(ctx_blocks + 4)[:ctx_blocks].astype(np.int32)
    cap = ctx_blocks * 16
    pool = nmx.KVPool(m, ctx_blocks + 4)
    g = m.forward(pool, [dict(tokens=prompt, start_pos=0, block_table=table)], nmx.OUT_LOGITS_LAST)
    cache = om.new_cache(cap)
    r = om.forward(cache, prompt, 0)
    err = check_logits(g, r)
    first = int(np.argmax(g[0]))
    determined = int(check_id(first, r, err))
    pos = prompt_len
    for _ in range(tf_steps):
        tok = int(rng.integers(0, cfg.vocab))
        g = m.forward(pool, [dict(tokens=[tok], start_pos=pos, block_table=table)], nmx.OUT_LOGITS_LAST)
        r = om.forward(cache, [tok], pos)
        err = max(err, check_logits(g, r))
        ids = m.forward(pool, [dict(tokens=[tok], start_pos=pos, block_table=table)], nmx.OUT_ARGMAX_LAST)
        assert ids[0] == int(np.argmax(g[0]))  # same logits → same id, lowest index on ties
        determined += int(check_id(ids[0], r, err))
        pos += 1
    # the benchmarked path: device greedy loop, one CUDA graph per step
    ids = m.decode_greedy(pool, [first], [prompt_len], table[None], greedy_steps)[:, 0]
    tok, pos = first, prompt_len
    for s in range(greedy_steps):
        g = m.forward(pool, [dict(tokens=[tok], start_pos=pos, block_table=table)], nmx.OUT_LOGITS_LAST)
        r = om.forward(cache, [tok], pos)
        e = check_logits(g, r)
        assert ids[s] == int(np.argmax(g[0])), s
        determined += int(check_id(ids[s], r, max(e, err)))
        tok, pos = int(ids[s]), pos + 1
    return determined, 1 + tf_steps + greedy_steps


def test_llama31_8b_full_depth_matches_oracle(nmx, ctx):
    """The benchmarked 32-layer 8B architecture: a 64-token prompt, four
    teacher-forced steps and six device-greedy steps."""
    cfg = nmx.llama31_8b(max_batch=1, max_tokens=128)
    m = nmx.Model(ctx, cfg)
    m.init_random(seed=0, std=0.02)
    om = O.OracleModel(oracle_cfg(cfg), gpu_tensors(m, cfg))
    determined, total = run_decode_parity(nmx, m, om, cfg, 64, 4, 6, seed=1, ctx_blocks=8)
    print(f"8B full depth: {determined}/{total} ids determined and equal to the oracle's")
    m.close()


@pytest.mark.parametrize("arch", ["qwen25_32b", "llama33_70b"])
def test_block_shapes_match_oracle(nmx, ctx, arch):
    """One block at the 32B (GQA 5, qkv bias, RoPE 1e6) and 70B (GQA 8,
    hidden 8192) widths, a 32K vocabulary."""
    cfg = getattr(nmx, arch)(n_layers=1, vocab=32768, max_batch=2, max_tokens=64)
    m = nmx.Model(ctx, cfg)
    m.init_random(seed=3, std=0.02)
    om = O.OracleModel(oracle_cfg(cfg), gpu_tensors(m, cfg))
    determined, total = run_decode_parity(nmx, m, om, cfg, 21, 3, 4, seed=4, ctx_blocks=4)
    print(f"{arch} block: {determined}/{total} ids determined and equal to the oracle's")
    m.close()


@pytest.mark.parametrize("Hq,Hkv", [(40, 8), (5, 1), (8, 1), (64, 8), (4, 4)])
@pytest.mark.parametrize("lens", [[1], [300, 17, 2048, 4097]])
def test_paged_decode_attention_gqa_ratios(ctx, Hq, Hkv, lens):
    """GQA ratios 5 and 8 (rep rows padded into the 16-row MMA tile) and 1,
    shuffled block tables, contexts across many key splits."""
    import torch
    rng = np.random.default_rng(Hq * 100 + Hkv + len(lens))
    B, D, BT = len(lens), 128, 16
    maxb = max((l + BT - 1) // BT for l in lens)
    nb = B * maxb + 3
    tables = rng.permutation(nb).astype(np.int32)[:B * maxb].reshape(B, maxb)
    kp = O.f32_to_f16bits(rng.standard_normal((nb, Hkv, BT, D), dtype=np.float32))
    vp = O.f32_to_f16bits(rng.standard_normal((nb, Hkv, BT, D), dtype=np.float32))
    q = O.f32_to_f16bits(rng.standard_normal((B, Hq, D), dtype=np.float32))
    t16 = lambda a: torch.from_numpy(a.view(np.int16)).view(torch.float16).cuda()
    out = ctx.paged_decode_attention(t16(q), t16(kp), t16(vp), torch.from_numpy(tables).cuda(),
                                     torch.tensor(lens, dtype=torch.int32).cuda(), Hkv, D ** -0.5)
    got = out.float().cpu().numpy().reshape(B, Hq, D)
    for b, L in enumerate(lens):
        j = np.arange(L)
        k, v = kp[tables[b, j // BT], :, j % BT], vp[tables[b, j // BT], :, j % BT]
        ref = O.f16bits_to_f32(O.attention(q[b][None], k, v, Hq, Hkv, D, L - 1, D ** -0.5))[0]
        assert O.max_rel_err(got[b], ref) <= 5e-3, (b, L)


def _tiny_long(nmx, T):
    d = dict(vocab=1024, hidden=512, n_layers=2, n_heads=8, n_kv_heads=2, head_dim=64, ffn=1024,
             rope_theta=500000.0, rope_factor=8.0, rope_low_freq_factor=1.0, rope_high_freq_factor=4.0,
             rope_original_max_pos=1024, rms_eps=1e-5)
    tensors = O.random_tensors(O.TinyCfg(**d), seed=9, std=0.05)
    return d, tensors


@pytest.mark.parametrize("T", [2048, 8192])
def test_long_prefill_matches_oracle(nmx, ctx, T):
    """A T-token prompt in one forward and in 512-token chunks: last logits
    vs the oracle, and the second layer's K/V at every position (which
    depend on the first layer's attention output at that position)."""
    d, tensors = _tiny_long(nmx, T)
    cfg = nmx.ModelConfig(**d, max_batch=1, max_tokens=T)
    m = nmx.Model(ctx, cfg)
    for k, v in tensors.items():
        m.load_tensor(k, v.view(np.float16) if v.dtype == np.uint16 else v)
    nblk = T // 16
    pool = nmx.KVPool(m, 2 * nblk + 8)
    rng = np.random.default_rng(T)
    prompt = rng.integers(0, d["vocab"], T)
    perm = rng.permutation(2 * nblk + 8).astype(np.int32)
    t_one, t_chunk = perm[:nblk], perm[nblk:2 * nblk]
    om = O.OracleModel(O.TinyCfg(**d), tensors)
    cache = om.new_cache(T)
    r = om.forward(cache, prompt, 0)
    kc, vc, _ = cache
    g_one = m.forward(pool, [dict(tokens=prompt, start_pos=0, block_table=t_one)], nmx.OUT_LOGITS_LAST)
    g_chunk = None
    for c0 in range(0, T, 512):
        g_chunk = m.forward(pool, [dict(tokens=prompt[c0:c0 + 512], start_pos=c0, block_table=t_chunk)],
                            nmx.OUT_LOGITS_LAST)
    for g in (g_one, g_chunk):
        err = check_logits(g, r)
        check_id(int(np.argmax(g[0])), r, err)
    for table in (t_one, t_chunk):
        blocks = pool.read_blocks(table)  # [nblk, L, 2, Hkv, 16, D]
        for kind, ref in ((0, kc), (1, vc)):
            got = O.f16bits_to_f32(blocks[:, 1, kind]).transpose(1, 0, 2, 3).reshape(d["n_kv_heads"], T, -1)
            want = O.f16bits_to_f32(ref[1])
            for p0 in range(0, T, 16):  # every page
                assert O.max_rel_err(got[:, p0:p0 + 16], want[:, p0:p0 + 16]) <= 2e-2, (kind, p0)
    m.close()


def test_scheduler_chunked_prefill_2048(nmx, ctx):
    """The scheduler's own 512-token prefill chunks over a 2048-token
    prompt: its first ids are the oracle's where determined."""
    T = 2048
    d, tensors = _tiny_long(nmx, T)
    cfg = nmx.ModelConfig(**d, max_batch=2, max_tokens=1024)
    m = nmx.Model(ctx, cfg)
    for k, v in tensors.items():
        m.load_tensor(k, v.view(np.float16) if v.dtype == np.uint16 else v)
    pool = nmx.KVPool(m, 2 * (T // 16) + 16)
    sched = nmx.Scheduler(m, pool, max_batch=2, max_step_tokens=1024, prefill_chunk=512, model_name="tiny",
                          kv_budget_bytes=1 << 30)
    prompt = np.random.default_rng(5).integers(0, d["vocab"], T)
    rid = sched.submit(prompt, 3)
    steps = 0
    while sched.poll(rid)[1] != nmx.REQ_DONE:
        sched.step()
        steps += 1
        assert steps < 64
    out = sched.poll(rid)[0]
    sched.close()
    assert steps >= T // 512  # the prompt went in 512-token chunks
    om = O.OracleModel(O.TinyCfg(**d), tensors)
    cache = om.new_cache(T + 8)
    r = om.forward(cache, prompt, 0)
    # GPU logits of the same steps, teacher-forced on the scheduler's ids
    t2 = np.arange(T // 16 + 1, dtype=np.int32) + (T // 16 + 8)
    g = None
    for c0 in range(0, T, 512):
        g = m.forward(pool, [dict(tokens=prompt[c0:c0 + 512], start_pos=c0, block_table=t2)], nmx.OUT_LOGITS_LAST)
    pos = T
    for tok in out:
        err = check_logits(g, r)
        assert int(tok) == int(np.argmax(g[0]))
        check_id(int(tok), r, err)
        g = m.forward(pool, [dict(tokens=[int(tok)], start_pos=pos, block_table=t2)], nmx.OUT_LOGITS_LAST)
        r = om.forward(cache, [int(tok)], pos)
        pos += 1
    m.close()
