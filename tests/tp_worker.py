"""One rank of the tensor-parallel parity check (test infrastructure; run
under torch.distributed.run by tests/test_tp.py). Every rank loads its shard
of the same tiny model, joins the communicator, and runs a ragged prefill, a
device greedy loop, the same steps teacher-forced with logits, and a
12-sequence batch through the decode-batch GEMM (with and without the
exchange fused into its epilogue). Each rank writes its results; the test
compares them with the oracle and with each other."""
import argparse
import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

GREEDY_STEPS = 6


def tiny(name):
    llama = dict(vocab=1024, hidden=512, n_layers=2, n_heads=8, n_kv_heads=2, head_dim=64, ffn=1024,
                 rope_theta=500000.0, rope_factor=8.0, rope_low_freq_factor=1.0, rope_high_freq_factor=4.0,
                 rope_original_max_pos=64, rms_eps=1e-5)
    qwen = dict(vocab=1024, hidden=512, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=128, ffn=1536,
                qkv_bias=True, rope_theta=1e6, rms_eps=1e-6)
    # eight kv heads: shard over 2, 4 and 8 ranks (one kv head per rank at 8)
    llama8kv = dict(llama, n_heads=16, n_kv_heads=8, ffn=2048)
    # the Qwen2.5-32B head layout (40 q heads / 8 kv heads of 128: 5 q heads
    # per kv head, 5/1 per rank at 8 ranks)
    qwen8kv = dict(qwen, n_heads=40, n_kv_heads=8, ffn=2048)
    return {"llama": llama, "qwen": qwen, "llama8kv": llama8kv, "qwen8kv": qwen8kv}[name]


def prompts_of(cfg, seed):
    rng = np.random.default_rng(seed)
    lens = [3, 40, 17, 70]
    prompts = [rng.integers(0, cfg.vocab, n) for n in lens]
    tables = [np.arange(8 * i + 1, 8 * i + 9, dtype=np.int32) for i in range(4)]
    return lens, prompts, tables


def run(nmx, m, pool, cfg, seed):
    lens, prompts, tables = prompts_of(cfg, seed)
    logits = m.forward(pool, [dict(tokens=p, start_pos=0, block_table=t) for p, t in zip(prompts, tables)],
                       nmx.OUT_LOGITS_LAST)
    first = m.forward(pool, [dict(tokens=p, start_pos=0, block_table=t) for p, t in zip(prompts, tables)])
    ids = m.decode_greedy(pool, first, lens, np.stack(tables), GREEDY_STEPS)
    # the same steps teacher-forced on the greedy ids, with logits
    step_logits = []
    cur = first.copy()
    for s in range(GREEDY_STEPS):
        step_logits.append(m.forward(pool, [dict(tokens=[int(cur[i])], start_pos=lens[i] + s, block_table=tables[i])
                                            for i in range(4)], nmx.OUT_LOGITS_LAST))
        cur = ids[s]
    return logits, first, ids, np.stack(step_logits)


def batch_inputs(cfg, seed):
    rng = np.random.default_rng(seed)
    prompts = [rng.integers(0, cfg.vocab, 8) for _ in range(12)]
    toks = rng.integers(0, cfg.vocab, 12)
    return prompts, toks


def run_batch(nmx, m, pool, cfg, seed):
    """12 short prompts prefilled together (96 rows) and one 12-row decode
    step: the decode-batch GEMM path, whose epilogue can do the exchange"""
    prompts, toks = batch_inputs(cfg, seed)
    tables = [np.array([100 + i], np.int32) for i in range(12)]
    pre = m.forward(pool, [dict(tokens=p, start_pos=0, block_table=t) for p, t in zip(prompts, tables)],
                    nmx.OUT_LOGITS_LAST)
    dec = m.forward(pool, [dict(tokens=[int(x)], start_pos=8, block_table=t) for x, t in zip(toks, tables)],
                    nmx.OUT_LOGITS_LAST)
    return np.concatenate([pre, dec])


def main():
    import torch
    import torch.distributed as dist
    from oracle import oracle as O
    from novamlx_b200 import nmx

    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama")
    ap.add_argument("--out", required=True)
    a = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dist.init_process_group("gloo", init_method="env://")
    torch.cuda.set_device(rank)
    d = tiny(a.model)
    full_cfg = nmx.ModelConfig(**d, max_batch=16, max_tokens=256)
    tensors = O.random_tensors(O.TinyCfg(**d), seed=5, std=0.05)
    shard = nmx.tp_shard(tensors, full_cfg, rank, world)
    ctx = nmx.Context(rank)
    m = nmx.Model(ctx, nmx.tp_config(full_cfg, world))
    for k, v in shard.items():
        m.load_tensor(k, v.view(np.float16) if v.dtype == np.uint16 else v)
    comm = nmx.tp_comm(ctx, rank, world, full_cfg.max_tokens * full_cfg.hidden * 2, nmx.torch_exchange(dist))
    m.set_comm(comm)
    pool = nmx.KVPool(m, 120)

    # op-level exchange: rank r contributes (r + 1) * base
    base = torch.arange(64 * 512, device=f"cuda:{rank}", dtype=torch.float32).reshape(64, 512) % 7 - 3
    part = ((rank + 1) * base).half()
    res = torch.ones_like(part)
    out = torch.empty_like(part)
    comm.allreduce_resid(part, res, out)
    torch.cuda.synchronize()
    ctx.synchronize()
    expect = (1 + base * sum(range(1, world + 1))).half()
    op_ok = bool(torch.equal(out, expect))

    tp_logits, tp_first, tp_ids, tp_step_logits = run(nmx, m, pool, full_cfg, 11)
    m.set_exchange_fusion(True)
    tp_batch = run_batch(nmx, m, pool, full_cfg, 12)       # exchange fused into the GEMM
    m.set_exchange_fusion(False)
    tp_batch_sep = run_batch(nmx, m, pool, full_cfg, 12)   # GEMM, then the exchange kernel
    dist.barrier()
    m.set_comm(None)
    comm.close()
    np.savez(f"{a.out}.rank{rank}.npz", op_ok=np.array(op_ok), tp_logits=tp_logits, tp_first=tp_first,
             tp_ids=tp_ids, tp_step_logits=tp_step_logits, tp_batch=tp_batch, tp_batch_sep=tp_batch_sep)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
