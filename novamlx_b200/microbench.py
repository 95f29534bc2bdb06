"""Per-kernel timings of the decode path, one kernel at a time.

  python -m novamlx_b200.microbench gemv [--n 28672] [--k 4096] [--m 1]
  python -m novamlx_b200.microbench qmm --m 4 --n 4096 --k 4096 --copies 32
  python -m novamlx_b200.microbench gemm [--m 2048] [--n 4096] [--k 4096]
  python -m novamlx_b200.microbench attn [--batch 1] [--ctx 2176]
  python -m novamlx_b200.microbench decode [--layers 2] [--ctx 2048] [--tokens 64] [--batch 1]
  python -m novamlx_b200.microbench serve [--layers 32] [--seqs 64] [--tokens 256]
  python -m novamlx_b200.microbench spec [--batch 16] [--ctx 4096] [--drafts 4] [--cycles 8] [--oracle-draft]
  torchrun --nproc-per-node T -m novamlx_b200.microbench tp [--batch 32] [--ctx 8192] [--steps 16] [--prefill 8192]
  torchrun --nproc-per-node T -m novamlx_b200.microbench spectp [--batch 16] [--ctx 4096] [--drafts 4] [--cycles 8]

gemv: the decode-record GEMV (nmx_op_qmatmul_records) over `copies` distinct
weight copies, so the weights come from HBM on every launch; the calls are
replayed from one CUDA graph (device time, not the host's launch rate).
gemm: the same entry point with many rows (the tcgen05 prefill GEMM); dense
f16 TFLOP/s = 2·M·N·K / t.
attn: paged decode attention (nmx_op_attn_paged_decode) at Llama-3.1-8B
head shapes (32 query heads, 8 KV heads, head dim 128, 16-token pages) over
a pool larger than L2, each rep reading a different set of pages.

decode: the model's decode step (nmx_decode_greedy, --batch sequences) on the
Llama-3.1-8B architecture cut to --layers layers (random 4-bit weights), at
context --ctx; the per-token time, and one short decode inside an NVTX range
named "decode" for a profiler to select.

serve: continuous batching (nmx_sched_*) on the Llama-3.1-8B architecture
(random 4-bit weights, --layers layers): --seqs sequences, half of them a
shared 2048-token random prefix plus a private suffix (total length uniform
in [2064, 4096]), the others uniform in [512, 4096] tokens; each decodes
--tokens greedy ids; 16-token pages, prefill chunks of 512. Reports the
aggregate generated tok/s over the whole run, the tok/s of the steps where
every running sequence decodes, the prefix-cache hit tokens, and the
distinct vs logical KV pages at the widest decode step.

spec: speculative decoding with a Llama-3.3-70B-style target and a
Llama-3.2-1B-style draft (random 4-bit weights, --layers / --draft-layers
layers): --batch sequences at context --ctx; per cycle the draft decodes
--drafts greedy ids per sequence (nmx_decode_greedy) and the target verifies
[last] + drafts in one forward (nmx_spec_verify, prefix rule: M = batch ×
(drafts + 1) rows). Random weights accept almost nothing, so the acceptance
is reported as measured; --oracle-draft replaces the drafts by the target's
own greedy continuation (computed before the timed cycles) for the
full-acceptance verify throughput. The pages before --ctx are left as
allocated (zeros): the timed work, reading ctx positions of K/V per row, is
the same as after a real prefill.

spectp: the same speculative decoding with the target tensor-parallel over
the ranks of torch.distributed.run and the draft sharded by sequence (each
rank drafts batch / N sequences with its own draft copy; the drafts are
all-gathered, then every rank verifies all sequences on its target shard).

tp: tensor-parallel decode of the Qwen2.5-32B-style architecture (random
4-bit weights, --layers layers) over the ranks of torch.distributed.run (one
GPU each; T = 1 runs without the exchange): batch --batch at context --ctx
(pages before --ctx left as allocated), --steps greedy steps timed with CUDA
events on every rank, the maximum taken; optionally one --prefill-token
prefill of a single sequence, timed the same way.

Prints one JSON line per run with the average launch duration measured by
CUDA events on the library's stream and the algorithmic bytes per launch.
"""
from __future__ import annotations

import argparse
import json
import time


def _time(torch, fn, reps, warm=5, graph=False):
    """Average device time per call. graph=True replays the reps calls from
    one CUDA graph (captured on the current stream), so the host's launch
    rate does not enter the time of a short kernel."""
    for i in range(warm):
        fn(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if graph:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=torch.cuda.current_stream()):
            for i in range(reps):
                fn(warm + i)
        g.replay()
        torch.cuda.synchronize()
        e0.record()
        g.replay()
        e1.record()
        torch.cuda.synchronize()
        del g
        return e0.elapsed_time(e1) * 1000.0 / reps
    e0.record()
    for i in range(reps):
        fn(warm + i)
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) * 1000.0 / reps


def gemv(ctx, torch, n, k, m, copies, reps):
    wf = torch.randn((n, k), device="cuda", dtype=torch.float32) * 0.02
    recs = []
    for _ in range(copies):
        wq, s, b = ctx.quantize(wf, 64, 4)
        recs.append(ctx.pack_records(wq, s, b))
        del wq, s, b
    del wf
    x = torch.randn((m, k), device="cuda", dtype=torch.float16)
    y = torch.empty((m, n), device="cuda", dtype=torch.float16)
    us = _time(torch, lambda i: ctx.quantized_matmul_records(x, recs[i % copies], n, out=y), reps, graph=True)
    nbytes = n * k // 2 + 2 * n * (k // 64) * 2 + m * k * 2 + m * n * 2
    return {"kernel": "qgemv_dl_kernel", "m": m, "n": n, "k": k, "us": round(us, 2), "bytes": nbytes,
            "gbs": round(nbytes / us / 1e3, 1), "timing": "CUDA graph of the calls"}


def qmm(ctx, torch, m, n, k, copies, reps):
    """The operator-level quantized matmul over MLX-layout weights
    (nmx_op_qmatmul, 4-bit g64, f16) rotating over `copies` weight copies."""
    wf = torch.randn((n, k), device="cuda", dtype=torch.float32) * 0.02
    ws = [ctx.quantize(wf, 64, 4) for _ in range(copies)]
    del wf
    x = torch.randn((m, k), device="cuda", dtype=torch.float16)
    y = torch.empty((m, n), device="cuda", dtype=torch.float16)
    us = _time(torch, lambda i: ctx.quantized_matmul(x, *ws[i % copies], out=y), reps)
    nbytes = n * k // 2 + 2 * n * (k // 64) * 2 + m * k * 2 + m * n * 2
    return {"kernel": "qgemv_mlx4_small_kernel", "m": m, "n": n, "k": k, "us": round(us, 2), "bytes": nbytes,
            "gbs": round(nbytes / us / 1e3, 1)}


def gemm(ctx, torch, m, n, k, reps, copies=1):
    wf = torch.randn((n, k), device="cuda", dtype=torch.float32) * 0.02
    recs = []
    for _ in range(copies):
        wq, s, b = ctx.quantize(wf, 64, 4)
        recs.append(ctx.pack_records(wq, s, b))
        del wq, s, b
    del wf
    x = torch.randn((m, k), device="cuda", dtype=torch.float16)
    y = torch.empty((m, n), device="cuda", dtype=torch.float16)
    us = _time(torch, lambda i: ctx.quantized_matmul_records(x, recs[i % copies], n, out=y), reps)
    flops = 2.0 * m * n * k
    wbytes = n * k // 2 + 2 * n * (k // 64) * 2
    return {"kernel": "qgemm_tc_kernel", "m": m, "n": n, "k": k, "copies": copies, "us": round(us, 2),
            "tflops": round(flops / us / 1e6, 1), "weight_gbs": round(wbytes / us / 1e3, 1)}


def attn(ctx, torch, batch, ctx_len, reps, hq=32, hkv=8, d=128, bt=16):
    nblk = (ctx_len + bt - 1) // bt
    # enough page sets that the pool (K and V) exceeds L2
    per_set = 2 * batch * nblk * hkv * bt * d * 2
    sets = max(2, (256 << 20) // per_set + 1)
    pool_blocks = sets * batch * nblk
    kc = torch.randn((pool_blocks, hkv, bt, d), device="cuda", dtype=torch.float16)
    vc = torch.randn_like(kc)
    q = torch.randn((batch, hq, d), device="cuda", dtype=torch.float16)
    lens = torch.full((batch,), ctx_len, dtype=torch.int32, device="cuda")
    tables = [torch.arange(s * batch * nblk, (s + 1) * batch * nblk, dtype=torch.int32, device="cuda")
              .view(batch, nblk) for s in range(sets)]
    out = torch.empty_like(q)
    us = _time(torch, lambda i: ctx.paged_decode_attention(q, kc, vc, tables[i % sets], lens, hkv, d ** -0.5, out=out),
               reps, graph=True)
    nbytes = 2 * batch * ctx_len * hkv * d * 2 + 2 * batch * hq * d * 2
    return {"kernel": "paged_decode_mma_kernel", "batch": batch, "ctx": ctx_len, "us": round(us, 2),
            "bytes": nbytes, "gbs": round(nbytes / us / 1e3, 1), "timing": "CUDA graph of the calls"}


def decode(ctx, torch, nmx, layers, ctx_len, tokens, batch=1):
    import numpy as np
    cfg = nmx.llama31_8b(n_layers=layers, max_batch=batch, max_tokens=max(ctx_len, batch))
    m = nmx.Model(ctx, cfg)
    m.init_random(seed=0, std=0.02)
    nblk = (ctx_len + tokens + 15) // 16 + 1
    pool = nmx.KVPool(m, batch * nblk + 4)
    tables = np.arange(batch * nblk, dtype=np.int32).reshape(batch, nblk)
    rng = np.random.default_rng(0)
    prompts = [rng.integers(0, cfg.vocab, ctx_len) for _ in range(batch)]
    first = []
    prefill_ms = 0.0
    for b in range(batch):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        first.append(int(m.forward(pool, [dict(tokens=prompts[b], start_pos=0, block_table=tables[b])])[0]))
        prefill_ms = (time.perf_counter() - t0) * 1000.0
    for _ in range(3):
        m.decode_greedy(pool, first, [ctx_len] * batch, tables, 8, want_ids=False)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    m.decode_greedy(pool, first, [ctx_len] * batch, tables, tokens, want_ids=False)
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / tokens
    torch.cuda.nvtx.range_push("decode")
    m.decode_greedy(pool, first, [ctx_len] * batch, tables, 2, want_ids=False)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_pop()
    return {"what": "decode step", "layers": layers, "batch": batch, "ctx": ctx_len, "us_per_step": round(us, 2),
            "tok_s": round(batch * 1e6 / us, 1), "prefill_ms": round(prefill_ms, 2),
            "weight_bytes_per_step": m.step_weight_bytes}


def serve(ctx, torch, nmx, layers, n_seqs, tokens, step_tokens, chunk, seed=0):
    import numpy as np
    rng = np.random.default_rng(seed)
    prefix = rng.integers(0, 128256, 2048)
    prompts = []
    for i in range(n_seqs):
        if i % 2 == 0:
            total = int(rng.integers(2064, 4097))
            prompts.append(np.concatenate([prefix, rng.integers(0, 128256, total - 2048)]))
        else:
            prompts.append(rng.integers(0, 128256, int(rng.integers(512, 4097))))
    cfg = nmx.llama31_8b(n_layers=layers, max_batch=n_seqs, max_tokens=step_tokens)
    m = nmx.Model(ctx, cfg)
    m.init_random(seed=0, std=0.02)
    bpt = m.kv_bytes_per_token
    logical_blocks = sum((len(p) + tokens + 15) // 16 for p in prompts)
    pool = nmx.KVPool(m, logical_blocks + 8)  # room for every page unshared: no preemption
    sched = nmx.Scheduler(m, pool, max_batch=n_seqs, max_step_tokens=step_tokens, prefill_chunk=chunk,
                          max_concurrent=n_seqs, kv_budget_bytes=160 << 30, model_name="llama-3.1-8b")
    ids = [sched.submit(p, tokens) for p in prompts]
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    dec_t = dec_tok = 0.0
    widest = (0, 0, 0)
    steps = 0
    while True:
        st0 = sched.stats()
        if st0["finished"] == n_seqs:
            break
        s0 = time.perf_counter()
        gen = sched.step()
        dt = time.perf_counter() - s0
        st = sched.stats()
        steps += 1
        if gen > 0 and st["tokens_in_steps"] - st0["tokens_in_steps"] == gen:  # every row a decode row
            dec_t += dt
            dec_tok += gen
            if gen > widest[0]:
                widest = (gen, st["blocks_in_use"], st["logical_blocks"])
        if steps > 100000:
            raise RuntimeError("scheduler did not drain")
    wall = time.perf_counter() - t0
    st = sched.stats()
    gen_total = st["generated"]
    assert all(len(sched.poll(r)[0]) == tokens for r in ids)
    sched.close()
    return {"what": "continuous batching", "layers": layers, "seqs": n_seqs, "tokens_each": tokens,
            "prompt_tokens": int(sum(len(p) for p in prompts)), "steps": st["steps"],
            "wall_s": round(wall, 3), "tok_s": round(gen_total / wall, 1),
            "decode_steps_tok_s": round(dec_tok / dec_t, 1) if dec_t else None,
            "prefix_hit_tokens": st["prefix_hit_tokens"], "tokens_in_steps": st["tokens_in_steps"],
            "widest_decode_step": {"seqs": widest[0], "distinct_pages": widest[1], "logical_pages": widest[2],
                                   "distinct_kv_gb": round(widest[1] * 16 * bpt / 1e9, 2),
                                   "logical_kv_gb": round(widest[2] * 16 * bpt / 1e9, 2)},
            "kv_bytes_per_token": bpt, "weight_bytes_per_step": m.step_weight_bytes}


def spec(ctx, torch, nmx, batch, ctx_len, n_drafts, cycles, layers, draft_layers, oracle_draft):
    import numpy as np
    D = n_drafts
    tcfg = nmx.llama33_70b(n_layers=layers, max_batch=batch, max_tokens=batch * (D + 1))
    target = nmx.Model(ctx, tcfg)
    target.init_random(seed=0, std=0.02)
    dcfg = nmx.llama32_1b(n_layers=draft_layers, max_batch=batch, max_tokens=batch)
    draft = nmx.Model(ctx, dcfg)
    draft.init_random(seed=1, std=0.02)
    span = ctx_len + (cycles + 2) * (D + 1) + 16
    nblk = (span + 15) // 16
    tables = np.arange(1, batch * nblk + 1, dtype=np.int32).reshape(batch, nblk)
    tpool = nmx.KVPool(target, batch * nblk + 2)
    dpool = nmx.KVPool(draft, batch * nblk + 2)
    rng = np.random.default_rng(0)
    last0 = rng.integers(0, tcfg.vocab, batch).astype(np.int32)
    oracle = None
    if oracle_draft:
        # drafts the target's verify accepts in full: start from its greedy
        # decode, then re-verify until every draft of every cycle is the
        # verify forward's own greedy id (each round fixes at least one more
        # position; the kernels are deterministic, so the timed run replays it)
        guess = target.decode_greedy(tpool, last0, [ctx_len] * batch, tables, cycles * (D + 1) + 1)
        oracle = []
        last = last0.copy()
        pos = np.full(batch, ctx_len, np.int64)
        for c in range(cycles + 1):
            dr = [guess[(D + 1) * c:(D + 1) * c + D, b].tolist() for b in range(batch)]
            for _ in range(D + 1):
                res = nmx.spec_verify(target, tpool, [dict(last_token=int(last[b]), drafts=dr[b], start_pos=int(pos[b]),
                                                           block_table=tables[b]) for b in range(batch)],
                                      nmx.VERIFY_PREFIX)
                if all(acc == D for _, acc in res):
                    break
                dr = [(toks + dr[b][len(toks):])[:D] for b, (toks, acc) in enumerate(res)]
            oracle.append(dr)
            for b, (toks, acc) in enumerate(res):
                pos[b] += 1 + acc
                last[b] = toks[-1]
    torch.cuda.synchronize()

    def run(n_cycles, record):
        last = last0.copy()
        pos = np.full(batch, ctx_len, np.int64)
        emitted = accepted = 0
        t0 = time.perf_counter()
        for c in range(n_cycles):
            d = draft.decode_greedy(dpool, last, pos.tolist(), tables, D)  # [D, B]
            seqs = []
            for b in range(batch):
                dr = oracle[c][b] if oracle is not None else d[:, b].tolist()
                seqs.append(dict(last_token=int(last[b]), drafts=dr, start_pos=int(pos[b]), block_table=tables[b]))
            res = nmx.spec_verify(target, tpool, seqs, nmx.VERIFY_PREFIX)
            for b, (toks, acc) in enumerate(res):
                emitted += len(toks)
                accepted += acc
                pos[b] += 1 + acc
                last[b] = toks[-1]
        torch.cuda.synchronize()
        return time.perf_counter() - t0, emitted, accepted

    if oracle is None:
        run(1, False)  # warm-up: graphs and kernel attributes (the oracle rounds warmed up otherwise)
    wall, emitted, accepted = run(cycles, True)
    return {"what": "speculative decoding", "target_layers": layers, "draft_layers": draft_layers, "batch": batch,
            "ctx": ctx_len, "drafts": D, "cycles": cycles, "oracle_draft": bool(oracle_draft),
            "ms_per_cycle": round(wall * 1000.0 / cycles, 3), "tok_s": round(emitted / wall, 1),
            "acceptance": round(accepted / (cycles * batch * D), 4),
            "target_weight_bytes": target.step_weight_bytes, "draft_weight_bytes": draft.step_weight_bytes}


def spec_tp(torch, nmx, batch, ctx_len, n_drafts, cycles, layers, draft_layers):
    """Speculative decoding with the 70B-style target tensor-parallel over
    the ranks of torch.distributed.run and the 1B-style draft sharded by
    sequence: rank r drafts sequences r·B/N .. (r+1)·B/N - 1 with its own
    copy of the draft (its own KV pool), the drafts are all-gathered (host
    ids over the process group), and every rank runs the same verify forward
    of all B sequences on its shard of the target (the exchange makes the
    results identical on every rank). Timed by wall clock per cycle, the
    maximum over ranks."""
    import numpy as np
    import os
    import torch.distributed as dist
    rank, world = int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1:
        dist.init_process_group("gloo", init_method="env://")
    if batch % world:
        raise ValueError("the batch must divide by the number of ranks")
    torch.cuda.set_device(rank)
    ctx = nmx.Context(rank)
    D, bl = n_drafts, batch // world
    tcfg = nmx.llama33_70b(n_layers=layers, max_batch=batch, max_tokens=batch * (D + 1))
    target = nmx.Model(ctx, nmx.tp_config(tcfg, world) if world > 1 else tcfg)
    target.init_random(seed=rank, std=0.02)
    comm = None
    if world > 1:
        comm = nmx.tp_comm(ctx, rank, world, batch * (D + 1) * tcfg.hidden * 2, nmx.torch_exchange(dist))
        target.set_comm(comm)
    dcfg = nmx.llama32_1b(n_layers=draft_layers, max_batch=bl, max_tokens=bl)
    draft = nmx.Model(ctx, dcfg)
    draft.init_random(seed=1, std=0.02)
    span = ctx_len + (cycles + 2) * (D + 1) + 16
    nblk = (span + 15) // 16
    tables = np.arange(1, batch * nblk + 1, dtype=np.int32).reshape(batch, nblk)
    dtables = np.arange(1, bl * nblk + 1, dtype=np.int32).reshape(bl, nblk)
    tpool = nmx.KVPool(target, batch * nblk + 2)
    dpool = nmx.KVPool(draft, bl * nblk + 2)
    last0 = np.random.default_rng(0).integers(0, tcfg.vocab, batch).astype(np.int32)
    mine = slice(rank * bl, (rank + 1) * bl)

    def gather(d_local):
        # [D, bl] per rank -> [D, batch] on every rank
        if world == 1:
            return d_local
        t = torch.from_numpy(np.ascontiguousarray(d_local.astype(np.int32)))
        parts = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(parts, t)
        return np.concatenate([p.numpy() for p in parts], axis=1)

    def run(n_cycles):
        last = last0.copy()
        pos = np.full(batch, ctx_len, np.int64)
        emitted = accepted = 0
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(n_cycles):
            d = gather(draft.decode_greedy(dpool, last[mine], pos[mine].tolist(), dtables, D))
            seqs = [dict(last_token=int(last[b]), drafts=d[:, b].tolist(), start_pos=int(pos[b]),
                         block_table=tables[b]) for b in range(batch)]
            res = nmx.spec_verify(target, tpool, seqs, nmx.VERIFY_PREFIX)
            for b, (toks, acc) in enumerate(res):
                emitted += len(toks)
                accepted += acc
                pos[b] += 1 + acc
                last[b] = toks[-1]
        torch.cuda.synchronize()
        wall = torch.tensor([time.perf_counter() - t0], dtype=torch.float64)
        if world > 1:
            dist.all_reduce(wall, op=dist.ReduceOp.MAX)
        return float(wall[0]), emitted, accepted

    run(1)  # warm-up: graphs and kernel attributes
    wall, emitted, accepted = run(cycles)
    out = {"what": "speculative decoding, tensor-parallel target, draft sharded by sequence", "tp": world,
           "target_layers": layers, "draft_layers": draft_layers, "batch": batch, "ctx": ctx_len, "drafts": D,
           "cycles": cycles, "ms_per_cycle": round(wall * 1000.0 / cycles, 3), "tok_s": round(emitted / wall, 1),
           "acceptance": round(accepted / (cycles * batch * D), 4),
           "target_weight_bytes_per_rank": target.step_weight_bytes, "draft_weight_bytes": draft.step_weight_bytes}
    if world > 1:
        target.set_comm(None)
        comm.close()
        dist.barrier()
        dist.destroy_process_group()
    return out if rank == 0 else None


def tp(torch, nmx, batch, ctx_len, steps, layers, prefill, fuse=False):
    import numpy as np
    import os
    import torch.distributed as dist
    rank, world = int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1:
        dist.init_process_group("gloo", init_method="env://")
    torch.cuda.set_device(rank)
    ctx = nmx.Context(rank)
    max_tokens = max(batch, prefill or 0, 16)
    cfg = nmx.qwen25_32b(n_layers=layers, max_batch=batch, max_tokens=max_tokens)
    local = nmx.tp_config(cfg, world)
    m = nmx.Model(ctx, local)
    m.init_random(seed=rank, std=0.02)
    comm = None
    if world > 1:
        comm = nmx.tp_comm(ctx, rank, world, max_tokens * cfg.hidden * 2, nmx.torch_exchange(dist))
        m.set_comm(comm)
        m.set_exchange_fusion(fuse)
    nblk = (ctx_len + steps + 64 + 15) // 16
    pblk = ((prefill or 0) + 15) // 16
    pool = nmx.KVPool(m, batch * nblk + pblk + 2)
    tables = np.arange(1, batch * nblk + 1, dtype=np.int32).reshape(batch, nblk)
    first = np.random.default_rng(0).integers(0, cfg.vocab, batch).astype(np.int32)

    def timed(fn):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(ctx.stream):
            e0.record()
            fn()
            e1.record()
        torch.cuda.synchronize()
        ms = torch.tensor([e0.elapsed_time(e1)])
        if world > 1:
            dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        return float(ms[0])

    m.decode_greedy(pool, first, [ctx_len] * batch, tables, 4, want_ids=False)  # graphs, attributes
    ms = timed(lambda: m.decode_greedy(pool, first, [ctx_len] * batch, tables, steps, want_ids=False))
    out = {"what": "tensor-parallel decode", "model": "qwen2.5-32b-style", "layers": layers, "tp": world,
           "exchange": "fused into the GEMM" if fuse else "separate kernel",
           "batch": batch, "ctx": ctx_len, "steps": steps, "ms_per_step": round(ms / steps, 3),
           "tok_s": round(batch * steps * 1000.0 / ms, 1),
           "weight_bytes_per_rank": m.step_weight_bytes, "kv_bytes_per_token_per_rank": m.kv_bytes_per_token}
    if prefill:
        ptab = np.arange(batch * nblk + 1, batch * nblk + 1 + pblk, dtype=np.int32)
        ptoks = np.random.default_rng(1).integers(0, cfg.vocab, prefill)
        m.forward(pool, [dict(tokens=ptoks[:256], start_pos=0, block_table=ptab)])  # warm
        pm = timed(lambda: m.forward(pool, [dict(tokens=ptoks, start_pos=0, block_table=ptab)]))
        out.update(prefill_tokens=prefill, prefill_ms=round(pm, 2))
    if world > 1:
        m.set_comm(None)
        comm.close()
        dist.barrier()
        dist.destroy_process_group()
    return out if rank == 0 else None


def main():
    import torch

    from novamlx_b200 import nmx

    ap = argparse.ArgumentParser()
    ap.add_argument("what", choices=["gemv", "qmm", "gemm", "attn", "decode", "serve", "spec", "spectp", "tp"])
    ap.add_argument("--n", type=int, default=None, help="gemv: 28672, gemm: 4096")
    ap.add_argument("--k", type=int, default=4096)
    ap.add_argument("--m", type=int, default=None, help="gemv: 1, gemm: 2048")
    ap.add_argument("--copies", type=int, default=None, help="gemv: 3, gemm: 1")
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--ctx", type=int, default=2048)
    ap.add_argument("--reps", type=int, default=30)
    ap.add_argument("--layers", type=int, default=None, help="decode: 2, serve: 32")
    ap.add_argument("--tokens", type=int, default=None, help="decode: 64, serve: 256")
    ap.add_argument("--seqs", type=int, default=64)
    ap.add_argument("--step-tokens", type=int, default=4096)
    ap.add_argument("--chunk", type=int, default=512)
    ap.add_argument("--drafts", type=int, default=4)
    ap.add_argument("--cycles", type=int, default=8)
    ap.add_argument("--draft-layers", type=int, default=16)
    ap.add_argument("--oracle-draft", action="store_true")
    ap.add_argument("--steps", type=int, default=16)
    ap.add_argument("--prefill", type=int, default=0)
    ap.add_argument("--fuse", action="store_true", help="tp: exchange fused into the decode-batch GEMM epilogue")
    a = ap.parse_args()
    if a.copies is None:
        a.copies = 1 if a.what == "gemm" else 3
    if a.layers is None:
        a.layers = {"serve": 32, "spec": 80, "spectp": 80, "tp": 64}.get(a.what, 2)
    if a.tokens is None:
        a.tokens = 256 if a.what == "serve" else 64
    if a.n is None:
        a.n = 4096 if a.what == "gemm" else 28672
    if a.m is None:
        a.m = 2048 if a.what == "gemm" else 1
    if a.what == "spectp":
        r = spec_tp(torch, nmx, a.batch if a.batch != 1 else 16, a.ctx if a.ctx != 2048 else 4096, a.drafts,
                    a.cycles, a.layers, a.draft_layers)
        if r is not None:
            print(json.dumps(r), flush=True)
        return
    if a.what == "tp":
        r = tp(torch, nmx, a.batch if a.batch != 1 else 32, a.ctx if a.ctx != 2048 else 8192, a.steps, a.layers,
               a.prefill, a.fuse)
        if r is not None:
            print(json.dumps(r), flush=True)
        return
    torch.cuda.set_device(0)
    c = nmx.Context(0)
    with torch.cuda.stream(c.stream):
        if a.what == "gemv":
            r = gemv(c, torch, a.n, a.k, a.m, a.copies, a.reps)
        elif a.what == "qmm":
            r = qmm(c, torch, a.m, a.n, a.k, a.copies, a.reps)
        elif a.what == "gemm":
            r = gemm(c, torch, a.m, a.n, a.k, a.reps, a.copies)
        elif a.what == "attn":
            r = attn(c, torch, a.batch, a.ctx, a.reps)
        elif a.what == "spec":
            r = spec(c, torch, nmx, a.batch if a.batch != 1 else 16, a.ctx if a.ctx != 2048 else 4096, a.drafts,
                     a.cycles, a.layers, a.draft_layers, a.oracle_draft)
        elif a.what == "serve":
            r = serve(c, torch, nmx, a.layers, a.seqs, a.tokens, a.step_tokens, a.chunk)
        else:
            r = decode(c, torch, nmx, a.layers, a.ctx, a.tokens, a.batch)
    print(json.dumps(r), flush=True)


if __name__ == "__main__":
    main()
