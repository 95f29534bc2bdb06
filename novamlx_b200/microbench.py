"""Per-kernel timings of the decode path, one kernel at a time.

  python -m novamlx_b200.microbench gemv [--n 28672] [--k 4096] [--m 1]
  python -m novamlx_b200.microbench gemm [--m 2048] [--n 4096] [--k 4096]
  python -m novamlx_b200.microbench attn [--batch 1] [--ctx 2176]
  python -m novamlx_b200.microbench decode [--layers 2] [--ctx 2048] [--tokens 64]

gemv: the decode-record GEMV (nmx_op_qmatmul_records) over `copies` distinct
weight copies, so the weights come from HBM on every launch.
gemm: the same entry point with many rows (the tcgen05 prefill GEMM); dense
f16 TFLOP/s = 2·M·N·K / t.
attn: paged decode attention (nmx_op_attn_paged_decode) at Llama-3.1-8B
head shapes (32 query heads, 8 KV heads, head dim 128, 16-token pages) over
a pool larger than L2, each rep reading a different set of pages.

decode: the model's batch-1 decode step (nmx_decode_greedy) on the
Llama-3.1-8B architecture cut to --layers layers (random 4-bit weights), at
context --ctx; the per-token time, and one short decode inside an NVTX range
named "decode" for a profiler to select.

Prints one JSON line per run with the average launch duration measured by
CUDA events on the library's stream and the algorithmic bytes per launch.
"""
from __future__ import annotations

import argparse
import json
import time


def _time(torch, fn, reps, warm=5):
    for i in range(warm):
        fn(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
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
    us = _time(torch, lambda i: ctx.quantized_matmul_records(x, recs[i % copies], n, out=y), reps)
    nbytes = n * k // 2 + 2 * n * (k // 64) * 2 + m * k * 2 + m * n * 2
    return {"kernel": "qgemv_dl_kernel", "m": m, "n": n, "k": k, "us": round(us, 2), "bytes": nbytes,
            "gbs": round(nbytes / us / 1e3, 1)}


def gemm(ctx, torch, m, n, k, reps):
    wf = torch.randn((n, k), device="cuda", dtype=torch.float32) * 0.02
    wq, s, b = ctx.quantize(wf, 64, 4)
    rec = ctx.pack_records(wq, s, b)
    del wf, wq, s, b
    x = torch.randn((m, k), device="cuda", dtype=torch.float16)
    y = torch.empty((m, n), device="cuda", dtype=torch.float16)
    us = _time(torch, lambda i: ctx.quantized_matmul_records(x, rec, n, out=y), reps)
    flops = 2.0 * m * n * k
    return {"kernel": "qgemm_tc_kernel", "m": m, "n": n, "k": k, "us": round(us, 2),
            "tflops": round(flops / us / 1e6, 1)}


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
    us = _time(torch, lambda i: ctx.paged_decode_attention(q, kc, vc, tables[i % sets], lens, hkv, d ** -0.5), reps)
    nbytes = 2 * batch * ctx_len * hkv * d * 2 + 2 * batch * hq * d * 2
    return {"kernel": "paged_decode_mma_kernel", "batch": batch, "ctx": ctx_len, "us": round(us, 2),
            "bytes": nbytes, "gbs": round(nbytes / us / 1e3, 1)}


def decode(ctx, torch, nmx, layers, ctx_len, tokens):
    import numpy as np
    cfg = nmx.llama31_8b(n_layers=layers, max_batch=1, max_tokens=ctx_len)
    m = nmx.Model(ctx, cfg)
    m.init_random(seed=0, std=0.02)
    nblk = (ctx_len + tokens + 15) // 16 + 1
    pool = nmx.KVPool(m, nblk + 4)
    table = np.arange(nblk, dtype=np.int32)
    prompt = np.random.default_rng(0).integers(0, cfg.vocab, ctx_len)
    first = int(m.forward(pool, [dict(tokens=prompt, start_pos=0, block_table=table)])[0])
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    m.forward(pool, [dict(tokens=prompt, start_pos=0, block_table=table)])
    prefill_ms = (time.perf_counter() - t0) * 1000.0
    for _ in range(3):
        m.decode_greedy(pool, [first], [ctx_len], table[None], 8, want_ids=False)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    m.decode_greedy(pool, [first], [ctx_len], table[None], tokens, want_ids=False)
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / tokens
    torch.cuda.nvtx.range_push("decode")
    m.decode_greedy(pool, [first], [ctx_len], table[None], 2, want_ids=False)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_pop()
    return {"what": "decode step", "layers": layers, "ctx": ctx_len, "us_per_token": round(us, 2),
            "prefill_ms": round(prefill_ms, 2), "weight_bytes_per_token": m.step_weight_bytes}


def main():
    import torch

    from novamlx_b200 import nmx

    ap = argparse.ArgumentParser()
    ap.add_argument("what", choices=["gemv", "gemm", "attn", "decode"])
    ap.add_argument("--n", type=int, default=None, help="gemv: 28672, gemm: 4096")
    ap.add_argument("--k", type=int, default=4096)
    ap.add_argument("--m", type=int, default=None, help="gemv: 1, gemm: 2048")
    ap.add_argument("--copies", type=int, default=3)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--ctx", type=int, default=2048)
    ap.add_argument("--reps", type=int, default=30)
    ap.add_argument("--layers", type=int, default=2)
    ap.add_argument("--tokens", type=int, default=64)
    a = ap.parse_args()
    if a.n is None:
        a.n = 4096 if a.what == "gemm" else 28672
    if a.m is None:
        a.m = 2048 if a.what == "gemm" else 1
    torch.cuda.set_device(0)
    c = nmx.Context(0)
    with torch.cuda.stream(c.stream):
        if a.what == "gemv":
            r = gemv(c, torch, a.n, a.k, a.m, a.copies, a.reps)
        elif a.what == "gemm":
            r = gemm(c, torch, a.m, a.n, a.k, a.reps)
        elif a.what == "attn":
            r = attn(c, torch, a.batch, a.ctx, a.reps)
        else:
            r = decode(c, torch, nmx, a.layers, a.ctx, a.tokens)
    print(json.dumps(r), flush=True)


if __name__ == "__main__":
    main()
