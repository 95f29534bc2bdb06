"""Benchmark: 4-bit Llama-3.1-8B-architecture greedy decode on B200.

Workload (the one the headline metric is quoted on): random-init N(0, 0.02)
weights quantized MLX-affine 4-bit g64 (hidden 4096, 32 layers, 32/8 heads,
head_dim 128, SwiGLU 14336, vocab 128256, RMSNorm 1e-5, RoPE θ 5e5 with the
Llama-3.1 scaling), batch 1, a prompt of 2048 uniform-random ids prefilled
once, then one STEP = greedy decode of 256 tokens from position 2048 (each
step rewrites the same KV pages). value = tokens/s over the K timed steps,
summed over GPUs. With N GPUs every rank decodes its own sequence (replicas,
weak scaling; the path needs no collective at batch 1).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

--impl reference times the CPU restatement of the same decode step (the
reference itself is Swift + Apple Metal and cannot run here) on all host
cores, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

PROMPT = 2048
GEN = 256
METRIC = "4-bit decode tok/s (Llama-3.1-8B arch, batch 1, ctx 2048+256)"
WORKLOAD = ("Llama-3.1-8B architecture, MLX-affine 4-bit g64 random-init weights, batch 1 per GPU, "
            "2048-token random prompt, 256 greedy tokens per step")


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


class Clocks:
    """nvidia-smi sampling during the timed region."""

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"nmx_clocks_{os.getpid()}.csv"

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.device}", f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.f,
                                         stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.f.close()

    def summary(self) -> dict:
        if not self.proc or not self.path.exists():
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.path.read_text().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        self.path.unlink(missing_ok=True)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------ CPU legs

def host_model_8b(seed: int = 0):
    """Host copy of an 8B-architecture 4-bit model for the CPU restatement:
    random packed codes and per-group scale/bias of the magnitude
    N(0, 0.02) weights produce (the CPU arithmetic does not depend on the
    values). Returns an OracleModel."""
    from oracle import oracle as O
    cfg = O.TinyCfg(vocab=128256, hidden=4096, n_layers=32, n_heads=32, n_kv_heads=8, head_dim=128, ffn=14336,
                    rope_theta=500000.0, rope_factor=8.0, rope_low_freq_factor=1.0, rope_high_freq_factor=4.0,
                    rope_original_max_pos=8192)
    rng = np.random.default_rng(seed)
    t = {}

    def lin(name, N, K):
        t[f"{name}.weight"] = rng.integers(0, 2 ** 32, (N, K // 8), dtype=np.uint32)
        t[f"{name}.scales"] = O.f32_to_f16bits(np.full((N, K // 64), 0.0064, np.float32)
                                               * (1 + 0.1 * rng.standard_normal((N, K // 64), np.float32)))
        t[f"{name}.biases"] = O.f32_to_f16bits(np.full((N, K // 64), -0.048, np.float32)
                                               * (1 + 0.1 * rng.standard_normal((N, K // 64), np.float32)))

    H, F, V = 4096, 14336, 128256
    t["model.embed_tokens.weight"] = O.f32_to_f16bits(rng.standard_normal((V, H), np.float32) * 0.02)
    t["model.norm.weight"] = O.f32_to_f16bits(np.ones(H, np.float32))
    lin("lm_head", V, H)
    for i in range(32):
        p = f"model.layers.{i}"
        t[f"{p}.input_layernorm.weight"] = O.f32_to_f16bits(np.ones(H, np.float32))
        t[f"{p}.post_attention_layernorm.weight"] = O.f32_to_f16bits(np.ones(H, np.float32))
        lin(f"{p}.self_attn.q_proj", 4096, H)
        lin(f"{p}.self_attn.k_proj", 1024, H)
        lin(f"{p}.self_attn.v_proj", 1024, H)
        lin(f"{p}.self_attn.o_proj", H, 4096)
        lin(f"{p}.mlp.gate_proj", F, H)
        lin(f"{p}.mlp.up_proj", F, H)
        lin(f"{p}.mlp.down_proj", H, F)
    return O.OracleModel(cfg, t)


def host_threads() -> int:
    """Every host core this process may run on, whatever OMP_NUM_THREADS the
    launcher set (torch.distributed.run sets 1)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_decode_sample(max_seconds: float, min_tokens: int, max_tokens: int, seed: int = 0):
    """Times the CPU restatement's decode step at context 2048 (random KV of
    the right size; a CPU prefill of 2048 tokens would take tens of minutes).
    Returns (tok/s, tokens, seconds, threads)."""
    from oracle import oracle as O
    O.set_threads(host_threads())
    om = host_model_8b(seed)
    kc, vc, cap = om.new_cache(PROMPT + max_tokens + 8)
    rng = np.random.default_rng(seed + 1)
    kc[:, :, :PROMPT] = O.f32_to_f16bits(rng.standard_normal(kc[:, :, :PROMPT].shape, np.float32))
    vc[:, :, :PROMPT] = O.f32_to_f16bits(rng.standard_normal(vc[:, :, :PROMPT].shape, np.float32))
    cache = (kc, vc, cap)
    om.forward(cache, [1], PROMPT)  # warm-up token
    n, t0 = 0, time.perf_counter()
    tok = 1
    while n < max_tokens and (n < min_tokens or time.perf_counter() - t0 < max_seconds):
        lg = om.forward(cache, [tok], PROMPT + 1 + n)
        tok = int(np.argmax(lg[0]))
        n += 1
    dt = time.perf_counter() - t0
    return n / dt, n, dt, O.max_threads()


def run_reference(args, rank: int, world: int) -> None:
    if rank != 0:
        return
    from oracle import oracle as O
    O.set_threads(host_threads())
    om = host_model_8b(0)
    kc, vc, cap = om.new_cache(PROMPT + args.warmup + args.steps + 8)
    rng = np.random.default_rng(1)
    kc[:, :, :PROMPT] = O.f32_to_f16bits(rng.standard_normal(kc[:, :, :PROMPT].shape, np.float32))
    vc[:, :, :PROMPT] = O.f32_to_f16bits(rng.standard_normal(vc[:, :, :PROMPT].shape, np.float32))
    cache = (kc, vc, cap)
    pos, tok = PROMPT, 1
    for _ in range(args.warmup):
        tok = int(np.argmax(om.forward(cache, [tok], pos)[0]))
        pos += 1
    t0 = time.perf_counter()
    for _ in range(args.steps):
        tok = int(np.argmax(om.forward(cache, [tok], pos)[0]))
        pos += 1
    dt = time.perf_counter() - t0
    v = args.steps / dt
    cores = O.max_threads()
    sample = (f"{args.steps} decode tokens of the 8B-architecture 4-bit model at context {PROMPT}, one token "
              f"per step (C restatement, OpenMP)")
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * dt / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic", "config": {"workload": WORKLOAD, "global_batch": 1, "seq_len": PROMPT + GEN,
                                            "parallelism": "cpu"},
            "cpu_baseline": {"value": v, "unit": "tok/s", "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "reference is Swift + Apple Metal (MLX); its arithmetic restated in C runs on the host cores"}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ GPU leg

def time_gemv_roofline(torch, nmx, ctx, peaks, N=2 * 14336, K=4096, copies=3, reps=30):
    """Average duration of the decode-record GEMV (the kernel every linear of
    the decode step runs) at the gate/up shape (M=1, N=28672, K=4096, Q4 g64),
    rotating over `copies` distinct weight copies so no launch finds its
    weights in L2. Timed with CUDA events on the library's stream."""
    wf = torch.randn((N, K), device="cuda", dtype=torch.float32) * 0.02
    recs = []
    for _ in range(copies):
        wq, s, b = ctx.quantize(wf, 64, 4)
        recs.append(ctx.pack_records(wq, s, b))
        del wq, s, b
    del wf
    x = torch.randn((1, K), device="cuda", dtype=torch.float16)
    y = torch.empty((1, N), device="cuda", dtype=torch.float16)
    for i in range(5):
        ctx.quantized_matmul_records(x, recs[i % copies], N, out=y)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(reps):
        ctx.quantized_matmul_records(x, recs[i % copies], N, out=y)
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / reps
    nbytes = N * K // 2 + 2 * N * (K // 64) * 2 + K * 2 + N * 2
    ach = nbytes / (us * 1e-6) / 1e9
    return {"bound": "hbm", "achieved": round(ach, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
            "frac": round(ach / peaks["hbm_gbs"], 4), "traffic": None,
            "kernel": f"qgemv_dl8_kernel (decode-record GEMV, M=1, N={N}, K={K}, 4-bit g64)",
            "bytes_per_launch": nbytes, "us_per_launch": round(us, 2),
            "peak_source": f"{peaks['source']} (MEASURED_PEAKS.json hbm_gbs)"}


TRAFFIC_PROFILE = ROOT / "profiles" / "qgemv_dl_m1_n28672_k4096.md"


def profiled_traffic():
    """DRAM bytes (read + write) per launch of the roofline kernel, from the
    committed ncu summary of the same shape (`traffic_bytes_per_launch:`)."""
    try:
        for line in TRAFFIC_PROFILE.read_text().splitlines():
            if line.strip().startswith("traffic_bytes_per_launch:"):
                return int(line.split(":", 1)[1].strip())
    except OSError:
        pass
    return None


def time_c1(torch, ctx, peaks, copies=32, reps=64):
    """C1: x f16[4,4096] · Q4g64 W[4096,4096]^T over 32 rotating W copies (> L2)."""
    wf = torch.randn((4096, 4096), device="cuda", dtype=torch.float32) * 0.02
    ws = [ctx.quantize(wf, 64, 4) for _ in range(copies)]
    x = torch.randn((4, 4096), device="cuda", dtype=torch.float16)
    y = torch.empty((4, 4096), device="cuda", dtype=torch.float16)
    for i in range(copies):
        ctx.quantized_matmul(x, *ws[i], out=y)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(reps):
        ctx.quantized_matmul(x, *ws[i % copies], out=y)
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / reps
    nbytes = 9_502_720
    return {"us_per_call": round(us, 2), "achieved_gbs": round(nbytes / (us * 1e-6) / 1e9, 1),
            "frac_of_measured_hbm": round(nbytes / (us * 1e-6) / 1e9 / peaks["hbm_gbs"], 4),
            "bytes_per_call": nbytes}


def run_ours(args, rank: int, world: int, dist) -> None:
    import torch
    from novamlx_b200 import nmx

    dev = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(dev)
    peaks = measured_peaks()
    ctx = nmx.Context(dev)
    # every torch op and event below runs on the library's stream
    with torch.cuda.stream(ctx.stream):
        _run_ours(args, rank, world, dist, torch, nmx, ctx, peaks, dev)


def _run_ours(args, rank, world, dist, torch, nmx, ctx, peaks, dev):
    cfg = nmx.llama31_8b(max_batch=1, max_tokens=PROMPT)
    model = nmx.Model(ctx, cfg)
    model.init_random(seed=0, std=0.02)
    nblk = (PROMPT + GEN + 15) // 16
    pool = nmx.KVPool(model, nblk + 8)
    table = np.arange(nblk, dtype=np.int32)
    prompt = np.random.default_rng(rank).integers(0, cfg.vocab, PROMPT)
    first = int(model.forward(pool, [dict(tokens=prompt, start_pos=0, block_table=table)])[0])

    def step(want_ids=False):
        return model.decode_greedy(pool, [first], [PROMPT], table[None], GEN, want_ids=want_ids)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    def barrier():
        if dist is not None:
            dist.barrier()

    launches0 = ctx.launches
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(dev) as clk:
        barrier()
        torch.cuda.synchronize()
        e0.record()
        torch.cuda.nvtx.range_push("timed")  # lets a profiler capture only the timed steps
        for _ in range(args.steps):
            step()
        torch.cuda.nvtx.range_pop()
        e1.record()
        torch.cuda.synchronize()
        barrier()
    ms = e0.elapsed_time(e1)
    launches = ctx.launches - launches0
    if dist is not None:
        t = torch.tensor([ms], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    tokens = world * args.steps * GEN
    value = tokens / (ms / 1000.0)
    ids = step(want_ids=True)[:, 0]

    # end to end through the host-facing forward: one call per token, host ids in/out
    e2e_steps = max(1, min(args.steps, 2))
    cur = first
    for _ in range(8):
        model.forward(pool, [dict(tokens=[cur], start_pos=PROMPT, block_table=table)])
    barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        cur = first
        for i in range(GEN):
            cur = int(model.forward(pool, [dict(tokens=[cur], start_pos=PROMPT + i, block_table=table)])[0])
    e2e_s = time.perf_counter() - t0
    if dist is not None:
        t = torch.tensor([e2e_s], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e = world * e2e_steps * GEN / e2e_s
    h2d = GEN * (4 * 4 + 4 * len(table))
    d2h = GEN * 4

    roof = time_gemv_roofline(torch, nmx, ctx, peaks)
    c1 = time_c1(torch, ctx, peaks)
    roof["traffic"] = profiled_traffic()
    step_bytes = model.step_weight_bytes + model.kv_bytes_per_token * (PROMPT + GEN // 2)
    per_gpu_tps = value / world
    step_gbs = step_bytes * per_gpu_tps / 1e9

    if rank != 0:
        return
    cpu = None
    if world == 1 and not args.no_cpu:
        tps, n, secs, thr = cpu_decode_sample(max_seconds=args.cpu_seconds, min_tokens=2, max_tokens=64)
        cpu = {"value": round(tps, 4), "unit": "tok/s", "cores": thr, "kind": "port",
               "sample": f"{n} decode tokens at context {PROMPT} in {secs:.1f} s (C restatement, OpenMP, "
                         f"{thr} threads)"}
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {"workload": WORKLOAD, "global_batch": world, "seq_len": PROMPT + GEN,
                   "parallelism": f"replicas x{world} (independent sequence per GPU)",
                   "l2": "inputs larger than L2: ~4.5 GB of weights+KV read per token"},
        "roofline": roof,
        "step_roofline": {"bytes_per_token": step_bytes, "achieved": round(step_gbs, 1),
                          "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": round(step_gbs / peaks["hbm_gbs"], 4)},
        "c1_qmatmul": c1,
        "cpu_baseline": cpu,
        "e2e": {"value": round(e2e, 2), "unit": "tok/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "call": "nmx_forward, one call per token, host token in / host id out"},
        "gpu_launches": launches,
        "clocks": clk.summary(),
        "sample_ids": [int(i) for i in ids[:8]],
    }
    print(json.dumps(line), flush=True)


def main():
    global PROMPT, GEN
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--prompt", type=int, default=PROMPT, help="prompt length (profiling runs only)")
    ap.add_argument("--gen", type=int, default=GEN, help="tokens per step (profiling runs only)")
    args = ap.parse_args()
    PROMPT, GEN = args.prompt, args.gen
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    dist = None
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    try:
        run_ours(args, rank, world, dist)
    finally:
        if dist is not None:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
