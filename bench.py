"""Benchmark: 4-bit decode on B200, the Qwen2.5-32B-style tensor-parallel config.

Headline workload (the configuration the decode tok/s metric is quoted on at
1/2/4/8 GPUs): Qwen2.5-32B-style architecture (hidden 5120, 64 layers, 40/8
heads of 128, qkv bias, SwiGLU 27648, vocab 152064, RMSNorm 1e-6, RoPE 1e6),
random-init N(0, 0.02) weights quantized MLX-affine 4-bit g64, tensor-parallel
over the N ranks (q/k/v/gate/up by output rows, o/down by K; one exchange
after o_proj and after down_proj through the library's peer-memory kernel);
32 sequences at context 8192 (KV pages filled with seeded random values: a
cache of that context without running its 262k-token prefill). One STEP =
16 greedy decode tokens for each of the 32 sequences (512 tokens), every
step from context 8192 (rewriting the same pages). value = tokens/s of the
whole job (max over ranks of the device time); scaling "strong" (the same 32
sequences at every N).

Secondary keys: `e2e` (the same decode through nmx_forward, host ids in and
out), the exchange per call next to an NCCL all-reduce of the same 327,680
bytes (N > 1), the 8192-token prefill of one sequence, the dominant kernels'
rooflines; at N = 1 also the Llama-3.1-8B batch-1 decode (`c2_decode`), the
single quantized matmul (`c1_qmatmul`, CUDA-graph timed), continuous
batching (`c3_serve`), speculative decoding (`c5_spec`) and the CPU
baseline.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

--impl reference times the CPU restatement of the same decode step (the
reference itself is Swift + Apple Metal and cannot run here) on all host
cores, rank 0 only, extrapolated from one layer (see cpu_c4_step).
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

# the headline workload
C4_BATCH, C4_CTX, C4_GEN = 32, 8192, 16
C4_PREFILL = 8192
METRIC = "4-bit decode tok/s (Qwen2.5-32B-style, batch 32 at context 8192, tensor-parallel over the GPUs)"
WORKLOAD = ("Qwen2.5-32B-style architecture, MLX-affine 4-bit g64 random-init weights, tensor-parallel over the "
            "GPUs, 32 sequences at context 8192, 16 greedy tokens per sequence per step")
# the batch-1 8B decode (secondary key)
PROMPT = 2048
GEN = 256


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

def host_model(arch: str, n_layers: int, seed: int = 0):
    """Host copy of a 4-bit model of the given architecture for the CPU
    restatement: random packed codes and per-group scale/bias of the
    magnitude N(0, 0.02) weights produce (the CPU arithmetic does not depend
    on the values). arch: "llama31_8b" or "qwen25_32b". Returns an
    OracleModel."""
    from oracle import oracle as O
    if arch == "llama31_8b":
        dims = dict(vocab=128256, hidden=4096, n_heads=32, n_kv_heads=8, head_dim=128, ffn=14336,
                    rope_theta=500000.0, rope_factor=8.0, rope_low_freq_factor=1.0, rope_high_freq_factor=4.0,
                    rope_original_max_pos=8192)
    else:
        dims = dict(vocab=152064, hidden=5120, n_heads=40, n_kv_heads=8, head_dim=128, ffn=27648, qkv_bias=True,
                    rms_eps=1e-6, rope_theta=1e6)
    cfg = O.TinyCfg(n_layers=n_layers, **dims)
    return O.OracleModel(cfg, host_tensors(cfg, seed))


def host_tensors(cfg, seed: int = 0) -> dict:
    """MLX-named random 4-bit tensors of an oracle config (see host_model)."""
    from oracle import oracle as O
    n_layers = cfg.n_layers
    rng = np.random.default_rng(seed)
    t = {}

    def lin(name, N, K):
        t[f"{name}.weight"] = rng.integers(0, 2 ** 32, (N, K // 8), dtype=np.uint32)
        t[f"{name}.scales"] = O.f32_to_f16bits(np.full((N, K // 64), 0.0064, np.float32)
                                               * (1 + 0.1 * rng.standard_normal((N, K // 64), np.float32)))
        t[f"{name}.biases"] = O.f32_to_f16bits(np.full((N, K // 64), -0.048, np.float32)
                                               * (1 + 0.1 * rng.standard_normal((N, K // 64), np.float32)))

    H, F, V = cfg.hidden, cfg.ffn, cfg.vocab
    Nq, Nkv = cfg.n_heads * cfg.head_dim, cfg.n_kv_heads * cfg.head_dim
    # a decode step reads one embedding row per token: the first 4096 rows
    # hold values of magnitude ~0.02 (random f16 mantissas and signs,
    # exponents 2^-7..2^-5), the rest stay zero (values do not change CPU time)
    emb = np.zeros((V, H), np.uint16)
    emb[:4096] = (rng.integers(0x2000, 0x2800, (4096, H), dtype=np.uint16)
                  | (rng.integers(0, 2, (4096, H), dtype=np.uint16) << 15))
    t["model.embed_tokens.weight"] = emb
    t["model.norm.weight"] = O.f32_to_f16bits(np.ones(H, np.float32))
    lin("lm_head", V, H)
    for i in range(n_layers):
        p = f"model.layers.{i}"
        t[f"{p}.input_layernorm.weight"] = O.f32_to_f16bits(np.ones(H, np.float32))
        t[f"{p}.post_attention_layernorm.weight"] = O.f32_to_f16bits(np.ones(H, np.float32))
        lin(f"{p}.self_attn.q_proj", Nq, H)
        lin(f"{p}.self_attn.k_proj", Nkv, H)
        lin(f"{p}.self_attn.v_proj", Nkv, H)
        lin(f"{p}.self_attn.o_proj", H, Nq)
        lin(f"{p}.mlp.gate_proj", F, H)
        lin(f"{p}.mlp.up_proj", F, H)
        lin(f"{p}.mlp.down_proj", H, F)
        if cfg.qkv_bias:
            for nm, n in (("q", Nq), ("k", Nkv), ("v", Nkv)):
                t[f"{p}.self_attn.{nm}_proj.bias"] = O.f32_to_f16bits(0.02 * rng.standard_normal(n, np.float32))
    return t


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
    om = host_model("llama31_8b", 32, seed)
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


class CpuC4:
    """The CPU restatement of the headline decode step (Qwen2.5-32B-style,
    32 sequences at context 8192), sampled so that a sample takes seconds:
    1- and 3-layer copies of the model instead of 64 layers, and
    `sample_seqs` of the 32 sequences (every sequence does the same work).
    Per sequence and token: layer = (t(3 layers) - t(1 layer)) / 2, head
    (embedding, final norm, LM head) = t(1 layer) - layer; the full step is
    extrapolated as 32 x (head + 64 x layer). Each copy's KV cache is one
    shared random 8192-token cache (values do not change CPU time)."""

    def __init__(self, sample_seqs: int = 4):
        from oracle import oracle as O
        O.set_threads(host_threads())
        self.n = sample_seqs
        self.m3 = host_model("qwen25_32b", 3, seed=0)
        # the 1-layer copy shares the 3-layer copy's embedding, head and layer 0
        self.m1 = O.OracleModel(O.TinyCfg(**{**self.m3.cfg.__dict__, "n_layers": 1}), self.m3.t)
        rng = np.random.default_rng(1)
        # moderate random f16 values: random mantissas and signs, exponents 2^-3..2^0
        bits = lambda shape: (rng.integers(0x3000, 0x3C00, shape, dtype=np.uint16)
                              | (rng.integers(0, 2, shape, dtype=np.uint16) << 15))
        self.caches = []
        for m in (self.m1, self.m3):
            kc, vc, cap = m.new_cache(C4_CTX + 8)
            kc[:, :, :C4_CTX] = bits(kc[:, :, :C4_CTX].shape)
            vc[:, :, :C4_CTX] = bits(vc[:, :, :C4_CTX].shape)
            self.caches.append((kc, vc, cap))
        self.cores = O.max_threads()
        for m, c in zip((self.m1, self.m3), self.caches):  # first touch of the weights and caches
            m.forward(c, [1], C4_CTX)

    def _time(self, model, cache) -> float:
        t0 = time.perf_counter()
        for i in range(self.n):
            model.forward(cache, [1 + i], C4_CTX)
        return (time.perf_counter() - t0) / self.n

    def step_seconds(self) -> float:
        """Extrapolated seconds of one decode step of all 32 sequences (one token each)."""
        t1 = self._time(self.m1, self.caches[0])
        t3 = self._time(self.m3, self.caches[1])
        layer = max(t3 - t1, 0.0) / 2
        head = max(t1 - layer, 0.0)
        return C4_BATCH * (head + 64 * layer)

    def sample_text(self) -> str:
        return (f"one decode token of {self.n} of the 32 sequences through 1- and 3-layer copies of the "
                f"Qwen2.5-32B-style 4-bit model at context {C4_CTX}, extrapolated to 64 layers and 32 sequences "
                f"(C restatement, OpenMP, {self.cores} threads)")


def run_reference(args, rank: int, world: int) -> None:
    """The reference arm: the C restatement of the headline decode step on
    the host cores (rank 0 only; other ranks exit without work)."""
    if rank != 0:
        return
    cpu = CpuC4()
    for _ in range(args.warmup):
        cpu.step_seconds()
    t = [cpu.step_seconds() for _ in range(args.steps)]
    sec = float(np.mean(t))
    v = C4_BATCH / sec  # one token per sequence per extrapolated step
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * sec * C4_GEN,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic", "config": {"workload": WORKLOAD, "global_batch": C4_BATCH, "seq_len": C4_CTX,
                                            "parallelism": f"tp{world}"},
            "cpu_baseline": {"value": v, "unit": "tok/s", "cores": cpu.cores, "kind": "port",
                             "sample": cpu.sample_text()},
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": ("reference is Swift + Apple Metal (MLX) and cannot run here; its arithmetic restated in C "
                     "runs on the host cores; the step time is extrapolated from one layer")}
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


def profiled_traffic(name: str):
    """DRAM bytes (read + write) per launch of a roofline kernel, from the
    committed ncu summary `profiles/<name>` (`traffic_bytes_per_launch:`)."""
    try:
        for line in (ROOT / "profiles" / name).read_text().splitlines():
            if line.strip().startswith("traffic_bytes_per_launch:"):
                return int(line.split(":", 1)[1].strip())
    except OSError:
        pass
    return None


def _events(torch):
    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def time_gemm_roofline(torch, ctx, peaks, M, N, K, reps=20):
    """Average duration of the decode-batch linear (nmx_op_qmatmul_records
    with M rows: the tcgen05 decode-batch GEMM) at one shape, rotating over
    `copies` weight copies so no launch finds its weights in L2. CUDA events
    on the library's stream."""
    wbytes = N * K * 9 // 16
    copies = max(3, 300_000_000 // wbytes + 1)  # together well above the 126 MB L2
    wf = torch.randn((N, K), device="cuda", dtype=torch.float32) * 0.02
    recs = []
    for _ in range(copies):
        wq, sc, bi = ctx.quantize(wf, 64, 4)
        recs.append(ctx.pack_records(wq, sc, bi))
        del wq, sc, bi
    del wf
    x = torch.randn((M, K), device="cuda", dtype=torch.float16)
    y = torch.empty((M, N), device="cuda", dtype=torch.float16)
    for i in range(5):
        ctx.quantized_matmul_records(x, recs[i % copies], N, out=y)
    torch.cuda.synchronize()
    e0, e1 = _events(torch)
    e0.record()
    for i in range(reps):
        ctx.quantized_matmul_records(x, recs[i % copies], N, out=y)
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / reps
    nbytes = N * K // 2 + 2 * N * (K // 64) * 2 + M * K * 2 + M * N * 2
    ach = nbytes / (us * 1e-6) / 1e9
    return {"bound": "hbm", "achieved": round(ach, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
            "frac": round(ach / peaks["hbm_gbs"], 4), "traffic": None,
            "kernel": f"qgemm_tcs_kernel (decode-batch linear, M={M}, N={N}, K={K}, 4-bit g64)",
            "bytes_per_launch": nbytes, "us_per_launch": round(us, 2),
            "peak_source": f"{peaks['source']} (MEASURED_PEAKS.json hbm_gbs)"}


def time_attention_roofline(torch, ctx, peaks, B, Hq, Hkv, L, reps=20):
    """Average duration of the paged decode attention (nmx_op_attn_paged_decode)
    for B rows at context L, over two page sets (each larger than L2)."""
    D, BT = 128, 16
    nblk = (L + BT - 1) // BT
    sets = max(2, 300_000_000 // (2 * B * nblk * Hkv * BT * D * 2) + 1)  # together well above L2
    kc = torch.empty((sets * B * nblk, Hkv, BT, D), device="cuda", dtype=torch.float16).normal_()
    vc = torch.empty_like(kc).normal_()
    q = torch.randn((B, Hq, D), device="cuda", dtype=torch.float16)
    lens = torch.full((B,), L, dtype=torch.int32, device="cuda")
    tables = [torch.arange(s * B * nblk, (s + 1) * B * nblk, dtype=torch.int32, device="cuda").view(B, nblk)
              for s in range(sets)]
    for i in range(4):
        ctx.paged_decode_attention(q, kc, vc, tables[i % sets], lens, Hkv, D ** -0.5)
    torch.cuda.synchronize()
    e0, e1 = _events(torch)
    e0.record()
    for i in range(reps):
        ctx.paged_decode_attention(q, kc, vc, tables[i % sets], lens, Hkv, D ** -0.5)
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / reps
    nbytes = 2 * B * L * Hkv * D * 2 + 2 * B * Hq * D * 2
    ach = nbytes / (us * 1e-6) / 1e9
    del kc, vc
    return {"bound": "hbm", "achieved": round(ach, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
            "frac": round(ach / peaks["hbm_gbs"], 4),
            "kernel": f"paged_decode_mma_kernel (B={B}, {Hq}/{Hkv} heads of 128, context {L})",
            "bytes_per_launch": nbytes, "us_per_launch": round(us, 2)}


def time_c1(torch, ctx, peaks, copies=32, reps=64):
    """C1: x f16[4,4096] · Q4g64 W[4096,4096]^T (nmx_op_qmatmul, MLX layout)
    over 32 rotating W copies (> L2). The `reps` calls are captured once in a
    CUDA graph and the graph is timed, so host dispatch is not in the number."""
    wf = torch.randn((4096, 4096), device="cuda", dtype=torch.float32) * 0.02
    ws = [ctx.quantize(wf, 64, 4) for _ in range(copies)]
    x = torch.randn((4, 4096), device="cuda", dtype=torch.float16)
    y = torch.empty((4, 4096), device="cuda", dtype=torch.float16)
    for i in range(copies):
        ctx.quantized_matmul(x, *ws[i], out=y)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=ctx.stream):
        for i in range(reps):
            ctx.quantized_matmul(x, *ws[i % copies], out=y)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = _events(torch)
    e0.record()
    for _ in range(4):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / (4 * reps)
    # the same calls issued one by one from Python (the op-level API a host calls)
    e0.record()
    for i in range(reps):
        ctx.quantized_matmul(x, *ws[i % copies], out=y)
    e1.record()
    torch.cuda.synchronize()
    us_eager = e0.elapsed_time(e1) * 1000.0 / reps
    del g
    nbytes = 9_502_720
    ach = nbytes / (us * 1e-6) / 1e9
    return {"us_per_call": round(us, 2), "achieved_gbs": round(ach, 1),
            "frac_of_measured_hbm": round(ach / peaks["hbm_gbs"], 4), "bytes_per_call": nbytes,
            "timing": f"CUDA graph of {reps} calls over {copies} weight copies",
            "us_per_call_python_dispatch": round(us_eager, 2)}


def _barrier(dist):
    if dist is not None:
        dist.barrier()


def _max_over_ranks(torch, dist, v: float) -> float:
    if dist is None:
        return v
    t = torch.tensor([v], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def run_c4(args, rank, world, dist, torch, nmx, ctx, peaks, dev, clk_box):
    """The headline: Qwen2.5-32B-style decode, batch 32 at context 8192,
    tensor-parallel over the ranks."""
    cfg = nmx.qwen25_32b(max_batch=C4_BATCH, max_tokens=C4_PREFILL)
    local = nmx.tp_config(cfg, world) if world > 1 else cfg
    m = nmx.Model(ctx, local)
    m.init_random(seed=rank, std=0.02)
    comm = None
    if world > 1:
        comm = nmx.tp_comm(ctx, rank, world, cfg.max_tokens * cfg.hidden * 2, nmx.torch_exchange(dist))
        m.set_comm(comm)
    nblk = (C4_CTX + C4_GEN + 15) // 16 + 1
    pblk = C4_PREFILL // 16 + 1
    pool = nmx.KVPool(m, C4_BATCH * nblk + pblk + 2)
    pool.fill_random(seed=7 + rank, std=1.0)
    tables = np.arange(1, C4_BATCH * nblk + 1, dtype=np.int32).reshape(C4_BATCH, nblk)
    first = np.random.default_rng(0).integers(0, cfg.vocab, C4_BATCH).astype(np.int32)
    start = [C4_CTX] * C4_BATCH

    def step():
        m.decode_greedy(pool, first, start, tables, C4_GEN, want_ids=False)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    launches0 = ctx.launches
    e0, e1 = _events(torch)
    with clk_box(dev) as clk:
        _barrier(dist)
        torch.cuda.synchronize()
        e0.record()
        torch.cuda.nvtx.range_push("timed")  # lets a profiler capture only the timed steps
        for _ in range(args.steps):
            step()
        torch.cuda.nvtx.range_pop()
        e1.record()
        torch.cuda.synchronize()
        _barrier(dist)
    ms = _max_over_ranks(torch, dist, e0.elapsed_time(e1))
    launches = ctx.launches - launches0
    tokens = args.steps * C4_GEN * C4_BATCH
    value = tokens / (ms / 1000.0)
    out = {"value": value, "ms": ms, "launches": launches, "clocks": clk.summary()}

    # end to end through the host-facing forward: one call per decode step
    # (32 sequences), host token ids in, host ids out
    def fwd(toks, s):
        return m.forward(pool, [dict(tokens=[int(toks[b])], start_pos=C4_CTX + s, block_table=tables[b])
                                for b in range(C4_BATCH)])
    cur = first.copy()
    for s in range(3):
        cur = fwd(cur, s)
    e2e_steps = max(1, min(args.steps, 3))
    _barrier(dist)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        cur = first.copy()
        for s in range(C4_GEN):
            cur = fwd(cur, s)
    e2e_s = _max_over_ranks(torch, dist, time.perf_counter() - t0)
    out["e2e"] = {"value": round(e2e_steps * C4_GEN * C4_BATCH / e2e_s, 2), "unit": "tok/s",
                  "h2d_bytes_per_step": C4_GEN * (C4_BATCH * 16 + C4_BATCH * nblk * 4),
                  "d2h_bytes_per_step": C4_GEN * C4_BATCH * 4,
                  "call": "nmx_forward, one call per decode step of the 32 sequences, host ids in / host ids out"}

    # one 8192-token prefill of a single sequence (the workload's prefill)
    ptab = np.arange(C4_BATCH * nblk + 1, C4_BATCH * nblk + 1 + pblk, dtype=np.int32)
    ptoks = np.random.default_rng(1).integers(0, cfg.vocab, C4_PREFILL)
    m.forward(pool, [dict(tokens=ptoks[:1024], start_pos=0, block_table=ptab)])  # warm
    _barrier(dist)
    torch.cuda.synchronize()
    e0.record()
    m.forward(pool, [dict(tokens=ptoks, start_pos=0, block_table=ptab)])
    e1.record()
    torch.cuda.synchronize()
    pms = _max_over_ranks(torch, dist, e0.elapsed_time(e1))
    lin_params = (64 * (5120 * (5120 + 2 * 1024) + 5120 * 5120 + 3 * 5120 * 27648))
    flop = 2.0 * C4_PREFILL * lin_params + 64 * 2 * 40 * 128 * C4_PREFILL ** 2
    out["prefill"] = {"tokens": C4_PREFILL, "ms": round(pms, 2), "tflops": round(flop / (pms * 1e-3) / 1e12, 1),
                      "flop": flop, "peak_tflops": peaks["bf16_tflops"] * world,
                      "frac_of_measured_bf16": round(flop / (pms * 1e-3) / 1e12 / (peaks["bf16_tflops"] * world), 4),
                      "note": "whole prompt in one nmx_forward, host call included"}

    # the same decode over 4-bit KV pages (groups of 64 along head_dim): the
    # quantized-KV path, pages filled with seeded random records
    pool.close()
    qpool = nmx.KVPool(m, C4_BATCH * nblk + 2, kv_bits=4, kv_group_size=64)
    qpool.fill_random(seed=11 + rank, std=1.0)
    m.decode_greedy(qpool, first, start, tables, 2, want_ids=False)
    _barrier(dist)
    torch.cuda.synchronize()
    e0.record()
    for _ in range(args.steps):
        m.decode_greedy(qpool, first, start, tables, C4_GEN, want_ids=False)
    e1.record()
    torch.cuda.synchronize()
    qms = _max_over_ranks(torch, dist, e0.elapsed_time(e1))
    out["kv4"] = {"value": round(args.steps * C4_GEN * C4_BATCH / (qms / 1000.0), 2), "unit": "tok/s",
                  "ms_per_step": round(qms / args.steps, 3), "kv_bits": 4, "kv_group_size": 64,
                  "kv_bytes_per_token_per_rank": qpool.bytes_per_token,
                  "note": "same decode, K/V pages quantized on append and dequantized in the attention kernel"}
    qpool.close()

    # the exchange per call vs an NCCL all-reduce of the same 32 x 5120 f16
    if world > 1:
        part = torch.randn((C4_BATCH, cfg.hidden), device="cuda", dtype=torch.float16)
        res = torch.zeros_like(part)
        o = torch.empty_like(part)
        reps = 200

        def per_call_us(fn, stream):
            # device time per call: the calls replayed from one CUDA graph
            # (as in the decode step), so host launch cost is not measured
            with torch.cuda.stream(stream):
                for _ in range(10):
                    fn()
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for _ in range(reps):
                    fn()
            torch.cuda.synchronize()
            _barrier(dist)
            with torch.cuda.stream(stream):
                g.replay()
                torch.cuda.synchronize()
                _barrier(dist)
                e0.record(stream)
                g.replay()
                e1.record(stream)
            torch.cuda.synchronize()
            t = e0.elapsed_time(e1) * 1000.0 / reps
            del g
            return _max_over_ranks(torch, dist, t)

        ours_us = per_call_us(lambda: comm.allreduce_resid(part, res, o), ctx.stream)
        nc = part.clone()
        nccl_us = per_call_us(lambda: dist.all_reduce(nc), torch.cuda.Stream())
        out["exchange"] = {"bytes": C4_BATCH * cfg.hidden * 2, "ours_us_per_call": round(ours_us, 2),
                           "nccl_allreduce_us_per_call": round(nccl_us, 2), "calls_per_step_token": 128,
                           "ours_share_estimate": round(128 * C4_GEN * args.steps * ours_us / 1000.0 / ms, 4),
                           "kernel": "allreduce_resid_kernel (peer loads, rank-ordered sum + residual)"}
        m.set_comm(None)
        comm.close()

    # rooflines of the step's two dominant kernels at this rank's shapes
    H, F = cfg.hidden, cfg.ffn // world
    out["roofline_gemm"] = time_gemm_roofline(torch, ctx, peaks, C4_BATCH, 2 * F, H)
    out["roofline_attention"] = time_attention_roofline(torch, ctx, peaks, C4_BATCH, 40 // world, 8 // world,
                                                        C4_CTX + 1)
    out["weight_bytes_per_rank"] = m.step_weight_bytes
    out["kv_bytes_per_token_per_rank"] = m.kv_bytes_per_token
    m.close()
    return out


def run_c2(args, torch, nmx, ctx, peaks):
    """The Llama-3.1-8B batch-1 decode: prompt 2048 prefilled once, then
    steps of 256 greedy tokens from position 2048."""
    cfg = nmx.llama31_8b(max_batch=1, max_tokens=PROMPT)
    model = nmx.Model(ctx, cfg)
    model.init_random(seed=0, std=0.02)
    nblk = (PROMPT + GEN + 15) // 16
    pool = nmx.KVPool(model, nblk + 8)
    table = np.arange(nblk, dtype=np.int32)
    prompt = np.random.default_rng(0).integers(0, cfg.vocab, PROMPT)
    first = int(model.forward(pool, [dict(tokens=prompt, start_pos=0, block_table=table)])[0])

    def step(want_ids=False):
        return model.decode_greedy(pool, [first], [PROMPT], table[None], GEN, want_ids=want_ids)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    steps = max(args.steps, 3)
    e0, e1 = _events(torch)
    e0.record()
    for _ in range(steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    value = steps * GEN / (ms / 1000.0)
    ids = step(want_ids=True)[:, 0]
    cur = first
    for _ in range(8):
        model.forward(pool, [dict(tokens=[cur], start_pos=PROMPT, block_table=table)])
    t0 = time.perf_counter()
    for i in range(GEN):
        cur = int(model.forward(pool, [dict(tokens=[cur], start_pos=PROMPT + i, block_table=table)])[0])
    e2e = GEN / (time.perf_counter() - t0)
    step_bytes = model.step_weight_bytes + model.kv_bytes_per_token * (PROMPT + GEN // 2)
    gbs = step_bytes * value / 1e9
    roof = time_gemv_roofline(torch, nmx, ctx, peaks)
    roof["traffic"] = profiled_traffic("qgemv_dl_m1_n28672_k4096.md")
    model.close()
    pool.close()
    return {"workload": "Llama-3.1-8B architecture, 4-bit g64, batch 1, prompt 2048, 256 greedy tokens per step",
            "value": round(value, 2), "unit": "tok/s", "ms_per_step": round(ms / steps, 3), "steps": steps,
            "e2e": {"value": round(e2e, 2), "unit": "tok/s", "call": "nmx_forward, one call per token"},
            "step_roofline": {"bytes_per_token": step_bytes, "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"],
                              "unit": "GB/s", "frac": round(gbs / peaks["hbm_gbs"], 4)},
            "roofline": roof, "sample_ids": [int(i) for i in ids[:8]]}


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
    c4 = run_c4(args, rank, world, dist, torch, nmx, ctx, peaks, dev, Clocks)
    torch.cuda.empty_cache()
    extra = {}
    if world == 1 and not args.headline_only:
        from novamlx_b200 import microbench as mb
        extra["c2_decode"] = run_c2(args, torch, nmx, ctx, peaks)
        extra["c1_qmatmul"] = time_c1(torch, ctx, peaks)
        torch.cuda.empty_cache()
        extra["c3_serve"] = mb.serve(ctx, torch, nmx, 32, 64, 256, 4096, 512)
        torch.cuda.empty_cache()
        extra["c5_spec"] = mb.spec(ctx, torch, nmx, 16, 4096, 4, 8, 80, 16, False)
        torch.cuda.empty_cache()
    if rank != 0:
        return
    cpu = None
    if world == 1 and not args.no_cpu:
        c = CpuC4()
        sec = c.step_seconds()
        cpu = {"value": round(C4_BATCH / sec, 4), "unit": "tok/s", "cores": c.cores, "kind": "port",
               "sample": c.sample_text()}
    per_rank_bytes = c4["weight_bytes_per_rank"] + c4["kv_bytes_per_token_per_rank"] * C4_BATCH * (C4_CTX + C4_GEN // 2)
    step_tok_s = c4["value"] / C4_BATCH  # decode steps per second (each step reads every rank's bytes once)
    gbs = per_rank_bytes * step_tok_s / 1e9
    roof = dict(c4["roofline_gemm"])
    roof["traffic"] = profiled_traffic(f"qgemm_tcs_m32_n{roof['kernel'].split('N=')[1].split(',')[0]}_k5120.md")
    line = {
        "metric": METRIC, "value": round(c4["value"], 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(c4["ms"] / args.steps, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {"workload": WORKLOAD, "global_batch": C4_BATCH, "seq_len": C4_CTX,
                   "parallelism": f"tp{world}" if world > 1 else "tp1",
                   "tokens_per_step": C4_GEN * C4_BATCH,
                   "l2": "inputs larger than L2: every step reads each rank's weights and 32 x 8192 positions of KV"},
        "roofline": roof,
        "roofline_attention": c4["roofline_attention"],
        "step_roofline": {"bytes_per_rank_per_decode_step": per_rank_bytes, "achieved": round(gbs, 1),
                          "peak": peaks["hbm_gbs"], "unit": "GB/s (per GPU)", "frac": round(gbs / peaks["hbm_gbs"], 4)},
        "prefill_8192": c4["prefill"],
        "kv4_decode": c4["kv4"],
        "cpu_baseline": cpu,
        "e2e": c4["e2e"],
        "gpu_launches": c4["launches"],
        "clocks": c4["clocks"],
    }
    if "exchange" in c4:
        line["exchange"] = c4["exchange"]
    line.update(extra)
    print(json.dumps(line), flush=True)


def main():
    global C4_GEN
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--headline-only", action="store_true", help="skip the secondary workloads")
    ap.add_argument("--c4-gen", type=int, default=C4_GEN, help="decode tokens per sequence per step (profiling)")
    args = ap.parse_args()
    C4_GEN = args.c4_gen
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
