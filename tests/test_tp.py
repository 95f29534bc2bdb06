"""Tensor parallelism: the host-side sharding of MLX-layout tensors and the
rank rendezvous (CPU, gloo, world size 2), and on two GPUs the sharded model
with the peer-memory exchange against the unsharded model (same tiny
weights): logits within the workload tolerance, the same greedy ids, the
same bits on every rank, and the exchange op exact on integers."""
import os
import socket
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _torchrun(n, script, *args, timeout=600):
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()), str(script), *args]
    return subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=timeout)


@pytest.fixture(scope="module")
def nmx():
    from novamlx_b200 import nmx as mod
    return mod


def _tiny(nmx, name):
    sys.path.insert(0, str(ROOT / "tests"))
    from tp_worker import tiny
    return tiny(name)


@pytest.mark.parametrize("name", ["llama", "qwen"])
@pytest.mark.parametrize("world", [2, 4])
def test_shards_reassemble(nmx, name, world):
    from oracle import oracle as O
    d = _tiny(nmx, name)
    cfg = nmx.ModelConfig(**d)
    if cfg.n_kv_heads % world:
        pytest.skip("kv heads do not split")
    full = O.random_tensors(O.TinyCfg(**d), seed=3, std=0.05)
    shards = [nmx.tp_shard(full, cfg, r, world) for r in range(world)]
    for k, v in full.items():
        mod = k.split(".")[-2]
        if mod in ("q_proj", "k_proj", "v_proj", "gate_proj", "up_proj"):
            assert np.array_equal(np.concatenate([s[k] for s in shards], axis=0), v), k
        elif mod in ("o_proj", "down_proj"):
            assert np.array_equal(np.concatenate([s[k] for s in shards], axis=1), v), k
        else:
            assert all(s[k] is v for s in shards), k
    local = nmx.tp_config(cfg, world)
    assert local.n_heads * world == cfg.n_heads and local.ffn * world == cfg.ffn
    # the local shapes are what a model of the local config expects
    s0 = shards[0]
    nq = local.n_heads * local.head_dim
    assert s0[f"model.layers.0.self_attn.q_proj.weight"].shape == (nq, cfg.hidden * cfg.bits // 32)
    assert s0[f"model.layers.0.self_attn.o_proj.weight"].shape == (cfg.hidden, nq * cfg.bits // 32)
    assert s0[f"model.layers.0.mlp.down_proj.scales"].shape == (cfg.hidden, local.ffn // cfg.group_size)


def test_tp_config_rejects_uneven(nmx):
    cfg = nmx.ModelConfig(**_tiny(nmx, "llama"))
    with pytest.raises(ValueError):
        nmx.tp_config(cfg, 3)


def test_rendezvous_gloo_world2():
    r = _torchrun(2, ROOT / "tests" / "tp_exchange_check.py", timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert "rank 0 ok" in r.stdout and "rank 1 ok" in r.stdout


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["llama", "qwen"])
def test_tp2_matches_unsharded(nmx, tmp_path, name):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from oracle import oracle as O
    out = tmp_path / "tp"
    r = _torchrun(2, ROOT / "tests" / "tp_worker.py", "--model", name, "--out", str(out))
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    r0 = np.load(f"{out}.rank0.npz")
    r1 = np.load(f"{out}.rank1.npz")
    assert bool(r0["op_ok"]) and bool(r1["op_ok"])
    # every rank holds the same hidden states, hence the same bits
    assert np.array_equal(r0["tp_logits"], r1["tp_logits"])
    assert np.array_equal(r0["tp_ids"], r1["tp_ids"])
    for g, f in zip(r0["tp_logits"], r0["full_logits"]):
        assert O.cosine(g, f) >= 0.999
        assert O.max_rel_err(g, f) <= 2e-2
    assert np.array_equal(r0["tp_first"], r0["full_first"])
    agree = float(np.mean(r0["tp_ids"] == r0["full_ids"]))
    assert agree >= 0.9, agree
    # decode-batch GEMM with the exchange in its epilogue: the same bits as
    # GEMM + exchange kernel, the same bits on both ranks, close to unsharded
    assert np.array_equal(r0["tp_batch"], r0["tp_batch_sep"])
    assert np.array_equal(r0["tp_batch"], r1["tp_batch"])
    for g, f in zip(r0["tp_batch"], r0["full_batch"]):
        assert O.cosine(g, f) >= 0.999
        assert O.max_rel_err(g, f) <= 2e-2
