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


@pytest.mark.parametrize("name", ["llama", "qwen", "llama8kv", "qwen8kv"])
@pytest.mark.parametrize("world", [2, 4, 8])
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
@pytest.mark.parametrize("world,name", [(2, "llama"), (2, "qwen"), (2, "qwen8kv"), (4, "llama8kv"),
                                        (4, "qwen8kv"), (8, "llama8kv"), (8, "qwen8kv")])
def test_tp_matches_oracle(nmx, tmp_path, world, name):
    """The sharded model on `world` GPUs against the oracle's unsharded
    forward: prefill and every greedy step's logits within the bars, every
    determined id equal (tests/parity.py), the same bits on every rank, the
    exchange fused into the decode-batch GEMM equal to GEMM + exchange
    kernel, and the op-level exchange exact on integers."""
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from oracle import oracle as O
    from parity import check_id, check_logits
    from tp_worker import GREEDY_STEPS, batch_inputs, prompts_of
    out = tmp_path / "tp"
    r = _torchrun(world, ROOT / "tests" / "tp_worker.py", "--model", name, "--out", str(out))
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    res = [np.load(f"{out}.rank{k}.npz") for k in range(world)]
    r0 = res[0]
    for rk in res:
        assert bool(rk["op_ok"])
        # every rank holds the same hidden states, hence the same bits
        for key in ("tp_logits", "tp_ids", "tp_step_logits", "tp_batch"):
            assert np.array_equal(rk[key], r0[key]), key
        # decode-batch GEMM with the exchange in its epilogue: the same bits
        # as GEMM + exchange kernel
        assert np.array_equal(rk["tp_batch"], rk["tp_batch_sep"])
    d = _tiny(nmx, name)
    cfg = nmx.ModelConfig(**d)
    om = O.OracleModel(O.TinyCfg(**d), O.random_tensors(O.TinyCfg(**d), seed=5, std=0.05))
    lens, prompts, _ = prompts_of(cfg, 11)
    determined = 0
    for i, (n, p) in enumerate(zip(lens, prompts)):
        cache = om.new_cache(128)
        ref = om.forward(cache, p, 0)
        err = check_logits(r0["tp_logits"][i], ref)
        determined += check_id(int(r0["tp_first"][i]), ref, err)
        tok = int(r0["tp_first"][i])
        for s in range(GREEDY_STEPS):
            ref = om.forward(cache, [tok], n + s)
            e = check_logits(r0["tp_step_logits"][s, i], ref)
            determined += check_id(int(r0["tp_ids"][s, i]), ref, max(e, err))
            tok = int(r0["tp_ids"][s, i])
    bp, btoks = batch_inputs(cfg, 12)
    for i, p in enumerate(bp):
        cache = om.new_cache(32)
        check_logits(r0["tp_batch"][i], om.forward(cache, p, 0))
        check_logits(r0["tp_batch"][12 + i], om.forward(cache, [int(btoks[i])], 8))
    print(f"tp{world} {name}: {determined}/{4 * (GREEDY_STEPS + 1)} ids determined and equal to the oracle's")


def test_lost_rank_detected_on_host_gloo():
    """A rank that leaves before the rendezvous: the other learns of it on
    the host (an error from the exchange), not by waiting for good."""
    r = _torchrun(2, ROOT / "tests" / "tp_failure_check.py", timeout=120)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert "rank 0 detected" in r.stdout, r.stdout[-2000:] + r.stderr[-2000:]


@pytest.mark.gpu
def test_exchange_wait_runs_out_with_timeout(tmp_path):
    """Two GPUs: one rank starts an exchange its peer never joins; with a
    short wait limit its kernel gives up, the host gets NMX_ERR_TIMEOUT,
    and the context still runs work (bounded form only: no fault, no
    spin without a limit)."""
    import json
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    out = tmp_path / "to"
    r = _torchrun(2, ROOT / "tests" / "tp_timeout_worker.py", "--out", str(out), timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    r0 = json.loads(open(f"{out}.rank0.json").read())
    r1 = json.loads(open(f"{out}.rank1.json").read())
    assert r0["together"] and r1["together"]
    assert r0["status"] == "timeout", r0
    assert "peer rank" in r0["message"]
    assert r0["usable_after"]
    assert r0["seconds"] < 30
