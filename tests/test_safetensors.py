"""safetensors on the host side of the ABI: the reader against an
independent writer (json + struct), the writer against an independent
reader, the header checks of SafetensorsHeader.swift:12-31; on the GPU, an
MLX checkpoint file loads into the model exactly as load_tensor does (whole,
or as a tensor-parallel rank's shard), and prefix blocks saved in the SSD
store's format (SSDCacheStore.swift:132-135,194-269) reload into other pages
with identical K/V."""
import json
import struct

import numpy as np
import pytest


@pytest.fixture(scope="module")
def nmx():
    from novamlx_b200 import nmx as mod
    return mod


def write_plain(path, tensors, meta=None):
    """an independent safetensors writer"""
    hdr, off, blobs = {}, 0, []
    if meta:
        hdr["__metadata__"] = meta
    for name, (dt, arr) in tensors.items():
        b = np.ascontiguousarray(arr).tobytes()
        hdr[name] = {"dtype": dt, "shape": list(arr.shape), "data_offsets": [off, off + len(b)]}
        off += len(b)
        blobs.append(b)
    h = json.dumps(hdr).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def read_plain(path):
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        hdr = json.loads(f.read(n))
        data = f.read()
    return hdr, data


def test_reader_reads_independent_file(nmx, tmp_path):
    rng = np.random.default_rng(0)
    t = {"a.weight": ("U32", rng.integers(0, 2**32, (4, 6), dtype=np.uint32)),
         "a.scales": ("F16", rng.standard_normal((4, 3)).astype(np.float16)),
         "b": ("F32", rng.standard_normal(5).astype(np.float32)),
         "eé\"q": ("I32", np.arange(3, dtype=np.int32))}
    p = str(tmp_path / "x.safetensors")
    write_plain(p, t, {"format": "mlx", "note": "a \"quoted\" value"})
    f = nmx.SafetensorsFile(p)
    info = f.tensors()
    assert set(info) == set(t)
    for k, (dt, arr) in t.items():
        assert info[k][0] == dt and info[k][1] == arr.shape
        assert np.array_equal(f.read(k), arr)
    assert f.metadata("format") == "mlx" and f.metadata("note") == 'a "quoted" value'
    assert f.metadata("missing") is None


def test_writer_read_by_independent_reader(nmx, tmp_path):
    rng = np.random.default_rng(1)
    t = {"0.0": rng.standard_normal((1, 2, 16, 8)).astype(np.float16), "x": np.arange(10, dtype=np.uint32)}
    p = str(tmp_path / "y.safetensors")
    nmx.safetensors_write(p, t, {"num_layers": "1", "k\n": "v\t"})
    hdr, data = read_plain(p)
    assert hdr["__metadata__"] == {"num_layers": "1", "k\n": "v\t"}
    for k, a in t.items():
        b, e = hdr[k]["data_offsets"]
        assert hdr[k]["shape"] == list(a.shape)
        assert np.array_equal(np.frombuffer(data[b:e], dtype=a.dtype).reshape(a.shape), a)


def test_header_checks(nmx, tmp_path):
    p = tmp_path / "bad.safetensors"
    p.write_bytes(struct.pack("<Q", 0))
    with pytest.raises(nmx.NmxError):
        nmx.SafetensorsFile(str(p))
    p.write_bytes(struct.pack("<Q", 32 << 20) + b"{}")
    with pytest.raises(nmx.NmxError):
        nmx.SafetensorsFile(str(p))
    h = json.dumps({"t": {"dtype": "F16", "shape": [4], "data_offsets": [0, 6]}}).encode()
    p.write_bytes(struct.pack("<Q", len(h)) + h + b"\0" * 8)
    with pytest.raises(nmx.NmxError):  # offsets disagree with the shape
        nmx.SafetensorsFile(str(p))
    with pytest.raises(nmx.NmxError):
        nmx.SafetensorsFile(str(tmp_path / "absent.safetensors"))


def _tiny():
    return dict(vocab=1024, hidden=512, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=128, ffn=1536,
                qkv_bias=True, rope_theta=1e6, rms_eps=1e-6)


def _checkpoint(tmp_path, nmx):
    from oracle import oracle as O
    d = _tiny()
    tensors = O.random_tensors(O.TinyCfg(**d), seed=9, std=0.05)
    dts = {k: ("U32" if v.dtype == np.uint32 else "F16") for k, v in tensors.items()}
    arrs = {k: (v.view(np.float16) if v.dtype == np.uint16 else v) for k, v in tensors.items()}
    p = str(tmp_path / "model.safetensors")
    nmx.safetensors_write(p, arrs, {"format": "mlx"}, dtypes=dts)
    return d, tensors, p


@pytest.mark.gpu
def test_model_loads_checkpoint_file(nmx, tmp_path):
    d, tensors, p = _checkpoint(tmp_path, nmx)
    ctx = nmx.Context(0)
    cfg = nmx.ModelConfig(**d, max_batch=4, max_tokens=128)
    a = nmx.Model(ctx, cfg)
    for k, v in tensors.items():
        a.load_tensor(k, v.view(np.float16) if v.dtype == np.uint16 else v)
    b = nmx.Model(ctx, cfg)
    loaded, skipped = nmx.load_safetensors(b, p)
    assert loaded == len(tensors) and skipped == 0
    prompt = np.random.default_rng(2).integers(0, 1024, 37)
    la = a.forward(nmx.KVPool(a, 8), [dict(tokens=prompt, start_pos=0, block_table=[1, 2, 3])], nmx.OUT_LOGITS_LAST)
    lb = b.forward(nmx.KVPool(b, 8), [dict(tokens=prompt, start_pos=0, block_table=[1, 2, 3])], nmx.OUT_LOGITS_LAST)
    assert np.array_equal(la, lb)


@pytest.mark.gpu
def test_checkpoint_shard_equals_host_shard(nmx, tmp_path):
    d, tensors, p = _checkpoint(tmp_path, nmx)
    ctx = nmx.Context(0)
    full = nmx.ModelConfig(**d, max_batch=4, max_tokens=128)
    for rank in range(2):
        m = nmx.Model(ctx, nmx.tp_config(full, 2))
        nmx.load_safetensors(m, p, rank, 2)
        ref = nmx.Model(ctx, nmx.tp_config(full, 2))
        for k, v in nmx.tp_shard(tensors, full, rank, 2).items():
            ref.load_tensor(k, v.view(np.float16) if v.dtype == np.uint16 else v)
        for name in ("model.layers.1.self_attn.q_proj.weight", "model.layers.0.self_attn.o_proj.weight",
                     "model.layers.1.mlp.down_proj.scales", "model.layers.0.self_attn.k_proj.bias"):
            sh = nmx.tp_shard(tensors, full, rank, 2)[name]
            got = m.get_tensor(name, sh.shape, sh.dtype)
            assert np.array_equal(got, sh), name
            assert np.array_equal(got, ref.get_tensor(name, sh.shape, sh.dtype)), name


@pytest.mark.gpu
def test_ssd_block_roundtrip(nmx, tmp_path):
    d, tensors, p = _checkpoint(tmp_path, nmx)
    ctx = nmx.Context(0)
    cfg = nmx.ModelConfig(**d, max_batch=4, max_tokens=128)
    m = nmx.Model(ctx, cfg)
    nmx.load_safetensors(m, p)
    pool = nmx.KVPool(m, 16)
    prompt = np.random.default_rng(3).integers(0, 1024, 48)
    m.forward(pool, [dict(tokens=prompt, start_pos=0, block_table=[1, 2, 3])])
    hashes = nmx.BlockHasher.compute_chain_hashes(prompt.tolist(), 16, "tiny")
    cache = str(tmp_path / "ssd")
    for i, h in enumerate(hashes):
        nmx.ssd_save_block(pool, 1 + i, h, 16, "tiny", cache)
    # the file layout and metadata of the reference store
    f = nmx.SafetensorsFile(f"{cache}/{hashes[0].hex()[0]}/{hashes[0].hex()}.safetensors")
    info = f.tensors()
    assert set(info) == {f"{l}.{j}" for l in range(2) for j in range(2)}
    assert info["1.0"][:2] == ("F16", (1, 2, 16, 128))
    assert f.metadata("block_hash") == hashes[0].hex() and f.metadata("num_layers") == "2"
    assert f.metadata("token_count") == "16" and f.metadata("model_name") == "tiny"
    assert json.loads(f.metadata("layer_cache_types")) == ["KVCacheSimple"] * 2
    # reload into other pages: the same K/V bytes, and decoding on them agrees
    for i, h in enumerate(hashes):
        assert nmx.ssd_load_block(pool, h, cache, 10 + i) == 16
    assert np.array_equal(pool.read_blocks([1, 2, 3]), pool.read_blocks([10, 11, 12]))
    tok = [int(prompt[-1])]
    x = m.forward(pool, [dict(tokens=tok, start_pos=48, block_table=[1, 2, 3, 4])], nmx.OUT_LOGITS_LAST)
    y = m.forward(pool, [dict(tokens=tok, start_pos=48, block_table=[10, 11, 12, 13])], nmx.OUT_LOGITS_LAST)
    assert np.array_equal(x, y)
