"""Python access to the CPU oracle (liboracle.so built from oracle/oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline legs, never by the product path. See oracle.c's
header for what is restated from where and the parity status.

Arrays: f16/bf16 values travel as raw uint16 numpy arrays; packed weights
as uint32.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from dataclasses import dataclass
from pathlib import Path
from typing import Optional

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"


def build() -> Path:
    src = HERE / "oracle.c"
    if not LIB.exists() or LIB.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-C", str(HERE), "-s"], check=True)
    return LIB


def _load():
    if not LIB.exists():
        build()
    return C.CDLL(str(LIB))


lib = _load()
_vp, _i, _f = C.c_void_p, C.c_int, C.c_float


def _p(fn, res, *args):
    f = getattr(lib, fn)
    f.restype = res
    f.argtypes = list(args)


_p("oracle_h2f", C.c_float, C.c_uint16)
_p("oracle_f2h", C.c_uint16, C.c_float)
_p("oracle_bf2f", C.c_float, C.c_uint16)
_p("oracle_f2bf", C.c_uint16, C.c_float)
_p("oracle_set_threads", None, _i)
_p("oracle_max_threads", _i)
_p("oracle_quantize", None, _vp, _i, _i, _i, _i, _i, _vp, _vp, _vp)
_p("oracle_unpack", None, _vp, _i, _i, _i, _vp)
_p("oracle_dequantize", None, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp)
_p("oracle_qmatmul", None, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _vp)
_p("oracle_rmsnorm", None, _vp, _vp, _i, _i, _f, _i, _vp)
_p("oracle_rope_inv_freq", None, _i, _f, _f, _f, _f, _i, _vp)
_p("oracle_rope", None, _vp, _i, _i, _i, _vp, _vp, _i)
_p("oracle_attention", None, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _f, _i, _vp)
_p("oracle_quantized_sdpa", None, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _f, _i, _i, _i, _vp)
_p("oracle_argmax", None, _vp, _i, _i, _i, _vp)
_p("oracle_penalized_argmax", None, _vp, _i, _i, _i, _vp, _vp, _i, _f, _vp)
_p("oracle_forward", _i, _vp, _vp, _vp, _i, _vp, _i, _i, _vp, _i)

F16, BF16, F32 = 0, 1, 2


def _c(a):
    return np.ascontiguousarray(a)


def f32_to_f16bits(a) -> np.ndarray:
    return np.asarray(a, dtype=np.float32).astype(np.float16).view(np.uint16)


def f16bits_to_f32(a) -> np.ndarray:
    return np.asarray(a, dtype=np.uint16).view(np.float16).astype(np.float32)


def bf16bits_to_f32(a) -> np.ndarray:
    return (np.asarray(a, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def to_f32(a, dt=F16) -> np.ndarray:
    return bf16bits_to_f32(a) if dt == BF16 else f16bits_to_f32(a)


def set_threads(n: int) -> None:
    lib.oracle_set_threads(n)


def max_threads() -> int:
    return lib.oracle_max_threads()


def quantize(w: np.ndarray, bits: int = 4, group_size: int = 64, sdt: int = F16):
    w = _c(np.asarray(w, dtype=np.float32))
    N, K = w.shape
    wq = np.empty((N, K * bits // 32), dtype=np.uint32)
    s = np.empty((N, K // group_size), dtype=np.uint16)
    b = np.empty_like(s)
    lib.oracle_quantize(w.ctypes.data, N, K, bits, group_size, sdt, wq.ctypes.data, s.ctypes.data, b.ctypes.data)
    return wq, s, b


def unpack(wq: np.ndarray, K: int, bits: int) -> np.ndarray:
    wq = _c(wq)
    q = np.empty((wq.shape[0], K), dtype=np.uint8)
    lib.oracle_unpack(wq.ctypes.data, wq.shape[0], K, bits, q.ctypes.data)
    return q


def dequantize(wq, s, b, bits=4, group_size=64, sdt=F16) -> np.ndarray:
    wq, s, b = _c(wq), _c(s), _c(b)
    N = wq.shape[0]
    K = wq.shape[1] * 32 // bits
    w = np.empty((N, K), dtype=np.float32)
    lib.oracle_dequantize(wq.ctypes.data, s.ctypes.data, b.ctypes.data, N, K, bits, group_size, sdt, w.ctypes.data)
    return w


def qmatmul(x: np.ndarray, wq, s, b, bits=4, group_size=64, dt=F16) -> np.ndarray:
    """x: uint16 [M, K] (f16/bf16 bits) → uint16 [M, N]."""
    x, wq, s, b = _c(x), _c(wq), _c(s), _c(b)
    M, K = x.shape
    N = wq.shape[0]
    y = np.empty((M, N), dtype=np.uint16)
    lib.oracle_qmatmul(x.ctypes.data, wq.ctypes.data, s.ctypes.data, b.ctypes.data, M, N, K, bits, group_size, dt,
                       y.ctypes.data)
    return y


def rmsnorm(x, g, eps=1e-5, dt=F16):
    x, g = _c(x), _c(g)
    M, H = x.shape
    y = np.empty_like(x)
    lib.oracle_rmsnorm(x.ctypes.data, g.ctypes.data, M, H, eps, dt, y.ctypes.data)
    return y


def rope_inv_freq(D, theta, factor=0.0, low=1.0, high=4.0, orig=8192) -> np.ndarray:
    out = np.empty(D // 2, dtype=np.float32)
    lib.oracle_rope_inv_freq(D, theta, factor, low, high, orig, out.ctypes.data)
    return out


def attention(q, k, v, Hq, Hkv, D, q_start, scale, dt=F16):
    """q [T, Hq, D], k/v [S, Hkv, D] as uint16 → uint16 [T, Hq, D]."""
    q, k, v = _c(q), _c(k), _c(v)
    T, S = q.shape[0], k.shape[0]
    out = np.empty_like(q)
    lib.oracle_attention(q.ctypes.data, k.ctypes.data, v.ctypes.data, T, Hq, Hkv, D, S, q_start, scale, dt,
                         out.ctypes.data)
    return out


def quantized_sdpa(q, kw, ks, kb, vw, vs, vb, gqa, scale, group_size, bits, dt=F16):
    """q [BH, L, D] uint16; kw/vw [BHkv, N, D*bits/32] uint32; scales/biases [BHkv, N, D/gs]."""
    q, kw, ks, kb, vw, vs, vb = map(_c, (q, kw, ks, kb, vw, vs, vb))
    BH, L, D = q.shape
    N = kw.shape[1]
    out = np.empty_like(q)
    lib.oracle_quantized_sdpa(q.ctypes.data, kw.ctypes.data, ks.ctypes.data, kb.ctypes.data, vw.ctypes.data,
                              vs.ctypes.data, vb.ctypes.data, BH, gqa, N, L, D, scale, group_size, bits, dt,
                              out.ctypes.data)
    return out


def argmax(logits, dt=F32) -> np.ndarray:
    logits = _c(logits)
    M, V = logits.shape
    out = np.empty(M, dtype=np.int32)
    lib.oracle_argmax(logits.ctypes.data, M, V, dt, out.ctypes.data)
    return out


def penalized_argmax(logits, recent, n_recent, penalty, dt=F32) -> np.ndarray:
    logits, recent, n_recent = _c(logits), _c(np.asarray(recent, np.int32)), _c(np.asarray(n_recent, np.int32))
    M, V = logits.shape
    out = np.empty(M, dtype=np.int32)
    lib.oracle_penalized_argmax(logits.ctypes.data, M, V, dt, recent.ctypes.data, n_recent.ctypes.data,
                                recent.shape[1], penalty, out.ctypes.data)
    return out


# ------------------------------------------------------------------ the model

class _CModel(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("vocab", "hidden", "n_layers", "n_heads", "n_kv_heads", "head_dim", "ffn",
                                        "bits", "gs", "dt", "qkv_bias", "tie")] + [("eps", C.c_float)] + \
               [(n, C.c_void_p) for n in (
                   "inv_freq", "embed", "final_norm", "lm_w", "lm_s", "lm_b", "attn_norm", "mlp_norm",
                   "q_w", "k_w", "v_w", "o_w", "g_w", "u_w", "d_w",
                   "q_s", "k_s", "v_s", "o_s", "g_s", "u_s", "d_s",
                   "q_b", "k_b", "v_b", "o_b", "g_b", "u_b", "d_b",
                   "q_bias", "k_bias", "v_bias")] + [("kv_bits", C.c_int), ("kv_gs", C.c_int)]


_LIN = {"q": "self_attn.q_proj", "k": "self_attn.k_proj", "v": "self_attn.v_proj", "o": "self_attn.o_proj",
        "g": "mlp.gate_proj", "u": "mlp.up_proj", "d": "mlp.down_proj"}


@dataclass
class TinyCfg:
    """Architecture fields the oracle needs (same meaning as nmx.ModelConfig)."""
    vocab: int
    hidden: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    ffn: int
    bits: int = 4
    group_size: int = 64
    qkv_bias: bool = False
    rms_eps: float = 1e-5
    rope_theta: float = 10000.0
    rope_factor: float = 0.0
    rope_low_freq_factor: float = 1.0
    rope_high_freq_factor: float = 4.0
    rope_original_max_pos: int = 8192
    kv_bits: int = 0      # quantized KV cache: 4 or 8 (0: f16 cache)
    kv_group_size: int = 64


class OracleModel:
    """A Llama/Qwen2 model held as MLX-named numpy tensors, run by oracle_forward."""

    def __init__(self, cfg, tensors: dict):
        self.cfg = cfg
        self.t = tensors
        c = cfg
        L = c.n_layers
        st = lambda key: _c(np.stack([tensors[f"model.layers.{i}.{key}"] for i in range(L)]))
        self._keep = {}
        m = _CModel()
        for k in ("vocab", "hidden", "n_layers", "n_heads", "n_kv_heads", "head_dim", "ffn", "bits"):
            setattr(m, k, int(getattr(c, k)))
        m.gs = int(c.group_size)
        m.dt = F16
        m.qkv_bias = int(bool(c.qkv_bias))
        m.tie = 0
        m.eps = float(c.rms_eps)
        m.kv_bits = int(getattr(c, "kv_bits", 0))
        m.kv_gs = int(getattr(c, "kv_group_size", 64))

        def keep(name, arr):
            arr = _c(arr)
            self._keep[name] = arr
            return arr.ctypes.data

        m.inv_freq = keep("inv_freq", rope_inv_freq(c.head_dim, c.rope_theta, c.rope_factor, c.rope_low_freq_factor,
                                                    c.rope_high_freq_factor, c.rope_original_max_pos))
        m.embed = keep("embed", tensors["model.embed_tokens.weight"])
        m.final_norm = keep("final_norm", tensors["model.norm.weight"])
        m.lm_w = keep("lm_w", tensors["lm_head.weight"])
        m.lm_s = keep("lm_s", tensors["lm_head.scales"])
        m.lm_b = keep("lm_b", tensors["lm_head.biases"])
        m.attn_norm = keep("attn_norm", st("input_layernorm.weight"))
        m.mlp_norm = keep("mlp_norm", st("post_attention_layernorm.weight"))
        for short, full in _LIN.items():
            setattr(m, f"{short}_w", keep(f"{short}_w", st(f"{full}.weight")))
            setattr(m, f"{short}_s", keep(f"{short}_s", st(f"{full}.scales")))
            setattr(m, f"{short}_b", keep(f"{short}_b", st(f"{full}.biases")))
        if c.qkv_bias:
            for short in ("q", "k", "v"):
                setattr(m, f"{short}_bias", keep(f"{short}_bias", st(f"{_LIN[short]}.bias")))
        self.m = m

    def new_cache(self, max_ctx: int):
        c = self.cfg
        shape = (c.n_layers, c.n_kv_heads, max_ctx, c.head_dim)
        return np.zeros(shape, np.uint16), np.zeros(shape, np.uint16), max_ctx

    def forward(self, cache, tokens, start_pos: int, all_logits: bool = False) -> np.ndarray:
        kc, vc, max_ctx = cache
        toks = _c(np.asarray(tokens, np.int32))
        T = len(toks)
        rows = T if all_logits else 1
        out = np.empty((rows, self.cfg.vocab), dtype=np.float32)
        rc = lib.oracle_forward(C.byref(self.m), kc.ctypes.data, vc.ctypes.data, max_ctx, toks.ctypes.data, T,
                                start_pos, out.ctypes.data, int(all_logits))
        if rc != 0:
            raise ValueError("oracle_forward: context overflow")
        return out


def random_tensors(cfg, seed: int = 0, std: float = 0.02) -> dict:
    """MLX-named tensors of a random-init model: linears N(0, std) quantized
    with the oracle's rule, embeddings N(0, std) f16, norms 1 + N(0, 0.1)."""
    rng = np.random.default_rng(seed)
    c = cfg
    H, F, V = c.hidden, c.ffn, c.vocab
    Nq, Nkv = c.n_heads * c.head_dim, c.n_kv_heads * c.head_dim
    t = {}

    def lin(name, N, K):
        w = (rng.standard_normal((N, K), dtype=np.float32) * std).astype(np.float32)
        wq, s, b = quantize(w, c.bits, c.group_size)
        t[f"{name}.weight"], t[f"{name}.scales"], t[f"{name}.biases"] = wq, s, b

    t["model.embed_tokens.weight"] = f32_to_f16bits(rng.standard_normal((V, H), dtype=np.float32) * std)
    t["model.norm.weight"] = f32_to_f16bits(1.0 + 0.1 * rng.standard_normal(H, dtype=np.float32))
    lin("lm_head", V, H)
    for i in range(c.n_layers):
        p = f"model.layers.{i}"
        t[f"{p}.input_layernorm.weight"] = f32_to_f16bits(1.0 + 0.1 * rng.standard_normal(H, dtype=np.float32))
        t[f"{p}.post_attention_layernorm.weight"] = f32_to_f16bits(
            1.0 + 0.1 * rng.standard_normal(H, dtype=np.float32))
        lin(f"{p}.self_attn.q_proj", Nq, H)
        lin(f"{p}.self_attn.k_proj", Nkv, H)
        lin(f"{p}.self_attn.v_proj", Nkv, H)
        lin(f"{p}.self_attn.o_proj", H, Nq)
        lin(f"{p}.mlp.gate_proj", F, H)
        lin(f"{p}.mlp.up_proj", F, H)
        lin(f"{p}.mlp.down_proj", H, F)
        if c.qkv_bias:
            for nm, n in (("q", Nq), ("k", Nkv), ("v", Nkv)):
                t[f"{p}.self_attn.{nm}_proj.bias"] = f32_to_f16bits(0.5 * rng.standard_normal(n, dtype=np.float32))
    return t


def cosine(a, b) -> float:
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-300))


def max_rel_err(y, r) -> float:
    """Normwise max relative error max|y - r| / max|r|."""
    y = np.asarray(y, np.float64)
    r = np.asarray(r, np.float64)
    return float(np.max(np.abs(y - r)) / max(np.max(np.abs(r)), 1e-30))
