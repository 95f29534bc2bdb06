"""ctypes binding of libnovamlx_cuda.so (the C ABI in include/nmx.h).

This is the host-side mirror of the engine-facing interface: the names follow
the reference's Swift API where one exists (MLX.quantizedMM →
``quantized_matmul``, FusedQuantizedSDPA.attention → ``fused_quantized_sdpa``,
BlockHasher / PagedBlockPool → the classes of the same names, the model's
``callAsFunction(tokens, cache:)`` → ``Model.forward``). Device tensors are
passed as torch CUDA tensors (torch is only used for device memory here);
everything else is plain Python / numpy.

There is no CPU fallback: if the shared library is missing, importing this
module raises.
"""
from __future__ import annotations

import ctypes as C
import os
import sys
from dataclasses import dataclass, field
from pathlib import Path
from typing import Optional, Sequence

import numpy as np

_LIB_PATH = Path(__file__).resolve().parent / "libnovamlx_cuda.so"

NMX_OK, NMX_ERR_INVALID, NMX_ERR_UNSUPPORTED, NMX_ERR_CUDA, NMX_ERR_OOM, NMX_ERR_TIMEOUT, NMX_ERR_STATE, \
    NMX_ERR_NOT_FOUND = range(8)
F16, BF16, F32, U32, I32 = range(5)
OUT_ARGMAX_LAST, OUT_LOGITS_LAST, OUT_ARGMAX_ALL, OUT_LOGITS_ALL = range(4)


class NmxError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"nmx status {status}: {msg}")
        self.status = status


def _load() -> C.CDLL:
    if not _LIB_PATH.exists():
        raise ImportError(f"{_LIB_PATH} is missing; build it with `python -m novamlx_b200.build`")
    return C.CDLL(str(_LIB_PATH))


lib = _load()

_vp, _i, _u64, _f, _sz = C.c_void_p, C.c_int, C.c_uint64, C.c_float, C.c_size_t
_ip = C.POINTER(C.c_int32)
_u8p = C.POINTER(C.c_uint8)


class ModelCfg(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("vocab", "hidden", "n_layers", "n_heads", "n_kv_heads", "head_dim", "ffn",
                                        "bits", "group_size", "dtype", "qkv_bias", "tie_embeddings")] + \
               [("rms_eps", C.c_float), ("rope_theta", C.c_float), ("rope_factor", C.c_float),
                ("rope_low_freq_factor", C.c_float), ("rope_high_freq_factor", C.c_float),
                ("rope_original_max_pos", C.c_int), ("max_batch", C.c_int), ("max_tokens", C.c_int)]


class Seq(C.Structure):
    _fields_ = [("n_new_tokens", C.c_int), ("token_ids", _ip), ("start_pos", C.c_int),
                ("block_table", _ip), ("n_blocks", C.c_int)]


def _proto(name, res, *args):
    fn = getattr(lib, name)
    fn.restype = res
    fn.argtypes = list(args)
    return fn


_proto("nmx_last_error", C.c_char_p)
_proto("nmx_version", C.c_char_p)
_proto("nmx_ctx_create", _i, _i, C.POINTER(_vp))
_proto("nmx_ctx_destroy", _i, _vp)
_proto("nmx_ctx_set_stream", _i, _vp, _vp)
_proto("nmx_ctx_stream", _vp, _vp)
_proto("nmx_ctx_synchronize", _i, _vp)
_proto("nmx_ctx_kernel_launches", _u64, _vp)
_proto("nmx_ctx_set_wait_limit", _i, _vp, C.c_uint32)
_proto("nmx_op_qmatmul", _i, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _vp)
_proto("nmx_op_pack_records", _i, _vp, _vp, _vp, _vp, _i, _i, _vp)
_proto("nmx_op_qmatmul_records", _i, _vp, _vp, _vp, _i, _i, _i, _vp)
_proto("nmx_op_quantize", _i, _vp, _vp, _i, _i, _i, _i, _i, _vp, _vp, _vp)
_proto("nmx_op_dequantize", _i, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp)
_proto("nmx_op_rmsnorm", _i, _vp, _vp, _vp, _i, _i, _f, _i, _vp)
_proto("nmx_op_argmax", _i, _vp, _vp, _i, _i, _i, _vp)
_proto("nmx_op_penalized_argmax", _i, _vp, _vp, _i, _i, _i, _vp, _vp, _i, _f, _vp)
_proto("nmx_op_attn_quantized_decode", _i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _f,
       _i, _i, _i, _i, _vp)
_proto("nmx_op_attn_paged_decode", _i, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _f, _vp)
_proto("nmx_op_attn_paged_decode_noalloc", _i, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _f, _vp)
_proto("nmx_model_create", _i, _vp, C.POINTER(ModelCfg), C.POINTER(_vp))
_proto("nmx_model_destroy", _i, _vp)
_proto("nmx_model_init_random", _i, _vp, _u64, _f)
_proto("nmx_model_load_tensor", _i, _vp, C.c_char_p, _vp, _i, C.POINTER(C.c_int64), _i)
_proto("nmx_model_get_tensor", _i, _vp, C.c_char_p, _vp, _sz)
_proto("nmx_model_weight_bytes", _u64, _vp)
_proto("nmx_model_step_weight_bytes", _u64, _vp)
_proto("nmx_kv_pool_create", _i, _vp, _i, _i, C.POINTER(_vp))
_proto("nmx_kv_pool_destroy", _i, _vp)
_proto("nmx_kv_copy_blocks", _i, _vp, _ip, _ip, _i)
_proto("nmx_kv_read_blocks", _i, _vp, _ip, _i, _vp)
_proto("nmx_kv_write_blocks", _i, _vp, _ip, _i, _vp)
_proto("nmx_kv_pool_layer_ptrs", _i, _vp, _i, C.POINTER(_vp), C.POINTER(_vp))
_proto("nmx_kv_pool_num_blocks", _i, _vp)
_proto("nmx_kv_pool_fill_random", _i, _vp, _u64, C.c_float)
_proto("nmx_kv_pool_create_quantized", _i, _vp, _i, _i, _i, _i, C.POINTER(_vp))
_proto("nmx_kv_pool_bytes_per_token", _u64, _vp)
_proto("nmx_kv_bytes_per_token", _u64, _vp)
_proto("nmx_forward", _i, _vp, _vp, C.POINTER(Seq), _i, _i, _vp)
_proto("nmx_decode_greedy", _i, _vp, _vp, _ip, _ip, _ip, _i, _i, _i, _ip)
_proto("nmx_block_hash", None, _u8p, _ip, _i, C.c_char_p, _u8p)
_proto("nmx_chain_hashes", _i, _ip, _i, _i, C.c_char_p, _u8p, _i)
_proto("nmx_block_pool_create", _i, _i, _i, _i, C.c_char_p, C.POINTER(_vp))


class SchedCfg(C.Structure):
    _fields_ = [("max_batch", C.c_int), ("max_step_tokens", C.c_int), ("prefill_chunk", C.c_int),
                ("max_concurrent", C.c_int), ("headroom_percent", C.c_int), ("kv_budget_bytes", C.c_uint64),
                ("model_name", C.c_char_p)]


class SchedStats(C.Structure):
    _fields_ = [("steps", C.c_uint64), ("generated", C.c_uint64), ("finished", C.c_uint64),
                ("preemptions", C.c_uint64), ("prefix_hit_tokens", C.c_uint64), ("tokens_in_steps", C.c_uint64),
                ("running", C.c_int), ("waiting", C.c_int), ("blocks_in_use", C.c_int),
                ("logical_blocks", C.c_uint64), ("kv_available_bytes", C.c_uint64)]


_proto("nmx_budget_create", _i, C.c_uint64, _i, C.POINTER(_vp))
_proto("nmx_budget_destroy", None, _vp)
_proto("nmx_budget_add_weights", None, _vp, C.c_uint64)
_proto("nmx_budget_can_admit", _i, _vp, C.c_uint64, C.c_uint64)
_proto("nmx_budget_reserve", None, _vp, C.c_int64, C.c_uint64, C.c_uint64)
_proto("nmx_budget_release", None, _vp, C.c_int64)
_proto("nmx_budget_available", C.c_uint64, _vp)
_proto("nmx_sched_create", _i, _vp, _vp, C.POINTER(SchedCfg), C.POINTER(_vp))
_proto("nmx_sched_destroy", None, _vp)
_proto("nmx_sched_submit", _i, _vp, _vp, _i, _i, _i, C.POINTER(C.c_int64))
_proto("nmx_sched_step", _i, _vp, C.POINTER(C.c_int))
_proto("nmx_sched_poll", _i, _vp, C.c_int64, _vp, _i, C.POINTER(C.c_int), C.POINTER(C.c_int))
_proto("nmx_sched_stats", _i, _vp, C.POINTER(SchedStats))
REQ_WAITING, REQ_PREFILL, REQ_DECODE, REQ_DONE, REQ_PREEMPTED = range(5)


class SpecSeq(C.Structure):
    _fields_ = [("last_token", C.c_int32), ("drafts", C.POINTER(C.c_int32)), ("n_drafts", C.c_int),
                ("start_pos", C.c_int), ("block_table", C.POINTER(C.c_int32)), ("n_blocks", C.c_int)]


_proto("nmx_ngram_create", _i, _i, _i, _i, _i, C.POINTER(_vp))
_proto("nmx_ngram_destroy", None, _vp)
_proto("nmx_ngram_record_token", None, _vp, C.c_int32)
_proto("nmx_ngram_record_tokens", None, _vp, C.POINTER(C.c_int32), _i)
_proto("nmx_ngram_speculate", _i, _vp, C.POINTER(C.c_int32), _i, C.POINTER(C.c_int32), _i)
_proto("nmx_ngram_record_accepted", None, _vp, C.POINTER(C.c_int32), _i, _i)
_proto("nmx_ngram_stats", None, _vp, C.POINTER(_i), C.POINTER(C.c_longlong), C.POINTER(_i), C.POINTER(C.c_double))
_proto("nmx_spec_verify", _i, _vp, _vp, C.POINTER(SpecSeq), _i, _i, C.POINTER(C.c_int32), C.POINTER(_i),
       C.POINTER(_i))
VERIFY_NGRAM, VERIFY_PREFIX = 0, 1
IPC_HANDLE_BYTES = 64
_proto("nmx_op_sample", _i, _vp, _vp, _i, _i, _i, _f, _f, C.c_uint64, C.c_uint64, _vp, _vp, _i, _vp, _vp)
_proto("nmx_safetensors_open", _i, C.c_char_p, C.POINTER(_vp))
_proto("nmx_safetensors_close", None, _vp)
_proto("nmx_safetensors_count", _i, _vp)
_proto("nmx_safetensors_info", _i, _vp, _i, C.c_char_p, _i, C.c_char_p, C.POINTER(C.c_int64), C.POINTER(_i),
       C.POINTER(C.c_uint64))
_proto("nmx_safetensors_metadata", _i, _vp, C.c_char_p, C.c_char_p, _i)
_proto("nmx_safetensors_read", _i, _vp, C.c_char_p, _vp, C.c_uint64)
_proto("nmx_safetensors_write", _i, C.c_char_p, _i, C.POINTER(C.c_char_p), C.POINTER(C.c_char_p),
       C.POINTER(C.POINTER(C.c_int64)), C.POINTER(_i), C.POINTER(_vp), _i, C.POINTER(C.c_char_p),
       C.POINTER(C.c_char_p))
_proto("nmx_model_load_safetensors", _i, _vp, C.c_char_p, _i, _i, C.POINTER(_i), C.POINTER(_i))
_proto("nmx_ssd_save_block", _i, _vp, _i, C.c_char_p, _i, C.c_char_p, C.c_char_p)
_proto("nmx_ssd_load_block", _i, _vp, C.c_char_p, C.c_char_p, _i, C.POINTER(_i))
_proto("nmx_comm_create", _i, _vp, _i, _i, _sz, C.POINTER(_vp))
_proto("nmx_comm_ipc_handle", _i, _vp, _vp)
_proto("nmx_comm_connect", _i, _vp, _vp)
_proto("nmx_comm_destroy", None, _vp)
_proto("nmx_model_set_comm", _i, _vp, _vp)
_proto("nmx_op_allreduce_resid", _i, _vp, _vp, _i, _i, _vp, _vp)
_proto("nmx_model_set_exchange_fusion", _i, _vp, _i)
_proto("nmx_block_pool_destroy", None, _vp)
_proto("nmx_block_pool_allocate", _i, _vp)
_proto("nmx_block_pool_free", None, _vp, _i)
_proto("nmx_block_pool_incref", None, _vp, _i)
_proto("nmx_block_pool_refcount", _i, _vp, _i)
_proto("nmx_block_pool_register", None, _vp, _i, _u8p, _ip, _i)
_proto("nmx_block_pool_find_prefix", _i, _vp, _ip, _i, _ip, _i, C.POINTER(_i))
_proto("nmx_block_pool_stats", None, _vp, C.POINTER(_i), C.POINTER(_i), C.POINTER(_i), C.POINTER(_i))
_proto("nmx_block_pool_clear", None, _vp)
_proto("nmx_block_pool_table_create", _i, _vp, C.c_char_p)
_proto("nmx_block_pool_table_append", _i, _vp, C.c_char_p, _i)
_proto("nmx_block_pool_table_get", _i, _vp, C.c_char_p, _ip, _i)
_proto("nmx_block_pool_table_delete", _i, _vp, C.c_char_p)
_proto("nmx_block_pool_table_fork", _i, _vp, C.c_char_p, C.c_char_p)


def check(status: int) -> None:
    if status != NMX_OK:
        raise NmxError(status, lib.nmx_last_error().decode())


def version() -> str:
    return lib.nmx_version().decode()


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.int32))


def _iptr(a: np.ndarray):
    return a.ctypes.data_as(_ip)


def _dt_of(t) -> int:
    import torch
    if t.dtype == torch.float16:
        return F16
    if t.dtype == torch.bfloat16:
        return BF16
    if t.dtype == torch.float32:
        return F32
    raise ValueError(f"unsupported dtype {t.dtype}")


def _ptr(t) -> int:
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("device tensor required")
    if not t.is_contiguous():
        raise ValueError("contiguous tensor required")
    return t.data_ptr()


# --------------------------------------------------------------------- context

class Context:
    """One device + one stream (nmx_ctx_t)."""

    def __init__(self, device: int = 0):
        import torch
        h = _vp()
        check(lib.nmx_ctx_create(device, C.byref(h)))
        self.h = h
        self.device = device
        # a side stream owned by torch (capturable, unlike the legacy default
        # stream); op wrappers order it against torch's current stream
        self.stream = torch.cuda.Stream(device=device)
        check(lib.nmx_ctx_set_stream(self.h, self.stream.cuda_stream))

    def _enter(self):
        import torch
        cur = torch.cuda.current_stream(self.device)
        if cur.cuda_stream != self.stream.cuda_stream:
            self.stream.wait_stream(cur)
        return cur

    def _leave(self, cur):
        if cur.cuda_stream != self.stream.cuda_stream:
            cur.wait_stream(self.stream)

    def _op(self, status_fn):
        cur = self._enter()
        st = status_fn()
        self._leave(cur)
        return st

    def synchronize(self):
        check(lib.nmx_ctx_synchronize(self.h))

    def set_wait_limit(self, polls: int = 0):
        """Polls a device-side wait makes before giving up with
        NMX_ERR_TIMEOUT (0: the default, 2^24)."""
        check(lib.nmx_ctx_set_wait_limit(self.h, int(polls)))

    @property
    def launches(self) -> int:
        return int(lib.nmx_ctx_kernel_launches(self.h))

    def close(self):
        if self.h:
            lib.nmx_ctx_destroy(self.h)
            self.h = None

    def __del__(self, _finalizing=sys.is_finalizing):
        if _finalizing():
            return  # the process is exiting; the driver reclaims device memory
        try:
            self.close()
        except Exception:
            pass

    # ---- op level (MLX names) -------------------------------------------
    def quantized_matmul(self, x, w, scales, biases, transpose: bool = True, group_size: int = 64,
                         bits: int = 4, out=None):
        """y = x @ dequant(w).T — MLX.quantizedMM (BailingHybridModel.swift:213)."""
        import torch
        M, K = x.shape
        N = w.shape[0]
        if out is None:
            out = torch.empty((M, N), dtype=x.dtype, device=x.device)
        check(self._op(lambda: lib.nmx_op_qmatmul(self.h, _ptr(x), _ptr(w), _ptr(scales), _ptr(biases), M, N, K,
                                                  bits, group_size, 1 if transpose else 0, _dt_of(x), _ptr(out))))
        return out

    def pack_records(self, wq, scales, biases):
        """Decode-record copy of a 4-bit g64 f16 linear (uint8 tensor of N*K*9/16 bytes)."""
        import torch
        N = wq.shape[0]
        K = wq.shape[1] * 8
        rec = torch.empty((N * K * 9 // 16,), dtype=torch.uint8, device=wq.device)
        check(self._op(lambda: lib.nmx_op_pack_records(self.h, _ptr(wq), _ptr(scales), _ptr(biases), N, K,
                                                       _ptr(rec))))
        return rec

    def quantized_matmul_records(self, x, records, N: int, out=None):
        import torch
        M, K = x.shape
        if out is None:
            out = torch.empty((M, N), dtype=x.dtype, device=x.device)
        check(self._op(lambda: lib.nmx_op_qmatmul_records(self.h, _ptr(x), _ptr(records), M, N, K, _ptr(out))))
        return out

    def quantize(self, w, group_size: int = 64, bits: int = 4, scale_dtype=None):
        """MLX.quantized (BailingHybridModel.swift:179): returns (packed u32 as int32, scales, biases)."""
        import torch
        N, K = w.shape
        sdt = scale_dtype or torch.float16
        wq = torch.empty((N, K * bits // 32), dtype=torch.int32, device=w.device)
        s = torch.empty((N, K // group_size), dtype=sdt, device=w.device)
        b = torch.empty_like(s)
        check(self._op(lambda: lib.nmx_op_quantize(self.h, _ptr(w), N, K, bits, group_size, _dt_of(s), _ptr(wq),
                                                   _ptr(s), _ptr(b))))
        return wq, s, b

    def dequantize(self, wq, scales, biases, group_size: int = 64, bits: int = 4):
        import torch
        N = wq.shape[0]
        K = wq.shape[1] * 32 // bits
        w = torch.empty((N, K), dtype=torch.float32, device=wq.device)
        check(self._op(lambda: lib.nmx_op_dequantize(self.h, _ptr(wq), _ptr(scales), _ptr(biases), N, K, bits,
                                                     group_size, _dt_of(scales), _ptr(w))))
        return w

    def rms_norm(self, x, weight, eps: float = 1e-5):
        import torch
        M, H = x.shape
        y = torch.empty_like(x)
        check(self._op(lambda: lib.nmx_op_rmsnorm(self.h, _ptr(x), _ptr(weight), M, H, eps, _dt_of(x), _ptr(y))))
        return y

    def argmax(self, logits):
        import torch
        M, V = logits.shape
        out = torch.empty((M,), dtype=torch.int32, device=logits.device)
        check(self._op(lambda: lib.nmx_op_argmax(self.h, _ptr(logits), M, V, _dt_of(logits), _ptr(out))))
        return out

    def sample(self, logits, temperature: float, top_p: float = 1.0, seed: int = 0, counter: int = 0,
               top_k: int = 0):
        """temperature / top-p categorical per row; returns (ids, chosen logprobs,
        top ids, top logprobs) as device tensors (the last two None when top_k == 0)"""
        import torch
        M, V = logits.shape
        ids = torch.empty((M,), dtype=torch.int32, device=logits.device)
        lp = torch.empty((M,), dtype=torch.float32, device=logits.device)
        tid = torch.empty((M, max(top_k, 1)), dtype=torch.int32, device=logits.device)
        tlp = torch.empty((M, max(top_k, 1)), dtype=torch.float32, device=logits.device)
        check(self._op(lambda: lib.nmx_op_sample(self.h, _ptr(logits), M, V, _dt_of(logits), float(temperature),
                                                 float(top_p), int(seed), int(counter), _ptr(ids), _ptr(lp),
                                                 int(top_k), _ptr(tid), _ptr(tlp))))
        return ids, lp, (tid if top_k else None), (tlp if top_k else None)

    def penalized_argmax(self, logits, recent, n_recent, penalty: float):
        import torch
        M, V = logits.shape
        out = torch.empty((M,), dtype=torch.int32, device=logits.device)
        check(self._op(lambda: lib.nmx_op_penalized_argmax(self.h, _ptr(logits), M, V, _dt_of(logits), _ptr(recent),
                                                           _ptr(n_recent), recent.shape[1], penalty, _ptr(out))))
        return out

    def fused_quantized_sdpa(self, queries, k_w, k_s, k_b, v_w, v_s, v_b, scale: float, group_size: int, bits: int,
                             n_kv_heads: int, allow_multi_query: bool = False):
        """FusedQuantizedSDPA.attention (FusedQuantizedSDPA.swift:168-250). queries [B, Hq, L, D];
        K/V arrays [B, Hkv, N, ...]. Returns None where the reference returns nil."""
        import torch
        B, Hq, L, D = queries.shape
        N = k_w.shape[-2]
        out = torch.empty_like(queries)
        st = self._op(lambda: lib.nmx_op_attn_quantized_decode(
            self.h, _ptr(queries), _ptr(k_w), _ptr(k_s), _ptr(k_b), _ptr(v_w), _ptr(v_s), _ptr(v_b), B, Hq,
            n_kv_heads, N, L, D, scale, group_size, bits, 1 if allow_multi_query else 0, _dt_of(queries), _ptr(out)))
        if st == NMX_ERR_UNSUPPORTED:
            return None
        check(st)
        return out

    def paged_decode_attention(self, q, k_cache, v_cache, block_tables, seq_lens, n_kv_heads: int, scale: float,
                               block_tokens: int = 16, out=None):
        import torch
        B, Hq, D = q.shape
        if out is None:
            out = torch.empty_like(q)
        kp = k_cache if isinstance(k_cache, int) else _ptr(k_cache)
        vp = v_cache if isinstance(v_cache, int) else _ptr(v_cache)
        check(self._op(lambda: lib.nmx_op_attn_paged_decode(self.h, _ptr(q), kp, vp, _ptr(block_tables),
                                                            _ptr(seq_lens), B, Hq, n_kv_heads, D, block_tokens,
                                                            block_tables.shape[1], scale, _ptr(out))))
        return out


    def paged_decode_attention_noalloc(self, q, k_cache, v_cache, block_tables, seq_lens, n_kv_heads: int,
                                       scale: float, block_tokens: int = 16, out=None):
        """paged_decode_attention through the entry point that never allocates
        device memory (its scratch is a fixed array inside the library)."""
        import torch
        B, Hq, D = q.shape
        if out is None:
            out = torch.empty_like(q)
        kp = k_cache if isinstance(k_cache, int) else _ptr(k_cache)
        vp = v_cache if isinstance(v_cache, int) else _ptr(v_cache)
        check(self._op(lambda: lib.nmx_op_attn_paged_decode_noalloc(
            self.h, _ptr(q), kp, vp, _ptr(block_tables), _ptr(seq_lens), B, Hq, n_kv_heads, D, block_tokens,
            block_tables.shape[1], scale, _ptr(out))))
        return out


# ----------------------------------------------------------------------- model

@dataclass
class ModelConfig:
    vocab: int
    hidden: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    ffn: int
    bits: int = 4
    group_size: int = 64
    dtype: int = F16
    qkv_bias: bool = False
    tie_embeddings: bool = False
    rms_eps: float = 1e-5
    rope_theta: float = 10000.0
    rope_factor: float = 0.0
    rope_low_freq_factor: float = 1.0
    rope_high_freq_factor: float = 4.0
    rope_original_max_pos: int = 8192
    max_batch: int = 8
    max_tokens: int = 2048

    def to_c(self) -> ModelCfg:
        c = ModelCfg()
        for k in ("vocab", "hidden", "n_layers", "n_heads", "n_kv_heads", "head_dim", "ffn", "bits", "group_size",
                  "dtype", "rope_original_max_pos", "max_batch", "max_tokens"):
            setattr(c, k, int(getattr(self, k)))
        c.qkv_bias = int(self.qkv_bias)
        c.tie_embeddings = int(self.tie_embeddings)
        for k in ("rms_eps", "rope_theta", "rope_factor", "rope_low_freq_factor", "rope_high_freq_factor"):
            setattr(c, k, float(getattr(self, k)))
        return c

    @property
    def nqkv(self) -> int:
        return (self.n_heads + 2 * self.n_kv_heads) * self.head_dim


def llama31_8b(**kw) -> ModelConfig:
    """Llama-3.1-8B architecture (hidden 4096, 32 layers, 32/8 heads, ffn 14336, vocab 128256,
    RoPE θ 5e5 with the "llama3" scaling factor 8 / low 1 / high 4 / original 8192)."""
    base = dict(vocab=128256, hidden=4096, n_layers=32, n_heads=32, n_kv_heads=8, head_dim=128, ffn=14336,
                rms_eps=1e-5, rope_theta=500000.0, rope_factor=8.0, rope_low_freq_factor=1.0,
                rope_high_freq_factor=4.0, rope_original_max_pos=8192)
    base.update(kw)
    return ModelConfig(**base)


def llama33_70b(**kw) -> ModelConfig:
    """Llama-3.3-70B-style architecture (hidden 8192, 80 layers, 64/8 heads, ffn 28672, vocab 128256,
    RoPE θ 5e5 with the llama3 scaling)."""
    base = dict(vocab=128256, hidden=8192, n_layers=80, n_heads=64, n_kv_heads=8, head_dim=128, ffn=28672,
                rms_eps=1e-5, rope_theta=500000.0, rope_factor=8.0, rope_low_freq_factor=1.0,
                rope_high_freq_factor=4.0, rope_original_max_pos=8192)
    base.update(kw)
    return ModelConfig(**base)


def llama32_1b(**kw) -> ModelConfig:
    """Llama-3.2-1B-style draft architecture (hidden 2048, 16 layers, 32/8 heads of 64, ffn 8192,
    vocab 128256). The original ties the output head to the embedding; here the head is its own
    quantized [vocab, hidden] matrix, which streams the same bytes per token."""
    base = dict(vocab=128256, hidden=2048, n_layers=16, n_heads=32, n_kv_heads=8, head_dim=64, ffn=8192,
                rms_eps=1e-5, rope_theta=500000.0, rope_factor=32.0,
                rope_low_freq_factor=1.0, rope_high_freq_factor=4.0, rope_original_max_pos=8192)
    base.update(kw)
    return ModelConfig(**base)


def qwen25_32b(**kw) -> ModelConfig:
    """Qwen2.5-32B-style architecture (hidden 5120, 64 layers, 40/8 heads, qkv bias, ffn 27648,
    vocab 152064, RoPE θ 1e6, RMSNorm eps 1e-6)."""
    base = dict(vocab=152064, hidden=5120, n_layers=64, n_heads=40, n_kv_heads=8, head_dim=128, ffn=27648,
                qkv_bias=True, rms_eps=1e-6, rope_theta=1000000.0)
    base.update(kw)
    return ModelConfig(**base)


class Model:
    """nmx_model_t: weights on one device plus the forward entry points."""

    def __init__(self, ctx: Context, cfg: ModelConfig):
        self.ctx = ctx
        self.cfg = cfg
        self._c = cfg.to_c()
        h = _vp()
        check(lib.nmx_model_create(ctx.h, C.byref(self._c), C.byref(h)))
        self.h = h

    def close(self):
        if self.h:
            lib.nmx_model_destroy(self.h)
            self.h = None

    def __del__(self, _finalizing=sys.is_finalizing):
        if _finalizing():
            return  # the process is exiting; the driver reclaims device memory
        try:
            self.close()
        except Exception:
            pass

    def init_random(self, seed: int = 0, std: float = 0.02):
        check(lib.nmx_model_init_random(self.h, seed, std))

    def set_comm(self, comm: Optional["Comm"]):
        """tensor parallelism: join o_proj / down_proj outputs over the ranks"""
        check(lib.nmx_model_set_comm(self.h, comm.h if comm is not None else None))
        self.comm = comm  # keep it alive while the model uses it

    def set_exchange_fusion(self, enable: bool):
        check(lib.nmx_model_set_exchange_fusion(self.h, int(bool(enable))))

    def load_tensor(self, name: str, arr: np.ndarray):
        arr = np.ascontiguousarray(arr)
        if arr.dtype == np.uint32:
            dt = U32
        elif arr.dtype == np.float16:
            dt = F16
        elif arr.dtype == np.uint16:  # raw bf16 bits
            dt = BF16
        else:
            raise ValueError(f"unsupported array dtype {arr.dtype}")
        shape = (C.c_int64 * arr.ndim)(*arr.shape)
        check(lib.nmx_model_load_tensor(self.h, name.encode(), arr.ctypes.data, dt, shape, arr.ndim))

    def get_tensor(self, name: str, shape: Sequence[int], dtype) -> np.ndarray:
        out = np.empty(shape, dtype=dtype)
        check(lib.nmx_model_get_tensor(self.h, name.encode(), out.ctypes.data, out.nbytes))
        return out

    @property
    def weight_bytes(self) -> int:
        return int(lib.nmx_model_weight_bytes(self.h))

    @property
    def step_weight_bytes(self) -> int:
        return int(lib.nmx_model_step_weight_bytes(self.h))

    @property
    def kv_bytes_per_token(self) -> int:
        return int(lib.nmx_kv_bytes_per_token(self.h))

    def forward(self, pool: "KVPool", seqs: Sequence[dict], mode: int = OUT_ARGMAX_LAST) -> np.ndarray:
        """One forward over sequences given as dicts {tokens, start_pos, block_table}."""
        n = len(seqs)
        arr = (Seq * n)()
        keep = []
        total = 0
        for i, s in enumerate(seqs):
            toks = _i32(s["tokens"])
            tbl = _i32(s["block_table"])
            keep += [toks, tbl]
            arr[i].n_new_tokens = len(toks)
            arr[i].token_ids = _iptr(toks)
            arr[i].start_pos = int(s["start_pos"])
            arr[i].block_table = _iptr(tbl)
            arr[i].n_blocks = len(tbl)
            total += len(toks)
        rows = total if mode in (OUT_ARGMAX_ALL, OUT_LOGITS_ALL) else n
        if mode in (OUT_LOGITS_LAST, OUT_LOGITS_ALL):
            out = np.empty((rows, self.cfg.vocab), dtype=np.float32)
        else:
            out = np.empty((rows,), dtype=np.int32)
        check(lib.nmx_forward(self.h, pool.h, arr, n, mode, out.ctypes.data))
        return out

    def decode_greedy(self, pool: "KVPool", first_tokens, start_pos, block_tables: np.ndarray, n_steps: int,
                      want_ids: bool = True) -> Optional[np.ndarray]:
        ft = _i32(first_tokens)
        sp = _i32(start_pos)
        bt = _i32(block_tables)
        n = len(ft)
        out = np.empty((n_steps, n), dtype=np.int32) if want_ids else None
        check(lib.nmx_decode_greedy(self.h, pool.h, _iptr(ft), _iptr(sp), _iptr(bt), bt.shape[1], n, n_steps,
                                    _iptr(out) if out is not None else None))
        return out


class KVPool:
    """nmx_kv_pool_t: K/V pages of `block_tokens` tokens for every layer, fp16 or
    (kv_bits 4 / 8) MLX-affine quantized in groups of kv_group_size along head_dim."""

    def __init__(self, model: Model, num_blocks: int, block_tokens: int = 16, kv_bits: int = 0,
                 kv_group_size: int = 64):
        h = _vp()
        if kv_bits:
            check(lib.nmx_kv_pool_create_quantized(model.h, block_tokens, num_blocks, kv_bits, kv_group_size,
                                                   C.byref(h)))
        else:
            check(lib.nmx_kv_pool_create(model.h, block_tokens, num_blocks, C.byref(h)))
        self.h = h
        self.model = model
        self.num_blocks = num_blocks
        self.block_tokens = block_tokens
        self.kv_bits = kv_bits
        self._gs = kv_group_size

    @property
    def bytes_per_token(self) -> int:
        return int(lib.nmx_kv_pool_bytes_per_token(self.h))

    def fill_random(self, seed: int = 0, std: float = 1.0):
        """Every page of every layer N(0, std): a cache of a given context without its prefill."""
        check(lib.nmx_kv_pool_fill_random(self.h, seed, std))

    def layer_ptrs(self, layer: int):
        k, v = _vp(), _vp()
        check(lib.nmx_kv_pool_layer_ptrs(self.h, layer, C.byref(k), C.byref(v)))
        return k.value, v.value

    def read_blocks(self, ids) -> np.ndarray:
        """Host copy [n, layers, 2, Hkv, block_tokens, head_dim] (raw f16 bits);
        quantized pools: the raw page records [n, layers, 2, block bytes] (uint8)."""
        c = self.model.cfg
        ids = _i32(ids)
        if self.kv_bits:
            rec = 16 * (c.head_dim * self.kv_bits // 8 + 2 * (c.head_dim // self._gs) * 2)
            out = np.empty((len(ids), c.n_layers, 2, c.n_kv_heads * rec), np.uint8)
            check(lib.nmx_kv_read_blocks(self.h, _iptr(ids), len(ids), out.ctypes.data))
            return out
        out = np.empty((len(ids), c.n_layers, 2, c.n_kv_heads, self.block_tokens, c.head_dim), np.uint16)
        check(lib.nmx_kv_read_blocks(self.h, _iptr(ids), len(ids), out.ctypes.data))
        return out

    def write_blocks(self, ids, data: np.ndarray):
        ids = _i32(ids)
        data = np.ascontiguousarray(data, dtype=np.uint16)
        check(lib.nmx_kv_write_blocks(self.h, _iptr(ids), len(ids), data.ctypes.data))

    def copy_blocks(self, src, dst):
        s, d = _i32(src), _i32(dst)
        check(lib.nmx_kv_copy_blocks(self.h, _iptr(s), _iptr(d), len(s)))

    def close(self):
        if self.h:
            lib.nmx_kv_pool_destroy(self.h)
            self.h = None

    def __del__(self, _finalizing=sys.is_finalizing):
        if _finalizing():
            return  # the process is exiting; the driver reclaims device memory
        try:
            self.close()
        except Exception:
            pass


# ------------------------------------------------------------- prefix cache

class BlockHasher:
    """BlockHasher (Sources/NovaMLXPrefixCache/BlockHasher.swift:4-55)."""

    @staticmethod
    def compute_block_hash(parent_hash: Optional[bytes], token_ids: Sequence[int], model_name: str) -> bytes:
        toks = _i32(token_ids)
        out = (C.c_uint8 * 20)()
        par = (C.c_uint8 * 20).from_buffer_copy(parent_hash) if parent_hash is not None else None
        lib.nmx_block_hash(par, _iptr(toks) if len(toks) else None, len(toks), model_name.encode(), out)
        return bytes(out)

    @staticmethod
    def compute_chain_hashes(token_ids: Sequence[int], block_size: int, model_name: str) -> list:
        toks = _i32(token_ids)
        nmax = len(toks) // block_size if block_size > 0 else 0
        buf = (C.c_uint8 * max(1, 20 * nmax))()
        n = lib.nmx_chain_hashes(_iptr(toks) if len(toks) else None, len(toks), block_size, model_name.encode(),
                                 buf, nmax)
        raw = bytes(buf)
        return [raw[20 * i:20 * (i + 1)] for i in range(n)]


class PagedBlockPool:
    """PagedBlockPool (Sources/NovaMLXPrefixCache/PagedBlockPool.swift:108-291)."""

    def __init__(self, block_size: int = 64, max_blocks: int = 4096, initial_blocks: int = 256, model_name: str = ""):
        h = _vp()
        check(lib.nmx_block_pool_create(block_size, max_blocks, initial_blocks, model_name.encode(), C.byref(h)))
        self.h = h
        self.block_size = block_size

    def __del__(self, _finalizing=sys.is_finalizing):
        if getattr(self, "h", None) and not _finalizing():
            lib.nmx_block_pool_destroy(self.h)
            self.h = None

    def allocate_block(self) -> Optional[int]:
        b = lib.nmx_block_pool_allocate(self.h)
        return None if b < 0 else b

    def free_block(self, block_id: int):
        lib.nmx_block_pool_free(self.h, block_id)

    def increment_ref(self, block_id: int):
        lib.nmx_block_pool_incref(self.h, block_id)

    def ref_count(self, block_id: int) -> int:
        return lib.nmx_block_pool_refcount(self.h, block_id)

    def register_block(self, block_id: int, token_ids: Sequence[int], parent_hash: Optional[bytes]):
        toks = _i32(token_ids)
        par = (C.c_uint8 * 20).from_buffer_copy(parent_hash) if parent_hash is not None else None
        lib.nmx_block_pool_register(self.h, block_id, par, _iptr(toks) if len(toks) else None, len(toks))

    def find_shared_prefix(self, token_ids: Sequence[int]):
        toks = _i32(token_ids)
        nmax = max(1, len(toks) // self.block_size)
        ids = np.zeros(nmax, dtype=np.int32)
        rem = C.c_int(0)
        n = lib.nmx_block_pool_find_prefix(self.h, _iptr(toks) if len(toks) else None, len(toks), _iptr(ids), nmax,
                                           C.byref(rem))
        return [int(x) for x in ids[:n]], int(rem.value)

    def get_stats(self):
        t, a, f, s = C.c_int(), C.c_int(), C.c_int(), C.c_int()
        lib.nmx_block_pool_stats(self.h, C.byref(t), C.byref(a), C.byref(f), C.byref(s))
        return t.value, a.value, f.value, s.value

    def clear(self):
        lib.nmx_block_pool_clear(self.h)

    def create_block_table(self, request_id: str):
        check(lib.nmx_block_pool_table_create(self.h, request_id.encode()))

    def append_block(self, request_id: str, block_id: int):
        check(lib.nmx_block_pool_table_append(self.h, request_id.encode(), block_id))

    def block_table(self, request_id: str) -> Optional[list]:
        n = lib.nmx_block_pool_table_get(self.h, request_id.encode(), None, 0)
        if n < 0:
            return None
        ids = np.zeros(max(1, n), dtype=np.int32)
        lib.nmx_block_pool_table_get(self.h, request_id.encode(), _iptr(ids), n)
        return [int(x) for x in ids[:n]]

    def delete_block_table(self, request_id: str):
        check(lib.nmx_block_pool_table_delete(self.h, request_id.encode()))

    def fork_block_table(self, source_request_id: str, new_request_id: str):
        check(lib.nmx_block_pool_table_fork(self.h, source_request_id.encode(), new_request_id.encode()))


class MemoryBudget:
    """nmx_budget_t: MemoryBudgetTracker's admission arithmetic (10% headroom by default)."""

    def __init__(self, limit_bytes: int, headroom_percent: int = 10):
        h = _vp()
        check(lib.nmx_budget_create(limit_bytes, headroom_percent, C.byref(h)))
        self.h = h

    def add_weights(self, nbytes: int):
        lib.nmx_budget_add_weights(self.h, nbytes)

    def can_admit(self, estimated_tokens: int, bytes_per_token: int) -> bool:
        return bool(lib.nmx_budget_can_admit(self.h, estimated_tokens, bytes_per_token))

    def reserve(self, seq_id: int, estimated_tokens: int, bytes_per_token: int):
        lib.nmx_budget_reserve(self.h, seq_id, estimated_tokens, bytes_per_token)

    def release(self, seq_id: int):
        lib.nmx_budget_release(self.h, seq_id)

    @property
    def available(self) -> int:
        return int(lib.nmx_budget_available(self.h))

    def __del__(self, _finalizing=sys.is_finalizing):
        if not _finalizing() and getattr(self, "h", None):
            lib.nmx_budget_destroy(self.h)
            self.h = None


class Scheduler:
    """nmx_sched_t: continuous batching (admission, prefix reuse, chunked prefill,
    one batched forward per step, preemption of the newest sequence)."""

    def __init__(self, model: Model, pool: KVPool, max_batch: int, max_step_tokens: int, prefill_chunk: int = 512,
                 max_concurrent: int = 64, headroom_percent: int = 10, kv_budget_bytes: int = 0,
                 model_name: str = ""):
        self._name = model_name.encode()
        cfg = SchedCfg(max_batch, max_step_tokens, prefill_chunk, max_concurrent, headroom_percent, kv_budget_bytes,
                       self._name)
        h = _vp()
        check(lib.nmx_sched_create(model.h, pool.h, C.byref(cfg), C.byref(h)))
        self.h = h
        self.model = model
        self.pool = pool  # the scheduler hands out this pool's blocks: keep it alive

    def submit(self, prompt, max_new_tokens: int, eos_id: int = -1) -> int:
        p = _i32(prompt)
        rid = C.c_int64()
        check(lib.nmx_sched_submit(self.h, _iptr(p), len(p), max_new_tokens, eos_id, C.byref(rid)))
        return int(rid.value)

    def step(self) -> int:
        n = C.c_int()
        check(lib.nmx_sched_step(self.h, C.byref(n)))
        return int(n.value)

    def poll(self, rid: int):
        n, st = C.c_int(), C.c_int()
        check(lib.nmx_sched_poll(self.h, rid, None, 0, C.byref(n), C.byref(st)))
        out = np.empty(n.value, np.int32)
        if n.value:
            check(lib.nmx_sched_poll(self.h, rid, out.ctypes.data, n.value, C.byref(n), C.byref(st)))
        return out, int(st.value)

    def stats(self) -> dict:
        st = SchedStats()
        check(lib.nmx_sched_stats(self.h, C.byref(st)))
        return {f: getattr(st, f) for f, _ in SchedStats._fields_}

    def close(self):
        if self.h:
            lib.nmx_sched_destroy(self.h)
            self.h = None

    def __del__(self, _finalizing=sys.is_finalizing):
        if _finalizing():
            return
        self.close()


class NGramSpeculator:
    """nmx_ngram_t: NGramSpeculator + SpeculativeDecoder's acceptance count."""

    def __init__(self, ngram_size: int = 4, max_draft: int = 5, min_hits: int = 1, max_cache_size: int = 65536):
        h = _vp()
        check(lib.nmx_ngram_create(ngram_size, max_draft, min_hits, max_cache_size, C.byref(h)))
        self.h = h
        self.max_draft = max_draft

    def record_token(self, token: int):
        lib.nmx_ngram_record_token(self.h, int(token))

    def record_tokens(self, tokens):
        t = _i32(tokens)
        lib.nmx_ngram_record_tokens(self.h, _iptr(t), len(t))

    def speculate(self, context=None):
        out = np.zeros(max(self.max_draft, 1), np.int32)
        if context is None:
            n = lib.nmx_ngram_speculate(self.h, None, 0, _iptr(out), len(out))
        else:
            c = _i32(context)
            n = lib.nmx_ngram_speculate(self.h, _iptr(c), len(c), _iptr(out), len(out))
        return [int(v) for v in out[:n]]

    def record_accepted(self, tokens, accepted: int):
        t = _i32(tokens)
        lib.nmx_ngram_record_accepted(self.h, _iptr(t), len(t), int(accepted))

    @property
    def stats(self):
        cs, hits, buf, rate = C.c_int(), C.c_longlong(), C.c_int(), C.c_double()
        lib.nmx_ngram_stats(self.h, C.byref(cs), C.byref(hits), C.byref(buf), C.byref(rate))
        return {"cache_size": cs.value, "total_hits": hits.value, "buffer_size": buf.value,
                "acceptance_rate": rate.value}

    def __del__(self, _finalizing=sys.is_finalizing):
        if not _finalizing() and getattr(self, "h", None):
            lib.nmx_ngram_destroy(self.h)
            self.h = None


def spec_verify(model: Model, pool: KVPool, seqs, rule: int = VERIFY_PREFIX):
    """nmx_spec_verify over dicts {last_token, drafts, start_pos, block_table};
    returns [(tokens, accepted)] per sequence."""
    keep = []
    arr = (SpecSeq * len(seqs))()
    max_d = 0
    for i, sq in enumerate(seqs):
        d = _i32(sq.get("drafts", []))
        t = _i32(sq["block_table"])
        keep += [d, t]
        arr[i].last_token = int(sq["last_token"])
        arr[i].drafts = _iptr(d)
        arr[i].n_drafts = len(d)
        arr[i].start_pos = int(sq["start_pos"])
        arr[i].block_table = _iptr(t)
        arr[i].n_blocks = len(t)
        max_d = max(max_d, len(d))
    out = np.zeros((len(seqs), max_d + 1), np.int32)
    cnt = np.zeros(len(seqs), np.int32)
    acc = np.zeros(len(seqs), np.int32)
    check(lib.nmx_spec_verify(model.h, pool.h, arr, len(seqs), int(rule), _iptr(out),
                              cnt.ctypes.data_as(C.POINTER(_i)), acc.ctypes.data_as(C.POINTER(_i))))
    return [(out[i, :cnt[i]].tolist(), int(acc[i])) for i in range(len(seqs))]


class Comm:
    """nmx_comm_t: this rank's end of the tensor-parallel exchange (peer
    partials over CUDA IPC)."""

    def __init__(self, ctx: Context, rank: int, world: int, region_bytes: int):
        h = _vp()
        check(lib.nmx_comm_create(ctx.h, rank, world, region_bytes, C.byref(h)))
        self.h, self.ctx, self.rank, self.world = h, ctx, rank, world

    def handle(self) -> bytes:
        buf = (C.c_ubyte * IPC_HANDLE_BYTES)()
        check(lib.nmx_comm_ipc_handle(self.h, buf))
        return bytes(buf)

    def connect(self, handles):
        assert len(handles) == self.world and all(len(b) == IPC_HANDLE_BYTES for b in handles)
        blob = b"".join(handles)
        buf = (C.c_ubyte * len(blob)).from_buffer_copy(blob)
        check(lib.nmx_comm_connect(self.h, buf))

    def allreduce_resid(self, partial, res, out):
        """out = res + sum over ranks of partial (device tensors, [rows, cols] f16)"""
        rows, cols = partial.shape
        check(self.ctx._op(lambda: lib.nmx_op_allreduce_resid(self.h, partial.data_ptr(), rows, cols, res.data_ptr(),
                                                              out.data_ptr())))
        return out

    def close(self):
        if self.h:
            lib.nmx_comm_destroy(self.h)
            self.h = None

    def __del__(self, _finalizing=sys.is_finalizing):
        if not _finalizing():
            self.close()


def tp_comm(ctx: Context, rank: int, world: int, region_bytes: int, exchange) -> Comm:
    """Create this rank's communicator and connect it; exchange(bytes) must
    return every rank's bytes in rank order (e.g. torch.distributed
    all_gather_object)."""
    comm = Comm(ctx, rank, world, region_bytes)
    comm.connect(exchange(comm.handle()))
    return comm


def torch_exchange(dist):
    """exchange() over an initialised torch.distributed process group"""
    def ex(b: bytes):
        out = [None] * dist.get_world_size()
        dist.all_gather_object(out, b)
        return out
    return ex


def tp_config(cfg: ModelConfig, world: int) -> ModelConfig:
    """The model config of one tensor-parallel rank: heads and ffn split."""
    import dataclasses
    if cfg.n_heads % world or cfg.n_kv_heads % world or cfg.ffn % world:
        raise ValueError("heads, kv heads and ffn must divide by the tensor-parallel size")
    if (cfg.ffn // world) % cfg.group_size or (cfg.n_heads // world * cfg.head_dim) % cfg.group_size:
        raise ValueError("a rank's K shard of o_proj / down_proj must be whole quantization groups")
    return dataclasses.replace(cfg, n_heads=cfg.n_heads // world, n_kv_heads=cfg.n_kv_heads // world,
                               ffn=cfg.ffn // world)


def tp_shard(tensors: dict, cfg: ModelConfig, rank: int, world: int) -> dict:
    """This rank's slice of MLX-layout tensors (names unchanged): rows of
    q/k/v/gate/up (and q/k/v biases), K columns of o/down (packed words,
    scales, biases); everything else replicated."""
    D, bits, gs = cfg.head_dim, cfg.bits, cfg.group_size
    nq, nkv, f = cfg.n_heads // world * D, cfg.n_kv_heads // world * D, cfg.ffn // world
    per_word = 32 // bits
    out = {}
    for name, t in tensors.items():
        parts = name.split(".")
        kind = parts[-1]  # weight | scales | biases | bias
        mod = parts[-2] if len(parts) >= 2 else ""
        rows = {"q_proj": nq, "k_proj": nkv, "v_proj": nkv, "gate_proj": f, "up_proj": f}.get(mod)
        cols = {"o_proj": nq, "down_proj": f}.get(mod)
        if rows is not None:
            out[name] = np.ascontiguousarray(t[rank * rows:(rank + 1) * rows])
        elif cols is not None:
            if kind == "weight":
                w = cols // per_word
            elif kind in ("scales", "biases"):
                w = cols // gs
            else:
                out[name] = t
                continue
            out[name] = np.ascontiguousarray(t[:, rank * w:(rank + 1) * w])
        else:
            out[name] = t
    return out


_ST_NP = {"U32": np.uint32, "F16": np.float16, "BF16": np.uint16, "F32": np.float32, "I32": np.int32,
          "U8": np.uint8, "I64": np.int64, "U16": np.uint16}


def safetensors_write(path: str, tensors: dict, metadata: Optional[dict] = None, dtypes: Optional[dict] = None):
    """Write numpy arrays (name -> array) with an optional string metadata map.
    dtypes overrides the stored dtype per name (e.g. "BF16" for raw uint16 bits)."""
    names = list(tensors)
    arrs = [np.ascontiguousarray(tensors[n]) for n in names]
    rev = {np.dtype(np.uint32): "U32", np.dtype(np.float16): "F16", np.dtype(np.float32): "F32",
           np.dtype(np.int32): "I32", np.dtype(np.uint8): "U8", np.dtype(np.int64): "I64",
           np.dtype(np.uint16): "U16"}
    dts = [(dtypes or {}).get(n) or rev[a.dtype] for n, a in zip(names, arrs)]
    shapes = [(C.c_int64 * max(a.ndim, 1))(*a.shape) for a in arrs]
    meta = metadata or {}
    check(lib.nmx_safetensors_write(
        path.encode(), len(names), (C.c_char_p * len(names))(*[n.encode() for n in names]),
        (C.c_char_p * len(names))(*[d.encode() for d in dts]),
        (C.POINTER(C.c_int64) * len(names))(*[C.cast(sh, C.POINTER(C.c_int64)) for sh in shapes]),
        (_i * len(names))(*[a.ndim for a in arrs]), (_vp * len(names))(*[a.ctypes.data for a in arrs]),
        len(meta), (C.c_char_p * len(meta))(*[k.encode() for k in meta]),
        (C.c_char_p * len(meta))(*[str(v).encode() for v in meta.values()])))


class SafetensorsFile:
    """nmx_safetensors_t: read-only view of a .safetensors file."""

    def __init__(self, path: str):
        h = _vp()
        check(lib.nmx_safetensors_open(path.encode(), C.byref(h)))
        self.h = h

    def tensors(self) -> dict:
        out = {}
        for i in range(lib.nmx_safetensors_count(self.h)):
            name = C.create_string_buffer(1024)
            dt = C.create_string_buffer(8)
            shape = (C.c_int64 * 8)()
            nd, nb = C.c_int(), C.c_uint64()
            check(lib.nmx_safetensors_info(self.h, i, name, 1024, dt, shape, C.byref(nd), C.byref(nb)))
            out[name.value.decode()] = (dt.value.decode(), tuple(shape[:nd.value]), nb.value)
        return out

    def read(self, name: str) -> np.ndarray:
        dt, shape, nb = self.tensors()[name]
        arr = np.empty(shape, dtype=_ST_NP[dt])
        check(lib.nmx_safetensors_read(self.h, name.encode(), arr.ctypes.data, nb))
        return arr

    def metadata(self, key: str) -> Optional[str]:
        n = lib.nmx_safetensors_metadata(self.h, key.encode(), None, 0)
        if n < 0:
            return None
        buf = C.create_string_buffer(n + 1)
        lib.nmx_safetensors_metadata(self.h, key.encode(), buf, n + 1)
        return buf.value.decode()

    def close(self):
        if self.h:
            lib.nmx_safetensors_close(self.h)
            self.h = None

    def __del__(self, _finalizing=sys.is_finalizing):
        if not _finalizing():
            self.close()


def load_safetensors(model: "Model", path: str, tp_rank: int = 0, tp_size: int = 1):
    """nmx_model_load_safetensors: returns (tensors loaded, tensors skipped)"""
    n, k = C.c_int(), C.c_int()
    check(lib.nmx_model_load_safetensors(model.h, path.encode(), tp_rank, tp_size, C.byref(n), C.byref(k)))
    return n.value, k.value


def ssd_save_block(pool: "KVPool", block_id: int, hash20: bytes, token_count: int, model_name: str, cache_dir: str):
    check(lib.nmx_ssd_save_block(pool.h, block_id, hash20, token_count, model_name.encode(), cache_dir.encode()))


def ssd_load_block(pool: "KVPool", hash20: bytes, cache_dir: str, block_id: int) -> int:
    tc = C.c_int()
    check(lib.nmx_ssd_load_block(pool.h, hash20, cache_dir.encode(), block_id, C.byref(tc)))
    return tc.value
