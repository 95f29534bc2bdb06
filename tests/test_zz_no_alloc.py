"""The decode attention entry point that never allocates device memory.

Some hosts cannot let a library call allocate: an engine that reserves its
whole device budget at start-up and admits work against it, or one that
cannot afford the device synchronisation cudaMalloc/cudaFree can cause.
nmx_op_attn_paged_decode_noalloc keeps its scratch in a fixed array inside
the library instead. This file is collected last, so a run that stops at its
first failure has already run every other test; it also passes on its own in
a fresh process (its first call sets up the array's address).
"""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _case(torch, rng, lens, Hq=32, Hkv=8, D=128, BT=16):
    B = len(lens)
    maxb = max((l + BT - 1) // BT for l in lens)
    nb = B * maxb + 5
    tables = rng.permutation(nb)[:B * maxb].astype(np.int32).reshape(B, maxb)
    to16 = lambda a: torch.from_numpy(O.f32_to_f16bits(a).view(np.int16)).view(torch.float16).cuda()
    kp = to16(rng.standard_normal((nb, Hkv, BT, D), dtype=np.float32))
    vp = to16(rng.standard_normal((nb, Hkv, BT, D), dtype=np.float32))
    q = to16(rng.standard_normal((B, Hq, D), dtype=np.float32))
    return q, kp, vp, torch.from_numpy(tables).cuda(), torch.tensor(lens, dtype=torch.int32).cuda(), Hkv, D


def test_noalloc_matches_allocating_entry_point_twice():
    import torch
    from novamlx_b200 import nmx
    ctx = nmx.Context(0)
    rng = np.random.default_rng(21)
    # two calls in a row: the second must not see the first call's scratch
    for lens in ([33, 700, 5], [1, 2048, 129, 16]):
        q, kp, vp, tables, seq_lens, Hkv, D = _case(torch, rng, lens)
        ref = ctx.paged_decode_attention(q, kp, vp, tables, seq_lens, Hkv, D ** -0.5)
        got = ctx.paged_decode_attention_noalloc(q, kp, vp, tables, seq_lens, Hkv, D ** -0.5)
        torch.cuda.synchronize()
        g = got.float().cpu().numpy().reshape(len(lens), -1)
        r = ref.float().cpu().numpy().reshape(len(lens), -1)
        for b in range(len(lens)):
            assert O.max_rel_err(g[b], r[b]) <= 5e-3, (lens, b)


def test_noalloc_rejects_batches_beyond_its_scratch():
    import torch
    from novamlx_b200 import nmx
    ctx = nmx.Context(0)
    q, kp, vp, tables, seq_lens, Hkv, D = _case(torch, np.random.default_rng(0), [16])
    out = torch.empty_like(q)
    # 1<<20 rows x 8 kv heads of tickets alone exceed the fixed array; the
    # call is refused before anything is launched
    st = nmx.lib.nmx_op_attn_paged_decode_noalloc(ctx.h, q.data_ptr(), kp.data_ptr(), vp.data_ptr(),
                                                  tables.data_ptr(), seq_lens.data_ptr(), 1 << 20, 32, 8, D,
                                                  16, tables.shape[1], 0.1, out.data_ptr())
    assert st == nmx.NMX_ERR_UNSUPPORTED
    assert "scratch" in nmx.lib.nmx_last_error().decode()
