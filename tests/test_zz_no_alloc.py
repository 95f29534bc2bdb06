"""The decode attention entry point that never allocates device memory.

Some hosts cannot let a library call allocate: an engine that reserves its
whole device budget at start-up and admits work against it, or one that
cannot afford the device synchronisation cudaMalloc/cudaFree can cause.
nmx_op_attn_paged_decode_noalloc keeps its scratch (the per-row descriptors)
in a fixed array inside the library instead. This file is collected last, so
a run that stops at its first failure has already run every other test; it
also passes on its own in a fresh process (its first call sets up the
array's address).
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
    # two calls in a row, the larger batch first: the array keeps the first
    # call's four row descriptors, so a second call that read past its own
    # three rows, or did not rewrite them, would give different bits
    for lens in ([1, 2048, 129, 16], [33, 700, 5]):
        q, kp, vp, tables, seq_lens, Hkv, D = _case(torch, rng, lens)
        ref = ctx.paged_decode_attention(q, kp, vp, tables, seq_lens, Hkv, D ** -0.5)
        got = ctx.paged_decode_attention_noalloc(q, kp, vp, tables, seq_lens, Hkv, D ** -0.5)
        torch.cuda.synchronize()
        # same kernel, same key splits: the same bits
        assert torch.equal(got.view(torch.int16), ref.view(torch.int16)), lens
        # and the allocating entry point is the oracle's attention
        g = got.float().cpu().numpy().reshape(len(lens), -1)
        kpc, vpc = kp.cpu().numpy().view(np.uint16), vp.cpu().numpy().view(np.uint16)
        tab = tables.cpu().numpy()
        for b, n in enumerate(lens):
            j = np.arange(n)
            kk, vv = kpc[tab[b, j // 16], :, j % 16], vpc[tab[b, j // 16], :, j % 16]
            qq = q[b:b + 1].cpu().numpy().view(np.uint16)
            r = O.f16bits_to_f32(O.attention(qq, kk, vv, 32, Hkv, D, n - 1, D ** -0.5)).reshape(-1)
            assert O.max_rel_err(g[b], r) <= 2e-2, (lens, b)


def test_noalloc_rejects_batches_beyond_its_scratch():
    import torch
    from novamlx_b200 import nmx
    ctx = nmx.Context(0)
    q, kp, vp, tables, seq_lens, Hkv, D = _case(torch, np.random.default_rng(0), [16])
    out = torch.empty_like(q)
    # 32769 rows need 8 bytes of descriptors each, one row more than the
    # fixed array holds; the call is refused before anything is launched
    st = nmx.lib.nmx_op_attn_paged_decode_noalloc(ctx.h, q.data_ptr(), kp.data_ptr(), vp.data_ptr(),
                                                  tables.data_ptr(), seq_lens.data_ptr(), 32769, 32, 8, D,
                                                  16, tables.shape[1], 0.1, out.data_ptr())
    assert st == nmx.NMX_ERR_UNSUPPORTED
    assert "scratch" in nmx.lib.nmx_last_error().decode()
