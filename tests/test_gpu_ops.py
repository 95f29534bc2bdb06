"""GPU parity of the op-level C ABI against the CPU oracle (same seeded
inputs). Tolerances (from the workload definition): integer work bit-exact;
bf16/f16 outputs max_rel_err = max|y-r|/max|r| <= 2e-2 vs the fp32
dequant reference (the kernels are far tighter; the asserted bounds below
are what they meet)."""
import json
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu
KAT = json.loads((Path(__file__).parent / "golden" / "kat.json").read_text())
TOL = 2e-2


@pytest.fixture(scope="module")
def env():
    import torch
    from novamlx_b200 import nmx
    ctx = nmx.Context(0)
    return torch, nmx, ctx


def dev(torch, a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.view(dtype)
    return t.cuda()


def u16(torch, a):
    return dev(torch, a.view(np.int16), torch.float16)


def host16(t):
    return t.view(__import__("torch").int16).cpu().numpy().view(np.uint16)


def test_quantize_bit_exact(env):
    torch, nmx, ctx = env
    rng = np.random.default_rng(0)
    for bits, gs in [(4, 64), (4, 32), (4, 128), (8, 64), (8, 32)]:
        w = rng.standard_normal((64, 512), dtype=np.float32) * 0.02
        w[5, :gs] = 0.25
        wq, s, b = ctx.quantize(dev(torch, w), gs, bits)
        torch.cuda.synchronize()
        rq, rs, rb = O.quantize(w, bits, gs)
        assert np.array_equal(wq.cpu().numpy().view(np.uint32), rq)
        assert np.array_equal(host16(s), rs)
        assert np.array_equal(host16(b), rb)
        wd = ctx.dequantize(wq, s, b, gs, bits)
        assert np.array_equal(wd.cpu().numpy(), O.dequantize(rq, rs, rb, bits, gs))


@pytest.mark.parametrize("i", range(len(KAT["quantize"])))
def test_quantize_kat_gpu(env, i):
    torch, nmx, ctx = env
    case = KAT["quantize"][i]
    w = np.array([case["w"]] * 16, dtype=np.float32)
    wq, s, b = ctx.quantize(dev(torch, w), case["group"], case["bits"])
    q = O.unpack(wq.cpu().numpy().view(np.uint32), w.shape[1], case["bits"])
    assert q[0].tolist() == case["q"]


def _qmm_case(torch, ctx, M, N, K, bits, gs, seed):
    rng = np.random.default_rng(seed)
    w = rng.standard_normal((N, K), dtype=np.float32) * 0.02
    wq, s, b = O.quantize(w, bits, gs)
    x = O.f32_to_f16bits(rng.standard_normal((M, K), dtype=np.float32))
    ref = O.f16bits_to_f32(O.qmatmul(x, wq, s, b, bits, gs))
    y = ctx.quantized_matmul(u16(torch, x), dev(torch, wq.view(np.int32)), u16(torch, s), u16(torch, b),
                             group_size=gs, bits=bits)
    got = O.f16bits_to_f32(host16(y))
    return got, ref


def test_qmatmul_kat(env):
    torch, nmx, ctx = env
    k = KAT["qmatmul"]
    w = np.tile(np.array(k["w_row"], np.float32), (k["rows"], 1))
    wq, s, b = O.quantize(w, k["bits"], k["group"])
    x = O.f32_to_f16bits(np.array([k["x"]], np.float32))
    y = ctx.quantized_matmul(u16(torch, x), dev(torch, wq.view(np.int32)), u16(torch, s), u16(torch, b),
                             group_size=k["group"], bits=k["bits"])
    assert np.all(O.f16bits_to_f32(host16(y)) == k["y"])


def test_qmatmul_c1_config(env):
    """x f16[4,4096] ~ N(0,1); W [4096,4096] ~ N(0,0.02) → Q4 g64; seed 0."""
    torch, nmx, ctx = env
    got, ref = _qmm_case(torch, ctx, 4, 4096, 4096, 4, 64, 0)
    assert O.max_rel_err(got, ref) <= 2e-3
    assert O.cosine(got, ref) > 0.99999


@pytest.mark.parametrize("M,N,K,bits,gs", [
    (1, 4096, 4096, 4, 64), (1, 1024, 4096, 4, 64), (2, 14336, 4096, 4, 64), (1, 4096, 14336, 4, 64),
    (3, 512, 1024, 4, 32), (5, 256, 2048, 4, 128), (8, 512, 512, 4, 64), (9, 256, 512, 4, 64),
    (16, 512, 1024, 4, 64), (32, 256, 512, 4, 64), (40, 128, 512, 4, 64),
    (1, 1024, 1024, 8, 64), (4, 512, 2048, 8, 32), (7, 256, 1024, 8, 128), (24, 256, 512, 8, 64),
    (1, 640, 3456, 4, 64),  # a TP8 down-proj shard (54 groups: ragged k-split)
    (8, 1024, 4096, 4, 64),  # eight activation rows, the most the few-row kernel takes
    (5, 512, 8192, 4, 128),  # g128: eight 128-k steps per warp
    (4, 256, 14336, 4, 32),  # g32: fourteen 128-k steps per warp
])
def test_qmatmul_shapes(env, M, N, K, bits, gs):
    torch, nmx, ctx = env
    got, ref = _qmm_case(torch, ctx, M, N, K, bits, gs, M * 7 + N + K)
    assert O.max_rel_err(got, ref) <= 2e-3, (M, N, K, bits, gs)


@pytest.mark.parametrize("M", [1, 2, 3, 4, 5, 8, 9, 13, 32])
@pytest.mark.parametrize("N,K", [(4096, 4096), (256, 512), (4096, 14336), (768, 512), (6144, 4096), (5120, 1024)])
def test_qmatmul_records(env, M, N, K):
    """The decode-record GEMV (the model's layout) equals the oracle."""
    torch, nmx, ctx = env
    rng = np.random.default_rng(M * 31 + N + K)
    w = rng.standard_normal((N, K), dtype=np.float32) * 0.02
    wq, s, b = O.quantize(w, 4, 64)
    x = O.f32_to_f16bits(rng.standard_normal((M, K), dtype=np.float32))
    ref = O.f16bits_to_f32(O.qmatmul(x, wq, s, b, 4, 64))
    rec = ctx.pack_records(dev(torch, wq.view(np.int32)), u16(torch, s), u16(torch, b))
    y = ctx.quantized_matmul_records(u16(torch, x), rec, N)
    got = O.f16bits_to_f32(host16(y))
    for m in range(M):
        assert O.max_rel_err(got[m], ref[m]) <= 2e-3, (m, M)


@pytest.mark.parametrize("M,N,K", [(64, 256, 512), (128, 512, 1024), (200, 768, 512), (333, 256, 2048),
                                   (130, 4096, 4096)])
def test_qmatmul_records_tensor_core_gemm(env, M, N, K):
    """Many rows go through the tcgen05 GEMM (weights dequantised to f16 in
    shared memory, f32 accumulation in TMEM): equals the oracle, ragged M."""
    torch, nmx, ctx = env
    rng = np.random.default_rng(M + 3 * N + K)
    w = rng.standard_normal((N, K), dtype=np.float32) * 0.02
    wq, s, b = O.quantize(w, 4, 64)
    x = O.f32_to_f16bits(rng.standard_normal((M, K), dtype=np.float32))
    ref = O.f16bits_to_f32(O.qmatmul(x, wq, s, b, 4, 64))
    rec = ctx.pack_records(dev(torch, wq.view(np.int32)), u16(torch, s), u16(torch, b))
    n0 = ctx.launches
    y = ctx.quantized_matmul_records(u16(torch, x), rec, N)
    got = O.f16bits_to_f32(host16(y))
    assert ctx.launches - n0 == 1  # one GEMM launch for all rows
    assert O.max_rel_err(got, ref) <= 2e-3, (M, N, K)
    assert O.cosine(got.ravel(), ref.ravel()) > 0.99999


@pytest.mark.parametrize("M,N,K", [(9, 4096, 4096), (16, 1024, 512), (33, 6144, 1024), (64, 4096, 4096),
                                   (80, 16384, 1024), (128, 1024, 2048), (100, 512, 14336), (21, 6144, 4096),
                                   (21, 4096, 14336), (32, 55296, 5120), (112, 4096, 4096), (21, 896, 5120),
                                   (40, 384, 1024), (17, 128, 4096), (64, 1280, 27648), (65, 1792, 5120)])
def test_qmatmul_records_decode_batch_gemm(env, M, N, K):
    """9..112 rows go through the decode-batch tcgen05 GEMM (weights as the
    MMA's rows, rows of x as its columns, K split over the SMs with a
    deterministic last-arriver sum; 113..128 rows through the prefill GEMM),
    odd tile counts and a single tile included: equals the oracle in one
    launch, and repeated calls agree bit for bit."""
    torch, nmx, ctx = env
    rng = np.random.default_rng(7 * M + N + K)
    w = rng.standard_normal((N, K), dtype=np.float32) * 0.02
    wq, s, b = O.quantize(w, 4, 64)
    x = O.f32_to_f16bits(rng.standard_normal((M, K), dtype=np.float32))
    ref = O.f16bits_to_f32(O.qmatmul(x, wq, s, b, 4, 64))
    rec = ctx.pack_records(dev(torch, wq.view(np.int32)), u16(torch, s), u16(torch, b))
    xd = u16(torch, x)
    n0 = ctx.launches
    y = ctx.quantized_matmul_records(xd, rec, N)
    assert ctx.launches - n0 == 1
    got = O.f16bits_to_f32(host16(y))
    assert O.max_rel_err(got, ref) <= 2e-3, (M, N, K)
    assert O.cosine(got.ravel(), ref.ravel()) > 0.99999
    again = host16(ctx.quantized_matmul_records(xd, rec, N))
    assert np.array_equal(again, host16(y))


@pytest.mark.parametrize("M,N,K", [(1, 6144, 4096), (1, 4096, 4096), (3, 5120, 1024), (1, 512, 640 // 128 * 128)])
def test_qmatmul_records_deterministic(env, M, N, K):
    """Split tile groups are summed in a fixed order: repeated calls agree bit for bit."""
    torch, nmx, ctx = env
    rng = np.random.default_rng(N + K + M)
    w = rng.standard_normal((N, K), dtype=np.float32) * 0.02
    wq, s, b = O.quantize(w, 4, 64)
    x = u16(torch, O.f32_to_f16bits(rng.standard_normal((M, K), dtype=np.float32)))
    rec = ctx.pack_records(dev(torch, wq.view(np.int32)), u16(torch, s), u16(torch, b))
    ys = [host16(ctx.quantized_matmul_records(x, rec, N)) for _ in range(4)]
    for y in ys[1:]:
        assert np.array_equal(y, ys[0])


@pytest.mark.parametrize("M,N,K", [(1, 6144, 4096), (3, 4096, 14336), (8, 512, 1024)])
def test_qmatmul_records_unaligned_activations(env, M, N, K):
    """Activations at an address that is not 16-byte aligned are staged
    element by element: the same bits as the aligned call."""
    torch, nmx, ctx = env
    rng = np.random.default_rng(N + 3 * K + M)
    w = rng.standard_normal((N, K), dtype=np.float32) * 0.02
    wq, s, b = O.quantize(w, 4, 64)
    xd = u16(torch, O.f32_to_f16bits(rng.standard_normal((M, K), dtype=np.float32)))
    buf = torch.zeros(M * K + 8, dtype=xd.dtype, device=xd.device)
    xm = buf[1:1 + M * K].view(M, K)
    xm.copy_(xd)
    assert xm.data_ptr() % 16 != 0
    rec = ctx.pack_records(dev(torch, wq.view(np.int32)), u16(torch, s), u16(torch, b))
    y0 = host16(ctx.quantized_matmul_records(xd, rec, N))
    y1 = host16(ctx.quantized_matmul_records(xm, rec, N))
    assert np.array_equal(y0, y1)


def test_qmatmul_records_rejects_tiny(env):
    """Fewer than eight (tile group, block) units: not served by the records kernel."""
    torch, nmx, ctx = env
    wq, s, b = O.quantize(np.ones((16, 128), np.float32), 4, 64)
    rec = ctx.pack_records(dev(torch, wq.view(np.int32)), u16(torch, s), u16(torch, b))
    x = u16(torch, O.f32_to_f16bits(np.ones((1, 128), np.float32)))
    with pytest.raises(nmx.NmxError) as e:
        ctx.quantized_matmul_records(x, rec, 16)
    assert e.value.status == nmx.NMX_ERR_UNSUPPORTED


def test_qmatmul_bf16(env):
    torch, nmx, ctx = env
    rng = np.random.default_rng(4)
    M, N, K, bits, gs = 3, 512, 1024, 4, 64
    w = rng.standard_normal((N, K), dtype=np.float32) * 0.02
    wq, s, b = O.quantize(w, bits, gs, sdt=O.BF16)
    xf = rng.standard_normal((M, K), dtype=np.float32) * 3
    xf[1] *= 5e4  # exercises the power-of-two range guard of the f16 MMA operand
    x = dev(torch, xf).to(torch.bfloat16)
    xb = x.view(torch.int16).cpu().numpy().view(np.uint16)
    ref = O.bf16bits_to_f32(O.qmatmul(xb, wq, s, b, bits, gs, dt=O.BF16))
    y = ctx.quantized_matmul(x, dev(torch, wq.view(np.int32)), dev(torch, s.view(np.int16), torch.bfloat16),
                             dev(torch, b.view(np.int16), torch.bfloat16), group_size=gs, bits=bits)
    got = y.float().cpu().numpy()
    for m in range(M):
        assert O.max_rel_err(got[m], ref[m]) <= 1e-2


def test_qmatmul_rejects_bad_shapes(env):
    torch, nmx, ctx = env
    x = torch.zeros((1, 100), dtype=torch.float16, device="cuda")
    w = torch.zeros((16, 100 // 8), dtype=torch.int32, device="cuda")
    s = torch.zeros((16, 1), dtype=torch.float16, device="cuda")
    with pytest.raises(nmx.NmxError) as e:
        ctx.quantized_matmul(x, w, s, s, group_size=64, bits=4)
    assert e.value.status == nmx.NMX_ERR_UNSUPPORTED
    with pytest.raises(nmx.NmxError):
        ctx.quantized_matmul(x[:, :64].contiguous(), w[:, :8].contiguous(), s, s, group_size=64, bits=3)


@pytest.mark.parametrize("M,H", [(5, 4096), (32, 5120), (3, 8192), (2, 24576), (4, 1000)])
def test_rmsnorm(env, M, H):
    """Vectorised rows (H % 8 == 0: one or two 16-byte chunks per thread)
    and the scalar fallback (H = 1000)."""
    torch, nmx, ctx = env
    rng = np.random.default_rng(2)
    x = O.f32_to_f16bits(rng.standard_normal((M, H), dtype=np.float32) * 3)
    g = O.f32_to_f16bits(1 + 0.1 * rng.standard_normal(H, dtype=np.float32))
    y = host16(ctx.rms_norm(u16(torch, x), u16(torch, g), 1e-5))
    ref = O.rmsnorm(x, g, 1e-5)
    d = np.abs(O.f16bits_to_f32(y) - O.f16bits_to_f32(ref))
    assert np.max(d) <= 2 ** -9 * np.max(np.abs(O.f16bits_to_f32(ref)))


def test_argmax_bit_exact(env):
    torch, nmx, ctx = env
    rng = np.random.default_rng(8)
    V = 128256
    lg = rng.standard_normal((6, V)).astype(np.float32)
    lg[1, 77] = lg[1, 100000] = 50.0  # tie → lowest index
    lg[2, :] = 1.0                    # all equal → 0
    lg[3, V - 1] = 99.0
    for dt in (torch.float32, torch.float16, torch.bfloat16):
        t = dev(torch, lg).to(dt)
        got = ctx.argmax(t).cpu().numpy()
        ref = O.argmax(t.float().cpu().numpy())
        assert np.array_equal(got, ref)
        assert got[1] == 77 and got[2] == 0 and got[3] == V - 1


def test_penalized_argmax(env):
    torch, nmx, ctx = env
    rng = np.random.default_rng(9)
    V = 32000
    lg = rng.standard_normal((4, V)).astype(np.float32)
    recent = rng.integers(0, V, (4, 64)).astype(np.int32)
    recent[0, :10] = int(np.argmax(lg[0]))  # penalise the winner heavily
    n = np.array([64, 10, 0, 33], np.int32)
    got = ctx.penalized_argmax(dev(torch, lg), dev(torch, recent), dev(torch, n), 0.7).cpu().numpy()
    assert np.array_equal(got, O.penalized_argmax(lg, recent, n, 0.7))


@pytest.mark.parametrize("D,gs,bits,N", [(128, 64, 4, 300), (64, 32, 8, 77), (96, 32, 4, 50), (256, 64, 8, 17)])
def test_quantized_sdpa_reference_semantics(env, D, gs, bits, N):
    """The reference's only GPU kernel (FusedQuantizedSDPA), same inputs."""
    torch, nmx, ctx = env
    rng = np.random.default_rng(D + N)
    B, Hq, Hkv = 2, 8, 2
    q = O.f32_to_f16bits(rng.standard_normal((B, Hq, 1, D), dtype=np.float32))
    kf = rng.standard_normal((B * Hkv * N, D), dtype=np.float32)
    vf = rng.standard_normal((B * Hkv * N, D), dtype=np.float32)
    kw, ks, kb = O.quantize(kf, bits, gs)
    vw, vs, vb = O.quantize(vf, bits, gs)
    sh4 = lambda a: a.reshape(B, Hkv, N, -1)
    ref = O.quantized_sdpa(q.reshape(B * Hq, 1, D), *(a.reshape(B * Hkv, N, -1) for a in (kw, ks, kb, vw, vs, vb)),
                           Hq // Hkv, D ** -0.5, gs, bits)
    out = ctx.fused_quantized_sdpa(u16(torch, q), dev(torch, sh4(kw).view(np.int32)), u16(torch, sh4(ks)),
                                   u16(torch, sh4(kb)), dev(torch, sh4(vw).view(np.int32)), u16(torch, sh4(vs)),
                                   u16(torch, sh4(vb)), D ** -0.5, gs, bits, Hkv)
    got = O.f16bits_to_f32(host16(out)).reshape(B * Hq, D)
    assert O.max_rel_err(got, O.f16bits_to_f32(ref).reshape(B * Hq, D)) <= 5e-3


def test_quantized_sdpa_guards(env):
    torch, nmx, ctx = env
    q = torch.zeros((1, 2, 2, 128), dtype=torch.float16, device="cuda")  # L = 2
    z = torch.zeros((1, 1, 4, 64), dtype=torch.int32, device="cuda")
    s = torch.zeros((1, 1, 4, 2), dtype=torch.float16, device="cuda")
    assert ctx.fused_quantized_sdpa(q, z, s, s, z, s, s, 0.1, 64, 4, 1) is None
    q1 = torch.zeros((1, 2, 1, 80), dtype=torch.float16, device="cuda")  # D = 80
    assert ctx.fused_quantized_sdpa(q1, z, s, s, z, s, s, 0.1, 16, 4, 1) is None


@pytest.mark.parametrize("lens", [[1], [17, 300, 2048], [16, 32, 5, 4095]])
def test_paged_decode_attention(env, lens):
    """Paged decode attention equals contiguous attention over the gathered
    pages, for shuffled (non-contiguous) block tables."""
    torch, nmx, ctx = env
    rng = np.random.default_rng(sum(lens))
    B, Hq, Hkv, D, BT = len(lens), 32, 8, 128, 16
    maxb = max((l + BT - 1) // BT for l in lens)
    nb = B * maxb + 3
    perm = rng.permutation(nb).astype(np.int32)
    tables = perm[:B * maxb].reshape(B, maxb)
    kp = O.f32_to_f16bits(rng.standard_normal((nb, Hkv, BT, D), dtype=np.float32))
    vp = O.f32_to_f16bits(rng.standard_normal((nb, Hkv, BT, D), dtype=np.float32))
    q = O.f32_to_f16bits(rng.standard_normal((B, Hq, D), dtype=np.float32))
    out = ctx.paged_decode_attention(u16(torch, q), u16(torch, kp), u16(torch, vp), dev(torch, tables),
                                     dev(torch, np.array(lens, np.int32)), Hkv, D ** -0.5)
    got = O.f16bits_to_f32(host16(out))
    for b, L in enumerate(lens):
        blocks = tables[b, :(L + BT - 1) // BT]
        k = kp[blocks].transpose(0, 2, 1, 3).reshape(-1, Hkv, D)[:L]
        v = vp[blocks].transpose(0, 2, 1, 3).reshape(-1, Hkv, D)[:L]
        ref = O.f16bits_to_f32(O.attention(q[b][None], k, v, Hq, Hkv, D, L - 1, D ** -0.5))[0]
        assert O.max_rel_err(got[b], ref) <= 5e-3, (b, L)
