"""Second, independent restatement of the oracle's arithmetic in numpy.

Test infrastructure: used only to cross-check oracle/oracle.c on small
cases (two implementations of the same published rule must agree).
"""
import numpy as np


def quantize(w, bits=4, gs=64):
    w = np.asarray(w, np.float32)
    N, K = w.shape
    g = w.reshape(N, K // gs, gs)
    mn = g.min(axis=2)
    mx = g.max(axis=2)
    nb = np.float32((1 << bits) - 1)
    scale = ((mx - mn) / nb).astype(np.float32)
    bias = mn.astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.rint((g - bias[..., None]) / scale[..., None])
    q = np.where(scale[..., None] > 0, np.clip(q, 0, nb), 0).astype(np.uint32).reshape(N, K)
    vpw = 32 // bits
    qq = q.reshape(N, K // vpw, vpw)
    shifts = (np.arange(vpw, dtype=np.uint32) * bits)[None, None, :]
    packed = np.bitwise_or.reduce(qq << shifts, axis=2).astype(np.uint32)
    return packed, scale.astype(np.float16).view(np.uint16), bias.astype(np.float16).view(np.uint16)


def unpack(wq, K, bits):
    vpw = 32 // bits
    k = np.arange(K)
    words = wq[:, k // vpw]
    return ((words >> ((k % vpw) * bits).astype(np.uint32)) & ((1 << bits) - 1)).astype(np.uint8)


def dequantize(wq, s, b, bits=4, gs=64):
    N = wq.shape[0]
    K = wq.shape[1] * 32 // bits
    q = unpack(wq, K, bits).astype(np.float32)
    sf = s.view(np.float16).astype(np.float32)
    bf = b.view(np.float16).astype(np.float32)
    return q * np.repeat(sf, gs, axis=1) + np.repeat(bf, gs, axis=1)


def qmatmul(x16, wq, s, b, bits=4, gs=64):
    x = x16.view(np.float16).astype(np.float64)
    w = dequantize(wq, s, b, bits, gs).astype(np.float64)
    return (x @ w.T).astype(np.float16).view(np.uint16)


def attention(q16, k16, v16, Hq, Hkv, D, q_start, scale):
    q = q16.view(np.float16).astype(np.float64)
    k = k16.view(np.float16).astype(np.float64)
    v = v16.view(np.float16).astype(np.float64)
    T, S = q.shape[0], k.shape[0]
    rep = Hq // Hkv
    out = np.zeros_like(q)
    for t in range(T):
        last = min(q_start + t, S - 1)
        for h in range(Hq):
            kk = k[: last + 1, h // rep]
            sc = kk @ q[t, h] * scale
            p = np.exp(sc - sc.max())
            out[t, h] = (p @ v[: last + 1, h // rep]) / p.sum()
    return out.astype(np.float16).view(np.uint16)
