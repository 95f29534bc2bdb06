// Attention over the paged KV pool (GQA, causal), plus the reference's
// quantized-KV single-query kernel restated for sm_100a.
//
// Paged layout per layer: K[num_blocks][Hkv][BT][D], V likewise, fp16. A
// CTA owns (query row, kv head, key split) and serves every q head of the
// GQA group, so each K/V block is read once per kv head. Long contexts are
// split over several CTAs whose partial (o, max, sum) are combined by the
// last CTA to finish (an atomic ticket per (row, kv head), reset by that
// CTA), which needs no grid-wide wait.
//
// The decode variant (FUSED) also applies RoPE to q and to the new key and
// appends the new k/v to its page: the CTA whose split contains the new
// position writes them before it reads the block, so the KV append and the
// attention are one launch. Replaces MLXFast.scaledDotProductAttention over
// KVCacheSimple (mlx-swift-lm; reached from
// Sources/NovaMLXEngine/FusedBatchScheduler.swift:1215) and the separate
// KVCache.update of the reference's batched decode
// (Sources/NovaMLXEngine/FusedBatchDecode.swift:7-147).
#include "common.cuh"
#include "kernels.h"

namespace nmx {

namespace {

constexpr int kAttnThreads = 128;
constexpr int kAttnWarps = 4;
constexpr int kMaxRep = 8;

__device__ __forceinline__ void rope_pair(float a, float b, float ang, float& ra, float& rb) {
  float sn, cs;
  sincosf(ang, &sn, &cs);
  ra = a * cs - b * sn;
  rb = b * cs + a * sn;
}

template <int D, bool FUSED>
__global__ void __launch_bounds__(kAttnThreads) paged_attn_kernel(AttnArgs a) {
  constexpr int BT = 16;
  constexpr int KST = D / 2 + 2;  // K row stride in 32-bit words (bank-conflict free)
  constexpr int DPL = D / 32;     // dims per lane in P·V
  constexpr int NH = kMaxRep / kAttnWarps;
  __shared__ float q_s[kMaxRep][D];
  __shared__ __align__(16) uint32_t k_s[BT * KST];
  __shared__ __align__(16) uint32_t v_s[BT * KST];
  __shared__ float p_s[kMaxRep][BT];
  __shared__ int s_last;

  const int split = blockIdx.x, h = blockIdx.y, row = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int Hq = a.Hq, Hkv = a.Hkv, rep = Hq / Hkv, S = gridDim.x;

  grid_wait();
  const int seq = a.tok_seq[row];
  const int pos = a.tok_pos[row];
  const int L = pos + 1;
  const int nblk = (L + BT - 1) / BT;
  const int bps = (nblk + S - 1) / S;
  const int b0 = split * bps;
  const int b1 = min(nblk, b0 + bps);
  const int* bt = a.block_tables + long(seq) * a.max_blocks;
  half* Kc = reinterpret_cast<half*>(a.k_cache);
  half* Vc = reinterpret_cast<half*>(a.v_cache);
  const half* Q = reinterpret_cast<const half*>(a.q) + long(row) * a.ldq;

  // ---- q (optionally roped), pre-scaled, fp32 in shared memory
  if (FUSED) {
    for (int i = tid; i < rep * (D / 2); i += kAttnThreads) {
      const int hi = i / (D / 2), d = i % (D / 2);
      const int hq = h * rep + hi;
      const float x0 = __half2float(Q[hq * D + d]), x1 = __half2float(Q[hq * D + d + D / 2]);
      float r0, r1;
      rope_pair(x0, x1, float(pos) * a.inv_freq[d], r0, r1);
      q_s[hi][d] = rnd<half>(r0) * a.scale;
      q_s[hi][d + D / 2] = rnd<half>(r1) * a.scale;
    }
    // append this row's k/v when its position falls in this split
    if (pos >= b0 * BT && pos < b1 * BT) {
      const long slot = (long(bt[pos / BT]) * Hkv + h) * BT + pos % BT;
      const half* kr = Q + (Hq + h) * D;
      const half* vr = Q + (Hq + Hkv + h) * D;
      for (int d = tid; d < D / 2; d += kAttnThreads) {
        float r0, r1;
        rope_pair(__half2float(kr[d]), __half2float(kr[d + D / 2]), float(pos) * a.inv_freq[d], r0, r1);
        Kc[slot * D + d] = __float2half_rn(r0);
        Kc[slot * D + d + D / 2] = __float2half_rn(r1);
      }
      for (int d = tid; d < D; d += kAttnThreads) Vc[slot * D + d] = vr[d];
    }
  } else {
    for (int i = tid; i < rep * D; i += kAttnThreads) {
      const int hi = i / D, d = i % D;
      q_s[hi][d] = __half2float(Q[(h * rep + hi) * D + d]) * a.scale;
    }
  }
  __syncthreads();

  float m_run[NH], l_run[NH], o[NH][DPL];
#pragma unroll
  for (int j = 0; j < NH; ++j) {
    m_run[j] = -INFINITY;
    l_run[j] = 0.f;
#pragma unroll
    for (int e = 0; e < DPL; ++e) o[j][e] = 0.f;
  }

  const int tok = lane >> 1, hv = lane & 1;
  for (int b = b0; b < b1; ++b) {
    const long base = (long(bt[b]) * Hkv + h) * BT * D;  // in halves
    // stage K and V blocks (BT*D halves each) with 16-byte loads
    {
      const uint4* ks = reinterpret_cast<const uint4*>(Kc + base);
      const uint4* vs = reinterpret_cast<const uint4*>(Vc + base);
      constexpr int NV = BT * D / 8;
      for (int i = tid; i < NV; i += kAttnThreads) {
        const int r = i / (D / 8), c = i % (D / 8);
        const uint4 kv = ks[i], vv = vs[i];
        uint32_t* kd = k_s + r * KST + c * 4;
        uint32_t* vd = v_s + r * KST + c * 4;
        kd[0] = kv.x; kd[1] = kv.y; kd[2] = kv.z; kd[3] = kv.w;
        vd[0] = vv.x; vd[1] = vv.y; vd[2] = vv.z; vd[3] = vv.w;
      }
    }
    __syncthreads();
    const bool valid = (b * BT + tok) <= pos;
#pragma unroll
    for (int j = 0; j < NH; ++j) {
      const int hi = warp + j * kAttnWarps;
      if (hi < rep) {
        // score of token `tok`, half of the words per lane (interleaved)
        float sc = 0.f;
#pragma unroll 8
        for (int w = 0; w < D / 4; ++w) {
          const int word = 2 * w + hv;
          const __half2 kk = *reinterpret_cast<const __half2*>(k_s + tok * KST + word);
          const float2 kf = __half22float2(kk);
          sc = fmaf(q_s[hi][2 * word], kf.x, fmaf(q_s[hi][2 * word + 1], kf.y, sc));
        }
        sc += __shfl_xor_sync(0xffffffffu, sc, 1);
        sc = valid ? sc : -INFINITY;
        float mb = sc;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, off));
        const float m_new = fmaxf(m_run[j], mb);
        const float f = expf(m_run[j] - m_new);
        const float p = valid ? expf(sc - m_new) : 0.f;
        float ps = hv == 0 ? p : 0.f;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
        l_run[j] = l_run[j] * f + ps;
        m_run[j] = m_new;
        if (hv == 0) p_s[hi][tok] = p;
        __syncwarp();
#pragma unroll
        for (int e = 0; e < DPL; ++e) o[j][e] *= f;
#pragma unroll
        for (int t2 = 0; t2 < BT; ++t2) {
          const float pt = p_s[hi][t2];
#pragma unroll
          for (int e = 0; e < DPL; e += 2) {
            const int word = lane + (e / 2) * 32;
            const float2 vf = __half22float2(*reinterpret_cast<const __half2*>(v_s + t2 * KST + word));
            o[j][e] = fmaf(pt, vf.x, o[j][e]);
            o[j][e + 1] = fmaf(pt, vf.y, o[j][e + 1]);
          }
        }
        __syncwarp();
      }
    }
    __syncthreads();
  }
  grid_launch_dependents();

  half* Out = reinterpret_cast<half*>(a.out) + long(row) * Hq * D;
  if (S == 1) {
#pragma unroll
    for (int j = 0; j < NH; ++j) {
      const int hi = warp + j * kAttnWarps;
      if (hi < rep) {
        const int hq = h * rep + hi;
        const float inv = l_run[j] > 0.f ? 1.0f / l_run[j] : 0.f;
#pragma unroll
        for (int e = 0; e < DPL; e += 2) {
          const int d = 2 * (lane + (e / 2) * 32);
          *reinterpret_cast<__half2*>(Out + hq * D + d) =
              __floats2half2_rn(o[j][e] * inv, o[j][e + 1] * inv);
        }
      }
    }
    return;
  }

  // ---- split-KV: publish partials; the last CTA of (row, h) combines
#pragma unroll
  for (int j = 0; j < NH; ++j) {
    const int hi = warp + j * kAttnWarps;
    if (hi < rep) {
      const int hq = h * rep + hi;
      const long pb = (long(row) * Hq + hq) * S + split;
#pragma unroll
      for (int e = 0; e < DPL; e += 2) {
        const int d = 2 * (lane + (e / 2) * 32);
        *reinterpret_cast<float2*>(a.part_o + pb * D + d) = make_float2(o[j][e], o[j][e + 1]);
      }
      if (lane == 0) *reinterpret_cast<float2*>(a.part_ml + pb * 2) = make_float2(m_run[j], l_run[j]);
    }
  }
  __threadfence();
  __syncthreads();
  unsigned* ctr = a.counters + long(row) * Hkv + h;
  if (tid == 0) s_last = (atomicAdd(ctr, 1u) == unsigned(S - 1)) ? 1 : 0;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int i = tid; i < rep * D; i += kAttnThreads) {
    const int hi = i / D, d = i % D;
    const int hq = h * rep + hi;
    const long pb = (long(row) * Hq + hq) * S;
    float mx = -INFINITY;
    for (int s2 = 0; s2 < S; ++s2) {
      const float2 ml = __ldcg(reinterpret_cast<const float2*>(a.part_ml + (pb + s2) * 2));
      if (ml.y > 0.f) mx = fmaxf(mx, ml.x);
    }
    float num = 0.f, den = 0.f;
    for (int s2 = 0; s2 < S; ++s2) {
      const float2 ml = __ldcg(reinterpret_cast<const float2*>(a.part_ml + (pb + s2) * 2));
      if (ml.y > 0.f) {
        const float w = expf(ml.x - mx);
        den = fmaf(ml.y, w, den);
        num = fmaf(__ldcg(a.part_o + (pb + s2) * D + d), w, num);
      }
    }
    Out[hq * D + d] = __float2half_rn(den > 0.f ? num / den : 0.f);
  }
  if (tid == 0) *ctr = 0u;
}

template <int D>
__global__ void __launch_bounds__(128) rope_append_kernel(half* qkv, long ldq, int Hq, int Hkv,
                                                          const int* tok_seq, const int* tok_pos,
                                                          const int* block_tables, int max_blocks,
                                                          int BT, half* Kc, half* Vc,
                                                          const float* inv_freq, half* q_out,
                                                          long ldqo) {
  grid_wait();
  const int row = blockIdx.x;
  const int seq = tok_seq[row], pos = tok_pos[row];
  half* r = qkv + long(row) * ldq;
  half* qo = q_out + long(row) * ldqo;
  const long slot0 = long(block_tables[long(seq) * max_blocks + pos / BT]) * Hkv;
  for (int i = threadIdx.x; i < (Hq + Hkv) * (D / 2); i += blockDim.x) {
    const int hh = i / (D / 2), d = i % (D / 2);
    float r0, r1;
    const half* src = r + hh * D;
    rope_pair(__half2float(src[d]), __half2float(src[d + D / 2]), float(pos) * inv_freq[d], r0, r1);
    if (hh < Hq) {
      qo[hh * D + d] = __float2half_rn(r0);
      qo[hh * D + d + D / 2] = __float2half_rn(r1);
    } else {
      const int kh = hh - Hq;
      const long slot = ((slot0 + kh) * BT + pos % BT) * D;
      Kc[slot + d] = __float2half_rn(r0);
      Kc[slot + d + D / 2] = __float2half_rn(r1);
    }
  }
  for (int i = threadIdx.x; i < Hkv * D; i += blockDim.x) {
    const int kh = i / D, d = i % D;
    const long slot = ((slot0 + kh) * BT + pos % BT) * D;
    Vc[slot + d] = r[(Hq + Hkv + kh) * D + d];
  }
  grid_launch_dependents();
}

// The reference kernel's semantics (FusedQuantizedSDPA.swift:17-135): per
// query row, keys i <= N - L + l, K/V dequantised on the fly. Four warps
// stride the keys; each lane owns D/32 consecutive dims; the warps' online
// softmax states are merged at the end.
template <typename T, int DPL>
__global__ void __launch_bounds__(128) qsdpa_kernel(const T* q, const uint32_t* kw, const T* ks,
                                                    const T* kb, const uint32_t* vw, const T* vs,
                                                    const T* vb, int gqa, int N, int L, float scale,
                                                    int gs, int bits, T* out) {
  constexpr int D = DPL * 32;
  __shared__ float s_m[4], s_l[4];
  __shared__ float s_o[4][D];
  grid_wait();
  const int bh = blockIdx.x, l = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kvh = bh / gqa;
  const int vpw = 32 / bits;
  const uint32_t mask = (1u << bits) - 1u;
  const int wstride = D * bits / 32, sstride = D / gs;
  float qv[DPL], o[DPL];
#pragma unroll
  for (int j = 0; j < DPL; ++j) {
    qv[j] = scale * tof<T>(q[(long(bh) * L + l) * D + lane * DPL + j]);
    o[j] = 0.f;
  }
  float mx = -1e30f, sum = 0.f;
  for (int i = warp; i < N; i += 4) {
    if (!(i <= N - L + l)) continue;
    const long kr = long(kvh) * N + i;
    float sc = 0.f;
#pragma unroll
    for (int j = 0; j < DPL; ++j) {
      const int d = lane * DPL + j;
      const float sv = tof<T>(ks[kr * sstride + d / gs]), bv = tof<T>(kb[kr * sstride + d / gs]);
      const float kv = float((kw[kr * wstride + d / vpw] >> ((d % vpw) * bits)) & mask) * sv + bv;
      sc = fmaf(qv[j], kv, sc);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) sc += __shfl_xor_sync(0xffffffffu, sc, off);
    const float nm = fmaxf(mx, sc);
    const float f = expf(mx - nm), e = expf(sc - nm);
    mx = nm;
    sum = sum * f + e;
#pragma unroll
    for (int j = 0; j < DPL; ++j) {
      const int d = lane * DPL + j;
      const float sv = tof<T>(vs[kr * sstride + d / gs]), bv = tof<T>(vb[kr * sstride + d / gs]);
      const float dv = float((vw[kr * wstride + d / vpw] >> ((d % vpw) * bits)) & mask) * sv + bv;
      o[j] = fmaf(o[j], f, e * dv);
    }
  }
  if (lane == 0) {
    s_m[warp] = mx;
    s_l[warp] = sum;
  }
#pragma unroll
  for (int j = 0; j < DPL; ++j) s_o[warp][lane * DPL + j] = o[j];
  __syncthreads();
  grid_launch_dependents();
  for (int d = threadIdx.x; d < D; d += 128) {
    float m = -1e30f;
    for (int w = 0; w < 4; ++w) m = fmaxf(m, s_m[w]);
    float den = 0.f, num = 0.f;
    for (int w = 0; w < 4; ++w) {
      const float f = expf(s_m[w] - m);
      den = fmaf(s_l[w], f, den);
      num = fmaf(s_o[w][d], f, num);
    }
    out[(long(bh) * L + l) * D + d] = fromf<T>(den == 0.f ? num : num / den);
  }
}

}  // namespace

nmx_status_t paged_attention(Ctx* c, const AttnArgs& a, bool fused) {
  NMX_CHECK(a.BT == 16, NMX_ERR_UNSUPPORTED, "paged attention: block size must be 16 tokens");
  NMX_CHECK(a.Hkv > 0 && a.Hq % a.Hkv == 0 && a.Hq / a.Hkv <= kMaxRep, NMX_ERR_UNSUPPORTED,
            "paged attention: q heads per kv head must be <= 8");
  NMX_CHECK(a.splits >= 1, NMX_ERR_INVALID, "paged attention: splits >= 1");
  if (a.T == 0) return NMX_OK;
  dim3 grid(a.splits, a.Hkv, a.T);
  if (a.D == 128) {
    return fused ? launch(c, paged_attn_kernel<128, true>, grid, dim3(kAttnThreads), 0, a)
                 : launch(c, paged_attn_kernel<128, false>, grid, dim3(kAttnThreads), 0, a);
  } else if (a.D == 64) {
    return fused ? launch(c, paged_attn_kernel<64, true>, grid, dim3(kAttnThreads), 0, a)
                 : launch(c, paged_attn_kernel<64, false>, grid, dim3(kAttnThreads), 0, a);
  }
  NMX_CHECK(false, NMX_ERR_UNSUPPORTED, "paged attention: head_dim must be 64 or 128");
}

nmx_status_t rope_append(Ctx* c, void* qkv, long ldq, int T, int Hq, int Hkv, int D,
                         const int* tok_seq, const int* tok_pos, const int* block_tables,
                         int max_blocks, int BT, void* k_cache, void* v_cache,
                         const float* inv_freq, void* q_out, long ldqo) {
  if (T == 0) return NMX_OK;
  auto* q = reinterpret_cast<half*>(qkv);
  if (D == 128)
    return launch(c, rope_append_kernel<128>, dim3(T), dim3(128), 0, q, ldq, Hq, Hkv, tok_seq,
                  tok_pos, block_tables, max_blocks, BT, reinterpret_cast<half*>(k_cache),
                  reinterpret_cast<half*>(v_cache), inv_freq, reinterpret_cast<half*>(q_out), ldqo);
  if (D == 64)
    return launch(c, rope_append_kernel<64>, dim3(T), dim3(128), 0, q, ldq, Hq, Hkv, tok_seq,
                  tok_pos, block_tables, max_blocks, BT, reinterpret_cast<half*>(k_cache),
                  reinterpret_cast<half*>(v_cache), inv_freq, reinterpret_cast<half*>(q_out), ldqo);
  NMX_CHECK(false, NMX_ERR_UNSUPPORTED, "rope_append: head_dim must be 64 or 128");
}

template <typename T>
static nmx_status_t qsdpa_t(Ctx* c, const void* q, const uint32_t* kw, const void* ks, const void* kb,
                            const uint32_t* vw, const void* vs, const void* vb, int BH, int gqa,
                            int N, int L, int D, float scale, int gs, int bits, void* out) {
  dim3 grid(BH, L);
#define NMX_QSDPA(DPLV)                                                                         \
  return launch(c, qsdpa_kernel<T, DPLV>, grid, dim3(128), 0, (const T*)q, kw, (const T*)ks,   \
                (const T*)kb, vw, (const T*)vs, (const T*)vb, gqa, N, L, scale, gs, bits, (T*)out)
  switch (D) {
    case 64: NMX_QSDPA(2);
    case 96: NMX_QSDPA(3);
    case 128: NMX_QSDPA(4);
    case 256: NMX_QSDPA(8);
  }
#undef NMX_QSDPA
  NMX_CHECK(false, NMX_ERR_UNSUPPORTED, "quantized sdpa: D must be 64, 96, 128 or 256");
}

nmx_status_t quantized_sdpa(Ctx* c, const void* q, const uint32_t* kw, const void* ks,
                            const void* kb, const uint32_t* vw, const void* vs, const void* vb,
                            int BH, int gqa, int N, int L, int D, float scale, int gs, int bits,
                            nmx_dtype_t dt, void* out) {
  if (BH == 0 || L == 0) return NMX_OK;
  if (dt == NMX_F16) return qsdpa_t<half>(c, q, kw, ks, kb, vw, vs, vb, BH, gqa, N, L, D, scale, gs, bits, out);
  if (dt == NMX_BF16)
    return qsdpa_t<__nv_bfloat16>(c, q, kw, ks, kb, vw, vs, vb, BH, gqa, N, L, D, scale, gs, bits, out);
  NMX_CHECK(false, NMX_ERR_UNSUPPORTED, "quantized sdpa: dtype must be f16 or bf16");
}

}  // namespace nmx
