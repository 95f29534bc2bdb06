// The paged-attention dispatcher, RoPE + KV append for prefill rows (f16 or
// quantized pages), and the reference's quantized-KV single-query kernel
// restated for sm_100a. The paged decode kernel itself is in
// attention_mma.cu, the prefill kernels in attention_prefill.cu and
// attention_prefill_tc.cu.
//
// Paged layout per layer: K[num_blocks][Hkv][BT][D], V likewise, fp16; or,
// for a quantized pool, one page record per (block, kv head) of K and of V
// (kv_page_bytes). Replaces MLXFast.scaledDotProductAttention over
// KVCacheSimple / the quantized KV cache (mlx-swift-lm; reached from
// Sources/NovaMLXEngine/FusedBatchScheduler.swift:1215) and the separate
// KVCache.update of the reference's batched decode
// (Sources/NovaMLXEngine/FusedBatchDecode.swift:7-147).
#include "attn_common.cuh"
#include "common.cuh"
#include "kernels.h"

namespace nmx {

namespace {

constexpr int kMaxRep = 8;

__device__ __forceinline__ void rope_pair(float a, float b, float ang, float& ra, float& rb) {
  float sn, cs;
  sincosf(ang, &sn, &cs);
  ra = a * cs - b * sn;
  rb = b * cs + a * sn;
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

// The same RoPE for q, with K and V appended to quantized page records: the
// CTA's warps take (k | v, kv head) rows; a row is roped (k), rounded to f16
// and quantized by the warp (quantize_row_warp) into its slot.
template <int D>
__global__ void __launch_bounds__(128) rope_append_q_kernel(half* qkv, long ldq, int Hq, int Hkv,
                                                            const int* tok_seq, const int* tok_pos,
                                                            const int* block_tables, int max_blocks, int BT,
                                                            unsigned char* Kc, unsigned char* Vc, int bits, int gs,
                                                            const float* inv_freq, half* q_out, long ldqo) {
  grid_wait();
  constexpr int VPL = D / 32;
  const int row = blockIdx.x;
  const int seq = tok_seq[row], pos = tok_pos[row];
  const half* r = qkv + long(row) * ldq;
  half* qo = q_out + long(row) * ldqo;
  for (int i = threadIdx.x; i < Hq * (D / 2); i += blockDim.x) {
    const int hh = i / (D / 2), d = i % (D / 2);
    float r0, r1;
    const half* src = r + hh * D;
    rope_pair(__half2float(src[d]), __half2float(src[d + D / 2]), float(pos) * inv_freq[d], r0, r1);
    qo[hh * D + d] = __float2half_rn(r0);
    qo[hh * D + d + D / 2] = __float2half_rn(r1);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long blk = block_tables[long(seq) * max_blocks + pos / BT];
  const int pq = 16 * (D * bits / 8 + 2 * (D / gs) * 2);
  for (int it = warp; it < 2 * Hkv; it += blockDim.x / 32) {
    const int kind = it / Hkv, kh = it % Hkv;
    const half* src = r + (Hq + kind * Hkv + kh) * D;
    float v[VPL];
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int d = lane * VPL + i;
      if (kind == 0) {
        const int d0 = d < D / 2 ? d : d - D / 2;
        float r0, r1;
        rope_pair(__half2float(src[d0]), __half2float(src[d0 + D / 2]), float(pos) * inv_freq[d0], r0, r1);
        v[i] = __half2float(__float2half_rn(d < D / 2 ? r0 : r1));
      } else {
        v[i] = __half2float(src[d]);
      }
    }
    unsigned char* rec = (kind == 0 ? Kc : Vc) + (blk * Hkv + kh) * pq;
    quantize_row_warp<D>(v, bits, gs, rec, pos % BT);
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
  NMX_CHECK(a.T >= 0 && a.T <= kMaxDecodeRows, NMX_ERR_UNSUPPORTED,
            "paged attention: at most " + std::to_string(kMaxDecodeRows) + " query rows per call");
  if (a.T == 0) return NMX_OK;
  return paged_attention_mma(c, a, fused);
}

nmx_status_t rope_append(Ctx* c, void* qkv, long ldq, int T, int Hq, int Hkv, int D,
                         const int* tok_seq, const int* tok_pos, const int* block_tables,
                         int max_blocks, int BT, void* k_cache, void* v_cache,
                         const float* inv_freq, void* q_out, long ldqo, int kv_bits, int kv_gs) {
  if (T == 0) return NMX_OK;
  auto* q = reinterpret_cast<half*>(qkv);
  if (kv_bits != 0) {
    NMX_CHECK((kv_bits == 4 || kv_bits == 8) && (kv_gs == 32 || kv_gs == 64), NMX_ERR_UNSUPPORTED,
              "rope_append: quantized pages need 4 or 8 bits, group 32 or 64");
    auto* kc = reinterpret_cast<unsigned char*>(k_cache);
    auto* vc = reinterpret_cast<unsigned char*>(v_cache);
    if (D == 128)
      return launch(c, rope_append_q_kernel<128>, dim3(T), dim3(128), 0, q, ldq, Hq, Hkv, tok_seq, tok_pos,
                    block_tables, max_blocks, BT, kc, vc, kv_bits, kv_gs, inv_freq,
                    reinterpret_cast<half*>(q_out), ldqo);
    if (D == 64)
      return launch(c, rope_append_q_kernel<64>, dim3(T), dim3(128), 0, q, ldq, Hq, Hkv, tok_seq, tok_pos,
                    block_tables, max_blocks, BT, kc, vc, kv_bits, kv_gs, inv_freq,
                    reinterpret_cast<half*>(q_out), ldqo);
    NMX_CHECK(false, NMX_ERR_UNSUPPORTED, "rope_append: head_dim must be 64 or 128");
  }
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
