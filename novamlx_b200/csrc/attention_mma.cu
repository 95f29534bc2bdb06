// Paged decode attention on the tensor cores (one query row per sequence).
//
// A CTA owns (query row, kv head, key split) and serves all q heads of the
// GQA group (rep <= 8 rows of a 16-row MMA tile). Its four warps take the
// split's 16-token blocks round-robin; each warp streams K and V blocks
// through its own two-stage cp.async ring into XOR-swizzled shared tiles
// (16 B chunk c of row r at chunk c ^ (r & 7): conflict-free ldmatrix), and
// per block runs S = Q·Kᵀ (mma.sync m16n8k16, f16 in, f32 out), an online
// softmax in the log2 domain on the accumulator fragments, and O += P·V with
// P taken straight from the S fragments and V fed by ldmatrix.trans. Over
// quantized pages (4/8-bit codes, group scales and biases) the ring holds the
// raw page records and each lane dequantizes its own code words straight
// into its K and V MMA registers (no f16 tile in between). Only rows 0-7 of
// the MMA tile carry q heads, so only their accumulators are kept. The
// warps' states merge through shared memory. The splits of one (row, kv
// head) run as one thread-block cluster (<= 16 CTAs): each CTA stores its
// (max, denominator) pairs into every CTA of the cluster and each of its
// numerators into the CTA that owns that output element (remote shared
// memory stores, which do not wait for an answer), then after one cluster
// barrier each CTA combines its slice of the outputs from its own shared
// memory; no global scratch, atomics or fences.
//
// In decode (FUSED) the CTA also applies RoPE to q; the split holding the new
// position writes the new token's roped k and its v to the page (for later
// steps) and adds the token to the softmax from shared memory, so the pages
// this kernel reads are never written by it or by the kernel before it: with
// kv_static the K/V stream starts before the programmatic-launch wait.
#include <algorithm>
#include <map>
#include <mutex>
#include <tuple>

#include "attn_common.cuh"
#include "common.cuh"
#include "kernels.h"

namespace nmx {

namespace {

constexpr int kAW = 4;        // warps per CTA
constexpr int kAStages = 2;   // cp.async stages per warp
constexpr int kMaxRepA = 8;   // q heads per kv head
constexpr int kMaxClusterA = kMaxDecodeSplits;  // key splits per (row, kv head): one cluster

// the two halves of a cluster barrier: arrive (relaxed: the start of the
// kernel, to mark that this CTA runs; release: after the remote stores) and
// wait (acquire)
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_arrive_release() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
// stores v to the shared memory of CTA `rank` of the cluster, at the address
// `p` has in this CTA
__device__ __forceinline__ void st_dsmem(void* p, unsigned rank, float v) {
  const unsigned la = static_cast<unsigned>(__cvta_generic_to_shared(p));
  unsigned ra;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(la), "r"(rank));
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(ra), "f"(v) : "memory");
}

// KQ = 0: f16 pages. KQ = 4 / 8: quantized pages (kv_page_bytes): each warp
// copies a block's K and V page records into its ring and dequantizes the
// codes straight into the MMA fragments (w = s·q + b rounded to f16, as a
// dequantized page holds them), see kfrag_q / vfrag_q.
template <int D, int KQ>
struct DecodeSmem {
  static constexpr int TILE = 16 * D * 2;
  static constexpr int PQ = KQ ? kv_page_bytes(D, KQ, 32) : TILE;  // the largest record (group 32)
  static constexpr int WARP = KQ ? kAStages * 2 * PQ : kAStages * 2 * TILE;
  // the warps' merge reuses the rings: [kAW][kMaxRepA][D] + [kMaxRepA][D] floats
  static constexpr int MERGE = (kAW + 1) * kMaxRepA * D * 4;
  static constexpr size_t BYTES = TILE + size_t(kAW * WARP > MERGE ? kAW * WARP : MERGE);
};

// ---- quantized pages: codes to MMA fragments -----------------------------
// S = Q·Kᵀ (m16n8k16, B = Kᵀ: k = head dim, n = token). The head dim is
// permuted inside each lane's span so that a lane's B registers come from
// whole code words: lane (g, t) of n-tile j supplies token 8j + g, dims
// t·D/4 .. t·D/4 + D/4 - 1 (one quantization group), and k32 step c the
// dims d0 + δ with d0 = t·D/4 + 8c. The q fragments follow the same order:
// block 2c + e, register a0 holds dims d0 + qd(e, 0), d0 + qd(e, 1) and a2
// holds d0 + qd(e, 2), d0 + qd(e, 3).
template <int KQ>
__device__ __forceinline__ int qd(int e, int i) {
  // 4-bit: a word's nibbles pair as (δ, δ + 4); 8-bit: bytes pair as (δ, δ + 1)
  if constexpr (KQ == 4) return 2 * e + (i >> 1) + 4 * (i & 1);
  else return 4 * e + i;
}
// (v0, v1) f16 bits from two exact f16 codes-plus-1024 x (1024 + q) and the
// page's scale and bias: w = (x - 1024)·s + b, one rounding
__device__ __forceinline__ uint32_t dq_pair(uint32_t x, __half2 s2, __half2 b2) {
  const __half2 k1024 = __float2half2_rn(1024.f);
  __half2 h = __hfma2(__hsub2(*reinterpret_cast<__half2*>(&x), k1024), s2, b2);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t nib_pair(uint32_t w, int sh) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;\n" : "=r"(r) : "r"(w >> sh), "r"(0x000F000Fu), "r"(0x64006400u));
  return r;
}
__device__ __forceinline__ uint32_t byte_pair(uint32_t w, uint32_t sel) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;\n" : "=r"(r) : "r"(__byte_perm(w, 0u, sel)), "r"(0x00FF00FFu), "r"(0x64006400u));
  return r;
}
// The lane's K code words of one token row (its D/4 dims).
template <int D, int KQ>
__device__ __forceinline__ void k_words(const unsigned char* row, int t, uint32_t* wd) {
  constexpr int NW = D / 4 * KQ / 32;  // 4-bit: D/32, 8-bit: D/16 words
  const unsigned char* p = row + t * (NW * 4);
  if constexpr (NW == 2) {
    const uint2 v = *reinterpret_cast<const uint2*>(p);
    wd[0] = v.x; wd[1] = v.y;
  } else {
#pragma unroll
    for (int i = 0; i < NW; i += 4) {
      const uint4 v = *reinterpret_cast<const uint4*>(p + 4 * i);
      wd[i] = v.x; wd[i + 1] = v.y; wd[i + 2] = v.z; wd[i + 3] = v.w;
    }
  }
}
// B registers of k16 blocks 2c (b[0], b[1]) and 2c + 1 (b[2], b[3]) from the
// lane's words of one token
template <int KQ>
__device__ __forceinline__ void kfrag_q(const uint32_t* wd, int c, __half2 s2, __half2 b2, uint32_t* b) {
  if constexpr (KQ == 4) {
    const uint32_t w = wd[c];
#pragma unroll
    for (int i = 0; i < 4; ++i) b[i] = dq_pair(nib_pair(w, 4 * i), s2, b2);  // (δi, δi+4)
  } else {
    const uint32_t w0 = wd[2 * c], w1 = wd[2 * c + 1];
    b[0] = dq_pair(byte_pair(w0, 0x5140), s2, b2);  // δ0, δ1
    b[1] = dq_pair(byte_pair(w0, 0x7362), s2, b2);  // δ2, δ3
    b[2] = dq_pair(byte_pair(w1, 0x5140), s2, b2);  // δ4, δ5
    b[3] = dq_pair(byte_pair(w1, 0x7362), s2, b2);  // δ6, δ7
  }
}
// O += P·V (B = V: k = token, n = head dim). Lane g's n columns are the dims
// g·D/8 .. g·D/8 + D/8 - 1 (n-tile j: dim g·D/8 + j), so the accumulator
// o[j][e] of lane (g, t) is dim (2t + e)·D/8 + j. The lane's B registers for
// tokens (A, A + 1) come from the two rows' words of its span: the rows'
// bytes are interleaved first so each register pairs token A with A + 1.
template <int D, int KQ>
__device__ __forceinline__ void vfrag_q(const unsigned char* rowA, const unsigned char* rowB, int g, __half2 s2,
                                        __half2 b2, uint32_t* b) {
  constexpr int NW = D / 8 * KQ / 32;  // words of the lane's span: 4-bit D/64, 8-bit D/32
  const unsigned char* pa = rowA + g * (NW * 4);
  const unsigned char* pb = rowB + g * (NW * 4);
  uint32_t wa[NW], wb[NW];
  if constexpr (NW == 1) {
    wa[0] = *reinterpret_cast<const uint32_t*>(pa);
    wb[0] = *reinterpret_cast<const uint32_t*>(pb);
  } else if constexpr (NW == 2) {
    const uint2 va = *reinterpret_cast<const uint2*>(pa), vb = *reinterpret_cast<const uint2*>(pb);
    wa[0] = va.x; wa[1] = va.y; wb[0] = vb.x; wb[1] = vb.y;
  } else {
    const uint4 va = *reinterpret_cast<const uint4*>(pa), vb = *reinterpret_cast<const uint4*>(pb);
    wa[0] = va.x; wa[1] = va.y; wa[2] = va.z; wa[3] = va.w;
    wb[0] = vb.x; wb[1] = vb.y; wb[2] = vb.z; wb[3] = vb.w;
  }
#pragma unroll
  for (int k = 0; k < NW; ++k) {
    if constexpr (KQ == 4) {
      // bytes (A0, A1, B0, B1) and (A2, A3, B2, B3): nibble i of each half
      const uint32_t lo = __byte_perm(wa[k], wb[k], 0x5410), hi = __byte_perm(wa[k], wb[k], 0x7632);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        b[8 * k + i] = dq_pair(nib_pair(lo, 4 * i), s2, b2);
        b[8 * k + 4 + i] = dq_pair(nib_pair(hi, 4 * i), s2, b2);
      }
    } else {
      // byte i of A and of B, each in the low byte of a half
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint32_t x;
        asm("lop3.b32 %0, %1, %2, %3, 0xEA;\n"
            : "=r"(x)
            : "r"(__byte_perm(wa[k], wb[k], ((4 + i) << 8) | i)), "r"(0x00FF00FFu), "r"(0x64006400u));
        b[4 * k + i] = dq_pair(x, s2, b2);
      }
    }
  }
}

template <int D, bool FUSED, int KQ>
__global__ void __launch_bounds__(kAW * 32, KQ ? 4 : 1) paged_decode_mma_kernel(AttnArgs a) {
  constexpr int BT = 16;
  constexpr int CH = D / 8;          // 16-byte chunks per row
  constexpr int TILE = BT * D * 2;   // bytes of one K (or V) block tile
  constexpr int KSTEPS = D / 16;
  constexpr int NT = D / 8;
  constexpr float kLog2e = 1.4426950408889634f;
  using SM = DecodeSmem<D, KQ>;
  extern __shared__ __align__(128) unsigned char sm[];
  unsigned char* q_sm = sm;
  unsigned char* ring_all = sm + TILE;
  // bytes of one page record (K or V of one block and kv head)
  const int pq = KQ ? kv_page_bytes(D, KQ, a.kv_gs) : TILE;
  // per-warp softmax states; entry kAW is the new token (FUSED, owner split)
  __shared__ float s_m[kAW + 1][kMaxRepA], s_l[kAW + 1][kMaxRepA];
  __shared__ float c_ml[kMaxRepA][2];  // this split's (max, denominator) per q head
  // every split's (max, denominator) per q head, stored here by the splits
  __shared__ float s_cm[kMaxRepA][kMaxClusterA], s_cl[kMaxRepA][kMaxClusterA];
  // numerators of this CTA's output slice, one row of slot_len per split
  __shared__ float s_rnum[kMaxRepA * D + kMaxClusterA];
  __shared__ float s_w[kMaxRepA][kMaxClusterA];
  __shared__ float s_f[kAW + 1][kMaxRepA];  // per state and q head: exp2(m - M)
  __shared__ float s_den[kMaxRepA];
  __shared__ __align__(16) half s_knew[D];
  __shared__ __align__(16) half s_vnew[D];

  const int split = blockIdx.x, h = blockIdx.y, row = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int Hq = a.Hq, Hkv = a.Hkv, rep = Hq / Hkv, S = gridDim.x;
  // phase 1 of the cluster barrier: this CTA runs (its shared memory may be
  // written by the others once the phase completes)
  if (S > 1) cluster_arrive_relaxed();
  half* Kc = reinterpret_cast<half*>(a.k_cache);
  half* Vc = reinterpret_cast<half*>(a.v_cache);

  int pos = 0, b0 = 0, b1 = 0;
  const int* bt = nullptr;
  auto locate = [&]() {
    const int seq = a.tok_seq[row];
    pos = a.tok_pos[row];
    const int nblk = (pos + 1 + BT - 1) / BT;
    const int bps = (nblk + S - 1) / S;
    b0 = split * bps;
    b1 = min(nblk, b0 + bps);
    bt = a.block_tables + long(seq) * a.max_blocks;
  };
  unsigned char* ring = ring_all + warp * SM::WARP;
  auto issue = [&](int stage, int b) {
    if (b < b1) {
      if constexpr (KQ == 0) {
        const long base = (long(bt[b]) * Hkv + h) * BT * D;  // halves
        const unsigned char* ks = reinterpret_cast<const unsigned char*>(Kc + base);
        const unsigned char* vs = reinterpret_cast<const unsigned char*>(Vc + base);
        unsigned char* kd = ring + stage * 2 * TILE;
        unsigned char* vd = kd + TILE;
#pragma unroll
        for (int i = lane; i < BT * CH; i += 32) {
          const int r = i / CH, c = i % CH;
          cp_async16a(kd + swz<D>(r, c), ks + i * 16);
          cp_async16a(vd + swz<D>(r, c), vs + i * 16);
        }
      } else {
        const long base = (long(bt[b]) * Hkv + h) * pq;  // bytes
        const unsigned char* ks = reinterpret_cast<const unsigned char*>(Kc) + base;
        const unsigned char* vs = reinterpret_cast<const unsigned char*>(Vc) + base;
        unsigned char* kd = ring + stage * 2 * SM::PQ;
        unsigned char* vd = kd + SM::PQ;
        for (int i = lane; i < pq / 16; i += 32) {
          cp_async16a(kd + i * 16, ks + i * 16);
          cp_async16a(vd + i * 16, vs + i * 16);
        }
      }
    }
    cp_commit();
  };
  // The pages read here never hold the new token (FUSED masks it and adds it
  // from registers), so when the caller says the cache is not written by the
  // previous kernel, the stream starts before the programmatic-launch wait.
  if (a.kv_static) {
    locate();
    issue(0, b0 + warp);
    issue(1, b0 + warp + kAW);
    grid_wait();
  } else {
    grid_wait();
    locate();
    issue(0, b0 + warp);
    issue(1, b0 + warp + kAW);
  }
  const half* Q = reinterpret_cast<const half*>(a.q) + long(row) * a.ldq;
  const int bpos = pos / BT;
  const bool owner = FUSED && bpos >= b0 && bpos < b1;

  // ---- q tile: rows < rep hold the (roped) q heads, rows >= rep are zero
  for (int i = tid; i < (BT - rep) * CH; i += kAW * 32) {
    const int r = rep + i / CH, c = i % CH;
    *reinterpret_cast<uint4*>(q_sm + swz<D>(r, c)) = make_uint4(0, 0, 0, 0);
  }
  if (FUSED) {
    for (int i = tid; i < rep * (D / 2); i += kAW * 32) {
      const int hi = i / (D / 2), d = i % (D / 2);
      const int hq = h * rep + hi;
      float r0, r1;
      rope2(__half2float(Q[hq * D + d]), __half2float(Q[hq * D + d + D / 2]), float(pos) * a.inv_freq[d], r0, r1);
      half* q0 = reinterpret_cast<half*>(q_sm + swz<D>(hi, d / 8)) + (d % 8);
      half* q1 = reinterpret_cast<half*>(q_sm + swz<D>(hi, (d + D / 2) / 8)) + (d % 8);
      *q0 = __float2half_rn(r0);
      *q1 = __float2half_rn(r1);
    }
    if (owner) {
      // the new token: roped k and v to its page (for later steps) and to
      // shared memory (for this one)
      const half* kr = Q + (Hq + h) * D;
      const half* vr = Q + (Hq + Hkv + h) * D;
      if constexpr (KQ == 0) {
        const long slot = (long(bt[bpos]) * Hkv + h) * BT + pos % BT;
        for (int d = tid; d < D / 2; d += kAW * 32) {
          float r0, r1;
          rope2(__half2float(kr[d]), __half2float(kr[d + D / 2]), float(pos) * a.inv_freq[d], r0, r1);
          const half k0 = __float2half_rn(r0), k1 = __float2half_rn(r1);
          Kc[slot * D + d] = k0;
          Kc[slot * D + d + D / 2] = k1;
          s_knew[d] = k0;
          s_knew[d + D / 2] = k1;
        }
        for (int d = tid; d < D; d += kAW * 32) {
          Vc[slot * D + d] = vr[d];
          s_vnew[d] = vr[d];
        }
      } else if (warp < 2) {
        // warp 0: k (roped, rounded to f16), warp 1: v; quantized into the
        // page record, and the dequantized values are what this step uses
        // (the cache holds nothing finer)
        constexpr int VPL = D / 32;
        const long rec = (long(bt[bpos]) * Hkv + h) * pq;
        float v[VPL];
#pragma unroll
        for (int i = 0; i < VPL; ++i) {
          const int d = lane * VPL + i;
          if (warp == 0) {
            const int d0 = d < D / 2 ? d : d - D / 2;
            float r0, r1;
            rope2(__half2float(kr[d0]), __half2float(kr[d0 + D / 2]), float(pos) * a.inv_freq[d0], r0, r1);
            v[i] = __half2float(__float2half_rn(d < D / 2 ? r0 : r1));
          } else {
            v[i] = __half2float(vr[d]);
          }
        }
        unsigned char* page = reinterpret_cast<unsigned char*>(warp == 0 ? a.k_cache : a.v_cache) + rec;
        quantize_row_warp<D>(v, KQ, a.kv_gs, page, pos % BT);
        half* dst = warp == 0 ? s_knew : s_vnew;
#pragma unroll
        for (int i = 0; i < VPL; ++i) dst[lane * VPL + i] = __float2half_rn(v[i]);
      }
    }
  } else {
    for (int i = tid; i < rep * CH; i += kAW * 32) {
      const int r = i / CH, c = i % CH;
      *reinterpret_cast<uint4*>(q_sm + swz<D>(r, c)) =
          *reinterpret_cast<const uint4*>(Q + (h * rep + r) * D + c * 8);
    }
  }
  __syncthreads();

  // q fragments (rows 8-15 are zero: a1 = a3 = 0); quantized pages: in the
  // permuted head-dim order of kfrag_q
  uint32_t qa[KSTEPS][2];
  if constexpr (KQ == 0) {
#pragma unroll
    for (int kk = 0; kk < KSTEPS; ++kk) {
      const int r = lane & 7, c = 2 * kk + ((lane >> 3) & 1);
      ldsm_x2(qa[kk], q_sm + swz<D>(r, c));
    }
  } else {
#pragma unroll
    for (int kk = 0; kk < KSTEPS; ++kk) {
      const int c = kk >> 1, e = kk & 1, d0 = t * (D / 4) + 8 * c;
      const half* qc = reinterpret_cast<const half*>(q_sm + swz<D>(g, d0 / 8));  // dims d0 .. d0 + 7
      qa[kk][0] = pack_half2(__half2float(qc[qd<KQ>(e, 0)]), __half2float(qc[qd<KQ>(e, 1)]));
      qa[kk][1] = pack_half2(__half2float(qc[qd<KQ>(e, 2)]), __half2float(qc[qd<KQ>(e, 3)]));
    }
  }

  const float sl2 = a.scale * kLog2e;
  // keys up to `last` come from the pages (FUSED: the new token is added apart)
  const int last = FUSED ? pos - 1 : pos;
  float o[NT][2];  // rows 0-7 of the MMA tile (rows 8-15 are the zero padding)
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) o[nt][0] = o[nt][1] = 0.f;
  float m_r = -INFINITY, l_r = 0.f;

  int stage = 0;
  for (int b = b0 + warp; b < b1; b += kAW) {
    cp_wait<1>();
    __syncwarp();
    const unsigned char* kt = ring + stage * 2 * TILE;
    const unsigned char* vt = kt + TILE;
    float s[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
    // quantized pages: V's B registers (tokens 2t, 2t + 1 | 2t + 8, 2t + 9)
    uint32_t vb[2][KQ ? NT : 1];
    if constexpr (KQ == 0) {
#pragma unroll
      for (int kk = 0; kk < KSTEPS; ++kk) {
        uint32_t r[4];
        const int rr = (lane & 7) + ((lane >> 4) << 3), cc = 2 * kk + ((lane >> 3) & 1);
        ldsm_x4(r, kt + swz<D>(rr, cc));
        mma_f16_top(s[0], qa[kk][0], qa[kk][1], r[0], r[1]);
        mma_f16_top(s[1], qa[kk][0], qa[kk][1], r[2], r[3]);
      }
    } else {
      // page record: codes [16][R], scales [16][ng], biases [16][ng]
      constexpr int R = D * KQ / 8;
      const unsigned char* kraw = ring + stage * 2 * SM::PQ;
      const unsigned char* vraw = kraw + SM::PQ;
      const int ng = D / a.kv_gs;
      const half* ksc = reinterpret_cast<const half*>(kraw + 16 * R);
      const half* vsc = reinterpret_cast<const half*>(vraw + 16 * R);
      const int kgrp = t * (D / 4) / a.kv_gs, vgrp = g * (D / 8) / a.kv_gs;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int tok = 8 * j + g;
        uint32_t wd[D / 4 * KQ / 32];
        k_words<D, KQ>(kraw + tok * R, t, wd);
        const __half2 s2 = __half2half2(ksc[tok * ng + kgrp]), b2 = __half2half2(ksc[16 * ng + tok * ng + kgrp]);
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t bq[4];
          kfrag_q<KQ>(wd, c, s2, b2, bq);
          mma_f16_top(s[j], qa[2 * c][0], qa[2 * c][1], bq[0], bq[1]);
          mma_f16_top(s[j], qa[2 * c + 1][0], qa[2 * c + 1][1], bq[2], bq[3]);
        }
      }
#pragma unroll
      for (int tp = 0; tp < 2; ++tp) {
        const int A = 2 * t + 8 * tp;
        const __half2 s2 = __halves2half2(vsc[A * ng + vgrp], vsc[(A + 1) * ng + vgrp]);
        const __half2 b2 = __halves2half2(vsc[16 * ng + A * ng + vgrp], vsc[16 * ng + (A + 1) * ng + vgrp]);
        vfrag_q<D, KQ>(vraw + A * R, vraw + (A + 1) * R, g, s2, b2, vb[tp]);
      }
    }
    // scale to log2 units, mask keys past `last`, online softmax of row g
    const int tb = b * BT;
    float v[4];
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int tok = tb + 8 * j + 2 * t + e;
        v[2 * j + e] = tok <= last ? s[j][e] * sl2 : -INFINITY;
      }
    float mx = fmaxf(fmaxf(v[0], v[1]), fmaxf(v[2], v[3]));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float m_new = fmaxf(m_r, mx);
    // a block with every key masked leaves the state as it was
    const float m_use = m_new == -INFINITY ? 0.f : m_new;
    const float corr = exp2f(m_r - m_use);
    float p[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) p[e] = exp2f(v[e] - m_use);
    l_r = l_r * corr + (p[0] + p[1] + p[2] + p[3]);
    m_r = m_new;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      o[nt][0] *= corr;
      o[nt][1] *= corr;
    }
    const uint32_t pa0 = pack_half2(p[0], p[1]), pa2 = pack_half2(p[2], p[3]);
    if constexpr (KQ == 0) {
#pragma unroll
      for (int np = 0; np < NT / 2; ++np) {
        uint32_t r[4];
        const int rr = (lane & 7) + (((lane >> 3) & 1) << 3), cc = 2 * np + (lane >> 4);
        ldsm_x4_t(r, vt + swz<D>(rr, cc));
        mma_f16_top(o[2 * np], pa0, pa2, r[0], r[1]);
        mma_f16_top(o[2 * np + 1], pa0, pa2, r[2], r[3]);
      }
    } else {
#pragma unroll
      for (int j = 0; j < NT; ++j) mma_f16_top(o[j], pa0, pa2, vb[0][j], vb[1][j]);
    }
    __syncwarp();
    issue(stage, b + 2 * kAW);
    stage ^= 1;
  }
  cp_wait<0>();
  l_r += __shfl_xor_sync(0xffffffffu, l_r, 1);
  l_r += __shfl_xor_sync(0xffffffffu, l_r, 2);

  // ---- merge the warps (rows g < rep hold results) and the new token
  __syncthreads();  // every warp is done with its ring: reuse it
  float* s_o = reinterpret_cast<float*>(ring_all);           // [kAW][kMaxRepA][D]
  float* c_num = s_o + kAW * kMaxRepA * D;                   // [kMaxRepA][D] this split's numerators
  if (g < rep) {
    if (t == 0) {
      s_m[warp][g] = m_r;
      s_l[warp][g] = l_r;
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      if constexpr (KQ == 0) {
        *reinterpret_cast<float2*>(s_o + (warp * kMaxRepA + g) * D + nt * 8 + 2 * t) = make_float2(o[nt][0], o[nt][1]);
      } else {
        // n-tile nt, column 2t + e: dim (2t + e)·D/8 + nt
        s_o[(warp * kMaxRepA + g) * D + (2 * t) * (D / 8) + nt] = o[nt][0];
        s_o[(warp * kMaxRepA + g) * D + (2 * t + 1) * (D / 8) + nt] = o[nt][1];
      }
    }
  }
  {
    // new token score per q head (warp w takes heads w, w + kAW): f16 q ·
    // f16 k summed in f32, log2 units
    for (int hi = warp; hi < rep; hi += kAW) {
      float sc = 0.f;
      if (owner) {
        for (int d = lane; d < D; d += 32) {
          const half qv = reinterpret_cast<const half*>(q_sm + swz<D>(hi, d / 8))[d % 8];
          sc = fmaf(__half2float(qv), __half2float(s_knew[d]), sc);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) sc += __shfl_xor_sync(0xffffffffu, sc, off);
      }
      if (lane == 0) {
        s_m[kAW][hi] = owner ? sc * sl2 : -INFINITY;
        s_l[kAW][hi] = owner ? 1.f : 0.f;
      }
    }
  }
  __syncthreads();
  grid_launch_dependents();

  // per q head (thread hi): the maximum over the warps' states and the new
  // token, each state's factor exp2(m - M) and the denominator
  if (tid < rep) {
    const int hi = tid;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w <= kAW; ++w)
      if (s_l[w][hi] > 0.f) M = fmaxf(M, s_m[w][hi]);
    float den = 0.f;
#pragma unroll
    for (int w = 0; w < kAW; ++w) {
      const float f = s_l[w][hi] > 0.f ? exp2f(s_m[w][hi] - M) : 0.f;
      s_f[w][hi] = f;
      if (s_l[w][hi] > 0.f) den = fmaf(s_l[w][hi], f, den);
    }
    const float fn = s_l[kAW][hi] > 0.f ? exp2f(s_m[kAW][hi] - M) : 0.f;
    s_f[kAW][hi] = fn;
    if (s_l[kAW][hi] > 0.f) den += fn;
    c_ml[hi][0] = M;
    c_ml[hi][1] = den;
  }
  __syncthreads();
  half* Out = reinterpret_cast<half*>(a.out) + long(row) * Hq * D;
  for (int e = tid; e < rep * D; e += kAW * 32) {
    const int hi = e / D, d = e % D;
    float num = 0.f;
#pragma unroll
    for (int w = 0; w < kAW; ++w)
      if (s_l[w][hi] > 0.f) num = fmaf(s_o[(w * kMaxRepA + hi) * D + d], s_f[w][hi], num);
    if (s_l[kAW][hi] > 0.f) num = fmaf(__half2float(s_vnew[d]), s_f[kAW][hi], num);
    if (S == 1) {
      const float den = c_ml[hi][1];
      Out[(h * rep + hi) * D + d] = __float2half_rn(den > 0.f ? num / den : 0.f);
    } else {
      c_num[hi * D + d] = num;
    }
  }
  if (S == 1) return;

  // ---- split-KV: the splits of (row, h) are one cluster. Output element e
  // of the rep * D belongs to split o with o E / S <= e < (o + 1) E / S.
  const int E = rep * D, slot_len = (E + S - 1) / S;
  __syncthreads();
  cluster_wait();  // phase 1: every CTA of the cluster runs
  for (int e = tid; e < E; e += kAW * 32) {
    const int o = ((e + 1) * S - 1) / E;
    st_dsmem(&s_rnum[split * slot_len + e - o * E / S], unsigned(o), c_num[e]);
  }
  if (tid < rep * S) {
    const int hi = tid / S, s2 = tid % S;
    st_dsmem(&s_cm[hi][split], unsigned(s2), c_ml[hi][0]);
    st_dsmem(&s_cl[hi][split], unsigned(s2), c_ml[hi][1]);
  }
  cluster_arrive_release();
  cluster_wait();  // phase 2: every store into this CTA has landed
  {
    // the splits' weights, thread (hi, s2) = (tid / 16, tid % 16): the
    // maximum over the head's live splits (a max of the half-warp), the
    // factor exp2(m - M), then the denominator in split order (thread hi)
    static_assert(kAW * 32 == kMaxRepA * kMaxClusterA, "one thread per (head, split)");
    const int hi = tid >> 4, s2 = tid & 15;
    const bool live = hi < rep && s2 < S && s_cl[hi][s2] > 0.f;
    float M = live ? s_cm[hi][s2] : -INFINITY;
#pragma unroll
    for (int off = 8; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
    s_w[hi][s2] = live ? exp2f(s_cm[hi][s2] - M) : 0.f;
    __syncthreads();
    if (tid < rep) {
      float den = 0.f;
#pragma unroll 4
      for (int k = 0; k < S; ++k)
        if (s_cl[tid][k] > 0.f) den = fmaf(s_cl[tid][k], s_w[tid][k], den);
      s_den[tid] = den > 0.f ? 1.f / den : 0.f;
    }
    __syncthreads();
    if (live) s_w[hi][s2] *= s_den[hi];
    __syncthreads();
  }
  const int e0 = split * E / S, e1 = (split + 1) * E / S;
  for (int e = e0 + tid; e < e1; e += kAW * 32) {
    const int hi = e / D, d = e % D;
    float num = 0.f;
#pragma unroll 4
    for (int s2 = 0; s2 < S; ++s2)
      if (s_w[hi][s2] != 0.f) num = fmaf(s_rnum[s2 * slot_len + e - e0], s_w[hi][s2], num);
    Out[(h * rep + hi) * D + d] = __float2half_rn(num);
  }
  // no remote access follows phase 2: a CTA may leave
}

template <int D, bool FUSED, int KQ>
nmx_status_t launch_mma(Ctx* c, const AttnArgs& a, int S) {
  const size_t smem = DecodeSmem<D, KQ>::BYTES;
  auto kern = paged_decode_mma_kernel<D, FUSED, KQ>;
  static std::mutex mu;
  static std::map<int, bool> attr;  // per device
  {
    std::lock_guard<std::mutex> lk(mu);
    if (!attr[c->device]) {
      NMX_CUDA_OK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
      NMX_CUDA_OK(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
      attr[c->device] = true;
    }
  }
  // the largest cluster not above S that the device can place
  static std::map<std::pair<int, int>, int> fit;  // (device, S) → usable S
  int s_use = S;
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = fit.find({c->device, S});
    if (it != fit.end()) {
      s_use = it->second;
    } else {
      while (s_use > 1) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(s_use, a.Hkv, 1);
        cfg.blockDim = dim3(kAW * 32);
        cfg.dynamicSmemBytes = smem;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = s_use;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) == cudaSuccess && n > 0) break;
        cudaGetLastError();
        s_use = s_use > 8 ? 8 : s_use / 2;
      }
      fit[{c->device, S}] = s_use;
    }
  }
  // The (row, kv head) clusters run in waves of as many clusters as the
  // device holds at once, which for 9-15 CTAs per cluster is not the CTA
  // slots over the cluster size (a cluster must fit in one GPC). A last wave
  // under half full streams its pages well below HBM speed (32 clusters of
  // 9: a second wave of two, 39 vs ~25 us), so take the largest split count
  // not above s_use whose clusters fit one wave or leave a last wave at
  // least half full (none: s_use).
  static std::map<std::tuple<int, int, long>, int> wave_fit;  // (device, s_use, clusters) → splits
  const long units = long(a.Hkv) * a.T;
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = wave_fit.find({c->device, s_use, units});
    if (it != wave_fit.end()) {
      s_use = it->second;
    } else {
      auto wave = [&](int s) -> long {  // clusters of s CTAs resident at once
        if (s == 1) {
          int per = 0;
          if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, kern, kAW * 32, smem) != cudaSuccess) {
            cudaGetLastError();
            return 0;
          }
          return long(per) * c->num_sms;
        }
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(s, a.Hkv, 1);
        cfg.blockDim = dim3(kAW * 32);
        cfg.dynamicSmemBytes = smem;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = s;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
          cudaGetLastError();
          return 0;
        }
        return n;
      };
      auto full_enough = [&](int s) {
        const long n = wave(s);
        if (n <= 0) return false;
        const long last = units % n;
        return units <= n || last == 0 || 2 * last >= n;
      };
      int pick = s_use;
      if (!full_enough(s_use)) {
        for (int s = s_use - 1; s >= 1; --s)
          if (full_enough(s)) {
            pick = s;
            break;
          }
      }
      wave_fit[{c->device, s_use, units}] = pick;
      s_use = pick;
    }
  }
  return launch_cluster(c, kern, dim3(s_use, a.Hkv, a.T), dim3(kAW * 32), smem, unsigned(s_use), a);
}

}  // namespace

nmx_status_t paged_attention_mma(Ctx* c, const AttnArgs& a, bool fused) {
  NMX_CHECK(a.splits >= 1, NMX_ERR_UNSUPPORTED, "paged attention: splits >= 1");
  // the splits of one (row, kv head) form a cluster: at most 16 CTAs
  const int S = std::min(a.splits, kMaxClusterA);
  NMX_CHECK(a.kv_bits == 0 || ((a.kv_bits == 4 || a.kv_bits == 8) && (a.kv_gs == 32 || a.kv_gs == 64)),
            NMX_ERR_UNSUPPORTED, "paged attention: quantized pages need 4 or 8 bits, group 32 or 64");
#define NMX_DEC(DD, KQ) \
  return fused ? launch_mma<DD, true, KQ>(c, a, S) : launch_mma<DD, false, KQ>(c, a, S)
  if (a.D == 128) {
    if (a.kv_bits == 4) NMX_DEC(128, 4);
    if (a.kv_bits == 8) NMX_DEC(128, 8);
    NMX_DEC(128, 0);
  }
  if (a.D == 64) {
    if (a.kv_bits == 4) NMX_DEC(64, 4);
    if (a.kv_bits == 8) NMX_DEC(64, 8);
    NMX_DEC(64, 0);
  }
#undef NMX_DEC
  NMX_CHECK(false, NMX_ERR_UNSUPPORTED, "paged attention: head_dim must be 64 or 128");
}

}  // namespace nmx
