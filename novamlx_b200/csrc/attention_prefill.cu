// Paged attention for prefill chunks and mixed batches: flash-style over
// query blocks, on the tensor cores (mma.sync m16n8k16, f16 in, f32 out).
//
// A work item is up to 16 consecutive query rows of one sequence (the host
// cuts every sequence's rows of the batch into items). A CTA owns (item, kv
// head) and has one warp per q head of the GQA group: warp w holds the 16
// rows' q of head h·rep + w as an MMA A operand. The CTA streams the
// sequence's 16-token K/V pages once, from the first page to the page of its
// last row's position, through a 3-stage cp.async ring into XOR-swizzled
// tiles shared by all its warps (ldmatrix, conflict-free); per page every
// warp runs S = Q·Kᵀ, the causal mask (key ≤ the row's position), an online
// softmax in the log2 domain on the accumulator fragments (rows g and g+8
// per thread), and O += P·V with P taken straight from the S fragments. So
// every K/V byte a CTA needs is read once for 16 query positions × rep heads,
// where the per-row decode kernel reads it once per position.
//
// The pages already hold the chunk's own keys (RoPE + append ran first), so
// keys up to each row's own position come from the pages.
#include <algorithm>
#include <map>
#include <mutex>
#include <vector>

#include "attn_common.cuh"
#include "common.cuh"
#include "kernels.h"

namespace nmx {

namespace {

constexpr int kPQB = 16;      // query rows per work item
constexpr int kPStages = 3;   // K/V ring stages
constexpr int kPMaxRep = 8;   // q heads per kv head (one warp each)

// KQ = 0: f16 pages; 4 / 8: quantized page records (kv_page_bytes) copied
// into the ring and dequantized by the CTA into one shared K/V tile pair per
// block before the warps read it.
template <int D, int KQ>
struct PrefillSmem {
  static constexpr int TILE = 16 * D * 2;
  static constexpr int PQ = KQ ? kv_page_bytes(D, KQ, 32) : TILE;  // the largest record (group 32)
  static constexpr size_t BYTES =
      size_t(kPMaxRep) * TILE + size_t(kPStages) * 2 * PQ + (KQ ? 2 * size_t(TILE) : 0);
};

template <int D, int KQ>
__global__ void __launch_bounds__(kPMaxRep * 32) paged_prefill_mma_kernel(AttnArgs a, const int2* items) {
  constexpr int BT = 16;
  constexpr int CH = D / 8;          // 16-byte chunks per row
  constexpr int TILE = BT * D * 2;   // bytes of one K (or V) page tile
  constexpr int KSTEPS = D / 16;
  constexpr int NT = D / 8;
  constexpr float kLog2e = 1.4426950408889634f;
  extern __shared__ __align__(128) unsigned char sm[];
  __shared__ int s_pos[kPQB];

  const int h = blockIdx.y;
  const int2 it = items[blockIdx.x];  // (first row, rows)
  const int r0 = it.x, nr = it.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int Hq = a.Hq, Hkv = a.Hkv, rep = Hq / Hkv;
  const int nthr = rep * 32;
  half* Kc = reinterpret_cast<half*>(a.k_cache);
  half* Vc = reinterpret_cast<half*>(a.v_cache);
  using PS = PrefillSmem<D, KQ>;
  unsigned char* q_sm = sm;                         // [rep][16][D] swizzled
  unsigned char* ring = sm + size_t(kPMaxRep) * TILE;  // [stage][K | V]
  unsigned char* kdq = ring + size_t(kPStages) * 2 * PS::PQ;  // quantized pages: the block's f16 K, V
  unsigned char* vdq = kdq + TILE;
  const int pq = KQ ? kv_page_bytes(D, KQ, a.kv_gs) : TILE;

  grid_wait();  // q rows and the pages (RoPE + append) come from the kernels before
  if (tid < kPQB) s_pos[tid] = tid < nr ? a.tok_pos[r0 + tid] : -1;
  const int seq = a.tok_seq[r0];
  const int* bt = a.block_tables + long(seq) * a.max_blocks;
  const int last_pos = a.tok_pos[r0 + nr - 1];  // rows of an item have increasing positions
  const int nblk = last_pos / BT + 1;

  auto issue = [&](int stage, int b) {
    if (b < nblk) {
      if constexpr (KQ == 0) {
        const long base = (long(bt[b]) * Hkv + h) * BT * D;  // halves
        const unsigned char* ks = reinterpret_cast<const unsigned char*>(Kc + base);
        const unsigned char* vs = reinterpret_cast<const unsigned char*>(Vc + base);
        unsigned char* kd = ring + stage * 2 * TILE;
        unsigned char* vd = kd + TILE;
        for (int i = tid; i < BT * CH; i += nthr) {
          const int r = i / CH, c = i % CH;
          cp_async16a(kd + swz<D>(r, c), ks + i * 16);
          cp_async16a(vd + swz<D>(r, c), vs + i * 16);
        }
      } else {
        const long base = (long(bt[b]) * Hkv + h) * pq;  // bytes
        const unsigned char* ks = reinterpret_cast<const unsigned char*>(Kc) + base;
        const unsigned char* vs = reinterpret_cast<const unsigned char*>(Vc) + base;
        unsigned char* kd = ring + stage * 2 * PS::PQ;
        unsigned char* vd = kd + PS::PQ;
        for (int i = tid; i < pq / 16; i += nthr) {
          cp_async16a(kd + i * 16, ks + i * 16);
          cp_async16a(vd + i * 16, vs + i * 16);
        }
      }
    }
    cp_commit();
  };
  issue(0, 0);
  issue(1, 1);

  // this warp's q tile: 16 rows of head h·rep + warp (rows past nr zero)
  {
    unsigned char* qw = q_sm + size_t(warp) * TILE;
    const half* Q = reinterpret_cast<const half*>(a.q);
    const int hq = h * rep + warp;
    for (int i = lane; i < kPQB * CH; i += 32) {
      const int r = i / CH, c = i % CH;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (r < nr) v = *reinterpret_cast<const uint4*>(Q + long(r0 + r) * a.ldq + hq * D + c * 8);
      *reinterpret_cast<uint4*>(qw + swz<D>(r, c)) = v;
    }
  }
  __syncthreads();
  uint32_t qa[KSTEPS][4];
  {
    const unsigned char* qw = q_sm + size_t(warp) * TILE;
#pragma unroll
    for (int kk = 0; kk < KSTEPS; ++kk) {
      const int r = lane & 15, c = 2 * kk + (lane >> 4);
      ldsm_x4(qa[kk], qw + swz<D>(r, c));
    }
  }
  const int pos_g = s_pos[g], pos_g8 = s_pos[g + 8];

  const float sl2 = a.scale * kLog2e;
  float o[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;  // rows g, g + 8

  for (int b = 0; b < nblk; ++b) {
    issue((b + 2) % kPStages, b + 2);
    cp_wait<2>();
    __syncthreads();
    const unsigned char* kt = ring + (b % kPStages) * 2 * TILE;
    const unsigned char* vt = kt + TILE;
    if constexpr (KQ != 0) {
      const unsigned char* kraw = ring + (b % kPStages) * 2 * PS::PQ;
      dequant_page<D>(kraw, KQ, a.kv_gs, kdq, tid, nthr);
      dequant_page<D>(kraw + PS::PQ, KQ, a.kv_gs, vdq, tid, nthr);
      __syncthreads();
      kt = kdq;
      vt = vdq;
    }
    float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int kk = 0; kk < KSTEPS; ++kk) {
      uint32_t r[4];
      const int rr = (lane & 7) + ((lane >> 4) << 3), cc = 2 * kk + ((lane >> 3) & 1);
      ldsm_x4(r, kt + swz<D>(rr, cc));
      mma_f16(s[0], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], r[0], r[1]);
      mma_f16(s[1], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], r[2], r[3]);
    }
    // causal mask in log2 units: s[j][0..1] row g, s[j][2..3] row g + 8
    const int tb = b * BT;
    float v[2][4];
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int tok = tb + 8 * j + 2 * t + e;
        v[j][e] = tok <= pos_g ? s[j][e] * sl2 : -INFINITY;
        v[j][2 + e] = tok <= pos_g8 ? s[j][2 + e] * sl2 : -INFINITY;
      }
    float mx0 = fmaxf(fmaxf(v[0][0], v[0][1]), fmaxf(v[1][0], v[1][1]));
    float mx1 = fmaxf(fmaxf(v[0][2], v[0][3]), fmaxf(v[1][2], v[1][3]));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);
    const float u0 = n0 == -INFINITY ? 0.f : n0, u1 = n1 == -INFINITY ? 0.f : n1;
    const float c0 = exp2f(m0 - u0), c1 = exp2f(m1 - u1);
    float p[2][4];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      p[j][0] = exp2f(v[j][0] - u0);
      p[j][1] = exp2f(v[j][1] - u0);
      p[j][2] = exp2f(v[j][2] - u1);
      p[j][3] = exp2f(v[j][3] - u1);
    }
    l0 = l0 * c0 + (p[0][0] + p[0][1] + p[1][0] + p[1][1]);
    l1 = l1 * c1 + (p[0][2] + p[0][3] + p[1][2] + p[1][3]);
    m0 = n0;
    m1 = n1;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      o[nt][0] *= c0;
      o[nt][1] *= c0;
      o[nt][2] *= c1;
      o[nt][3] *= c1;
    }
    // P as the A operand: (row g | g+8) × (tokens 2t.. | 8+2t..)
    const uint32_t pa0 = pack_half2(p[0][0], p[0][1]), pa1 = pack_half2(p[0][2], p[0][3]);
    const uint32_t pa2 = pack_half2(p[1][0], p[1][1]), pa3 = pack_half2(p[1][2], p[1][3]);
#pragma unroll
    for (int np = 0; np < NT / 2; ++np) {
      uint32_t r[4];
      const int rr = (lane & 7) + (((lane >> 3) & 1) << 3), cc = 2 * np + (lane >> 4);
      ldsm_x4_t(r, vt + swz<D>(rr, cc));
      mma_f16(o[2 * np], pa0, pa1, pa2, pa3, r[0], r[1]);
      mma_f16(o[2 * np + 1], pa0, pa1, pa2, pa3, r[2], r[3]);
    }
    __syncthreads();  // every warp is done with this stage before it is refilled
  }
  cp_wait<0>();
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  grid_launch_dependents();

  // rows g and g + 8 of head h·rep + warp
  half* Out = reinterpret_cast<half*>(a.out);
  const int hq = h * rep + warp;
  const float i0 = l0 > 0.f ? 1.f / l0 : 0.f, i1 = l1 > 0.f ? 1.f / l1 : 0.f;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int d = nt * 8 + 2 * t;
    if (g < nr)
      *reinterpret_cast<__half2*>(Out + long(r0 + g) * Hq * D + hq * D + d) =
          __floats2half2_rn(o[nt][0] * i0, o[nt][1] * i0);
    if (g + 8 < nr)
      *reinterpret_cast<__half2*>(Out + long(r0 + g + 8) * Hq * D + hq * D + d) =
          __floats2half2_rn(o[nt][2] * i1, o[nt][3] * i1);
  }
}

template <int D, int KQ>
nmx_status_t launch_prefill(Ctx* c, const AttnArgs& a, const int2* items, int n_items) {
  const int rep = a.Hq / a.Hkv;
  const size_t smem = PrefillSmem<D, KQ>::BYTES;
  auto kern = paged_prefill_mma_kernel<D, KQ>;
  static std::mutex mu;
  static std::map<int, bool> set;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (!set[c->device]) {
      NMX_CUDA_OK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
      set[c->device] = true;
    }
  }
  return launch(c, kern, dim3(n_items, a.Hkv), dim3(rep * 32), smem, a, items);
}

template <int D>
nmx_status_t launch_prefill_q(Ctx* c, const AttnArgs& a, const int2* items, int n_items) {
  if (a.kv_bits == 4) return launch_prefill<D, 4>(c, a, items, n_items);
  if (a.kv_bits == 8) return launch_prefill<D, 8>(c, a, items, n_items);
  return launch_prefill<D, 0>(c, a, items, n_items);
}

}  // namespace

int prefill_items(const int32_t* row_seq, int T, int D, int rep, int2* items_host, int* n_tc) {
  const bool tc = prefill_tc_supported(D, rep);
  const int qp = tc ? 128 / rep : kPQB;
  std::vector<int2> small;
  int n = 0;
  for (int r = 0; r < T;) {
    int e = r + 1;
    while (e < T && e - r < qp && row_seq[e] == row_seq[r]) ++e;
    const int nr = e - r;
    if (tc && !(nr <= kPQB && nr * rep < 64)) {
      items_host[n++] = make_int2(r, nr);
    } else {
      for (int s = r; s < e; s += kPQB) small.push_back(make_int2(s, std::min(kPQB, e - s)));
    }
    r = e;
  }
  *n_tc = n;
  for (const int2& it : small) items_host[n++] = it;
  return n;
}

nmx_status_t paged_prefill_attention(Ctx* c, const AttnArgs& a, const int2* items, int n_items) {
  NMX_CHECK(a.BT == 16, NMX_ERR_UNSUPPORTED, "prefill attention: block size must be 16 tokens");
  NMX_CHECK(a.Hkv > 0 && a.Hq % a.Hkv == 0 && a.Hq / a.Hkv <= kPMaxRep, NMX_ERR_UNSUPPORTED,
            "prefill attention: q heads per kv head must be <= 8");
  if (n_items == 0) return NMX_OK;
  NMX_CHECK(a.kv_bits == 0 || ((a.kv_bits == 4 || a.kv_bits == 8) && (a.kv_gs == 32 || a.kv_gs == 64)),
            NMX_ERR_UNSUPPORTED, "prefill attention: quantized pages need 4 or 8 bits, group 32 or 64");
  NMX_CHECK(a.kv_bits == 0 || a.prefill_tc_items == 0, NMX_ERR_INVALID,
            "prefill attention: quantized pages go through the small-item kernel");
  const int n_tc = std::min(a.prefill_tc_items, n_items);
  if (n_tc > 0) NMX_TRY(paged_prefill_attention_tc(c, a, items, n_tc));
  if (n_tc == n_items) return NMX_OK;
  items += n_tc;
  n_items -= n_tc;
  if (a.D == 128) return launch_prefill_q<128>(c, a, items, n_items);
  if (a.D == 64) return launch_prefill_q<64>(c, a, items, n_items);
  NMX_CHECK(false, NMX_ERR_UNSUPPORTED, "prefill attention: head_dim must be 64 or 128");
}

}  // namespace nmx
