// Paged prefill attention on the 5th-generation tensor cores (tcgen05).
//
// A work item is up to qp = 128 / rep consecutive query positions of one
// sequence; a CTA owns (item, kv head) and stacks the item's positions × the
// rep q heads of that kv head into one 128-row tile (row = position · rep +
// head), so every K/V byte the CTA streams serves 128 / rep positions × rep
// heads. Per chunk of 128 keys (8 pages of 16 tokens):
//   * warp 4 (one thread) brings the chunk's K and V pages with tensor-map
//     copies of this GPU's own KV pool (boxes of 16 tokens × 64 d, 128-byte
//     swizzle) into a 3-stage ring; pages past the last needed key are
//     copied from a row past the pool's end, which the copy fills with zeros;
//   * warp 5 (one thread) issues S = Q·Kᵀ (M 128 rows, N 128 keys, K = head
//     dim; Q from TMEM, K from shared memory, K-major) into one of two TMEM
//     S buffers, and warp 6 (one thread) O += P·V (P from TMEM, V from
//     shared memory read MN-major, i.e. straight from the page layout) into
//     the TMEM output: an issuing thread pays tens of cycles per MMA, so
//     the two streams go from two threads; a K/V stage is free once both
//     have committed it;
//   * warps 0-3 (thread i = tile row i = TMEM lane i) read their S row, mask
//     keys past the row's position, and run the online softmax in the log2
//     domain with a lazy reference maximum: p = exp2(s - m_ref) and m_ref
//     moves (rescaling O in TMEM and the denominator) only when the row's
//     maximum exceeds it by more than 8, so p <= 256 stays exact enough in
//     f16 and most chunks skip the O round trip; P (f16) goes to TMEM as the
//     next MMA's A operand.
// After the last chunk the same threads divide O by the denominator and
// store their rows. Every mbarrier wait is bounded by the context's poll
// limit: one that runs out sets kErrPipeWait and the CTA skips to its
// teardown (TMEM is always freed). No load uses cluster multicast.
#include <algorithm>
#include <map>
#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "tc_common.cuh"

namespace nmx {

namespace {

using tc::mbar_arrive;
using tc::mbar_expect_tx;
using tc::mbar_init;
using tc::mbar_wait;
using tc::sa_;

constexpr int kPTRows = 128;    // tile rows: (position, q head) pairs
constexpr int kPTKeys = 128;    // keys per chunk (8 pages)
constexpr int kPTStages = 3;    // K/V chunk stages
constexpr int kPTWarpTma = 4, kPTWarpMma = 5, kPTWarpMmaO = 6;  // S = Q·Kᵀ issuer, O += P·V issuer
constexpr int kPTThreads = 7 * 32;
constexpr int kBox = 16 * 64 * 2;  // one tensor copy: 16 tokens × 64 d of f16

template <int D>
struct PTL {
  static constexpr int kDH = D / 64;                // 64-wide d halves
  static constexpr int kKBytes = 8 * kDH * kBox;    // K (or V) of one chunk: [d half][page][16][64]
  static constexpr int kStage = 2 * kKBytes;
  static constexpr size_t kSmem = size_t(kPTStages) * kStage + 1024;
  // TMEM columns (512 allocated): O, two S buffers, Q and P as f16 pairs
  static constexpr uint32_t kColO = 0;
  static constexpr uint32_t kColS = 128;
  static constexpr uint32_t kColQ = 384;
  static constexpr uint32_t kColP = 448;
};

__device__ __forceinline__ void mma_ta(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p; }" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// MN-major operand in the 128-byte swizzle (a V page as stored: 64 d of one
// token per 128-byte row): `lbo` bytes between 64-wide MN atoms (d halves),
// `sbo` bytes between 8-row groups along K (tokens)
__device__ __forceinline__ uint64_t smem_desc_mn(const void* p, uint32_t lbo, uint32_t sbo) {
  const uint64_t a = sa_(p);
  return ((a >> 4) & 0x3FFFull) | (uint64_t((lbo >> 4) & 0x3FFFu) << 16) | (uint64_t((sbo >> 4) & 0x3FFFu) << 32) |
         (1ull << 46) | (2ull << 61);
}

__device__ __forceinline__ void tma_2d(void* dst, const CUtensorMap* tm, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          sa_(dst)),
      "l"(tm), "r"(x), "r"(y), "r"(sa_(bar))
      : "memory");
}

struct PTArgs {
  const half* q;  // [T][Hq * D], roped
  long ldq;
  half* out;      // [T][Hq * D]
  long ldo;
  const int* block_tables;
  int max_blocks;
  const int* tok_seq;
  const int* tok_pos;
  const int2* items;  // (first row, rows)
  int Hq, Hkv, rep;
  float sl2;          // softmax scale × log2(e)
  int pool_rows;      // rows of the K/V tensor maps (blocks × Hkv × 16): a copy from here reads zeros
  unsigned* err;
};

template <int D>
__global__ void __launch_bounds__(kPTThreads, 1) paged_prefill_tc_kernel(const __grid_constant__ CUtensorMap tm_k,
                                                                         const __grid_constant__ CUtensorMap tm_v,
                                                                         PTArgs a) {
  using L = PTL<D>;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((1024u - (sa_(smem_raw) & 1023u)) & 1023u);
  __shared__ __align__(8) uint64_t kv_full[kPTStages], kv_empty[kPTStages];
  __shared__ __align__(8) uint64_t s_full[2], s_free[2], p_full, o_done, q_ready;
  __shared__ uint32_t s_taddr;
  __shared__ int s_fail;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const unsigned lim = wait_polls(a.err);
  const int h = blockIdx.y;
  const int2 it = a.items[blockIdx.x];
  const int r0 = it.x, nr = it.y;

  if (tid == 0) {
    for (int s = 0; s < kPTStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 2);  // the S issuer (K read) and the O issuer (V read)
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&s_free[s], kPTRows / 32);  // one arrival per softmax warp
    }
    mbar_init(&p_full, kPTRows / 32);
    mbar_init(&o_done, 1);
    mbar_init(&q_ready, kPTRows / 32);
    s_fail = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kPTWarpMma) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(sa_(&s_taddr))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t taddr = s_taddr;

  grid_wait();  // q rows and the pages (RoPE + append) come from the kernels before
  const int seq = a.tok_seq[r0];
  const int pos_last = a.tok_pos[r0 + nr - 1];
  const int nchunks = pos_last / kPTKeys + 1;
  const int npages = pos_last / 16 + 1;

  if (warp == kPTWarpTma) {
    // ------------------------------------------------------- K/V pages
    if (lane == 0) {
      const int* bt = a.block_tables + long(seq) * a.max_blocks;
      for (int j = 0; j < nchunks; ++j) {
        const int st = j % kPTStages;
        if (j >= kPTStages && !mbar_wait(&kv_empty[st], ((j / kPTStages) - 1) & 1, lim)) {
          atomicOr(a.err, kErrPipeWait);
          s_fail = 1;
          break;
        }
        unsigned char* kd = smem + st * L::kStage;
        unsigned char* vd = kd + L::kKBytes;
        mbar_expect_tx(&kv_full[st], L::kStage);
#pragma unroll 1
        for (int p = 0; p < 8; ++p) {
          const int pg = j * 8 + p;
          const int row = pg < npages ? (bt[pg] * a.Hkv + h) * 16 : a.pool_rows;
#pragma unroll
          for (int dh = 0; dh < L::kDH; ++dh) {
            tma_2d(kd + (dh * 8 + p) * kBox, &tm_k, dh * 64, row, &kv_full[st]);
            tma_2d(vd + (dh * 8 + p) * kBox, &tm_v, dh * 64, row, &kv_full[st]);
          }
        }
      }
    }
  } else if (warp == kPTWarpMma) {
    // ------------------------------------------------------------ MMA issue
    if (lane == 0) {
      const uint32_t idS = tc::idesc_f16(128, kPTKeys);
      bool ok = mbar_wait(&q_ready, 0, lim);
      auto issue_s = [&](int j) -> bool {
        const int st = j % kPTStages, sb = j & 1;
        if (!mbar_wait(&kv_full[st], (j / kPTStages) & 1, lim)) return false;
        if (j >= 2 && !mbar_wait(&s_free[sb], ((j >> 1) - 1) & 1, lim)) return false;
        tc::tc_fence_after();
        const unsigned char* kd = smem + st * L::kStage;
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks)
          mma_ta(taddr + L::kColS + uint32_t(sb * kPTKeys), taddr + L::kColQ + uint32_t(8 * ks),
                 tc::smem_desc(kd + (ks >> 2) * 8 * kBox + 32 * (ks & 3)), idS, ks > 0 ? 1u : 0u);
        tc::mma_commit(&s_full[sb]);
        return true;
      };
      // one issuing thread pays tens of cycles per tcgen05.mma: the S
      // products and the P·V products come from two threads (two warps)
      for (int j = 0; ok && j < nchunks; ++j) {
        if (!issue_s(j)) ok = false;
        else tc::mma_commit(&kv_empty[j % kPTStages]);
      }
      if (!ok) {
        atomicOr(a.err, kErrPipeWait);
        s_fail = 1;
      }
    }
  } else if (warp == kPTWarpMmaO) {
    if (lane == 0) {
      const uint32_t idO = tc::idesc_f16(128, D) | (1u << 16);  // B (V) MN-major
      bool ok = true;
      for (int j = 0; ok && j < nchunks; ++j) {
        // P(j) is in TMEM (which also means S(j) and K(j) are done with)
        if (!mbar_wait(&p_full, j & 1, lim)) {
          ok = false;
          break;
        }
        tc::tc_fence_after();
        const unsigned char* vd = smem + (j % kPTStages) * L::kStage + L::kKBytes;
#pragma unroll
        for (int ks = 0; ks < kPTKeys / 16; ++ks)
          mma_ta(taddr + L::kColO, taddr + L::kColP + uint32_t(8 * ks), smem_desc_mn(vd + ks * 2048, 8 * kBox, 1024),
                 idO, (j > 0 || ks > 0) ? 1u : 0u);
        tc::mma_commit(&kv_empty[j % kPTStages]);
        tc::mma_commit(&o_done);
      }
      if (!ok) {
        atomicOr(a.err, kErrPipeWait);
        s_fail = 1;
      }
    }
  } else {
    // ---------------------------------------- softmax rows (warps 0-3)
    const int i = tid;  // tile row = TMEM lane
    const int pi = i / a.rep, hi = i % a.rep;
    const bool valid = pi < nr && pi * a.rep + a.rep <= kPTRows;
    const int pos = valid ? a.tok_pos[r0 + pi] : -1;
    const uint32_t lane_base = taddr + (uint32_t(32 * warp) << 16);
    {
      // this row's q (f16 pairs in k order) into the Q columns
      uint32_t qw[D / 2];
      const uint4* src = reinterpret_cast<const uint4*>(a.q + long(r0 + pi) * a.ldq + long(h * a.rep + hi) * D);
#pragma unroll
      for (int c = 0; c < D / 8; ++c) {
        const uint4 v = valid ? src[c] : make_uint4(0, 0, 0, 0);
        qw[4 * c] = v.x;
        qw[4 * c + 1] = v.y;
        qw[4 * c + 2] = v.z;
        qw[4 * c + 3] = v.w;
      }
#pragma unroll
      for (int c = 0; c < D / 64; ++c) tmem_st32(lane_base + L::kColQ + 32 * c, qw + 32 * c);
      tmem_st_wait();
      tc::tc_fence_before();
      tc::warp_arrive(&q_ready);
    }
    // tcgen05.ld / st are warp-collective: every branch around them below
    // is uniform over the warp (waits are agreed with __all_sync, the O
    // rescale runs for the whole warp with factor 1 on lanes that keep
    // their reference, the epilogue loads for every lane)
    float m_ref = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nchunks; ++j) {
      const int sb = j & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&s_full[sb], (j >> 1) & 1, lim));
      if (!ok) break;
      tc::tc_fence_after();
      const uint32_t scol = lane_base + L::kColS + uint32_t(sb * kPTKeys);
      const int key0 = j * kPTKeys;
      // pass 1: the row's maximum over this chunk's unmasked keys
      float mx = -INFINITY;
#pragma unroll 1
      for (int c0 = 0; c0 < kPTKeys; c0 += 32) {
        float v[32];
        tc::tmem_ld32(scol + c0, v);
#pragma unroll
        for (int e = 0; e < 32; ++e)
          if (key0 + c0 + e <= pos) mx = fmaxf(mx, v[e] * a.sl2);
      }
      // the reference moves when the maximum passes it by more than 8
      // (false for a fully masked chunk: mx = -inf)
      const bool move = mx > m_ref + 8.0f;
      float f = 1.f;
      if (move) {
        f = m_ref == -INFINITY ? 0.f : exp2f(m_ref - mx);
        l *= f;
        m_ref = mx;
      }
      bool waited = false;
      if (j > 0 && __any_sync(0xffffffffu, move && f != 0.f)) {
        // O holds P·V of chunks 0..j-1: scale it in place
        ok = __all_sync(0xffffffffu, mbar_wait(&o_done, (j - 1) & 1, lim));
        if (!ok) break;
        waited = true;
        tc::tc_fence_after();
#pragma unroll 1
        for (int c0 = 0; c0 < D; c0 += 32) {
          float v[32];
          tc::tmem_ld32(lane_base + L::kColO + c0, v);
          uint32_t u[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) u[e] = __float_as_uint(v[e] * f);
          tmem_st32(lane_base + L::kColO + c0, u);
        }
        tmem_st_wait();
      }
      // pass 2: p = exp2(s - m_ref) as f16 pairs, the denominator in f32
      uint32_t pw[kPTKeys / 2];
#pragma unroll
      for (int c0 = 0; c0 < kPTKeys; c0 += 32) {
        float v[32];
        tc::tmem_ld32(scol + c0, v);
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const float p0 = (key0 + c0 + e <= pos) ? exp2f(v[e] * a.sl2 - m_ref) : 0.f;
          const float p1 = (key0 + c0 + e + 1 <= pos) ? exp2f(v[e + 1] * a.sl2 - m_ref) : 0.f;
          const __half2 hp = __floats2half2_rn(p0, p1);
          l += __low2float(hp) + __high2float(hp);
          pw[(c0 + e) / 2] = *reinterpret_cast<const uint32_t*>(&hp);
        }
      }
      tc::tc_fence_before();
      tc::warp_arrive(&s_free[sb]);
      // P's columns are free once the previous P·V has completed
      if (j > 0 && !waited) {
        ok = __all_sync(0xffffffffu, mbar_wait(&o_done, (j - 1) & 1, lim));
        if (!ok) break;
      }
      tc::tc_fence_after();
      tmem_st32(lane_base + L::kColP, pw);
      tmem_st32(lane_base + L::kColP + 32, pw + 32);
      tmem_st_wait();
      tc::tc_fence_before();
      tc::warp_arrive(&p_full);
    }
    // ------------------------------------------------------------ epilogue
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&o_done, (nchunks - 1) & 1, lim));
    if (!ok) {
      atomicOr(a.err, kErrPipeWait);
      s_fail = 1;
    }
    tc::tc_fence_after();
    if (ok) {
      const float inv = l > 0.f ? 1.0f / l : 0.f;
      uint4* dst = reinterpret_cast<uint4*>(a.out + long(r0 + pi) * a.ldo + long(h * a.rep + hi) * D);
#pragma unroll 1
      for (int c0 = 0; c0 < D; c0 += 32) {
        float v[32];
        tc::tmem_ld32(lane_base + L::kColO + c0, v);
        if (valid) {
#pragma unroll
          for (int e = 0; e < 32; e += 8) {
            uint4 o;
            __half2* oh = reinterpret_cast<__half2*>(&o);
#pragma unroll
            for (int k = 0; k < 4; ++k) oh[k] = __floats2half2_rn(v[e + 2 * k] * inv, v[e + 2 * k + 1] * inv);
            dst[(c0 + e) / 8] = o;
          }
        }
      }
    }
  }
  grid_launch_dependents();
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  if (warp == kPTWarpMma)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(taddr) : "memory");
}

template <int D>
nmx_status_t launch_tc(Ctx* c, const AttnArgs& a, const int2* items, int n_items) {
  using L = PTL<D>;
  auto kern = paged_prefill_tc_kernel<D>;
  static std::mutex mu;
  static std::map<int, bool> set;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (!set[c->device]) {
      NMX_CUDA_OK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(L::kSmem)));
      set[c->device] = true;
    }
  }
  const long rows = long(a.pool_blocks) * a.Hkv * 16;
  NMX_CHECK(rows > 0 && rows < (1L << 31), NMX_ERR_UNSUPPORTED, "prefill attention: pool too large for a tensor map");
  CUtensorMap tk, tv;
  NMX_TRY(tc::encode_x_map(&tk, a.k_cache, D, int(rows), D, 16));
  NMX_TRY(tc::encode_x_map(&tv, a.v_cache, D, int(rows), D, 16));
  PTArgs p;
  p.q = static_cast<const half*>(a.q);
  p.ldq = a.ldq;
  p.out = static_cast<half*>(a.out);
  p.ldo = long(a.Hq) * D;
  p.block_tables = a.block_tables;
  p.max_blocks = a.max_blocks;
  p.tok_seq = a.tok_seq;
  p.tok_pos = a.tok_pos;
  p.items = items;
  p.Hq = a.Hq;
  p.Hkv = a.Hkv;
  p.rep = a.Hq / a.Hkv;
  p.sl2 = a.scale * 1.4426950408889634f;
  p.pool_rows = int(rows);
  p.err = a.err;
  return launch(c, kern, dim3(n_items, a.Hkv), dim3(kPTThreads), L::kSmem, tk, tv, p);
}

}  // namespace

bool prefill_tc_supported(int D, int rep) { return (D == 64 || D == 128) && rep >= 1 && rep <= 8; }

nmx_status_t paged_prefill_attention_tc(Ctx* c, const AttnArgs& a, const int2* items, int n_items) {
  NMX_CHECK(a.BT == 16, NMX_ERR_UNSUPPORTED, "prefill attention: block size must be 16 tokens");
  NMX_CHECK(a.Hkv > 0 && a.Hq % a.Hkv == 0 && prefill_tc_supported(a.D, a.Hq / a.Hkv), NMX_ERR_UNSUPPORTED,
            "prefill attention (tensor cores): head_dim 64 or 128, at most 8 q heads per kv head");
  NMX_CHECK(a.err != nullptr && a.pool_blocks > 0, NMX_ERR_INVALID, "prefill attention: no error word or pool size");
  NMX_CHECK(reinterpret_cast<uintptr_t>(a.q) % 16 == 0 && (a.ldq * 2) % 16 == 0 &&
                reinterpret_cast<uintptr_t>(a.out) % 16 == 0,
            NMX_ERR_UNSUPPORTED, "prefill attention: q and out must be 16-byte aligned");
  if (n_items == 0) return NMX_OK;
  return a.D == 128 ? launch_tc<128>(c, a, items, n_items) : launch_tc<64>(c, a, items, n_items);
}

}  // namespace nmx
