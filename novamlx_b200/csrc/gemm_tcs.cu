// Decode-batch GEMM on the 5th-generation tensor cores: y[M, N] = x[M, K] ·
// dequant(W)[N, K]ᵀ for 1..128 activation rows (a continuous-batching decode
// step, a speculative verify block), W in decode records (4-bit, group 64).
//
// At these row counts the product is bound by the weight stream, so the
// tile is turned around: 128 WEIGHT rows are the MMA's M (TMEM lanes) and
// the activation rows, rounded up to a multiple of 16 (NT), are its N
// (TMEM columns). A CTA owns a group of tg such weight tiles (for SiLU·up,
// gate/up pairs: both halves of an output tile sit in one TMEM lane) and a
// contiguous share of the K blocks (128 k); the grid is (groups × S
// K-shares), sized by the host to one wave over the SMs. Per K block:
//   * warp 21 brings the 8 records of each of the group's tiles into a ring
//     of raw slots with ONE 3-d tensor copy per tile (a copy per record
//     costs more issue time than its bytes take to arrive); these are
//     weights, so the copies may start before the programmatic-launch wait;
//   * warp 20 loads the block's x tile once for the whole group (two TMA
//     boxes of 64 k × NT rows, SWIZZLE_128B, rows past M read as zeros) and
//     warp 22 permutes it in place to the dequantizers' k order (see
//     dequant_row_words);
//   * three or four warpgroups (warps 0-15) take the (block, tile) units in
//     turn: each thread reads one weight row of the unit (64 bytes,
//     conflict-free: see lane_row) and writes its 128 f16 weights w = s·q + b
//     straight into its TMEM lane with tcgen05.st, into its warpgroup's
//     64-column A stage, so the dequantized tile never touches shared memory;
//   * lane 0 of warps 16-19 (up to four issuers; issuer j owns the tiles and
//     A stages ≡ j) issues eight tcgen05.mma (A from TMEM, x from shared
//     memory; M = 128, N = NT, K = 16) per unit into that tile's accumulator
//     (TMEM columns tile·NT ...), committing the A stage (and after its last
//     tile of the block the x tile) back to its producers.
// After the last block warps 0-15 read the accumulators (tcgen05.ld 32x32b;
// warp w: lanes 32 (w % 4) .., every fourth 8-column chunk). With one K share they run
// the epilogue directly; with S shares each CTA stores its f32 partial
// tiles, bumps the group's counter and waits (bounded) until all S have
// (the grid is a single wave of one CTA per SM, so they are resident or
// done); then each CTA sums its slice of the group's outputs over the S
// partials in share order (deterministic) and runs the epilogue; a second
// round of arrivals lets the last CTA reset the counter. Every mbarrier
// wait is bounded: one that runs out sets bit 0 of *err and the CTA skips
// to its teardown (TMEM is always freed).
#include <algorithm>
#include <map>
#include <mutex>

#include "comm.h"
#include "common.cuh"
#include "kernels.h"
#include "tc_common.cuh"

namespace nmx {

namespace {

using tc::kRecG;
using tc::mbar_arrive;
using tc::mbar_expect_tx;
using tc::mbar_init;
using tc::mbar_wait;
using tc::sa_;
using tc::smem_desc;

constexpr int kDG = 4;                      // dequant warpgroups (3 or 4 of them take units in turn)
constexpr int kSDW = 4 * kDG;               // dequant / epilogue warps
constexpr int kNIMax = 4;                   // MMA-issuing warps (one per dequant warpgroup at most)
constexpr int kSThreads = (kSDW + kNIMax + 3) * 32;  // + MMA-issue, x-tile, record-loader, x-permute warps
constexpr int kSWMma = kSDW, kSWTma = kSDW + kNIMax, kSWRec = kSDW + kNIMax + 1, kSWPerm = kSDW + kNIMax + 2;
constexpr int kAST = 4;                     // dequantized weight stages, in TMEM
constexpr int kAStageCols = 64;             // 128 k of f16, two per 32-bit column
constexpr int kAccCols = 512 - kAST * kAStageCols;  // accumulator columns
constexpr int kXSMax = 8;                   // x stages
constexpr int kRSMax = 24;                  // raw record slots
using tc::kRecPad;                          // shared-memory stride of a record
constexpr int kRawSlot = 8 * kRecPad;       // the 8 records of one tile and K block
constexpr int kMaxTG = 16;                  // weight tiles per CTA
constexpr int kMaxNT = kTcsMaxRows;
constexpr size_t kSmemCap = 225 * 1024;  // dynamic shared memory the kernel may ask for (plus 1 KB static)

struct TcsArgs {
  const unsigned char* w;  // decode records of the whole matrix
  int M, NT, K, nb;        // rows of x, MMA N, K, K / 128
  int n_atiles;            // weight tiles (SiLU: 2 per output tile)
  int tg, S;               // tiles per group, K shares
  int ndg;                 // dequant warpgroups taking units (3 or 4; each owns A stage dg)
  int ni;                  // MMA-issuing warps (divides ndg and tg)
  int rs, xs;              // raw slots, x stages
  uint32_t idesc;
  long long pair_tiles;    // SiLU: 16-row tile offset of the up rows
  const half* bias;
  half* y;
  long ldy;
  const half* res;
  long ldres;
  float* partials;         // [groups][S][tg][NT][128]
  unsigned* counters;      // [groups], zero between launches
  unsigned* err;
  bool weights_static;
  // tensor parallelism (residual epilogue only): this rank's partial goes
  // to its exchange region and the CTA sums every rank's (fused exchange)
  bool fused;
  ExchangeArgs x;
};

// 16-row record tile r8 (0..7) of weight tile `at`
template <int EPI>
__device__ __forceinline__ long long tile16(const TcsArgs& a, int at, int r8) {
  if constexpr (EPI == EPI_SILU) {
    const long long o = at >> 1;
    return (at & 1) ? a.pair_tiles + o * 8 + r8 : o * 8 + r8;
  } else {
    return (long long)at * 8 + r8;
  }
}

// one output value from the f32 accumulator(s), the GEMM epilogues' rounding
template <int EPI>
__device__ __forceinline__ half epi_value(const TcsArgs& a, float acc, float up, int m, long n) {
  if constexpr (EPI == EPI_SILU) {
    const float g16 = rnd<half>(acc), u16 = rnd<half>(up);
    return __float2half_rn(rnd<half>(g16 / (1.0f + expf(-g16))) * u16);
  } else {
    float v = rnd<half>(acc);
    if (a.bias) v = rnd<half>(v + __half2float(a.bias[n]));
    if constexpr (EPI == EPI_RESID) v += __half2float(a.res[(long)m * a.ldres + n]);
    return __float2half_rn(v);
  }
}

__device__ __forceinline__ void dq_bar() { asm volatile("bar.sync 1, %0;" ::"n"(kSDW * 32) : "memory"); }

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Fused exchange: this CTA's partial rows are in its region; publish slot
// `slot` at epoch e to every rank and wait (bounded) until every rank has
// published it. Called by all epilogue threads.
__device__ __forceinline__ bool tp_exchange(const ExchangeArgs& x, int slot, unsigned e, unsigned* err, int* s_ok) {
  __threadfence_system();
  dq_bar();
  if (threadIdx.x == 0) {
    for (int q = 0; q < x.world; ++q) st_release_sys(x.peer_tflags[q] + slot, e);
    int ok = 1;
    const unsigned lim = wait_polls(err);
    for (int q = 0; q < x.world && ok; ++q) {
      unsigned it = 0;
      while ((int)(ld_acquire_sys(x.my_tflags + size_t(q) * kMaxTileFlags + slot) - e) < 0)
        if (++it >= lim) {
          ok = 0;
          atomicOr(err, kErrPeerWait);
          break;
        }
    }
    *s_ok = ok;
  }
  dq_bar();
  return *s_ok != 0;
}

// y = res + Σ_ranks partial (f16 partials summed in rank order in f32, then
// rounded) — the rule of the separate exchange kernel
__device__ __forceinline__ half tp_combine(const ExchangeArgs& x, const half* res, long ldres, long ld, int m, long n) {
  float acc = 0.f;
  for (int q = 0; q < x.world; ++q) acc += __half2float(__ldcg(x.part[q] + (long)m * ld + n));
  return __float2half_rn(__half2float(res[(long)m * ldres + n]) + rnd<half>(acc));
}

// Weight row (record r8 of the tile, row g16 of the record) held by TMEM
// lane L. The eight lanes of each quarter warp take rows g, g+1 (g even) of
// four consecutive records, so with records kRecPad apart their 16-byte
// loads of a row fall in eight different bank groups.
__device__ __forceinline__ void lane_row(int L, int& r8, int& g16) {
  const int Q = L >> 3, j = L & 7;
  r8 = 4 * (Q & 1) + (j & 3);
  g16 = 8 * ((Q >> 1) & 1) + 2 * (Q >> 2) + (j >> 2);
}

// D[tmem] (+)= A[tmem] · B[smem]ᵀ, kind::f16
__device__ __forceinline__ void mma_f16_ta(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p; }" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 32 consecutive 32-bit columns of this thread's TMEM lane
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

// the 16 words of one record row (both groups) as 128 f16 weights
// w = s·q + b, two per 32-bit column: group gi in out[gi]. XP: word w's
// eight weights fill columns 4w .. 4w+3 as (w0, w4), (w1, w5), (w2, w6),
// (w3, w7), the order the nibble step makes them in, and the x block is
// permuted to match; otherwise in k order (four byte permutes per word).
template <bool XP>
__device__ __forceinline__ void dequant_row_words(const uint4* c, __half2 s2[2], __half2 s16[2], __half2 b2[2],
                                                  uint32_t out[2][32]) {
  const __half2 k1024 = __float2half2_rn(1024.f);
#pragma unroll
  for (int t = 0; t < 4; ++t) {
#pragma unroll
    for (int gi = 0; gi < 2; ++gi) {
#pragma unroll
      for (int ws = 0; ws < 2; ++ws) {
        const uint32_t word = gi ? (ws ? c[t].w : c[t].z) : (ws ? c[t].y : c[t].x);
        const int w = 2 * t + ws;  // word of the group: k 8w .. 8w+7
        uint32_t P[4];
        dequant_word<4>(word, P);  // (q0,q4), (16q1,16q5), (q2,q6), (16q3,16q7), each + 1024
        __half2 v0 = __hfma2(__hsub2(*reinterpret_cast<__half2*>(&P[0]), k1024), s2[gi], b2[gi]);
        __half2 v1 = __hfma2(__hsub2(*reinterpret_cast<__half2*>(&P[1]), k1024), s16[gi], b2[gi]);
        __half2 v2 = __hfma2(__hsub2(*reinterpret_cast<__half2*>(&P[2]), k1024), s2[gi], b2[gi]);
        __half2 v3 = __hfma2(__hsub2(*reinterpret_cast<__half2*>(&P[3]), k1024), s16[gi], b2[gi]);
        const uint32_t u0 = *reinterpret_cast<uint32_t*>(&v0), u1 = *reinterpret_cast<uint32_t*>(&v1);
        const uint32_t u2 = *reinterpret_cast<uint32_t*>(&v2), u3 = *reinterpret_cast<uint32_t*>(&v3);
        if constexpr (XP) {
          out[gi][4 * w + 0] = u0;
          out[gi][4 * w + 1] = u1;
          out[gi][4 * w + 2] = u2;
          out[gi][4 * w + 3] = u3;
        } else {
          out[gi][4 * w + 0] = __byte_perm(u0, u1, 0x5410);  // w0, w1
          out[gi][4 * w + 1] = __byte_perm(u2, u3, 0x5410);  // w2, w3
          out[gi][4 * w + 2] = __byte_perm(u0, u1, 0x7632);  // w4, w5
          out[gi][4 * w + 3] = __byte_perm(u2, u3, 0x7632);  // w6, w7
        }
      }
    }
  }
}

template <int EPI, bool XP>
__global__ void __launch_bounds__(kSThreads, 1) qgemm_tcs_kernel(const __grid_constant__ CUtensorMap tmap_x,
                                                                  const __grid_constant__ CUtensorMap tmap_w,
                                                                  TcsArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // 1024-byte aligned, derived from the shared array itself so that its
  // loads and stores compile to shared-memory (not generic) accesses
  unsigned char* smem = smem_raw + ((1024u - (tc::sa_(smem_raw) & 1023u)) & 1023u);
  __shared__ __align__(8) uint64_t a_full[kAST];
  __shared__ __align__(8) uint64_t a_empty[kAST];
  __shared__ __align__(8) uint64_t x_full[kXSMax];
  __shared__ __align__(8) uint64_t x_empty[kXSMax];
  __shared__ __align__(8) uint64_t x_ready[kXSMax];  // the x block is in the dequantizer's k order
  __shared__ __align__(8) uint64_t raw_full[kRSMax];
  __shared__ __align__(8) uint64_t raw_empty[kRSMax];
  __shared__ __align__(8) uint64_t acc_bar;
  __shared__ uint32_t s_taddr;
  __shared__ int s_fail;
  __shared__ unsigned s_last;  // every share of the group has stored its partials
  __shared__ unsigned s_epoch;  // fused exchange: this launch's epoch
  __shared__ int s_xok;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const unsigned lim = wait_polls(a.err);  // polls before a wait gives up
  const int grp = blockIdx.x, share = blockIdx.y;
  const int t0 = grp * a.tg;
  const int ntl = min(a.tg, a.n_atiles - t0);  // weight tiles of this CTA
  const int b0 = int((long long)share * a.nb / a.S), b1 = int((long long)(share + 1) * a.nb / a.S);
  const int nblk = b1 - b0;
  const int units = nblk * ntl;  // (block, tile) pairs, block-major
  // issuers: the largest of a.ni, a.ni / 2, .. dividing this CTA's tile count
  int ni = a.ni;
  while (ntl % ni) ni >>= 1;
  const int NT = a.NT;
  const int xhalf = NT * 128;    // bytes of one 64-k half of an x stage
  unsigned char* stX = smem;
  unsigned char* raw = stX + a.xs * 2 * xhalf;

  static_assert(kAST <= 32 && kXSMax <= 32 && kRSMax <= 32, "one barrier of each ring per lane");
  if (warp == 0) {
    // the lanes of warp 0 initialise the rings' barriers side by side
    if (lane < kAST) {
      mbar_init(&a_full[lane], 4);  // the four warps of one dequant warpgroup per unit
      mbar_init(&a_empty[lane], 1);
    }
    if (lane < kXSMax) {
      mbar_init(&x_full[lane], 1);
      mbar_init(&x_ready[lane], 1);   // the x-permute warp (warp_arrive)
      mbar_init(&x_empty[lane], ni);  // each issuer, after its last tile of the block
    }
    if (lane < kRSMax) {
      mbar_init(&raw_full[lane], 1);
      mbar_init(&raw_empty[lane], 4);
    }
    if (lane == 0) {
      mbar_init(&acc_bar, ni);
      s_fail = 0;
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kSWMma) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(sa_(&s_taddr))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t taddr = s_taddr;

  if (warp == kSWRec) {
    // ------------------------------------------------ raw records (weights)
    if (!a.weights_static) grid_wait();
    if (lane == 0) {
      // single-thread loops keep ring positions as counters: a runtime
      // division per unit would cost more than the unit's issue work
      int rs = 0, rph = 0, b = b0, ti = 0;
      for (int i = 0; i < units; ++i) {
        if (i >= a.rs && !mbar_wait(&raw_empty[rs], rph ^ 1, lim)) {
          atomicOr(a.err, kErrPipeWait);
          s_fail = 1;
          break;
        }
        mbar_expect_tx(&raw_full[rs], kRawSlot);
        tc::load_records(raw + rs * kRawSlot, &tmap_w, b, int(tile16<EPI>(a, t0 + ti, 0)), &raw_full[rs]);
        if (++rs == a.rs) {
          rs = 0;
          rph ^= 1;
        }
        if (++ti == ntl) {
          ti = 0;
          ++b;
        }
      }
    }
  } else if (warp == kSWTma) {
    // ------------------------------------------------------- x tiles (TMA)
    grid_wait();
    if (lane == 0) {
      int xs = 0, xph = 0;
      for (int bi = 0; bi < nblk; ++bi) {
        if (bi >= a.xs && !mbar_wait(&x_empty[xs], xph ^ 1, lim)) {
          atomicOr(a.err, kErrPipeWait);
          s_fail = 1;
          break;
        }
        unsigned char* dst = stX + xs * 2 * xhalf;
        mbar_expect_tx(&x_full[xs], 2 * xhalf);
#pragma unroll
        for (int h = 0; h < 2; ++h)
          asm volatile(
              "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
              "[%4];" ::"r"(sa_(dst + h * xhalf)),
              "l"(&tmap_x), "r"((b0 + bi) * 128 + h * 64), "r"(0), "r"(sa_(&x_full[xs]))
              : "memory");
        if (++xs == a.xs) {
          xs = 0;
          xph ^= 1;
        }
      }
    }
  } else if (warp == kSWPerm) {
    // ------------------------------------------- x blocks in the k order of A
    // The dequantizers write each record word's eight weights as the pairs
    // (w0, w4), (w1, w5), (w2, w6), (w3, w7) — the order the nibble-to-f16
    // step produces them in — so the x block is put in the same order: in
    // every 16-byte chunk (8 consecutive k; the 128-byte swizzle only moves
    // whole chunks) halves 0..7 become 0, 4, 1, 5, 2, 6, 3, 7.
    int xs = 0, xph = 0;
    const int chunks = 2 * xhalf / 16;
    for (int bi = 0; bi < nblk; ++bi) {
      if (!__all_sync(0xffffffffu, !s_fail && mbar_wait(&x_full[xs], xph, lim))) {
        atomicOr(a.err, kErrPipeWait);
        s_fail = 1;
        break;
      }
      uint4* st = reinterpret_cast<uint4*>(stX + xs * 2 * xhalf);
      for (int c = lane; XP && c < chunks; c += 32) {
        const uint4 v = st[c];
        st[c] = make_uint4(__byte_perm(v.x, v.z, 0x5410), __byte_perm(v.x, v.z, 0x7632), __byte_perm(v.y, v.w, 0x5410),
                           __byte_perm(v.y, v.w, 0x7632));
      }
      // generic-proxy writes, read by the tensor core's async proxy
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tc::warp_arrive(&x_ready[xs]);
      if (++xs == a.xs) {
        xs = 0;
        xph ^= 1;
      }
    }
  } else if (warp >= kSWMma && warp < kSWMma + kNIMax) {
    // ------------------------------------------------------------ MMA issue
    // Issuer j (lane 0 of warp kSWMma + j) takes the units i ≡ j (mod ni):
    // the tiles ti ≡ j and the A stages i mod ndg ≡ j (mod ni), so every
    // accumulator and every A stage has one issuer. An issuing thread pays
    // tens of cycles per tcgen05.mma, so one thread alone caps the tensor
    // pipe; ni threads keep up to ni instruction streams in flight.
    const int j = warp - kSWMma;
    if (lane == 0 && j < ni) {
      // per-MMA work is a few adds (descriptor start addresses advance in
      // 16-byte units)
      const uint64_t xdesc0 = smem_desc(stX);
      const uint32_t xstage_d = uint32_t(2 * xhalf) >> 4, xhalf_d = uint32_t(xhalf) >> 4;
      const uint32_t a0 = taddr + uint32_t(kAccCols), idesc = a.idesc;
      int ti = j, as = j, aph = 0, xs = 0, xph = 0;
      uint32_t first = 0u;  // 0 until the first block is in the accumulators
      for (int i = j; i < units; i += ni) {
        bool ok = !(ti == j && !mbar_wait(&x_ready[xs], xph, lim));
        if (ok && !mbar_wait(&a_full[as], aph, lim)) ok = false;
        if (!ok) {
          atomicOr(a.err, kErrPipeWait);
          s_fail = 1;
          break;
        }
        tc::tc_fence_after();
        const uint64_t bd = xdesc0 + uint64_t(xs * xstage_d);
        const uint32_t d = taddr + uint32_t(ti * NT);
        const uint32_t A = a0 + uint32_t(as * kAStageCols);
#pragma unroll
        for (int k16 = 0; k16 < 8; ++k16)
          mma_f16_ta(d, A + 8 * k16, bd + uint64_t((k16 >> 2) * xhalf_d + 2 * (k16 & 3)), idesc,
                     k16 ? 1u : first);
        tc::mma_commit(&a_empty[as]);
        as += ni;
        if (as >= a.ndg) {
          as -= a.ndg;
          aph ^= 1;
        }
        ti += ni;
        if (ti >= ntl) {
          tc::mma_commit(&x_empty[xs]);
          ti -= ntl;
          first = 1u;
          if (++xs == a.xs) {
            xs = 0;
            xph ^= 1;
          }
        }
      }
      tc::mma_commit(&acc_bar);
    }
  } else if (warp < kSDW) {
    // ------------------------------------------------ dequantize the tiles
    // warpgroup dg < ndg takes units dg, dg + ndg, ...; thread: TMEM lane L
    // (the warp's lane quarter), both groups of weight row lane_row(L)
    const int dg = warp >> 2, L = 32 * (warp & 3) + lane;
    int r8, g16;
    lane_row(L, r8, g16);
    const int rowoff = r8 * kRecPad + (g16 >> 3) * 512 + 64 * (g16 & 7);
    const int sboff = r8 * kRecPad + 1024 + (g16 & 7) * 4 + (g16 >> 3) * 2;
    const uint32_t lane_base = taddr + (uint32_t(32 * (warp & 3)) << 16);
    static_assert(kDG == kAST, "warpgroup dg owns A stage dg");
    const int as = dg, ndg = a.ndg;
    int rs = dg % a.rs, rph = (dg / a.rs) & 1;
    for (int i = dg; dg < ndg && i < units; i += ndg) {
      // waits agreed over the warp: its lanes arrive together (warp_arrive)
      if (!__all_sync(0xffffffffu, mbar_wait(&raw_full[rs], rph, lim))) {
        atomicOr(a.err, kErrPipeWait);
        s_fail = 1;
        break;
      }
      const unsigned char* slot = raw + rs * kRawSlot;
      uint4 c[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) c[t] = *reinterpret_cast<const uint4*>(slot + rowoff + 16 * t);
      __half2 s2[2], s16[2], b2[2];
#pragma unroll
      for (int gi = 0; gi < 2; ++gi) {
        const __half sc = *reinterpret_cast<const __half*>(slot + sboff + gi * 32);
        const __half bi = *reinterpret_cast<const __half*>(slot + sboff + 64 + gi * 32);
        s2[gi] = __halves2half2(sc, sc);
        s16[gi] = __hmul2(s2[gi], __float2half2_rn(0.0625f));
        b2[gi] = __halves2half2(bi, bi);
      }
      uint32_t out[2][32];
      dequant_row_words<XP>(c, s2, s16, b2, out);
      tc::warp_arrive(&raw_empty[rs]);  // the slot's bytes are in registers
      // only the TMEM stores wait for the stage's previous MMAs: the loads
      // and the dequantisation above overlap them
      if (!__all_sync(0xffffffffu, i < ndg || mbar_wait(&a_empty[as], ((i / ndg) - 1) & 1, lim))) {
        atomicOr(a.err, kErrPipeWait);
        s_fail = 1;
        break;
      }
      tc::tc_fence_after();         // after the wait for the stage's last MMAs
      const uint32_t acol = lane_base + uint32_t(kAccCols + as * kAStageCols);
      tmem_st32(acol, out[0]);
      tmem_st32(acol + 32, out[1]);
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      tc::tc_fence_before();
      tc::warp_arrive(&a_full[as]);
      rs += ndg;
      while (rs >= a.rs) {
        rs -= a.rs;
        rph ^= 1;
      }
    }

    // ------------------------------------------------------------ epilogue
    if (!mbar_wait(&acc_bar, 0, lim)) {
      atomicOr(a.err, kErrPipeWait);
      s_fail = 1;
    }
    tc::tc_fence_after();
    grid_wait();  // y, the residual and the partial scratch follow the previous kernel
    const int quad = warp & 3, part = warp >> 2;  // lane quarter; 8-column chunks part, part + kDG, ...
    const int tlane = 32 * quad + lane;  // this thread's TMEM lane
    int er8, eg16;
    lane_row(tlane, er8, eg16);
    const int trow = er8 * 16 + eg16;    // and the weight row of the tile it holds
    const uint32_t lane_addr = taddr + (uint32_t(32 * quad) << 16);
    const bool ok = !s_fail;
    const bool fused = EPI == EPI_RESID && a.fused;
    if (fused) {
      if (tid == 0) s_epoch = *reinterpret_cast<volatile unsigned*>(a.x.epoch) + 1u;
      dq_bar();
    }
    if (a.S == 1) {
      constexpr int STEP = EPI == EPI_SILU ? 2 : 1;
      for (int ti = 0; ti < ntl; ti += STEP) {
        const long n = EPI == EPI_SILU ? (long)((t0 + ti) >> 1) * 128 + trow : (long)(t0 + ti) * 128 + trow;
        for (int c0 = 8 * part; c0 < NT; c0 += 8 * kDG) {
          float v[8], u[8];
          tc::tmem_ld8(lane_addr + uint32_t(ti * NT + c0), v);
          if constexpr (EPI == EPI_SILU) tc::tmem_ld8(lane_addr + uint32_t((ti + 1) * NT + c0), u);
          if (ok) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const int m = c0 + j;
              if (m >= a.M) continue;
              if (fused)
                a.x.part_local[(long)m * a.ldy + n] = __float2half_rn(v[j]);
              else
                a.y[(long)m * a.ldy + n] = epi_value<EPI>(a, v[j], EPI == EPI_SILU ? u[j] : 0.f, m, n);
            }
          }
        }
      }
      if (fused && tp_exchange(a.x, grp, s_epoch, a.err, &s_xok) && ok) {
        for (int ti = 0; ti < ntl; ++ti) {
          const long n = (long)(t0 + ti) * 128 + trow;
          for (int c0 = 8 * part; c0 < NT; c0 += 8 * kDG)
            for (int j = 0; j < 8; ++j) {
              const int m = c0 + j;
              if (m < a.M) a.y[(long)m * a.ldy + n] = tp_combine(a.x, a.res, a.ldres, a.ldy, m, n);
            }
        }
      }
    } else {
      // partial tiles of this share: [tile][m][row], row fastest
      float* P = a.partials + ((size_t)grp * a.S + share) * a.tg * NT * 128;
      for (int ti = 0; ti < ntl; ++ti) {
        for (int c0 = 8 * part; c0 < NT; c0 += 8 * kDG) {
          float v[8];
          tc::tmem_ld8(lane_addr + uint32_t(ti * NT + c0), v);
#pragma unroll
          for (int j = 0; j < 8; ++j)
            if (c0 + j < a.M) __stcg(P + ((size_t)ti * NT + c0 + j) * 128 + tlane, v[j]);
        }
      }
      dq_bar();
      if (tid == 0) {
        // every share's partials are in place (the grid is one wave, so the
        // other shares are resident or done; the wait is bounded). The
        // barrier above orders the CTA's partial stores before this
        // thread's fence, which releases them with the count.
        unsigned* ctr = a.counters + grp;
        __threadfence();
        atomicAdd(ctr, 1u);
        unsigned v = 0;
        for (unsigned it = 0; it < lim; ++it) {
          asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
          if (v >= unsigned(a.S)) break;
          __nanosleep(64);
        }
        s_last = v >= unsigned(a.S) ? 1u : 0u;
        if (!s_last) atomicOr(a.err, kErrShareWait);
      }
      dq_bar();
      // this share's slice of the group's outputs, 4 rows per item, partials
      // summed in share order
      const bool all_in = s_last != 0u;
      const size_t share_stride = (size_t)a.tg * NT * 128;
      const float* Pg = a.partials + (size_t)grp * a.S * share_stride;
      constexpr int STEP = EPI == EPI_SILU ? 2 : 1;
      const int E4 = (ntl / STEP) * a.M * 32;
      const int e_lo = int((long long)share * E4 / a.S), e_hi = int((long long)(share + 1) * E4 / a.S);
      for (int e = e_lo + tid; e < e_hi; e += kSDW * 32) {
        const int r4 = e & 31, m = (e >> 5) % a.M, ti = ((e >> 5) / a.M) * STEP;
        const float* base = Pg + ((size_t)ti * NT + m) * 128 + 4 * r4;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f), up = acc;
        if constexpr (EPI == EPI_SILU) {
#pragma unroll 4
          for (int sh = 0; sh < a.S; ++sh) {
            const float4 v = __ldcg(reinterpret_cast<const float4*>(base + sh * share_stride));
            const float4 u = __ldcg(reinterpret_cast<const float4*>(base + NT * 128 + sh * share_stride));
            acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
            up.x += u.x; up.y += u.y; up.z += u.z; up.w += u.w;
          }
        } else {
          // eight shares' loads in flight at once (one L2 round trip per
          // eight shares), then added in share order
          for (int s0 = 0; s0 < a.S; s0 += 8) {
            float4 v[8];
#pragma unroll
            for (int q = 0; q < 8; ++q)
              if (s0 + q < a.S) v[q] = __ldcg(reinterpret_cast<const float4*>(base + (s0 + q) * share_stride));
#pragma unroll
            for (int q = 0; q < 8; ++q)
              if (s0 + q < a.S) {
                acc.x += v[q].x; acc.y += v[q].y; acc.z += v[q].z; acc.w += v[q].w;
              }
          }
        }
        const long n0 = (EPI == EPI_SILU ? (long)((t0 + ti) >> 1) : (long)(t0 + ti)) * 128;
        if (ok && all_in) {
          const float av[4] = {acc.x, acc.y, acc.z, acc.w}, uv[4] = {up.x, up.y, up.z, up.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            int pr8, pg16;
            lane_row(4 * r4 + q, pr8, pg16);
            const long n = n0 + pr8 * 16 + pg16;
            if (fused)
              a.x.part_local[(long)m * a.ldy + n] = __float2half_rn(av[q]);
            else
              a.y[(long)m * a.ldy + n] = epi_value<EPI>(a, av[q], uv[q], m, n);
          }
        }
      }
      if (fused && tp_exchange(a.x, grp * a.S + share, s_epoch, a.err, &s_xok) && ok && all_in) {
        for (int e = e_lo + tid; e < e_hi; e += kSDW * 32) {
          const int r4 = e & 31, m = (e >> 5) % a.M, ti = (e >> 5) / a.M;
          const long n0 = (long)(t0 + ti) * 128;
          for (int q = 0; q < 4; ++q) {
            int pr8, pg16;
            lane_row(4 * r4 + q, pr8, pg16);
            const long n = n0 + pr8 * 16 + pg16;
            a.y[(long)m * a.ldy + n] = tp_combine(a.x, a.res, a.ldres, a.ldy, m, n);
          }
        }
      }
      // the second round of arrivals: the last share resets the counter
      dq_bar();
      if (tid == 0 && atomicAdd(a.counters + grp, 1u) == unsigned(2 * a.S - 1)) a.counters[grp] = 0u;
    }
    if (fused && tid == 0) {
      // the last CTA records the epoch for the next exchange
      __threadfence();
      if (atomicAdd(a.x.ticket, 1u) == gridDim.x * gridDim.y - 1u) {
        *a.x.ticket = 0u;
        *a.x.epoch = s_epoch;
      }
    }
  }

  // ------------------------------------------------------------ teardown
  grid_launch_dependents();
  tc::tc_fence_before();
  __syncthreads();
  if (warp == kSWMma) {
    tc::tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(taddr) : "memory");
  }
}

struct TcsPlan {
  int NT = 0, tg = 0, groups = 0, S = 0, rs = 0, xs = 0, ni = 1, ndg = 4;
  size_t smem = 0, partial_floats = 0;
};

// Tiles per group and K shares: the fewest weight units (tile × K block) on
// the busiest CTA over one wave of SMs, with the x tile's L2 reads, the
// partial sums' round trip and the MMA issue rate counted against it: one
// issuing thread needs about twice a unit's streaming time for its eight
// MMAs, two or four issuers (tile counts divisible by them) do not.
TcsPlan plan_tcs(int M, int N_out, int K, int epi, int num_sms) {
  TcsPlan p;
  p.NT = (M + 15) / 16 * 16;
  const int apt = epi == EPI_SILU ? 2 : 1;
  const int n_ot = N_out / 128, nb = K / 128;
  const int tg_max = std::min(kMaxTG, kAccCols / p.NT) / apt * apt;
  double best = 1e30;
  for (int tgo = 1; tgo * apt <= tg_max; ++tgo) {
    const int tga = tgo * apt;
    const int groups = (n_ot + tgo - 1) / tgo;
    for (int S = 1; S <= nb; ++S) {
      const long long ctas = (long long)groups * S;
      const long long waves = (ctas + num_sms - 1) / num_sms;
      if (waves > 1 && S > 1) break;
      const int upc = tga * ((nb + S - 1) / S);
      // warpgroups and issuers: four and four, three and three, four and two
      const int ndg = tga % 4 == 0 ? 4 : (tga % 3 == 0 ? 3 : 4);
      const int ni = tga % 4 == 0 ? 4 : (tga % 3 == 0 ? 3 : (tga % 2 == 0 ? 2 : 1));
      // (more issuers also shorten each unit's hand-over: a small preference)
      const double issue = std::max(1.0, 1.9 / ni) * (1.0 + 0.03 * (4.0 / ni - 1.0));
      const double x_cost = 0.5 * double(p.NT) * 256.0 / (double(tga) * 8 * kRecG);
      const double p_cost = S > 1 ? 0.5 * double(tga) * p.NT * 128 * 8 / (double(upc) * 8 * kRecG) : 0.0;
      const double cost = double(waves) * upc * (issue + x_cost + p_cost) + 1e-6 * double(ctas);
      if (cost < best) {
        best = cost;
        p.tg = tga;
        p.groups = groups;
        p.S = S;
        p.ni = ni;
        p.ndg = ndg;
      }
    }
  }
  // Shared memory: three x stages (an x tile comes from L2; two stages at
  // three tiles per group measured half the MMA-issue rate), the rest raw
  // record slots: a record copy lands ~5 us after it is issued under a full
  // load, so the ring's depth sets how many units stream at once. The ndg
  // dequantising warpgroups take units round-robin from the raw ring, so it
  // holds a multiple of ndg slots: the unit a warpgroup waits for then reuses
  // a slot whose previous unit it consumed itself, and a phase-parity wait
  // can never run two phases ahead.
  const size_t xstage = size_t(2) * p.NT * 128;
  p.xs = 3;
  const size_t fixed = size_t(p.xs) * xstage + 1024;
  p.rs = int(std::min<size_t>(kRSMax, (kSmemCap - fixed) / kRawSlot)) / p.ndg * p.ndg;
  // a CTA with few units needs no more slots than units: the smaller
  // footprint lets it become resident (and start streaming its weights,
  // which may be read before the launch wait) while the previous kernel's
  // last CTAs still hold part of the SM
  const int upc_max = p.tg * ((nb + p.S - 1) / p.S);
  const int rs_need = (upc_max + p.ndg - 1) / p.ndg * p.ndg;
  p.rs = std::max(p.ndg, std::min(p.rs, rs_need));
  p.smem = fixed + size_t(p.rs) * kRawSlot;
  p.partial_floats = p.S > 1 ? size_t(p.groups) * p.S * p.tg * p.NT * 128 : 0;
  return p;
}

template <int EPI, bool XP>
nmx_status_t launch_tcs_xp(Ctx* c, const CUtensorMap& tm, const CUtensorMap& tw, const TcsArgs& g, const TcsPlan& p) {
  static std::mutex mu;
  static std::map<int, bool> set;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (!set[c->device]) {
      NMX_CUDA_OK(cudaFuncSetAttribute(qgemm_tcs_kernel<EPI, XP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       int(kSmemCap)));
      set[c->device] = true;
    }
  }
  return launch(c, qgemm_tcs_kernel<EPI, XP>, dim3(p.groups, p.S), dim3(kSThreads), p.smem, tm, tw, g);
}
// The x permute (one warp, once per K block of a CTA) pays off while an x
// block is small against the units it feeds: up to 64 rows. Wider x blocks
// keep the byte permutes in the dequantizers.
template <int EPI>
nmx_status_t launch_tcs(Ctx* c, const CUtensorMap& tm, const CUtensorMap& tw, const TcsArgs& g, const TcsPlan& p) {
  return p.NT <= 64 ? launch_tcs_xp<EPI, true>(c, tm, tw, g, p) : launch_tcs_xp<EPI, false>(c, tm, tw, g, p);
}

}  // namespace

bool qgemm_tcs_supported(int M, int N_out, int K, int epi) {
  if (M < 1 || M > kMaxNT || K <= 0 || K % 128 != 0 || N_out % 128 != 0) return false;
  return epi == EPI_STORE || epi == EPI_RESID || epi == EPI_SILU;
}

size_t qgemm_tcs_partials_floats(int M, int N_out, int K, int epi, int num_sms) {
  if (!qgemm_tcs_supported(M, N_out, K, epi)) return 0;
  return plan_tcs(M, N_out, K, epi, num_sms).partial_floats;
}

int qgemm_tcs_groups(int M, int N_out, int K, int epi, int num_sms) {
  if (!qgemm_tcs_supported(M, N_out, K, epi)) return 0;
  return plan_tcs(M, N_out, K, epi, num_sms).groups;
}

nmx_status_t qgemm_tcs(Ctx* c, const GemvDLArgs& a, int epi) {
  NMX_CHECK(qgemm_tcs_supported(a.M, a.N, a.K, epi), NMX_ERR_UNSUPPORTED, "qgemm_tcs: shape or epilogue");
  NMX_CHECK(a.gamma == nullptr, NMX_ERR_UNSUPPORTED, "qgemm_tcs: normalise x first");
  NMX_CHECK(a.err != nullptr, NMX_ERR_INVALID, "qgemm_tcs: no error word");
  NMX_CHECK(reinterpret_cast<uintptr_t>(a.x) % 16 == 0 && (a.ldx * 2) % 16 == 0, NMX_ERR_UNSUPPORTED,
            "qgemm_tcs: x must be 16-byte aligned with a 16-byte row pitch");
  NMX_CHECK(reinterpret_cast<uintptr_t>(a.w) % 16 == 0, NMX_ERR_INVALID, "qgemm_tcs: records must be 16-byte aligned");
  const TcsPlan p = plan_tcs(a.M, a.N, a.K, epi, c->num_sms);
  NMX_CHECK(p.rs >= p.ndg && p.rs % p.ndg == 0 && p.ni >= 1 && p.ndg % p.ni == 0 && p.smem <= kSmemCap,
            NMX_ERR_UNSUPPORTED,
            "qgemm_tcs: shared-memory plan does not fit");
  if (p.S > 1) {
    NMX_CHECK(a.partials != nullptr && a.partials_cap >= p.partial_floats && a.counters != nullptr,
              NMX_ERR_INVALID, "qgemm_tcs: partial-sum scratch too small");
  }
  CUtensorMap tm, tw;
  NMX_TRY(tc::encode_x_map(&tm, a.x, a.ldx, a.M, a.K, p.NT));
  const long long rows = epi == EPI_SILU ? (long long)a.pair_tiles * 16 + a.N : a.N;
  NMX_TRY(tc::encode_records_map(&tw, a.w, a.K / 128, rows / 16, 8));
  TcsArgs g;
  g.w = static_cast<const unsigned char*>(a.w);
  g.M = a.M;
  g.NT = p.NT;
  g.K = a.K;
  g.nb = a.K / 128;
  g.n_atiles = (a.N / 128) * (epi == EPI_SILU ? 2 : 1);
  g.tg = p.tg;
  g.S = p.S;
  g.ni = p.ni;
  g.ndg = p.ndg;
  g.rs = p.rs;
  g.xs = p.xs;
  g.idesc = tc::idesc_f16(128, p.NT);
  g.pair_tiles = a.pair_tiles;
  g.bias = static_cast<const half*>(a.bias);
  g.y = static_cast<half*>(a.y);
  g.ldy = a.ldy;
  g.res = static_cast<const half*>(a.res);
  g.ldres = a.ldres;
  g.partials = a.partials;
  g.counters = a.counters;
  g.err = a.err;
  g.weights_static = a.weights_static;
  g.fused = false;
  if (a.comm) {
    NMX_CHECK(epi == EPI_RESID && a.res != nullptr, NMX_ERR_INVALID, "qgemm_tcs: the exchange needs the residual epilogue");
    NMX_CHECK(long(p.groups) * p.S <= kMaxTileFlags, NMX_ERR_UNSUPPORTED, "qgemm_tcs: too many exchange slots");
    NMX_TRY(comm_exchange_args(static_cast<Comm*>(a.comm), a.comm_region, &g.x));
    g.fused = true;
  }
  switch (epi) {
    case EPI_STORE: return launch_tcs<EPI_STORE>(c, tm, tw, g, p);
    case EPI_RESID: return launch_tcs<EPI_RESID>(c, tm, tw, g, p);
    default: return launch_tcs<EPI_SILU>(c, tm, tw, g, p);
  }
}

}  // namespace nmx
