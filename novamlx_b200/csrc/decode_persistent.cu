// Batch-1 decode as one persistent, cooperative kernel: all layers of all
// greedy steps of a nmx_decode_greedy call (or the single step of a batch-1
// nmx_forward) in one launch.
//
// Why: at batch 1 every linear is a weight stream of 9-66 MB, and with one
// launch per operation each one pays a launch, a wait for the previous
// kernel's slowest CTA, an activation prologue and a tail while the memory
// system idles. Here one CTA of 16 warps runs on every SM for the whole
// call, and the weight stream never stops: every warp owns a fixed share of
// every GEMV phase (the same stream-K split as the stand-alone kernel) and
// walks the concatenation of its shares across phases, layers and tokens
// with a ring of 8 records in flight, so the records of the next GEMV are
// already arriving while the CTA waits at a grid barrier, runs attention or
// stages activations.
//
// Phases of one step (the host builds the list once per pool):
//   EMBED            h = embed[token]
//   per layer:  GEMV qkv (RMSNorm prologue, bias)     → qkv
//               ATTN     RoPE, append k/v to the page, one (kv head, key split)
//                        item per CTA → split partials
//               COMBINE  split partials → attn
//               GEMV o        (+ residual into h)
//               GEMV gate/up  (RMSNorm prologue, SiLU·up) → act
//               GEMV down     (+ residual into h)
//   GEMV lm_head (final RMSNorm prologue, argmax: one packed key per CTA)
//   ADVANCE          argmax over the CTA keys; token, position, history
// with a grid barrier (release-add on a monotonic arrival counter, bounded
// acquire spin) after each phase. Data made by another CTA within the launch is
// read through L2 (ld.global.cg / cp.async.cg), never from L1.
//
// GEMV phases reuse the small-batch kernel's arithmetic (qgemv_dl_small.cu):
// the one-row MMA layout with the lane-split group fold, shared-memory
// reduction of tile groups met by several warps of a CTA, and the early
// hand-over of tile groups shared by two CTAs. Attention runs on mma.sync as
// in attention_mma.cu, with warp pairs splitting head_dim for P·V so the
// accumulators fit the 128 registers a 512-thread CTA allows.
//
// Waits are bounded. A barrier whose wait runs out sets bit 1 of *err and
// every CTA leaves at its next barrier; a hand-over wait that runs out sets
// bit 0. Results of such a launch are not valid (nmx_ctx_synchronize and the
// model calls report it).
#include <algorithm>
#include <map>
#include <mutex>

#include "attn_common.cuh"
#include "common.cuh"
#include "kernels.h"
#include "qgemv_common.cuh"

namespace nmx {

namespace {

constexpr int kPW = 16;            // warps per CTA
constexpr int kPT = kPW * 32;      // threads per CTA
constexpr int kPRing = 8;          // records in flight per warp
constexpr int kPRec = 1152;        // bytes per decode record
constexpr int kPRecW = 512;
constexpr int kPairs = 8;          // attention: K/V blocks in flight per CTA
constexpr unsigned kPSpin = 1u << 24;

__device__ __forceinline__ void pcp16(void* smem_dst, const void* gsrc) {
  const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem_dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gsrc) : "memory");
}
__device__ __forceinline__ unsigned ld_acq(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_rel(unsigned* p, unsigned v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ float ldcg_h(const half* p) { return __half2float(__ldcg(p)); }
__device__ __forceinline__ unsigned ordered_bits_p(float v) {
  const unsigned u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
// part index owning item i when n items are cut into p parts by floor(k n / p)
__device__ __forceinline__ int owner_p(long long i, long long n, long long p) { return int(((i + 1) * p - 1) / n); }
__device__ __forceinline__ void pair_sync(int pair) {
  asm volatile("bar.sync %0, 64;" ::"r"(pair + 1) : "memory");
}

// units [u0, u1) of warp `warp` of CTA `cta` when U units go to G CTAs of kPW warps
__device__ __forceinline__ void warp_units(int U, int cta, int G, int warp, int& C0, int& C1, int& u0, int& u1) {
  if (cta >= G) {
    C0 = C1 = u0 = u1 = 0;
    return;
  }
  C0 = int((long long)cta * U / G);
  C1 = int((long long)(cta + 1) * U / G);
  const int n = C1 - C0;
  u0 = C0 + int((long long)warp * n / kPW);
  u1 = C0 + int((long long)(warp + 1) * n / kPW);
}

// the warp's position in the concatenated record stream of all GEMV phases
struct Cursor {
  int pi = 0, tok = 0;
  int u = 0, u1 = 0, tp = 0, tpt = 1;
  long long pair_off = 0;
  const unsigned char* src = nullptr;
};

__device__ void cursor_seek(Cursor& c, const PersistArgs& A, int cta, int warp) {
  for (;;) {
    if (c.pi >= A.n_ph) {
      c.pi = 0;
      ++c.tok;
    }
    if (c.tok >= A.steps) {
      c.src = nullptr;
      return;
    }
    const PPhase& P = A.ph[c.pi];
    if (P.kind == PH_GEMV) {
      int C0, C1, u0, u1;
      warp_units(P.n_tg * (P.K / 128), cta, P.G, warp, C0, C1, u0, u1);
      if (u0 < u1) {
        c.u = u0;
        c.u1 = u1;
        c.tp = 0;
        c.tpt = P.tpt;
        c.pair_off = P.pair_off;
        c.src = P.w + size_t(u0) * kPRec;
        return;
      }
    }
    ++c.pi;
  }
}

// the next record of the stream into ring slot `slot`: 72 chunks of 16 B
// copied by lanes 0-30 (lane 31 copies nothing, so it can publish flags and
// arrive at barriers without waiting for copies in flight); one commit group
// per record, empty past the end of the stream
__device__ __forceinline__ void cursor_issue(Cursor& c, const PersistArgs& A, unsigned char* ring_w, int slot,
                                             int lane, int cta, int warp) {
  if (c.src) {
    if (lane < 31) {
      const unsigned char* s = c.src + (c.tp ? c.pair_off : 0);
      unsigned char* d = ring_w + slot * kPRec;
      pcp16(d + 16 * lane, s + 16 * lane);
      pcp16(d + 16 * (lane + 31), s + 16 * (lane + 31));
      if (lane < 10) pcp16(d + 16 * (lane + 62), s + 16 * (lane + 62));
    }
    if (c.tpt == 2 && c.tp == 0) {
      c.tp = 1;
    } else {
      c.tp = 0;
      ++c.u;
      c.src += kPRec;
      if (c.u == c.u1) {
        ++c.pi;
        cursor_seek(c, A, cta, warp);
      }
    }
  }
  cp_commit();
}

// Grid barrier on a monotonic arrival counter: thread 31 (a lane that never
// has copies in flight) adds 1 with release semantics (no round trip) and
// waits until the counter reaches (barriers so far) x (CTAs). False when the
// launch is being abandoned.
__device__ bool grid_barrier(const PersistArgs& A, unsigned& episode, int* s_abort) {
  __syncthreads();
  if (threadIdx.x == 31) {
    int abort = *reinterpret_cast<volatile unsigned*>(A.err) != 0u;
    if (!abort) {
      ++episode;
      const unsigned target = episode * gridDim.x;
      asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(A.bar) : "memory");
      unsigned it = 0;
      while (ld_acq(A.bar) < target) {
        if (++it > kPSpin) {
          atomicOr(A.err, 2u);
          abort = 1;
          break;
        }
        if (it > 256) __nanosleep(32);
      }
    }
    *s_abort = abort;
  }
  __syncthreads();
  return *s_abort == 0;
}

// a warp's record ring in shared memory
struct Ring {
  unsigned char* mem;
  int cslot;  // next slot to consume
};

struct GemvSmem {
  uint32_t* xB;
  float2* CX;
  float* wout;   // [kPW][32]
  float* red;    // [lt_max][c_max][32]
  unsigned* cnt; // [lt_max]
  const unsigned char* zero;
};

// ------------------------------------------------------------ GEMV phase
template <int EPI, int TPT>
__device__ void gemv_phase(const PPhase& P, const PersistArgs& A, const GemvSmem& S, Ring& R, Cursor& cur,
                           unsigned long long* s_best, float* s_red, float* s_inv) {
  constexpr int ROWS = 16 * TPT;
  using C = QCfg<4, 64>;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int cta = blockIdx.x;
  const int K = P.K, nb = K / 128, ng = K / 64;
  const int U = P.n_tg * nb;
  int C0, C1, u0, u1;
  warp_units(U, cta, P.G, warp, C0, C1, u0, u1);
  const int n = C1 - C0;

  // ---- activations (made by the previous phase: read through L2)
  const half* X = P.x;
  if (P.gamma) {
    float ss = 0.f;
    for (int k = tid; k < K; k += kPT) {
      const float v = ldcg_h(X + k);
      ss = fmaf(v, v, ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) s_red[warp] = ss;
    __syncthreads();
    if (tid == 0) {
      float tot = 0.f;
      for (int w = 0; w < kPW; ++w) tot += s_red[w];
      *s_inv = 1.0f / sqrtf(tot / float(K) + A.eps);
    }
    __syncthreads();
  }
  const float inv = P.gamma ? *s_inv : 1.f;
  for (int it = tid; it < ng * 4; it += kPT) {
    const int G = it >> 2, tt = it & 3;
    const half* xr = X + G * 64;
    const half* gr = P.gamma ? P.gamma + G * 64 : nullptr;
    float bsum = 0.f, xsum = 0.f;
    uint32_t* dst = S.xB + (G * 4 + tt) * C::MP;
#pragma unroll
    for (int p = 0; p < C::MP; ++p) {
      int k0, k1;
      bool hi;
      pair_k<4, 64>(tt, p, k0, k1, hi);
      float x0 = ldcg_h(xr + k0), x1 = ldcg_h(xr + k1);
      if (gr) {
        x0 = rnd<half>(x0 * inv * __half2float(gr[k0]));
        x1 = rnd<half>(x1 * inv * __half2float(gr[k1]));
      }
      xsum += x0 + x1;
      const float f = hi ? 0.0625f : 1.0f;
      const __half h0 = __float2half_rn(x0 * f), h1 = __float2half_rn(x1 * f);
      bsum += __half2float(h0) + __half2float(h1);
      __half2 hh = __halves2half2(h0, h1);
      dst[p] = *reinterpret_cast<uint32_t*>(&hh);
    }
    const unsigned mask = __activemask();
    bsum += __shfl_xor_sync(mask, bsum, 1);
    bsum += __shfl_xor_sync(mask, bsum, 2);
    xsum += __shfl_xor_sync(mask, xsum, 1);
    xsum += __shfl_xor_sync(mask, xsum, 2);
    if (tt == 0) S.CX[G] = make_float2(-1024.f * bsum, xsum);
  }
  for (int i = tid; i < P.lt_max; i += kPT) S.cnt[i] = 0u;
  if (tid == 0) *s_best = 0ull;
  __syncthreads();

  const int t_first = nb ? C0 / nb : 0;
  float* wout = S.wout + warp * 32;

  auto finalize = [&](int T, const float* v) {
    if constexpr (EPI == EPI_ARGMAX) {
      unsigned long long best = 0ull;
      if (lane < 16) {
        const long nn = long(T) * 16 + lane;
        const float val = rnd<half>(v[lane]);
        if (!(val != val))
          best = (static_cast<unsigned long long>(ordered_bits_p(val)) << 32) |
                 static_cast<unsigned long long>(0xFFFFFFFFu - unsigned(nn));
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long ob = __shfl_xor_sync(0xffffffffu, best, o);
        best = ob > best ? ob : best;
      }
      if (lane == 0 && best) atomicMax(s_best, best);
    } else if (lane < 16) {
      const int r = lane;
      const long nn = long(T) * 16 + r;
      if constexpr (EPI == EPI_SILU) {
        const float g16 = rnd<half>(v[r]), u16 = rnd<half>(v[16 + r]);
        const float act = rnd<half>(g16 / (1.0f + expf(-g16)));
        P.y[nn] = __float2half_rn(act * u16);
      } else {
        float val = rnd<half>(v[r]);
        if (P.bias) val = rnd<half>(val + __half2float(P.bias[nn]));
        if constexpr (EPI == EPI_RESID) val += ldcg_h(P.res + nn);
        P.y[nn] = __float2half_rn(val);
      }
    }
  };

  float acc[TPT][2];
  auto zero_acc = [&]() {
#pragma unroll
    for (int tp = 0; tp < TPT; ++tp) acc[tp][0] = acc[tp][1] = 0.f;
  };
  zero_acc();
  auto put = [&](float* dst) {
#pragma unroll
    for (int tp = 0; tp < TPT; ++tp) {
      float v0 = acc[tp][0], v2 = acc[tp][1];
      v0 += __shfl_xor_sync(0xffffffffu, v0, 1);
      v2 += __shfl_xor_sync(0xffffffffu, v2, 1);
      v0 += __shfl_xor_sync(0xffffffffu, v0, 2);
      v2 += __shfl_xor_sync(0xffffffffu, v2, 2);
      if (t == 0) {
        dst[tp * 16 + g] = v0;
        dst[tp * 16 + g + 8] = v2;
      }
    }
  };
  auto flush = [&](int T) {
    const int li = T - t_first;
    const long long t0 = (long long)T * nb, t1 = (long long)(T + 1) * nb;
    const long long fu = t0 > C0 ? t0 : C0;
    const long long lu = (t1 < C1 ? t1 : C1) - 1;
    const int wa = owner_p(fu - C0, n, kPW), wb = owner_p(lu - C0, n, kPW);
    if (wa != wb) {
      float* slots = S.red + size_t(li) * P.c_max * 32;
      put(slots + (warp - wa) * 32);
      __syncwarp();
      unsigned last = 0;
      if (lane == 0) {
        __threadfence_block();
        last = (atomicAdd(&S.cnt[li], 1u) == unsigned(wb - wa)) ? 1u : 0u;
        __threadfence_block();
      }
      last = __shfl_sync(0xffffffffu, last, 0);
      __syncwarp();
      if (!last) return;
      if (lane < ROWS) {
        float v = 0.f;
        for (int k = 0; k <= wb - wa; ++k) v += slots[k * 32 + lane];
        wout[lane] = v;
      }
    } else {
      put(wout);
    }
    __syncwarp();
    if (fu == t0 && lu == t1 - 1) {
      finalize(T, wout);
    } else if (fu > t0) {
      float* part = A.hand + size_t(T) * 32;
      if (lane < ROWS) __stcg(part + lane, wout[lane]);
      __syncwarp();
      if (lane == 31) st_rel(A.flags + T, 1u);  // the lane with no copies in flight
    } else {
      unsigned ok = 1;
      if (lane == 0) {
        unsigned it = 0;
        while (ld_acq(A.flags + T) == 0u) {
          if (++it > kPSpin) {
            ok = 0;
            atomicOr(A.err, 1u);
            break;
          }
          if (it > 64) __nanosleep(64);
        }
        A.flags[T] = 0u;
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (lane < ROWS && ok) wout[lane] += __ldcg(A.hand + size_t(T) * 32 + lane);
      __syncwarp();
      finalize(T, wout);
    }
    __syncwarp();
  };

  // per-lane constants of the record math (one activation row)
  const int gi_t = t >> 1, term = t & 1;
  const int coef_off = 1024 + ((term * 2 + gi_t) * 8 + g) * 4;
  const unsigned char* xb_b = reinterpret_cast<const unsigned char*>(S.xB);
  const unsigned char* xA_base = g < 4 ? xb_b + t * 32 : S.zero;
  const int xA_step = g < 4 ? 256 : 0;
  const unsigned char* xB_base = g >= 4 ? xb_b + (4 + t) * 32 : S.zero;
  const int xB_step = g >= 4 ? 256 : 0;

  int tg = nb ? u0 / nb : 0, blk = u0 - tg * nb;
  for (int u = u0; u < u1; ++u) {
    if constexpr (TPT == 1)
      cp_wait<kPRing - 1>();
    else
      cp_wait<kPRing - 2>();
    __syncwarp();
    const float2 cx = S.CX[2 * blk + gi_t];
    const unsigned char* pa = xA_base + blk * xA_step;
    const unsigned char* pb = xB_base + blk * xB_step;
    const uint4 xa0 = *reinterpret_cast<const uint4*>(pa);
    const uint4 xa1 = *reinterpret_cast<const uint4*>(pa + 16);
    const uint4 xb0 = *reinterpret_cast<const uint4*>(pb);
    const uint4 xb1 = *reinterpret_cast<const uint4*>(pb + 16);
#pragma unroll
    for (int tp = 0; tp < TPT; ++tp) {
      const int sl = (R.cslot + tp) & (kPRing - 1);
      const unsigned char* r = R.mem + sl * kPRec;
      const uint4 w0 = *reinterpret_cast<const uint4*>(r + 16 * lane);
      const uint4 w1 = *reinterpret_cast<const uint4*>(r + kPRecW + 16 * lane);
      const __half2 ch = *reinterpret_cast<const __half2*>(r + coef_off);
      float d[4];
      uint32_t P0[8], P1[8];
      dequant_word<4>(w0.x, P0);
      dequant_word<4>(w0.y, P0 + 4);
      dequant_word<4>(w1.x, P1);
      dequant_word<4>(w1.y, P1 + 4);
      mma16816(d, P0[0], P1[0], P0[1], P1[1], xa0.x, xa0.y, cx.x, cx.x, cx.x, cx.x);
      mma16816(d, P0[2], P1[2], P0[3], P1[3], xa0.z, xa0.w, d[0], d[1], d[2], d[3]);
      mma16816(d, P0[4], P1[4], P0[5], P1[5], xa1.x, xa1.y, d[0], d[1], d[2], d[3]);
      mma16816(d, P0[6], P1[6], P0[7], P1[7], xa1.z, xa1.w, d[0], d[1], d[2], d[3]);
      dequant_word<4>(w0.z, P0);
      dequant_word<4>(w0.w, P0 + 4);
      dequant_word<4>(w1.z, P1);
      dequant_word<4>(w1.w, P1 + 4);
      mma16816(d, P0[0], P1[0], P0[1], P1[1], xb0.x, xb0.y, d[0], d[1], d[2], d[3]);
      mma16816(d, P0[2], P1[2], P0[3], P1[3], xb0.z, xb0.w, d[0], d[1], d[2], d[3]);
      mma16816(d, P0[4], P1[4], P0[5], P1[5], xb1.x, xb1.y, d[0], d[1], d[2], d[3]);
      mma16816(d, P0[6], P1[6], P0[7], P1[7], xb1.z, xb1.w, d[0], d[1], d[2], d[3]);
      const float v0 = term ? cx.y : d[0];
      const float v2 = term ? cx.y : d[2];
      acc[tp][0] = fmaf(__low2float(ch), v0, acc[tp][0]);
      acc[tp][1] = fmaf(__high2float(ch), v2, acc[tp][1]);
    }
    __syncwarp();
#pragma unroll
    for (int tp = 0; tp < TPT; ++tp) {
      cursor_issue(cur, A, R.mem, R.cslot, lane, cta, warp);
      R.cslot = (R.cslot + 1) & (kPRing - 1);
    }
    if (blk == nb - 1 || u == u1 - 1) {
      flush(tg);
      zero_acc();
    }
    if (++blk == nb) {
      blk = 0;
      ++tg;
    }
  }
  if constexpr (EPI == EPI_ARGMAX) {
    __syncthreads();
    if (tid == 0) A.best[cta] = *s_best;
  }
}

// ------------------------------------------------------- attention phase
// the K/V tiles of round 0 of this CTA's attention item (both warps of a
// pair copy half of the chunks each); issued at the end of the qkv phase so
// the pages stream during the grid barrier
template <int D>
__device__ void attn_prefetch(const PPhase& P, const PersistArgs& A, unsigned char* ua) {
  constexpr int BT = 16, CH = D / 8, TILE = BT * D * 2;
  const int item = blockIdx.x, S = A.S, Hkv = A.Hkv;
  if (item >= Hkv * S) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = item / S, split = item % S, pair = warp & (kPairs - 1), dh = warp >> 3;
  const int pos = __ldcg(A.tok_pos);
  const int nblk = (pos + 1 + BT - 1) / BT, bps = (nblk + S - 1) / S;
  const int b0 = split * bps, b1 = min(nblk, b0 + bps);
  const int b = b0 + pair;
  if (b < b1) {
    const half* Kc = reinterpret_cast<const half*>(A.kv_base + size_t(P.layer) * A.kv_layer_stride);
    const half* Vc = reinterpret_cast<const half*>(A.kv_base + size_t(P.layer) * A.kv_layer_stride +
                                                   A.kv_layer_stride / 2);
    const long base = (long(A.table[b]) * Hkv + h) * BT * D;
    const unsigned char* ks = reinterpret_cast<const unsigned char*>(Kc + base);
    const unsigned char* vs = reinterpret_cast<const unsigned char*>(Vc + base);
    unsigned char* kt = ua + TILE + pair * 2 * TILE;
    unsigned char* vt = kt + TILE;
    for (int i = dh * 32 + lane; i < BT * CH; i += 64) {
      const int r = i / CH, c = i % CH;
      cp_async16a(kt + swz<D>(r, c), ks + i * 16);
      cp_async16a(vt + swz<D>(r, c), vs + i * 16);
    }
  }
  cp_commit();
}

template <int D>
__device__ void attn_phase(const PPhase& P, const PersistArgs& A, unsigned char* ua, float* s_m, float* s_l,
                           half* s_knew, half* s_vnew, bool prefetched) {
  constexpr int BT = 16, CH = D / 8, TILE = BT * D * 2, KSTEPS = D / 16, NTH = D / 16;  // n-tiles per half
  constexpr float kLog2e = 1.4426950408889634f;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int Hq = A.Hq, Hkv = A.Hkv, rep = Hq / Hkv, S = A.S;
  const int item = blockIdx.x;
  if (item >= Hkv * S) return;
  const int h = item / S, split = item % S;
  const int pair = warp & (kPairs - 1), dh = warp >> 3;  // d-half of P·V
  unsigned char* q_sm = ua;
  unsigned char* tiles = ua + TILE;  // [kPairs][K tile, V tile]
  half* Kc = reinterpret_cast<half*>(A.kv_base + size_t(P.layer) * A.kv_layer_stride);
  half* Vc = reinterpret_cast<half*>(A.kv_base + size_t(P.layer) * A.kv_layer_stride + A.kv_layer_stride / 2);

  const int pos = __ldcg(A.tok_pos);
  const int nblk = (pos + 1 + BT - 1) / BT;
  const int bps = (nblk + S - 1) / S;
  const int b0 = split * bps, b1 = min(nblk, b0 + bps);
  const int* bt = A.table;
  const half* Q = A.qkv;
  const int bpos = pos / BT;
  const bool owner = bpos >= b0 && bpos < b1;

  for (int i = tid; i < (BT - rep) * CH; i += kPT) {
    const int r = rep + i / CH, c = i % CH;
    *reinterpret_cast<uint4*>(q_sm + swz<D>(r, c)) = make_uint4(0, 0, 0, 0);
  }
  for (int i = tid; i < rep * (D / 2); i += kPT) {
    const int hi = i / (D / 2), d = i % (D / 2);
    const int hq = h * rep + hi;
    float r0, r1;
    rope2(ldcg_h(Q + hq * D + d), ldcg_h(Q + hq * D + d + D / 2), float(pos) * A.inv_freq[d], r0, r1);
    reinterpret_cast<half*>(q_sm + swz<D>(hi, d / 8))[d % 8] = __float2half_rn(r0);
    reinterpret_cast<half*>(q_sm + swz<D>(hi, (d + D / 2) / 8))[d % 8] = __float2half_rn(r1);
  }
  if (owner) {
    const long slot = (long(bt[bpos]) * Hkv + h) * BT + pos % BT;
    const half* kr = Q + (Hq + h) * D;
    const half* vr = Q + (Hq + Hkv + h) * D;
    for (int d = tid; d < D / 2; d += kPT) {
      float r0, r1;
      rope2(ldcg_h(kr + d), ldcg_h(kr + d + D / 2), float(pos) * A.inv_freq[d], r0, r1);
      const half k0 = __float2half_rn(r0), k1 = __float2half_rn(r1);
      Kc[slot * D + d] = k0;
      Kc[slot * D + d + D / 2] = k1;
      s_knew[d] = k0;
      s_knew[d + D / 2] = k1;
    }
    for (int d = tid; d < D; d += kPT) {
      const half v = __ldcg(vr + d);
      Vc[slot * D + d] = v;
      s_vnew[d] = v;
    }
  }
  __syncthreads();

  uint32_t qa[KSTEPS][2];
#pragma unroll
  for (int kk = 0; kk < KSTEPS; ++kk) {
    const int r = lane & 7, c = 2 * kk + ((lane >> 3) & 1);
    ldsm_x2(qa[kk], q_sm + swz<D>(r, c));
  }
  const float sl2 = A.scale * kLog2e;
  const int last = pos - 1;  // the new token is added apart
  float o[NTH][4];
#pragma unroll
  for (int nt = 0; nt < NTH; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;
  float m_r = -INFINITY, l_r = 0.f;
  unsigned char* kt = tiles + pair * 2 * TILE;
  unsigned char* vt = kt + TILE;
  const int rounds = (b1 - b0 + kPairs - 1) / kPairs;
  for (int rd = 0; rd < rounds; ++rd) {
    const int b = b0 + rd * kPairs + pair;
    const bool have = b < b1;
    if (have && !(prefetched && rd == 0)) {
      // the two warps of the pair copy half of the chunks each
      const long base = (long(bt[b]) * Hkv + h) * BT * D;
      const unsigned char* ks = reinterpret_cast<const unsigned char*>(Kc + base);
      const unsigned char* vs = reinterpret_cast<const unsigned char*>(Vc + base);
      for (int i = dh * 32 + lane; i < BT * CH; i += 64) {
        const int r = i / CH, c = i % CH;
        cp_async16a(kt + swz<D>(r, c), ks + i * 16);
        cp_async16a(vt + swz<D>(r, c), vs + i * 16);
      }
    }
    cp_commit();
    cp_wait<0>();
    pair_sync(pair);
    if (have) {
      float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
      for (int kk = 0; kk < KSTEPS; ++kk) {
        uint32_t r[4];
        const int rr = (lane & 7) + ((lane >> 4) << 3), cc = 2 * kk + ((lane >> 3) & 1);
        ldsm_x4(r, kt + swz<D>(rr, cc));
        mma_f16(s[0], qa[kk][0], 0u, qa[kk][1], 0u, r[0], r[1]);
        mma_f16(s[1], qa[kk][0], 0u, qa[kk][1], 0u, r[2], r[3]);
      }
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
      const float m_use = m_new == -INFINITY ? 0.f : m_new;
      const float corr = exp2f(m_r - m_use);
      float p[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) p[e] = exp2f(v[e] - m_use);
      l_r = l_r * corr + (p[0] + p[1] + p[2] + p[3]);
      m_r = m_new;
#pragma unroll
      for (int nt = 0; nt < NTH; ++nt) {
        o[nt][0] *= corr;
        o[nt][1] *= corr;
      }
      const uint32_t pa0 = pack_half2(p[0], p[1]), pa2 = pack_half2(p[2], p[3]);
#pragma unroll
      for (int np = 0; np < NTH / 2; ++np) {
        uint32_t r[4];
        const int rr = (lane & 7) + (((lane >> 3) & 1) << 3), cc = dh * (CH / 2) + 2 * np + (lane >> 4);
        ldsm_x4_t(r, vt + swz<D>(rr, cc));
        mma_f16(o[2 * np], pa0, 0u, pa2, 0u, r[0], r[1]);
        mma_f16(o[2 * np + 1], pa0, 0u, pa2, 0u, r[2], r[3]);
      }
    }
    pair_sync(pair);  // both warps are done with the tiles before they are refilled
  }
  l_r += __shfl_xor_sync(0xffffffffu, l_r, 1);
  l_r += __shfl_xor_sync(0xffffffffu, l_r, 2);

  // merge the pairs and the new token into this item's partial
  __syncthreads();
  float* s_o = reinterpret_cast<float*>(tiles);  // [kPairs][8][D]
  if (g < rep) {
    if (t == 0 && dh == 0) {
      s_m[pair * 8 + g] = m_r;
      s_l[pair * 8 + g] = l_r;
    }
#pragma unroll
    for (int nt = 0; nt < NTH; ++nt)
      *reinterpret_cast<float2*>(s_o + (pair * 8 + g) * D + dh * (D / 2) + nt * 8 + 2 * t) =
          make_float2(o[nt][0], o[nt][1]);
  }
  if (warp == 0) {
    for (int hi = 0; hi < rep; ++hi) {
      float sc = 0.f;
      if (owner) {
        for (int d = lane; d < D; d += 32)
          sc = fmaf(__half2float(reinterpret_cast<const half*>(q_sm + swz<D>(hi, d / 8))[d % 8]),
                    __half2float(s_knew[d]), sc);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) sc += __shfl_xor_sync(0xffffffffu, sc, off);
      }
      if (lane == 0) {
        s_m[kPairs * 8 + hi] = owner ? sc * sl2 : -INFINITY;
        s_l[kPairs * 8 + hi] = owner ? 1.f : 0.f;
      }
    }
  }
  __syncthreads();
  for (int e = tid; e < rep * D; e += kPT) {
    const int hi = e / D, d = e % D;
    float M = -INFINITY;
    for (int w = 0; w <= kPairs; ++w)
      if (s_l[w * 8 + hi] > 0.f) M = fmaxf(M, s_m[w * 8 + hi]);
    float num = 0.f, den = 0.f;
    for (int w = 0; w < kPairs; ++w) {
      if (s_l[w * 8 + hi] > 0.f) {
        const float f = exp2f(s_m[w * 8 + hi] - M);
        num = fmaf(s_o[(w * 8 + hi) * D + d], f, num);
        den = fmaf(s_l[w * 8 + hi], f, den);
      }
    }
    if (s_l[kPairs * 8 + hi] > 0.f) {
      const float f = exp2f(s_m[kPairs * 8 + hi] - M);
      num = fmaf(__half2float(s_vnew[d]), f, num);
      den += f;
    }
    const long pb = long(item) * rep + hi;
    __stcg(A.part_o + pb * D + d, num);
    if (d == 0) __stcg(reinterpret_cast<float2*>(A.part_ml) + pb, make_float2(M, den));
  }
}

__global__ void __launch_bounds__(kPT, 1) decode_persistent_kernel(PersistArgs A) {
  extern __shared__ __align__(128) unsigned char sm[];
  __shared__ float s_red[kPW];
  __shared__ float s_inv;
  __shared__ unsigned long long s_best;
  __shared__ int s_abort;
  __shared__ float s_m[(kPairs + 1) * 8], s_l[(kPairs + 1) * 8];
  __shared__ __align__(16) half s_knew[128];
  __shared__ __align__(16) half s_vnew[128];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int cta = blockIdx.x, G = gridDim.x;
  Ring R;
  R.mem = sm + size_t(warp) * kPRing * kPRec;
  R.cslot = 0;
  unsigned char* ua = sm + size_t(kPW) * kPRing * kPRec;  // phase-local area
  GemvSmem gs;
  gs.xB = reinterpret_cast<uint32_t*>(ua + A.off_xb);
  gs.CX = reinterpret_cast<float2*>(ua + A.off_cx);
  gs.wout = reinterpret_cast<float*>(ua + A.off_wout);
  gs.red = reinterpret_cast<float*>(ua + A.off_red);
  gs.cnt = reinterpret_cast<unsigned*>(ua + A.off_cnt);
  gs.zero = ua + A.off_zero;

  unsigned episode = 0;  // barriers passed (the counter starts at 0 each launch)
  if (tid < 8) reinterpret_cast<uint32_t*>(ua + A.off_zero)[tid] = 0u;
  Cursor cur;
  cursor_seek(cur, A, cta, warp);
  for (int s = 0; s < kPRing; ++s) cursor_issue(cur, A, R.mem, s, lane, cta, warp);
  __syncthreads();

  bool prefetched = false;
  for (int step = 0; step < A.steps; ++step) {
    for (int p = 0; p < A.n_ph; ++p) {
      const PPhase P = A.ph[p];
      if (P.kind == PH_EMBED) {
        const int tok = __ldcg(A.tok_ids);
        const uint4* src = reinterpret_cast<const uint4*>(A.embed) + long(tok) * (A.H / 8);
        uint4* dst = reinterpret_cast<uint4*>(A.h);
        const int n8 = A.H / 8, i0 = int((long long)cta * n8 / G), i1 = int((long long)(cta + 1) * n8 / G);
        for (int i = i0 + tid; i < i1; i += kPT) dst[i] = src[i];
      } else if (P.kind == PH_GEMV) {
        if (tid < 8) reinterpret_cast<uint32_t*>(ua + A.off_zero)[tid] = 0u;
        switch (P.epi) {
          case EPI_STORE: gemv_phase<EPI_STORE, 1>(P, A, gs, R, cur, &s_best, s_red, &s_inv); break;
          case EPI_RESID: gemv_phase<EPI_RESID, 1>(P, A, gs, R, cur, &s_best, s_red, &s_inv); break;
          case EPI_SILU: gemv_phase<EPI_SILU, 2>(P, A, gs, R, cur, &s_best, s_red, &s_inv); break;
          default: gemv_phase<EPI_ARGMAX, 1>(P, A, gs, R, cur, &s_best, s_red, &s_inv); break;
        }
        if (p + 1 < A.n_ph && A.ph[p + 1].kind == PH_ATTN) {
          __syncthreads();  // the staging area is free: start the attention pages
          if (A.D == 128)
            attn_prefetch<128>(A.ph[p + 1], A, ua);
          else
            attn_prefetch<64>(A.ph[p + 1], A, ua);
          prefetched = true;
        }
      } else if (P.kind == PH_ATTN) {
        if (A.D == 128)
          attn_phase<128>(P, A, ua, s_m, s_l, s_knew, s_vnew, prefetched);
        else
          attn_phase<64>(P, A, ua, s_m, s_l, s_knew, s_vnew, prefetched);
        prefetched = false;
      } else if (P.kind == PH_COMBINE) {
        // (element, split) pairs over the threads: one round of loads, then
        // each element sums its splits in order from shared memory
        const int rep = A.Hq / A.Hkv, D = A.D, S = A.S;
        const int E = A.Hq * D, e0 = int((long long)cta * E / G), e1 = int((long long)(cta + 1) * E / G);
        float* bm = reinterpret_cast<float*>(ua);
        float* bl = bm + kPT;
        float* bo = bl + kPT;
        const int per = kPT / S;
        for (int base = e0; base < e1; base += per) {
          const int j = tid, e = base + j / S, s2 = j % S;
          if (j < per * S && e < e1) {
            const int hq = e / D, d = e % D, kvh = hq / rep, hi = hq % rep;
            const long pb = long(kvh * S + s2) * rep + hi;
            const float2 ml = __ldcg(reinterpret_cast<const float2*>(A.part_ml) + pb);
            bm[j] = ml.x;
            bl[j] = ml.y;
            bo[j] = __ldcg(A.part_o + pb * D + d);
          }
          __syncthreads();
          if (tid < per && base + tid < e1) {
            const float* m = bm + tid * S;
            const float* l = bl + tid * S;
            const float* o = bo + tid * S;
            float M = -INFINITY;
            for (int k = 0; k < S; ++k)
              if (l[k] > 0.f) M = fmaxf(M, m[k]);
            float num = 0.f, den = 0.f;
            for (int k = 0; k < S; ++k)
              if (l[k] > 0.f) {
                const float f = exp2f(m[k] - M);
                num = fmaf(o[k], f, num);
                den = fmaf(l[k], f, den);
              }
            A.attn[base + tid] = __float2half_rn(den > 0.f ? num / den : 0.f);
          }
          __syncthreads();
        }
      } else if (P.kind == PH_ADVANCE) {
        if (cta == 0 && tid == 0) {
          unsigned long long b = 0ull;
          for (int c = 0; c < G; ++c) {
            const unsigned long long k = __ldcg(A.best + c);
            b = k > b ? k : b;
          }
          const int id = b ? int(0xFFFFFFFFu - unsigned(b & 0xFFFFFFFFull)) : 0;
          const int st = *A.step;
          if (A.hist && st + 1 <= A.hist_cap) A.hist[st] = id;
          *A.step = st + 1;
          *A.tok_ids = id;
          *A.tok_pos = *A.tok_pos + 1;
          if (A.out_id) *A.out_id = id;
        }
      }
      if (!grid_barrier(A, episode, &s_abort)) {
        cp_wait<0>();  // abandoned: let the copies in flight land first
        return;
      }
    }
  }
  cp_wait<0>();
}

}  // namespace

// phase-local shared memory: the GEMV staging (activations in fragment order,
// group sums, per-warp outputs, reduction slots and tickets) and the attention
// tiles share one area after the record rings
size_t persist_smem_bytes(int K_max, int red_slots, int lt_max, int D) {
  const size_t xb = align_up(size_t(K_max) * 2, 128);
  const size_t cx = align_up(size_t(K_max / 64) * 8, 128);
  const size_t wout = size_t(kPW) * 32 * 4;
  const size_t red = align_up(size_t(red_slots) * 32 * 4, 128);
  const size_t cnt = align_up(size_t(lt_max) * 4, 128);
  const size_t gemv = xb + cx + wout + red + cnt + 128;
  const size_t attn = size_t(16) * D * 2 * (1 + 2 * kPairs);
  return size_t(kPW) * kPRing * kPRec + std::max(gemv, attn);
}

nmx_status_t persist_layout(int K_max, int red_slots, int lt_max, PersistArgs* A) {
  size_t off = 0;
  A->off_xb = int(off);
  off += align_up(size_t(K_max) * 2, 128);
  A->off_cx = int(off);
  off += align_up(size_t(K_max / 64) * 8, 128);
  A->off_wout = int(off);
  off += size_t(kPW) * 32 * 4;
  A->off_red = int(off);
  off += align_up(size_t(red_slots) * 32 * 4, 128);
  A->off_cnt = int(off);
  off += align_up(size_t(lt_max) * 4, 128);
  A->off_zero = int(off);
  return NMX_OK;
}

int persist_warps() { return kPW; }

nmx_status_t persist_launch(Ctx* c, const PersistArgs& A, size_t smem) {
  static std::mutex mu;
  static std::map<int, int> max_dyn;  // device → largest dynamic shared memory the kernel may ask for
  int lim = 0;
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = max_dyn.find(c->device);
    if (it == max_dyn.end()) {
      int coop = 0, optin = 0;
      NMX_CUDA_OK(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, c->device));
      NMX_CUDA_OK(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, c->device));
      cudaFuncAttributes fa;
      NMX_CUDA_OK(cudaFuncGetAttributes(&fa, decode_persistent_kernel));
      lim = coop ? optin - int(fa.sharedSizeBytes) : 0;
      if (lim > 0)
        NMX_CUDA_OK(cudaFuncSetAttribute(decode_persistent_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, lim));
      max_dyn[c->device] = lim;
    } else {
      lim = it->second;
    }
  }
  NMX_CHECK(lim > 0 && smem <= size_t(lim), NMX_ERR_UNSUPPORTED,
            "persistent decode: no cooperative launch or shared memory too large");
  int per_sm = 0;
  NMX_CUDA_OK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_persistent_kernel, kPT, smem));
  NMX_CHECK(per_sm >= 1, NMX_ERR_UNSUPPORTED, "persistent decode: a CTA does not fit an SM");
  NMX_CUDA_OK(cudaMemsetAsync(A.bar, 0, 4, c->stream));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(c->num_sms);
  cfg.blockDim = dim3(kPT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = c->stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, decode_persistent_kernel, A);
  if (e != cudaSuccess) {
    set_error(std::string("persistent decode launch: ") + cudaGetErrorString(e));
    return NMX_ERR_CUDA;
  }
  c->launches++;
  return NMX_OK;
}

}  // namespace nmx
