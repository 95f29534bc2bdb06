// Decode GEMV over decode records for 1..8 activation rows (the decode step
// at small batch): the model's linear layers at batch 1 run here.
//
// Split. The U = n_tg * nb (tile group, 128-k block) units of the launch are
// cut into one contiguous range per CTA, c(k) = floor(k U / G), and each
// CTA's range into one contiguous sub-range per warp the same way (stream-K
// at both levels: every warp streams the same number of records). A warp
// streams its sub-range through a private ring of cp.async stages and
// accumulates each tile group it meets in registers.
//
// Reduction. A tile group met by one warp only is finished by that warp. A
// tile group shared by several warps of the CTA is reduced in shared memory:
// each contributor writes its partial sums to its slot and the last to
// arrive (shared-memory ticket) sums the slots in warp order. The grid is
// chosen so that a tile group meets at most two CTAs (exactly one when there
// are at most two tile groups per SM). For a tile group two CTAs share, each
// writes its part to its own global slot and takes a ticket; the second to
// arrive adds the two parts and runs the epilogue, so no CTA waits for a
// neighbour that started late. All sums have a fixed order (a sum of two
// terms does not depend on which CTA adds them), so results are
// deterministic.
//
// One activation row (ONE): the eight MMA columns are split between the two
// groups of a block, columns 0-3 taking group 2B and columns 4-7 group 2B+1
// (the B operand is zero elsewhere). Lane (g, t) then holds the group
// (t >> 1) sums of rows g and g+8, and the group-affine fold is shared by the
// four lanes of a row: lanes with t even add scale * sum, lanes with t odd
// add bias * sum(x); the four lanes are summed when the tile group ends.
//
// Footprint: two CTAs per SM (a floor on the shared memory keeps a third
// off, so the grid spreads over all SMs).
#include <algorithm>
#include <map>
#include <mutex>
#include <tuple>

#include "common.cuh"
#include "kernels.h"
#include "qgemv_common.cuh"

namespace nmx {

namespace {

constexpr int kRecS = 1152;  // bytes per decode record
constexpr int kRecWS = 512;  // bytes of one row half of the packed words
constexpr int kMaxSmemS = 200 * 1024;
constexpr int kTwoPerSm = 110 * 1024;  // two CTAs per SM at or below this
// at least this much, so no SM takes a third CTA: the grid is sized for two
// per SM and a third would leave other SMs idle
constexpr int kMinSmemS = 78 * 1024;

struct SmallLayout {
  int xb_off = 0, cx_off = 0, out_off = 0, red_off = 0, cnt_off = 0, zero_off = 0, total = 0;
  int colstride = 0;  // words per staged activation row
  int lt_max = 0;     // tile groups a CTA range can meet
  int c_max = 0;      // warps of one CTA a tile group can meet
};

// 16-byte copy to a shared-space address
__device__ __forceinline__ void cp16(unsigned s, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

__device__ __forceinline__ unsigned ordered_bits_s(float v) {
  const unsigned u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// index of the part owning item i when n items are cut into p parts by
// floor(k n / p)
__host__ __device__ __forceinline__ int owner_of(long long i, long long n, long long p) {
  return int(((i + 1) * p - 1) / n);
}

template <int EPI, int TPT, int STAGES, bool ONE>
__global__ void __launch_bounds__(kThreads, 2) qgemv_dl8_kernel(GemvDLArgs a, SmallLayout L) {
  constexpr int ROWS = 16 * TPT;
  constexpr int NC = ONE ? 1 : 8;  // columns kept per row
  using C = QCfg<4, 64>;
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ float s_inv[8];
  __shared__ float s_wsum[kWarps][8];
  __shared__ unsigned long long s_best[8];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int K = a.K, M = a.M, nb = K / 128, ng = K / 64;
  const int U = a.n_tg * nb;
  const int Gd = gridDim.x, cta = blockIdx.x;
  const int C0 = int((long long)cta * U / Gd), C1 = int((long long)(cta + 1) * U / Gd);
  const int n = C1 - C0;
  const int u0 = C0 + int((long long)warp * n / kWarps), u1 = C0 + int((long long)(warp + 1) * n / kWarps);

  uint32_t* xB = reinterpret_cast<uint32_t*>(smem + L.xb_off);
  float2* CX = reinterpret_cast<float2*>(smem + L.cx_off);
  float* wout = reinterpret_cast<float*>(smem + L.out_off) + warp * (ROWS * NC);
  float* red = reinterpret_cast<float*>(smem + L.red_off);
  unsigned* cnt = reinterpret_cast<unsigned*>(smem + L.cnt_off);
  unsigned char* ring = smem + size_t(warp) * (STAGES * TPT * kRecS);

  // stream this warp's records: unit u is record u of the matrix, its up
  // half (EPI_SILU) pair_tiles * nb records further
  const unsigned char* src_cur = reinterpret_cast<const unsigned char*>(a.w) + size_t(u0) * kRecS + 16 * lane;
  const size_t pair_off = size_t(a.pair_tiles) * nb * kRecS;
  int is_u = u0;
  // this lane's 16-byte slice of ring stage 0 (shared-space address)
  const unsigned ring_s = static_cast<unsigned>(__cvta_generic_to_shared(ring)) + 16 * lane;
  auto issue = [&](int slot_off) {  // slot_off: byte offset of the stage in the ring
    if (is_u < u1) {
      const unsigned dst = ring_s + unsigned(slot_off);
#pragma unroll
      for (int tp = 0; tp < TPT; ++tp) {
        const unsigned char* src = src_cur + tp * pair_off;
        cp16(dst + tp * kRecS, src);
        cp16(dst + tp * kRecS + kRecWS, src + kRecWS);
        if (lane < 8) cp16(dst + tp * kRecS + 1024, src + 1024);
      }
      ++is_u;
      src_cur += kRecS;
    }
    cp_commit();
  };
  // model weights never change during a step: start streaming them before
  // the wait (records an op-level caller may just have written are not)
  if (!a.weights_static) grid_wait();
#pragma unroll
  for (int s = 0; s < STAGES; ++s) issue(s * TPT * kRecS);
  // the RMSNorm weights of this thread's first activation item, likewise
  const half* Gm = reinterpret_cast<const half*>(a.gamma);
  const bool g16 = Gm && (reinterpret_cast<uintptr_t>(Gm) & 15) == 0;
  uint4 gpre0 = make_uint4(0, 0, 0, 0), gpre1 = gpre0;
  if (g16 && a.weights_static && tid < M * ng * 4) {
    const uint4* gp = reinterpret_cast<const uint4*>(Gm + ((tid % (ng * 4)) >> 2) * 64 + (tid & 3) * 16);
    gpre0 = __ldg(gp);
    gpre1 = __ldg(gp + 1);
  }
  grid_wait();

  // ------------------------------------------------ activation prologue
  {
    // The activation rows are first copied into the xB area (row c at
    // c * colstride words, element k at byte 2k) with all of this thread's
    // loads in flight at once: one round trip to L2 instead of one per loop
    // pass. Item (G, tt) below then reads its 32 bytes there and rewrites
    // them in place as its MMA operand pairs (the same bytes, since both
    // layouts put item (G, tt) at byte 128 G + 32 tt of the row). The
    // arithmetic and its order are those of a direct read from global memory.
    const half* X = reinterpret_cast<const half*>(a.x);
    unsigned char* xs = smem + L.xb_off;
    const long rowb = long(L.colstride) * 4;
    const int cpr = K / 8;  // 16-byte chunks per row
    const int chunks = M * cpr;
    if (((reinterpret_cast<uintptr_t>(X) | (uintptr_t(a.ldx) * 2)) & 15) == 0) {
      for (int q0 = 0; q0 < chunks; q0 += 8 * kThreads) {
        uint4 v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int q = q0 + j * kThreads + tid;
          if (q < chunks) {
            const int c = q / cpr, r = q - c * cpr;
            v[j] = __ldcg(reinterpret_cast<const uint4*>(X + long(c) * a.ldx) + r);
          }
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int q = q0 + j * kThreads + tid;
          if (q < chunks) {
            const int c = q / cpr, r = q - c * cpr;
            *reinterpret_cast<uint4*>(xs + c * rowb + r * 16) = v[j];
          }
        }
      }
    } else {
      for (int q = tid; q < M * K; q += kThreads) {
        const int c = q / K, k = q - c * K;
        reinterpret_cast<half*>(xs + c * rowb)[k] = X[long(c) * a.ldx + k];
      }
    }
    __syncthreads();
    if (Gm) {
      for (int c = 0; c < M; ++c) {
        const half* xr_s = reinterpret_cast<const half*>(xs + c * rowb);
        float ss = 0.f;
        int k = tid;
        for (; k + 7 * kThreads < K; k += 8 * kThreads) {  // eight loads, then their FMAs in order
          float v[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) v[j] = __half2float(xr_s[k + j * kThreads]);
#pragma unroll
          for (int j = 0; j < 8; ++j) ss = fmaf(v[j], v[j], ss);
        }
        for (; k < K; k += kThreads) {
          const float v = __half2float(xr_s[k]);
          ss = fmaf(v, v, ss);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) s_wsum[warp][c] = ss;
      }
      __syncthreads();
      if (tid < M) {
        float ss = 0.f;
        for (int w = 0; w < kWarps; ++w) ss += s_wsum[w][tid];
        s_inv[tid] = 1.0f / sqrtf(ss / float(K) + a.eps);
      }
      __syncthreads();
    }
    const int items = M * ng * 4;
    for (int it = tid; it < items; it += kThreads) {
      const int c = it / (ng * 4);
      const int rem = it - c * (ng * 4);
      const int G = rem >> 2, tt = rem & 3;
      unsigned char* cell = xs + c * rowb + G * 128 + tt * 32;
      uint4 raw[2];
      raw[0] = *reinterpret_cast<const uint4*>(cell);
      raw[1] = *reinterpret_cast<const uint4*>(cell + 16);
      const half* xv = reinterpret_cast<const half*>(raw);
      uint4 graw[2];
      if (Gm) {
        if (it == tid && g16 && a.weights_static) {
          graw[0] = gpre0;
          graw[1] = gpre1;
        } else if (g16) {
          const uint4* gp = reinterpret_cast<const uint4*>(Gm + G * 64 + tt * 16);
          graw[0] = __ldg(gp);
          graw[1] = __ldg(gp + 1);
        } else {
          half* gh = reinterpret_cast<half*>(graw);
#pragma unroll
          for (int i = 0; i < 16; ++i) gh[i] = Gm[G * 64 + tt * 16 + i];
        }
      }
      const half* gv = reinterpret_cast<const half*>(graw);
      const float inv = Gm ? s_inv[c] : 1.f;
      float bsum = 0.f, xsum = 0.f;
      uint32_t outw[C::MP];
#pragma unroll
      for (int p = 0; p < C::MP; ++p) {
        int k0, k1;
        bool hi;
        pair_k<4, 64>(tt, p, k0, k1, hi);
        k0 -= tt * 16;  // offsets within this item's 16 elements
        k1 -= tt * 16;
        float x0 = __half2float(xv[k0]), x1 = __half2float(xv[k1]);
        if (Gm) {
          x0 = rnd<half>(x0 * inv * __half2float(gv[k0]));
          x1 = rnd<half>(x1 * inv * __half2float(gv[k1]));
        }
        xsum += x0 + x1;
        const float f = hi ? 0.0625f : 1.0f;
        const __half h0 = __float2half_rn(x0 * f), h1 = __float2half_rn(x1 * f);
        bsum += __half2float(h0) + __half2float(h1);
        __half2 hh = __halves2half2(h0, h1);
        outw[p] = *reinterpret_cast<uint32_t*>(&hh);
      }
      *reinterpret_cast<uint4*>(cell) = make_uint4(outw[0], outw[1], outw[2], outw[3]);
      *reinterpret_cast<uint4*>(cell + 16) = make_uint4(outw[4], outw[5], outw[6], outw[7]);
      const unsigned mask = __activemask();
      bsum += __shfl_xor_sync(mask, bsum, 1);
      bsum += __shfl_xor_sync(mask, bsum, 2);
      xsum += __shfl_xor_sync(mask, xsum, 1);
      xsum += __shfl_xor_sync(mask, xsum, 2);
      if (tt == 0) CX[ONE ? G : size_t(G) * 8 + c] = make_float2(-1024.f * bsum, xsum);
    }
    if constexpr (!ONE) {
      for (int it = tid; it < ng * (8 - M); it += kThreads) {
        const int G = it / (8 - M), c = M + it % (8 - M);
        CX[size_t(G) * 8 + c] = make_float2(0.f, 0.f);
      }
    }
    if (tid < 8) reinterpret_cast<uint32_t*>(smem + L.zero_off)[tid] = 0u;
    for (int i = tid; i < L.lt_max; i += kThreads) cnt[i] = 0u;
    if (tid < 8) s_best[tid] = 0ull;
  }
  __syncthreads();
  grid_launch_dependents();

  const int t_first = C0 / nb;

  // epilogue of tile group T; v[r * NC + m]
  auto finalize = [&](int T, const float* v) {
    const half* bias = reinterpret_cast<const half*>(a.bias);
    half* Y = reinterpret_cast<half*>(a.y);
    if constexpr (EPI == EPI_ARGMAX) {
      for (int m = 0; m < M; ++m) {
        unsigned long long best = 0ull;
        if (lane < 16) {
          const long nn = long(T) * 16 + lane;
          const float val = rnd<half>(v[lane * NC + m]);
          if (a.logits_f32) a.logits_f32[long(m) * a.N + nn] = val;
          if (!(val != val))
            best = (static_cast<unsigned long long>(ordered_bits_s(val)) << 32) |
                   static_cast<unsigned long long>(0xFFFFFFFFu - unsigned(nn));
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const unsigned long long ob = __shfl_xor_sync(0xffffffffu, best, o);
          best = ob > best ? ob : best;
        }
        if (lane == 0 && best) atomicMax(&s_best[m], best);
      }
    } else {
      for (int e = lane; e < 16 * M; e += 32) {
        const int r = e & 15, m = e >> 4;
        const long nn = long(T) * 16 + r;
        if constexpr (EPI == EPI_SILU) {
          const float g16 = rnd<half>(v[r * NC + m]), u16 = rnd<half>(v[(16 + r) * NC + m]);
          const float act = rnd<half>(g16 / (1.0f + expf(-g16)));
          Y[long(m) * a.ldy + nn] = __float2half_rn(act * u16);
        } else {
          float val = rnd<half>(v[r * NC + m]);
          if (bias) val = rnd<half>(val + __half2float(bias[nn]));
          if constexpr (EPI == EPI_RESID)
            val += __half2float(reinterpret_cast<const half*>(a.res)[long(m) * a.ldres + nn]);
          Y[long(m) * a.ldy + nn] = __float2half_rn(val);
        }
      }
    }
  };

  // accumulators: ONE → acc[tp][0] row g, acc[tp][2] row g+8; else d0..d3
  float acc[TPT][4];
  auto zero_acc = [&]() {
#pragma unroll
    for (int tp = 0; tp < TPT; ++tp) acc[tp][0] = acc[tp][1] = acc[tp][2] = acc[tp][3] = 0.f;
  };
  zero_acc();

  // write this warp's sums of the current tile group to dst[r * NC + m]
  auto put = [&](float* dst) {
    if constexpr (ONE) {
#pragma unroll
      for (int tp = 0; tp < TPT; ++tp) {
        float v0 = acc[tp][0], v2 = acc[tp][2];
        v0 += __shfl_xor_sync(0xffffffffu, v0, 1);
        v2 += __shfl_xor_sync(0xffffffffu, v2, 1);
        v0 += __shfl_xor_sync(0xffffffffu, v0, 2);
        v2 += __shfl_xor_sync(0xffffffffu, v2, 2);
        if (t == 0) {
          dst[tp * 16 + g] = v0;
          dst[tp * 16 + g + 8] = v2;
        }
      }
    } else {
#pragma unroll
      for (int tp = 0; tp < TPT; ++tp) {
        float* r0 = dst + (tp * 16 + g) * 8 + 2 * t;
        *reinterpret_cast<float2*>(r0) = make_float2(acc[tp][0], acc[tp][1]);
        *reinterpret_cast<float2*>(r0 + 64) = make_float2(acc[tp][2], acc[tp][3]);
      }
    }
  };

  // tile group T ends for this warp
  auto flush = [&](int T) {
    const int li = T - t_first;  // local tile index
    const long long t0 = (long long)T * nb, t1 = (long long)(T + 1) * nb;
    const long long fu = t0 > C0 ? t0 : C0;
    const long long lu = (t1 < C1 ? t1 : C1) - 1;
    const int wa = owner_of(fu - C0, n, kWarps), wb = owner_of(lu - C0, n, kWarps);
    float* mine = wout;
    if (wa != wb) {
      float* slots = red + size_t(li) * L.c_max * (ROWS * NC);
      put(slots + (warp - wa) * (ROWS * NC));
      __syncwarp();
      unsigned last = 0;
      if (lane == 0) {
        __threadfence_block();
        last = (atomicAdd(&cnt[li], 1u) == unsigned(wb - wa)) ? 1u : 0u;
        __threadfence_block();
      }
      last = __shfl_sync(0xffffffffu, last, 0);
      __syncwarp();
      if (!last) return;
      for (int i = lane; i < ROWS * NC; i += 32) {
        float v = 0.f;
        for (int k = 0; k <= wb - wa; ++k) v += slots[k * (ROWS * NC) + i];
        mine[i] = v;
      }
    } else {
      put(mine);
    }
    __syncwarp();
    if (fu == t0 && lu == t1 - 1) {
      finalize(T, mine);
    } else {
      // a tile group shared with the neighbouring CTA (this CTA holds its
      // start: side 1, or its end: side 0). Both publish their part; the
      // second to arrive adds the two and finishes the tile group, so
      // neither waits for the other. Two-term sums are order-free, so the
      // result is the same whichever CTA finishes it.
      const int side = fu > t0 ? 1 : 0;
      float* slot = a.partials + (size_t(T) * 2 + side) * (ROWS * NC);
      for (int i = lane; i < ROWS * NC; i += 32) __stcg(slot + i, mine[i]);
      __threadfence();
      __syncwarp();
      unsigned last = 0;
      if (lane == 0) {
        last = atomicAdd(a.counters + T, 1u) == 1u ? 1u : 0u;
        if (last) {
          __threadfence();
          a.counters[T] = 0u;  // zero again for the next launch
        }
      }
      last = __shfl_sync(0xffffffffu, last, 0);
      if (!last) return;
      const float* other = a.partials + (size_t(T) * 2 + (1 - side)) * (ROWS * NC);
      for (int i = lane; i < ROWS * NC; i += 32) mine[i] += __ldcg(other + i);
      __syncwarp();
      finalize(T, mine);
    }
    __syncwarp();
  };

  // per-lane constants of the record math
  const int gi_t = t >> 1, term = t & 1;
  const int coef_off = ONE ? 1024 + ((term * 2 + gi_t) * 8 + g) * 4 : 1024 + g * 4;
  const unsigned char* xb_b = reinterpret_cast<const unsigned char*>(xB);
  const unsigned char* zero_b = smem + L.zero_off;
  // ONE: B operand of the group-0 MMAs (columns 0-3) and the group-1 MMAs
  // (columns 4-7): real fragments for the lanes of those columns, zeros
  // for the others
  const unsigned char* xA_base = g < 4 ? xb_b + t * 32 : zero_b;
  const int xA_step = g < 4 ? 256 : 0;
  const unsigned char* xB_base = g >= 4 ? xb_b + (4 + t) * 32 : zero_b;
  const int xB_step = g >= 4 ? 256 : 0;
  const int colsel = ONE ? 0 : (g < M ? g : M - 1);
  const unsigned char* xcol_b = xb_b + size_t(colsel) * L.colstride * 4 + t * 32;

  // running state: tile group tg, the operand pointers of the current block
  // (blk at the start), the ring stage's byte offset, and the unit that ends
  // the current tile group's part of this warp's range
  int tg = u0 / nb, slot_off = 0;
  const int blk = u0 - tg * nb;
  int seg_end = min(u1, (tg + 1) * nb);
  const unsigned char* pa = xA_base + blk * xA_step;
  const unsigned char* pb = xB_base + blk * xB_step;
  const unsigned char* px = xcol_b + blk * 256;
  int cxi = ONE ? 2 * blk + gi_t : blk * 16 + 2 * t;
  for (int u = u0; u < u1;) {
    cp_wait<STAGES - 1>();
    __syncwarp();
    const unsigned char* rec0 = ring + slot_off;
    if constexpr (ONE) {
      const float2 cx = CX[cxi];
      const uint4 xa0 = *reinterpret_cast<const uint4*>(pa);
      const uint4 xa1 = *reinterpret_cast<const uint4*>(pa + 16);
      const uint4 xb0 = *reinterpret_cast<const uint4*>(pb);
      const uint4 xb1 = *reinterpret_cast<const uint4*>(pb + 16);
#pragma unroll
      for (int tp = 0; tp < TPT; ++tp) {
        const unsigned char* r = rec0 + tp * kRecS;
        const uint4 w0 = *reinterpret_cast<const uint4*>(r + 16 * lane);
        const uint4 w1 = *reinterpret_cast<const uint4*>(r + kRecWS + 16 * lane);
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
        acc[tp][2] = fmaf(__high2float(ch), v2, acc[tp][2]);
      }
    } else {
#pragma unroll
      for (int gi = 0; gi < 2; ++gi) {
        const uint4 xa = *reinterpret_cast<const uint4*>(px + gi * 128);
        const uint4 xc = *reinterpret_cast<const uint4*>(px + gi * 128 + 16);
        const float4 cx = *reinterpret_cast<const float4*>(CX + cxi + gi * 8);
#pragma unroll
        for (int tp = 0; tp < TPT; ++tp) {
          const unsigned char* r = rec0 + tp * kRecS;
          const uint2 w0 = *reinterpret_cast<const uint2*>(r + 16 * lane + 8 * gi);
          const uint2 w1 = *reinterpret_cast<const uint2*>(r + kRecWS + 16 * lane + 8 * gi);
          const __half2 sh = *reinterpret_cast<const __half2*>(r + coef_off + gi * 32);
          const __half2 bh = *reinterpret_cast<const __half2*>(r + coef_off + 64 + gi * 32);
          uint32_t P0[8], P1[8];
          dequant_word<4>(w0.x, P0);
          dequant_word<4>(w0.y, P0 + 4);
          dequant_word<4>(w1.x, P1);
          dequant_word<4>(w1.y, P1 + 4);
          float d[4];
          mma16816(d, P0[0], P1[0], P0[1], P1[1], xa.x, xa.y, cx.x, cx.z, cx.x, cx.z);
          mma16816(d, P0[2], P1[2], P0[3], P1[3], xa.z, xa.w, d[0], d[1], d[2], d[3]);
          mma16816(d, P0[4], P1[4], P0[5], P1[5], xc.x, xc.y, d[0], d[1], d[2], d[3]);
          mma16816(d, P0[6], P1[6], P0[7], P1[7], xc.z, xc.w, d[0], d[1], d[2], d[3]);
          const float s0 = __low2float(sh), s1 = __high2float(sh), b0 = __low2float(bh), b1 = __high2float(bh);
          acc[tp][0] = fmaf(s0, d[0], fmaf(b0, cx.y, acc[tp][0]));
          acc[tp][1] = fmaf(s0, d[1], fmaf(b0, cx.w, acc[tp][1]));
          acc[tp][2] = fmaf(s1, d[2], fmaf(b1, cx.y, acc[tp][2]));
          acc[tp][3] = fmaf(s1, d[3], fmaf(b1, cx.w, acc[tp][3]));
        }
      }
    }
    __syncwarp();
    issue(slot_off);
    slot_off = slot_off == (STAGES - 1) * TPT * kRecS ? 0 : slot_off + TPT * kRecS;
    if (++u == seg_end) {
      flush(tg);
      zero_acc();
      ++tg;
      seg_end = min(u1, seg_end + nb);
      pa = xA_base;
      pb = xB_base;
      px = xcol_b;
      cxi = ONE ? gi_t : 2 * t;
    } else {
      pa += xA_step;
      pb += xB_step;
      px += 256;
      cxi += ONE ? 2 : 16;
    }
  }
  cp_wait<0>();

  if constexpr (EPI == EPI_ARGMAX) {
    __syncthreads();
    if (warp != 0) return;
    __syncwarp();
    if (lane < M && s_best[lane]) atomicMax(a.keys + lane, s_best[lane]);
    __syncwarp();
    unsigned last = 0;
    if (lane == 0) {
      __threadfence();
      last = (atomicAdd(a.done, 1u) == unsigned(Gd - 1)) ? 1u : 0u;
      if (last) __threadfence();
    }
    last = __shfl_sync(0xffffffffu, last, 0);
    if (last) {
      if (lane < M) {
        const unsigned long long k = atomicExch(a.keys + lane, 0ull);
        const int id = k ? int(0xFFFFFFFFu - unsigned(k & 0xFFFFFFFFull)) : 0;
        a.out_ids[lane] = id;
        if (a.next_tokens) a.next_tokens[lane] = id;
      }
      if (lane == 0) *a.done = 0u;
    }
  }
}

// CTAs of a launch: one per tile group when there are at most two per SM
// and a tile group gives every warp a block (no tile group is split between
// CTAs), else at most two per SM with ranges of at least one tile group and
// at least one unit per warp, so a tile group meets at most two CTAs
int small_grid(int num_sms, int n_tg, int K) {
  const int nb = K / 128;
  const long long U = (long long)n_tg * nb;
  if (n_tg <= 2 * num_sms && nb >= kWarps) return n_tg;
  return int(std::max<long long>(1, std::min<long long>(std::min<long long>(2LL * num_sms, n_tg), U / kWarps)));
}

SmallLayout small_layout(int M, int K, int tpt, int stages, int grid, int n_tg) {
  SmallLayout L;
  const int ng = K / 64, nb = K / 128;
  const bool one = M == 1;
  const int rows = 16 * tpt, nc = one ? 1 : 8;
  const long long U = (long long)n_tg * nb;
  const long long nmax = (U + grid - 1) / grid, nmin = U / grid;
  L.lt_max = int(std::min<long long>(n_tg, (nmax + nb - 1) / nb + 1));
  const long long per_warp = nmin / kWarps;
  L.c_max = per_warp <= 0 ? kWarps : int(std::min<long long>(kWarps, (nb + per_warp - 1) / per_warp + 1));
  L.colstride = one ? ng * 32 : ng * 32 + 4;
  size_t off = size_t(kWarps) * stages * tpt * kRecS;
  L.xb_off = int(off);
  off += align_up(size_t(M) * L.colstride * 4, 16);
  L.cx_off = int(off);
  off += align_up(size_t(ng) * (one ? 1 : 8) * 8, 16);
  L.out_off = int(off);
  off += align_up(size_t(kWarps) * rows * nc * 4, 16);
  L.red_off = int(off);
  off += align_up(size_t(L.lt_max) * L.c_max * rows * nc * 4, 16);
  L.cnt_off = int(off);
  off += align_up(size_t(L.lt_max) * 4, 16);
  L.zero_off = int(off);
  off += 32;
  L.total = int(std::max<size_t>(off, kMinSmemS));
  return L;
}

// ring depth: the deepest that keeps two CTAs per SM, else the deepest that
// fits one
int small_stages(int M, int K, int tpt, int grid, int n_tg) {
  const int choices1[] = {8, 6, 4, 3};
  const int choices2[] = {4, 3, 2};
  const int* ch = tpt == 1 ? choices1 : choices2;
  const int nch = tpt == 1 ? 4 : 3;
  for (int i = 0; i < nch; ++i)
    if (small_layout(M, K, tpt, ch[i], grid, n_tg).total <= kTwoPerSm) return ch[i];
  for (int i = 0; i < nch; ++i)
    if (small_layout(M, K, tpt, ch[i], grid, n_tg).total <= kMaxSmemS) return ch[i];
  return 0;
}

template <int EPI, int TPT, int STAGES, bool ONE>
nmx_status_t launch_small(Ctx* c, const GemvDLArgs& a0, int grid, const SmallLayout& L) {
  auto kern = qgemv_dl8_kernel<EPI, TPT, STAGES, ONE>;
  static std::mutex mu;
  static std::map<int, bool> attr_set;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (!attr_set[c->device]) {
      NMX_CUDA_OK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmemS));
      attr_set[c->device] = true;
    }
  }
  return launch(c, kern, dim3(grid), dim3(kThreads), size_t(L.total), a0, L);
}

template <int EPI, int TPT, bool ONE>
nmx_status_t by_stages(Ctx* c, const GemvDLArgs& a, int grid, int stages, const SmallLayout& L) {
  if constexpr (TPT == 1) {
    switch (stages) {
      case 8: return launch_small<EPI, 1, 8, ONE>(c, a, grid, L);
      case 6: return launch_small<EPI, 1, 6, ONE>(c, a, grid, L);
      case 4: return launch_small<EPI, 1, 4, ONE>(c, a, grid, L);
      case 3: return launch_small<EPI, 1, 3, ONE>(c, a, grid, L);
    }
  } else {
    switch (stages) {
      case 4: return launch_small<EPI, 2, 4, ONE>(c, a, grid, L);
      case 3: return launch_small<EPI, 2, 3, ONE>(c, a, grid, L);
      case 2: return launch_small<EPI, 2, 2, ONE>(c, a, grid, L);
    }
  }
  NMX_CHECK(false, NMX_ERR_UNSUPPORTED, "qgemv_small: ring depth");
}

template <bool ONE>
nmx_status_t by_epi(Ctx* c, const GemvDLArgs& a, int epi, int grid, int stages, const SmallLayout& L) {
  switch (epi) {
    case EPI_STORE: return by_stages<EPI_STORE, 1, ONE>(c, a, grid, stages, L);
    case EPI_RESID: return by_stages<EPI_RESID, 1, ONE>(c, a, grid, stages, L);
    case EPI_SILU: return by_stages<EPI_SILU, 2, ONE>(c, a, grid, stages, L);
    case EPI_ARGMAX: return by_stages<EPI_ARGMAX, 1, ONE>(c, a, grid, stages, L);
  }
  NMX_CHECK(false, NMX_ERR_UNSUPPORTED, "qgemv_small: unknown epilogue");
}

}  // namespace

bool qgemv_small_fits(int M, int N_out, int K, int epi, int num_sms) {
  if (M < 1 || M > 8) return false;
  const int n_tg = N_out / 16;
  const int tpt = epi == EPI_SILU ? 2 : 1;
  return small_stages(M, K, tpt, small_grid(num_sms, n_tg, K), n_tg) > 0;
}

size_t qgemv_small_partials_floats(int N_out, int K, int epi, int num_sms) {
  (void)K;
  (void)num_sms;
  const int rows = epi == EPI_SILU ? 32 : 16;
  return size_t(N_out / 16) * rows * 8 * 2;  // two part slots per tile group
}

nmx_status_t qgemv_small(Ctx* c, const GemvDLArgs& a0, int epi) {
  NMX_CHECK(qgemv_small_fits(a0.M, a0.N, a0.K, epi, c->num_sms), NMX_ERR_UNSUPPORTED, "qgemv_small: shape");
  GemvDLArgs a = a0;
  const int tpt = epi == EPI_SILU ? 2 : 1;
  const int grid = small_grid(c->num_sms, a.n_tg, a.K);
  const int stages = small_stages(a.M, a.K, tpt, grid, a.n_tg);
  const SmallLayout L = small_layout(a.M, a.K, tpt, stages, grid, a.n_tg);
  const int nc = a.M == 1 ? 1 : 8;
  NMX_CHECK(size_t(a.n_tg) * 16 * tpt * nc * 2 <= a.partials_cap, NMX_ERR_UNSUPPORTED,
            "qgemv_small: partial-sum scratch too small");
  NMX_CHECK(a.err != nullptr, NMX_ERR_INVALID, "qgemv_small: no error word");
  return a.M == 1 ? by_epi<true>(c, a, epi, grid, stages, L) : by_epi<false>(c, a, epi, grid, stages, L);
}

}  // namespace nmx
