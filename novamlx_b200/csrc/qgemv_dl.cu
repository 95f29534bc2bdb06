// Decode GEMV over weights repacked into decode records (4-bit, group 64,
// f16 activations): the layout the model keeps its linears in.
//
// Record (tile T of 16 rows, block B of 128 k = two groups), 1152 bytes:
//   [   0,  512)  lane l = 4g+t: 16 B = words (2t, 2t+1) of groups 2B and
//                 2B+1 of row 16T+g (the words lane l feeds to the MMA)
//   [ 512, 1024)  the same for row 16T+g+8
//   [1024, 1152)  scales, then biases (f16): entry (kind, group gi, g) at
//                 1024 + ((kind * 2 + gi) * 8 + g) * 4 holds the pair
//                 (row 16T+g, row 16T+g+8), so one 4-byte load gives a lane
//                 the coefficient of both rows its MMA accumulators cover
// Records of a tile are consecutive in k, tiles consecutive in rows, so a
// linear is one stream of 1152-byte records and holds exactly the bytes of
// its MLX form (packed words + scales + biases).
//
// Each warp owns a contiguous share of the (tile group, block) units of the
// launch (stream-K split: every warp gets the same number of records) and
// streams it through a private ring of cp.async stages; lanes copy the bytes
// they consume (plus eight lanes the scales), so after the activation
// prologue no CTA-wide barrier is needed. A tile group split across warps
// is summed by its last-arriving warp in a fixed slot order (deterministic).
// The argmax epilogue folds every tile into one packed 64-bit key per row
// (ordered value, inverted index) with atomicMax: the maximum with the
// lowest index on ties, whatever the arrival order.
#include <algorithm>
#include <map>
#include <mutex>
#include <tuple>

#include "common.cuh"
#include "kernels.h"
#include "qgemv_common.cuh"

namespace nmx {

namespace {

constexpr int kRec = 1152;  // bytes per decode record
constexpr int kRecW = 512;  // bytes of one row half of the packed words
constexpr int kMaxDynSmemDL = 200 * 1024;

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
  const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem_dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

__device__ __forceinline__ unsigned ordered_bits(float v) {
  const unsigned u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

template <int NT, int EPI, int TPT, int STAGES>
__global__ void __launch_bounds__(kThreads, 2) qgemv_dl_kernel(GemvDLArgs a) {
  constexpr int NCOL = NT * 8;
  constexpr int ROWS = 16 * TPT;
  using C = QCfg<4, 64>;
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ float s_inv[32];
  __shared__ float s_wsum[kWarps][32];

  const int K = a.K, M = a.M;
  const int ng = K / 64, nb = K / 128;
  const int colstride = ng * 4 * C::MP + 4;
  uint32_t* xB = reinterpret_cast<uint32_t*>(smem);
  float2* CX = reinterpret_cast<float2*>(smem + ((size_t(M) * colstride * 4 + 15) & ~size_t(15)));
  unsigned char* ring0 = reinterpret_cast<unsigned char*>(CX) + size_t(ng) * NCOL * sizeof(float2);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  unsigned char* ring = ring0 + size_t(warp) * (STAGES * TPT * kRec + ROWS * NCOL * 4);
  float* stage_out = reinterpret_cast<float*>(ring + STAGES * TPT * kRec);

  // this warp's units [u0, u1) of U = n_tg * nb (U < 2^31; products in 64 bit)
  const int U = a.n_tg * nb;
  const int W = gridDim.x * kWarps;
  const int wg = blockIdx.x * kWarps + warp;
  const int u0 = int((long long)wg * U / W), u1 = int((long long)(wg + 1) * U / W);

  // unit u is record u of the matrix (tile-major, blocks inside a tile), so
  // the issue cursor is a pointer that advances one record per unit; the
  // paired up tile sits pair_tiles * nb records further
  const unsigned char* src_cur = reinterpret_cast<const unsigned char*>(a.w) + size_t(u0) * kRec + 16 * lane;
  const size_t pair_off = size_t(a.pair_tiles) * nb * kRec;
  int is_u = u0;
  auto issue = [&](int slot) {
    if (is_u < u1) {
      unsigned char* dst = ring + size_t(slot) * TPT * kRec + 16 * lane;
#pragma unroll
      for (int tp = 0; tp < TPT; ++tp) {
        const unsigned char* src = src_cur + tp * pair_off;
        cp_async16(dst + tp * kRec, src);
        cp_async16(dst + tp * kRec + kRecW, src + kRecW);
        if (lane < 8) cp_async16(dst + tp * kRec + 1024, src + 1024);
      }
      ++is_u;
      src_cur += kRec;
    }
    cp_async_commit();
  };

  // model weights never change during a step: start streaming them before
  // the wait (records an op-level caller may just have written are not)
  if (!a.weights_static) grid_wait();
#pragma unroll
  for (int s = 0; s < STAGES; ++s) issue(s);

  // ------------------------------------------------ activation prologue
  grid_wait();
  {
    const half* X = reinterpret_cast<const half*>(a.x);
    const half* Gm = reinterpret_cast<const half*>(a.gamma);
    if (Gm) {
      for (int c = 0; c < M; ++c) {
        float ss = 0.f;
        for (int k = tid; k < K; k += kThreads) {
          const float v = __half2float(X[long(c) * a.ldx + k]);
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
      const half* xr = X + long(c) * a.ldx + G * 64;
      const half* gr = Gm ? Gm + G * 64 : nullptr;
      const float inv = Gm ? s_inv[c] : 1.f;
      float bsum = 0.f, xsum = 0.f;
      uint32_t* dst = xB + size_t(c) * colstride + (G * 4 + tt) * C::MP;
#pragma unroll
      for (int p = 0; p < C::MP; ++p) {
        int k0, k1;
        bool hi;
        pair_k<4, 64>(tt, p, k0, k1, hi);
        float x0 = __half2float(xr[k0]), x1 = __half2float(xr[k1]);
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
      if (tt == 0) CX[size_t(G) * NCOL + c] = make_float2(-1024.f * bsum, xsum);
    }
    for (int it = tid; it < ng * (NCOL - M); it += kThreads) {
      const int G = it / (NCOL - M), c = M + it % (NCOL - M);
      CX[size_t(G) * NCOL + c] = make_float2(0.f, 0.f);
    }
  }
  __syncthreads();
  grid_launch_dependents();

  float acc[TPT][NT][4];
  auto zero_acc = [&]() {
#pragma unroll
    for (int tp = 0; tp < TPT; ++tp)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) acc[tp][nt][0] = acc[tp][nt][1] = acc[tp][nt][2] = acc[tp][nt][3] = 0.f;
  };
  zero_acc();

  // epilogue of one finished tile group: values v(r, m) come from `val`
  auto finalize = [&](int tg, auto val) {
    const half* bias = reinterpret_cast<const half*>(a.bias);
    half* Y = reinterpret_cast<half*>(a.y);
    if constexpr (EPI == EPI_ARGMAX) {
      for (int m = 0; m < M; ++m) {
        unsigned long long best = 0ull;
        if (lane < 16) {
          const long n = long(tg) * 16 + lane;
          const float v = rnd<half>(val(lane, m));
          if (a.logits_f32) a.logits_f32[long(m) * a.N + n] = v;
          if (!(v != v))
            best = (static_cast<unsigned long long>(ordered_bits(v)) << 32) |
                   static_cast<unsigned long long>(0xFFFFFFFFu - unsigned(n));
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const unsigned long long ob = __shfl_xor_sync(0xffffffffu, best, o);
          best = ob > best ? ob : best;
        }
        if (lane == 0 && best) atomicMax(a.keys + m, best);
      }
      __threadfence();
      unsigned last = 0;
      if (lane == 0) last = (atomicAdd(a.done, 1u) == unsigned(a.n_tg - 1)) ? 1u : 0u;
      last = __shfl_sync(0xffffffffu, last, 0);
      if (last) {
        __threadfence();
        if (lane < M) {
          const unsigned long long k = atomicExch(a.keys + lane, 0ull);
          const int id = k ? int(0xFFFFFFFFu - unsigned(k & 0xFFFFFFFFull)) : 0;
          a.out_ids[lane] = id;
          if (a.next_tokens) a.next_tokens[lane] = id;
        }
        if (lane == 0) *a.done = 0u;
      }
    } else {
      for (int e = lane; e < 16 * M; e += 32) {
        const int r = e & 15, m = e >> 4;
        const long n = long(tg) * 16 + r;
        if constexpr (EPI == EPI_SILU) {
          const float g16 = rnd<half>(val(r, m)), u16 = rnd<half>(val(16 + r, m));
          const float act = rnd<half>(g16 / (1.0f + expf(-g16)));
          Y[long(m) * a.ldy + n] = __float2half_rn(act * u16);
        } else {
          float v = rnd<half>(val(r, m));
          if (bias) v = rnd<half>(v + __half2float(bias[n]));
          if constexpr (EPI == EPI_RESID)
            v += __half2float(reinterpret_cast<const half*>(a.res)[long(m) * a.ldres + n]);
          Y[long(m) * a.ldy + n] = __float2half_rn(v);
        }
      }
    }
  };

  // flush the accumulators of tile group tg
  auto flush = [&](int tg) {
#pragma unroll
    for (int tp = 0; tp < TPT; ++tp)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        float* r = stage_out + (tp * 16) * NCOL + nt * 8 + 2 * t;
        r[g * NCOL] = acc[tp][nt][0];
        r[g * NCOL + 1] = acc[tp][nt][1];
        r[(g + 8) * NCOL] = acc[tp][nt][2];
        r[(g + 8) * NCOL + 1] = acc[tp][nt][3];
      }
    __syncwarp();
    // contributors of this tile group: warps owning its first and last unit
    const long long ufirst = (long long)tg * nb, ulast = ufirst + nb - 1;
    const int wfirst = int(((ufirst + 1) * W - 1) / U), wlast = int(((ulast + 1) * W - 1) / U);
    const int nctr = wlast - wfirst + 1;
    if (nctr == 1) {
      finalize(tg, [&](int r, int m) { return stage_out[r * NCOL + m]; });
    } else {
      const int pslot = wg - wfirst;
      float* part = a.partials + (size_t(tg) * a.max_contrib + pslot) * (ROWS * NCOL);
      for (int i = lane; i < ROWS * NCOL; i += 32) part[i] = stage_out[i];
      __threadfence();
      __syncwarp();
      unsigned last = 0;
      if (lane == 0) last = (atomicAdd(a.counters + tg, 1u) == unsigned(nctr - 1)) ? 1u : 0u;
      last = __shfl_sync(0xffffffffu, last, 0);
      if (last) {
        __threadfence();
        const float* base = a.partials + size_t(tg) * a.max_contrib * (ROWS * NCOL);
        for (int i = lane; i < ROWS * NCOL; i += 32) {
          float v = 0.f;
          for (int sl = 0; sl < nctr; ++sl) v += __ldcg(base + size_t(sl) * (ROWS * NCOL) + i);
          stage_out[i] = v;
        }
        __syncwarp();
        finalize(tg, [&](int r, int m) { return stage_out[r * NCOL + m]; });
        if (lane == 0) a.counters[tg] = 0u;
      }
    }
    __syncwarp();
  };

  int tg = u0 / nb, blk = u0 - (u0 / nb) * nb, slot = 0;
  for (int u = u0; u < u1; ++u) {
    cp_async_wait<STAGES - 1>();
    __syncwarp();
    const unsigned char* rec0 = ring + size_t(slot) * TPT * kRec;
#pragma unroll
    for (int tp = 0; tp < TPT; ++tp) {
      const unsigned char* rec = rec0 + tp * kRec;
      const uint4 w0 = *reinterpret_cast<const uint4*>(rec + 16 * lane);
      const uint4 w1 = *reinterpret_cast<const uint4*>(rec + kRecW + 16 * lane);
      // (row g, row g+8) pairs of scales / biases of groups 0 and 1
      const __half2 sA = *reinterpret_cast<const __half2*>(rec + 1024 + 4 * g);
      const __half2 sB = *reinterpret_cast<const __half2*>(rec + 1056 + 4 * g);
      const __half2 bA = *reinterpret_cast<const __half2*>(rec + 1088 + 4 * g);
      const __half2 bB = *reinterpret_cast<const __half2*>(rec + 1120 + 4 * g);
#pragma unroll
      for (int gi = 0; gi < 2; ++gi) {
        const int G = 2 * blk + gi;
        uint32_t P0[8], P1[8];
        dequant_word<4>(gi ? w0.z : w0.x, P0);
        dequant_word<4>(gi ? w0.w : w0.y, P0 + 4);
        dequant_word<4>(gi ? w1.z : w1.x, P1);
        dequant_word<4>(gi ? w1.w : w1.y, P1 + 4);
        const float fs0 = __low2float(gi ? sB : sA), fs1 = __high2float(gi ? sB : sA);
        const float fb0 = __low2float(gi ? bB : bA), fb1 = __high2float(gi ? bB : bA);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          int col = nt * 8 + g;
          col = col < M ? col : M - 1;
          const uint32_t* xb = xB + size_t(col) * colstride + (G * 4 + t) * C::MP;
          const uint4 xa = *reinterpret_cast<const uint4*>(xb);
          const uint4 xc = *reinterpret_cast<const uint4*>(xb + 4);
          const float4 cx = *reinterpret_cast<const float4*>(CX + size_t(G) * NCOL + nt * 8 + 2 * t);
          float d[4] = {cx.x, cx.z, cx.x, cx.z};
          mma16816(d, P0[0], P1[0], P0[1], P1[1], xa.x, xa.y, d[0], d[1], d[2], d[3]);
          mma16816(d, P0[2], P1[2], P0[3], P1[3], xa.z, xa.w, d[0], d[1], d[2], d[3]);
          mma16816(d, P0[4], P1[4], P0[5], P1[5], xc.x, xc.y, d[0], d[1], d[2], d[3]);
          mma16816(d, P0[6], P1[6], P0[7], P1[7], xc.z, xc.w, d[0], d[1], d[2], d[3]);
          acc[tp][nt][0] = fmaf(fs0, d[0], fmaf(fb0, cx.y, acc[tp][nt][0]));
          acc[tp][nt][2] = fmaf(fs1, d[2], fmaf(fb1, cx.y, acc[tp][nt][2]));
          acc[tp][nt][1] = fmaf(fs0, d[1], fmaf(fb0, cx.w, acc[tp][nt][1]));
          acc[tp][nt][3] = fmaf(fs1, d[3], fmaf(fb1, cx.w, acc[tp][nt][3]));
        }
      }
    }
    __syncwarp();
    issue(slot);
    if (blk == nb - 1 || u == u1 - 1) {
      flush(tg);
      zero_acc();
    }
    if (++slot == STAGES) slot = 0;
    if (++blk == nb) {
      blk = 0;
      ++tg;
    }
  }
  cp_async_wait<0>();
}

// every warp must own at least one unit: W = grid * 8 <= U
int dl_grid(int num_sms, int ctas_per_sm, int n_tg, int K) {
  const long long U = (long long)n_tg * (K / 128);
  return int(std::max<long long>(1, std::min<long long>((long long)num_sms * ctas_per_sm, U / kWarps)));
}

// largest number of warps whose unit ranges meet one tile group: with
// w(u) = floor(((u + 1) W - 1) / U) the owner of unit u, tile group tg meets
// w(last unit) - w(first unit) + 1 warps. Exact scan, cached per shape.
int dl_contrib(int n_tg, int K, int grid) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, int>, int> cache;
  const auto key = std::make_tuple(n_tg, K, grid);
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  const long long nb = K / 128, U = (long long)n_tg * nb, W = (long long)grid * kWarps;
  int best = 1;
  for (long long tg = 0; tg < n_tg; ++tg) {
    const long long a = tg * nb, b = a + nb - 1;
    best = std::max(best, int(((b + 1) * W - 1) / U - ((a + 1) * W - 1) / U + 1));
  }
  std::lock_guard<std::mutex> lk(mu);
  cache[key] = best;
  return best;
}

template <int NT, int EPI, int TPT, int STAGES>
nmx_status_t launch_dl(Ctx* c, const GemvDLArgs& a0, int M) {
  constexpr int NCOL = NT * 8;
  constexpr int ROWS = 16 * TPT;
  const int ng = a0.K / 64;
  const int colstride = ng * 4 * 8 + 4;
  const size_t ring = size_t(kWarps) * (STAGES * TPT * kRec + ROWS * NCOL * 4);
  const size_t smem = align_up(size_t(M) * colstride * 4, 16) + size_t(ng) * NCOL * sizeof(float2) + ring;
  NMX_CHECK(smem <= size_t(kMaxDynSmemDL), NMX_ERR_UNSUPPORTED, "qgemv_dl: staging too large");
  auto kern = qgemv_dl_kernel<NT, EPI, TPT, STAGES>;
  static std::mutex mu;
  static std::map<int, bool> attr_set;
  static std::map<std::pair<int, size_t>, int> occ;  // (device, smem) → resident CTAs per SM
  int per_sm = 0;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (!attr_set[c->device]) {
      NMX_CUDA_OK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxDynSmemDL));
      attr_set[c->device] = true;
    }
    const auto key = std::make_pair(c->device, smem);
    auto it = occ.find(key);
    if (it == occ.end()) {
      NMX_CUDA_OK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem));
      occ[key] = per_sm;
    } else {
      per_sm = it->second;
    }
  }
  NMX_CHECK(per_sm > 0, NMX_ERR_UNSUPPORTED, "qgemv_dl: does not fit on an SM");
  GemvDLArgs a = a0;
  a.M = M;
  // the split is static per warp: every CTA must be resident at once
  const int grid = dl_grid(c->num_sms, std::min(a.ctas_per_sm, per_sm), a.n_tg, a.K);
  a.max_contrib = dl_contrib(a.n_tg, a.K, grid);
  NMX_CHECK(size_t(a.n_tg) * a.max_contrib * ROWS * NCOL <= a.partials_cap, NMX_ERR_UNSUPPORTED,
            "qgemv_dl: partial-sum scratch too small");
  return launch(c, kern, dim3(grid), dim3(kThreads), smem, a);
}

constexpr int kStages1 = 6;  // ring depth, one tile per unit
constexpr int kStages2 = 3;  // ring depth, gate+up tile pairs

template <int NT>
nmx_status_t dispatch_dl(Ctx* c, const GemvDLArgs& a, int M, int epi) {
  switch (epi) {
    case EPI_STORE: return launch_dl<NT, EPI_STORE, 1, kStages1>(c, a, M);
    case EPI_RESID: return launch_dl<NT, EPI_RESID, 1, kStages1>(c, a, M);
    case EPI_SILU: return launch_dl<NT, EPI_SILU, 2, kStages2>(c, a, M);
    case EPI_ARGMAX: return launch_dl<NT, EPI_ARGMAX, 1, kStages1>(c, a, M);
  }
  NMX_CHECK(false, NMX_ERR_UNSUPPORTED, "qgemv_dl: unknown epilogue");
}

// MLX layout → decode records (or back): one thread per 16-byte lane chunk
// and per scale/bias pair.
__global__ void repack_kernel(const uint32_t* wq, const half* s, const half* b, int K, long row0,
                              unsigned char* rec, int part_mask, int inverse, uint32_t* wq_out, half* s_out,
                              half* b_out, int rows) {
  grid_wait();
  const int nb = K / 128, ng = K / 64, wpr = K / 8;
  const long total = long(rows / 16) * nb;
  for (long i = blockIdx.x * long(blockDim.x) + threadIdx.x; i < total * 32; i += long(gridDim.x) * blockDim.x) {
    const long rt = i / 32;
    const int lane = int(i % 32), g = lane >> 2, t = lane & 3;
    const long tl = rt / nb;          // tile within the slice
    const int blk = int(rt % nb);
    const long T = (row0 / 16) + tl;  // tile within the whole matrix
    unsigned char* r = rec + (size_t(T) * nb + blk) * kRec;
    for (int hf = 0; hf < 2; ++hf) {
      const long row = tl * 16 + g + 8 * hf;  // row within the slice
      uint32_t* dst = reinterpret_cast<uint32_t*>(r + hf * kRecW + 16 * lane);
      const long base = row * wpr + long(blk) * 16 + 2 * t;
      if (part_mask & 1) {
        if (!inverse) {
          dst[0] = wq[base];
          dst[1] = wq[base + 1];
          dst[2] = wq[base + 8];
          dst[3] = wq[base + 9];
        } else {
          wq_out[base] = dst[0];
          wq_out[base + 1] = dst[1];
          wq_out[base + 8] = dst[2];
          wq_out[base + 9] = dst[3];
        }
      }
    }
    if (t == 0) {
      for (int hf = 0; hf < 2; ++hf) {
        const long row = tl * 16 + g + 8 * hf;
        const long sb = row * ng + 2 * blk;
        for (int gi = 0; gi < 2; ++gi) {
          half* rs = reinterpret_cast<half*>(r + 1024 + ((0 * 2 + gi) * 8 + g) * 4) + hf;
          half* rb = reinterpret_cast<half*>(r + 1024 + ((1 * 2 + gi) * 8 + g) * 4) + hf;
          if (part_mask & 2) {
            if (!inverse) *rs = s[sb + gi];
            else s_out[sb + gi] = *rs;
          }
          if (part_mask & 4) {
            if (!inverse) *rb = b[sb + gi];
            else b_out[sb + gi] = *rb;
          }
        }
      }
    }
  }
  grid_launch_dependents();
}

}  // namespace

size_t qgemv_dl_partials_floats(int N_out, int K, int epi, int num_sms, int ctas_per_sm) {
  const int n_tg = N_out / 16;
  const int rows = epi == EPI_SILU ? 32 : 16;
  const int grid = dl_grid(num_sms, ctas_per_sm, n_tg, K);
  return std::max(size_t(n_tg) * dl_contrib(n_tg, K, grid) * rows * 32,
                  qgemv_small_partials_floats(N_out, K, epi, num_sms));
}

// at least one (tile group, block) unit per warp of a CTA
bool qgemv_dl_supported(int bits, int gs, nmx_dtype_t dt, int N, int K) {
  return bits == 4 && gs == 64 && dt == NMX_F16 && N % 16 == 0 && K % 128 == 0 &&
         (long long)(N / 16) * (K / 128) >= kWarps;
}

int qgemv_dl_max_m(int K, int epi) {
  const int ng = K / 64;
  const int stages = epi == EPI_SILU ? kStages2 : kStages1, tpt = epi == EPI_SILU ? 2 : 1;
  for (int m = 32; m >= 1; --m) {
    const int ncol = m <= 8 ? 8 : 32;
    const size_t ring = size_t(kWarps) * (stages * tpt * kRec + 16 * tpt * ncol * 4);
    const size_t smem = align_up(size_t(m) * (ng * 32 + 4) * 4, 16) + size_t(ng) * ncol * 8 + ring;
    if (smem <= size_t(kMaxDynSmemDL)) return m;
  }
  return 0;
}

nmx_status_t qgemv_dl(Ctx* c, const GemvDLArgs& a, int epi) {
  NMX_CHECK(a.M > 0 && a.N % 16 == 0 && a.K % 128 == 0 && (long long)(a.N / 16) * (a.K / 128) >= kWarps,
            NMX_ERR_UNSUPPORTED, "qgemv_dl: bad shape");
  // tensor-core GEMMs: decode batches (weights as the MMA rows, K split over
  // the SMs), and prefill row counts
  if (a.gamma == nullptr && a.err != nullptr) {
    if (a.M > kTcsMaxRows && qgemm_tc_supported(a.N, a.K, epi)) return qgemm_tc(c, a, epi);
    if (a.M >= kTcsMinRows && qgemm_tcs_supported(a.M, a.N, a.K, epi) && a.counters &&
        qgemm_tcs_partials_floats(a.M, a.N, a.K, epi, c->num_sms) <= (a.partials ? a.partials_cap : 0))
      return qgemm_tcs(c, a, epi);
    if (a.M >= kGemmMinRows && qgemm_tc_supported(a.N, a.K, epi)) return qgemm_tc(c, a, epi);
  }
  // up to eight rows: the small-batch kernel, in as few launches as its
  // staging allows
  if (a.M <= 8) {
    int mc = a.M;
    while (mc > 0 && !qgemv_small_fits(mc, a.N, a.K, epi, c->num_sms)) --mc;
    if (mc > 0) {
      for (int m0 = 0; m0 < a.M; m0 += mc) {
        GemvDLArgs b = a;
        b.M = std::min(mc, a.M - m0);
        b.x = static_cast<const char*>(a.x) + size_t(m0) * a.ldx * 2;
        if (a.y) b.y = static_cast<char*>(a.y) + size_t(m0) * a.ldy * 2;
        if (a.res) b.res = static_cast<const char*>(a.res) + size_t(m0) * a.ldres * 2;
        if (a.logits_f32) b.logits_f32 = a.logits_f32 + size_t(m0) * a.N;
        if (a.out_ids) b.out_ids = a.out_ids + m0;
        if (a.next_tokens) b.next_tokens = a.next_tokens + m0;
        b.n_tg = a.N / 16;
        NMX_TRY(qgemv_small(c, b, epi));
      }
      return NMX_OK;
    }
  }
  const int mmax = qgemv_dl_max_m(a.K, epi);
  NMX_CHECK(mmax > 0, NMX_ERR_UNSUPPORTED, "qgemv_dl: K too large");
  NMX_CHECK(epi != EPI_ARGMAX || a.M <= mmax, NMX_ERR_UNSUPPORTED, "qgemv_dl: argmax needs one launch");
  for (int m0 = 0; m0 < a.M; m0 += mmax) {
    const int mc = std::min(mmax, a.M - m0);
    GemvDLArgs b = a;
    b.x = static_cast<const char*>(a.x) + size_t(m0) * a.ldx * 2;
    if (a.y) b.y = static_cast<char*>(a.y) + size_t(m0) * a.ldy * 2;
    if (a.res) b.res = static_cast<const char*>(a.res) + size_t(m0) * a.ldres * 2;
    if (a.logits_f32) b.logits_f32 = a.logits_f32 + size_t(m0) * a.N;
    if (a.out_ids) b.out_ids = a.out_ids + m0;
    if (a.next_tokens) b.next_tokens = a.next_tokens + m0;
    b.n_tg = a.N / 16;
    nmx_status_t st;
    if (mc <= 8)
      st = dispatch_dl<1>(c, b, mc, epi);
    else
      st = dispatch_dl<4>(c, b, mc, epi);
    NMX_TRY(st);
  }
  return NMX_OK;
}

nmx_status_t repack_to_records(Ctx* c, const uint32_t* wq, const void* s, const void* b, int rows, int K,
                               long row0, void* rec, int part_mask) {
  if (rows == 0) return NMX_OK;
  NMX_CHECK(rows % 16 == 0 && row0 % 16 == 0 && K % 128 == 0, NMX_ERR_UNSUPPORTED, "repack: shape");
  const long n = long(rows / 16) * (K / 128) * 32;
  const int grid = int(std::min<long>((n + 255) / 256, long(c->num_sms) * 32));
  return launch(c, repack_kernel, dim3(grid), dim3(256), 0, wq, (const half*)s, (const half*)b, K, row0,
                (unsigned char*)rec, part_mask, 0, (uint32_t*)nullptr, (half*)nullptr, (half*)nullptr, rows);
}

nmx_status_t unpack_from_records(Ctx* c, const void* rec, int rows, int K, long row0, uint32_t* wq, void* s,
                                 void* b, int part_mask) {
  if (rows == 0) return NMX_OK;
  NMX_CHECK(rows % 16 == 0 && row0 % 16 == 0 && K % 128 == 0, NMX_ERR_UNSUPPORTED, "unpack: shape");
  const long n = long(rows / 16) * (K / 128) * 32;
  const int grid = int(std::min<long>((n + 255) / 256, long(c->num_sms) * 32));
  return launch(c, repack_kernel, dim3(grid), dim3(256), 0, (const uint32_t*)nullptr, (const half*)nullptr,
                (const half*)nullptr, K, row0, (unsigned char*)const_cast<void*>(rec), part_mask, 1, wq,
                (half*)s, (half*)b, rows);
}

}  // namespace nmx
