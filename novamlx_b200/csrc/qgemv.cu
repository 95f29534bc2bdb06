// Quantized GEMV / skinny GEMM for decode (M <= 32 rows of activations):
//   y[M, N] = epilogue( norm?(x)[M, K] · dequant(W)[N, K]^T )
// over MLX-affine packed weights (u32 words, 4- or 8-bit values low bits
// first; per-group scale and bias along K). Replaces MLX's quantized_matmul
// for the decode shapes reached from QuantizedLinear
// (Sources/NovaMLXEngine/Models/BailingHybridModel.swift:213) and the
// decode-step forward (Sources/NovaMLXEngine/FusedBatchScheduler.swift:1215).
//
// Design (sm_100a):
//  * A warp owns a 16-row tile of W and a contiguous range of K groups; the
//    eight warps of a CTA split K (or, for the gated MLP, pair a gate tile
//    with its up tile). Packed words are read straight from HBM with
//    8-32 B vector loads per lane, 16 rows × 32 B contiguous per instruction.
//  * The legacy tensor-core MMA (mma.sync m16n8k16, f16 in, f32 accumulate)
//    is the dot-product engine: A = dequantised weights, B = activations for
//    up to 8 batch rows per n-tile, so M <= 8 costs the same instructions as
//    M = 1.
//  * Dequant is one LOP3 per two values: a nibble OR'ed into the exponent
//    field of f16 1024.0 is exactly 1024 + q (or 1024 + 16q for the odd
//    nibble of a byte, whose activation is pre-scaled by 1/16). The constant
//    part, Σ offset·x, is precomputed per (column, group) and enters the MMA
//    as its accumulator input, so the MMA returns Σ q·x in fp32; the group's
//    scale and bias are folded after the group: acc += s·Σq·x + b·Σx.
//  * Activations are staged once per CTA in shared memory in the permuted
//    pair order the fragments need, after an optional RMSNorm (prologue
//    fusion), rounded to the activation dtype first as MLX would.
//  * Weights of the first k-batch are requested before griddepcontrol.wait,
//    so under programmatic dependent launch they stream in while the
//    previous kernel finishes.
#include <algorithm>
#include <map>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "kernels.h"
#include "qgemv_common.cuh"

namespace nmx {

namespace {

constexpr int kMaxDynSmem = 210 * 1024;  // dynamic smem ceiling of every qgemv launch

template <typename T>
struct Scale4 {
  T s0, s1, b0, b1;
};

template <typename T, int BITS, int GS, int NT, int EPI, int TPC>
__global__ void __launch_bounds__(kThreads, 2) qgemv_kernel(GemvArgs a, int num_tg) {
  using C = QCfg<BITS, GS>;
  constexpr int KS = kWarps / TPC;
  constexpr int NCOL = NT * 8;
  constexpr int kBatch = C::BATCH;
  extern __shared__ __align__(16) unsigned char smem[];

  const int K = a.K, M = a.M;
  const int ng = K / GS;
  const int wpr = K * BITS / 32;
  const int colstride = ng * 4 * C::MP + 4;  // in f16x2 units, +16 B pad
  uint32_t* xB = reinterpret_cast<uint32_t*>(smem);
  float2* CX = reinterpret_cast<float2*>(smem + ((size_t(M) * colstride * 4 + 15) & ~size_t(15)));
  float* red = reinterpret_cast<float*>(reinterpret_cast<unsigned char*>(CX) +
                                        size_t(ng) * NCOL * sizeof(float2));
  float* lg = red + TPC * KS * 16 * NCOL;  // [16*TPC][NCOL] rounded logits (argmax)
  __shared__ float s_inv[32];
  __shared__ float s_colmul[32];
  __shared__ float s_wsum[kWarps][32];
  __shared__ float s_wmax[kWarps][32];
  __shared__ int s_last;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int tile = warp / KS, ks = warp % KS;
  const int gb = ks * ng / KS, ge = (ks + 1) * ng / KS;

  const uint32_t* __restrict__ W = a.w;
  const T* __restrict__ S = reinterpret_cast<const T*>(a.s);
  const T* __restrict__ Bq = reinterpret_cast<const T*>(a.b);

  // rows of this warp's tile for tile group tg
  auto tile_row = [&](int tg) -> long {
    if constexpr (EPI == EPI_SILU) {
      return (tile == 0 ? 0 : a.pair_off) + long(tg) * 16;
    } else {
      return long(tg) * 16 * TPC + tile * 16;
    }
  };

  WordVec<C::WPT> wa0[kBatch], wa1[kBatch], wb0[kBatch], wb1[kBatch];
  Scale4<T> sa[kBatch], sb[kBatch];
  const uint32_t* w0 = nullptr;
  const T* s0p = nullptr;
  const T* b0p = nullptr;

  auto setup = [&](int tg) {
    const long r0 = tile_row(tg) + g;
    w0 = W + r0 * wpr + t * C::WPT;
    s0p = S + r0 * ng;
    b0p = Bq + r0 * ng;
  };
  auto load_batch = [&](WordVec<C::WPT>* v0, WordVec<C::WPT>* v1, Scale4<T>* sc, int G0) {
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
      const int G = G0 + i;
      if (G < ge) {
        load_words<C::WPT>(v0[i], w0 + G * C::WPG);
        load_words<C::WPT>(v1[i], w0 + 8L * wpr + G * C::WPG);
        sc[i].s0 = s0p[G];
        sc[i].s1 = s0p[8L * ng + G];
        sc[i].b0 = b0p[G];
        sc[i].b1 = b0p[8L * ng + G];
      }
    }
  };

  float acc[NT][4];
  auto compute_batch = [&](WordVec<C::WPT>* v0, WordVec<C::WPT>* v1, Scale4<T>* sc, int G0) {
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
      const int G = G0 + i;
      if (G < ge) {
        uint32_t P0[C::MP], P1[C::MP];
#pragma unroll
        for (int j = 0; j < C::WPT; ++j) {
          dequant_word<BITS>(v0[i].v[j], P0 + j * (BITS == 4 ? 4 : 2));
          dequant_word<BITS>(v1[i].v[j], P1 + j * (BITS == 4 ? 4 : 2));
        }
        const float fs0 = tof<T>(sc[i].s0), fs1 = tof<T>(sc[i].s1);
        const float fb0 = tof<T>(sc[i].b0), fb1 = tof<T>(sc[i].b1);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          int col = nt * 8 + g;
          col = col < M ? col : M - 1;
          const uint32_t* xb = xB + size_t(col) * colstride + (G * 4 + t) * C::MP;
          uint32_t bf[C::MP];
#pragma unroll
          for (int p = 0; p < C::MP; p += 4) {
            uint4 u = *reinterpret_cast<const uint4*>(xb + p);
            bf[p] = u.x; bf[p + 1] = u.y; bf[p + 2] = u.z; bf[p + 3] = u.w;
          }
          const float4 cx = *reinterpret_cast<const float4*>(CX + size_t(G) * NCOL + nt * 8 + 2 * t);
          float d[4] = {cx.x, cx.z, cx.x, cx.z};  // -C of columns 2t, 2t+1
#pragma unroll
          for (int u = 0; u < C::NMMA; ++u) {
            mma16816(d, P0[2 * u], P1[2 * u], P0[2 * u + 1], P1[2 * u + 1], bf[2 * u],
                     bf[2 * u + 1], d[0], d[1], d[2], d[3]);
          }
          float m0 = 1.f, m1 = 1.f;
          if constexpr (!std::is_same<T, half>::value) {
            m0 = s_colmul[min(nt * 8 + 2 * t, 31)];
            m1 = s_colmul[min(nt * 8 + 2 * t + 1, 31)];
          }
          acc[nt][0] = fmaf(fs0 * m0, d[0], fmaf(fb0, cx.y, acc[nt][0]));
          acc[nt][1] = fmaf(fs0 * m1, d[1], fmaf(fb0, cx.w, acc[nt][1]));
          acc[nt][2] = fmaf(fs1 * m0, d[2], fmaf(fb1, cx.y, acc[nt][2]));
          acc[nt][3] = fmaf(fs1 * m1, d[3], fmaf(fb1, cx.w, acc[nt][3]));
        }
      }
    }
  };

  int tg = blockIdx.x;
  const bool early = a.weights_static;
  if (early && tg < num_tg) {
    setup(tg);
    load_batch(wa0, wa1, sa, gb);
  }

  // ---------------------------------------------------------------- prologue
  grid_wait();
  {
    const T* X = reinterpret_cast<const T* __restrict__>(a.x);
    const T* Gm = reinterpret_cast<const T* __restrict__>(a.gamma);
    // pass A: per-column inverse RMS (M <= 32)
    if (Gm) {
      for (int c = 0; c < M; ++c) {
        float ss = 0.f;
        for (int k = tid; k < K; k += kThreads) {
          const float v = tof<T>(X[long(c) * a.ldx + k]);
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
    } else if (tid < M) {
      s_inv[tid] = 1.0f;
    }
    if (tid < 32) s_colmul[tid] = 1.0f;
    __syncthreads();
    if constexpr (!std::is_same<T, half>::value) {
      // pass B (bf16 only): the MMA operand is f16, so scale each column by a
      // power of two that keeps max|x| <= 2^14; the fold multiplies it back.
      for (int c = 0; c < M; ++c) {
        float mx = 0.f;
        for (int k = tid; k < K; k += kThreads) {
          float v = tof<T>(X[long(c) * a.ldx + k]);
          if (Gm) v = rnd<T>(v * s_inv[c] * tof<T>(Gm[k]));
          mx = fmaxf(mx, fabsf(v));
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if (lane == 0) s_wmax[warp][c] = mx;
      }
      __syncthreads();
      if (tid < M) {
        float mx = 0.f;
        for (int w = 0; w < kWarps; ++w) mx = fmaxf(mx, s_wmax[w][tid]);
        float mul = 1.f;
        while (mx / mul > 16384.f) mul *= 2.f;
        s_colmul[tid] = mul;
      }
      __syncthreads();
    }
    // pass C: permuted, pre-scaled f16 pairs and per-(column, group) sums.
    // The MMA sees A = 1024 + q (low nibble / byte) against B = x, or
    // A = 1024 + 16q (high nibble) against B = x/16; either way the constant
    // part of A·B is 1024·B, so C = 1024·ΣB and D - C = Σ q·x.
    const int items = M * ng * 4;
    for (int it = tid; it < items; it += kThreads) {
      const int c = it / (ng * 4);
      const int rem = it - c * (ng * 4);
      const int G = rem >> 2, tt = rem & 3;
      const float inv = s_inv[c];
      const float cm = 1.0f / s_colmul[c];
      const T* xr = X + long(c) * a.ldx + G * GS;
      const T* gr = Gm ? Gm + G * GS : nullptr;
      float bsum = 0.f, xsum = 0.f;
      uint32_t* dst = xB + size_t(c) * colstride + (G * 4 + tt) * C::MP;
#pragma unroll 4
      for (int p = 0; p < C::MP; ++p) {
        int k0, k1;
        bool hi;
        pair_k<BITS, GS>(tt, p, k0, k1, hi);
        float x0 = tof<T>(xr[k0]), x1 = tof<T>(xr[k1]);
        if (gr) {
          x0 = rnd<T>(x0 * inv * tof<T>(gr[k0]));
          x1 = rnd<T>(x1 * inv * tof<T>(gr[k1]));
        }
        xsum += x0 + x1;
        const float f = (hi ? 0.0625f : 1.0f) * cm;
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

  float best_v = -INFINITY;
  int best_i = 0x7fffffff;

  for (; tg < num_tg; tg += gridDim.x) {
    if (!early || tg != int(blockIdx.x)) {
      setup(tg);
      load_batch(wa0, wa1, sa, gb);
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;

    for (int G0 = gb; G0 < ge; G0 += 2 * kBatch) {
      if (G0 + kBatch < ge) load_batch(wb0, wb1, sb, G0 + kBatch);
      compute_batch(wa0, wa1, sa, G0);
      if (G0 + kBatch < ge) {
        if (G0 + 2 * kBatch < ge) load_batch(wa0, wa1, sa, G0 + 2 * kBatch);
        compute_batch(wb0, wb1, sb, G0 + kBatch);
      }
    }

    // cross-warp (k-split) reduction through shared memory
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      float* r = red + ((tile * KS + ks) * 16) * NCOL + nt * 8 + 2 * t;
      r[g * NCOL] = acc[nt][0];
      r[g * NCOL + 1] = acc[nt][1];
      r[(g + 8) * NCOL] = acc[nt][2];
      r[(g + 8) * NCOL + 1] = acc[nt][3];
    }
    __syncthreads();

    constexpr int OUT_ROWS = (EPI == EPI_SILU) ? 16 : 16 * TPC;
    const long n_base = long(tg) * OUT_ROWS;
    T* Y = reinterpret_cast<T*>(a.y);
    for (int e = tid; e < OUT_ROWS * M; e += kThreads) {
      const int r = e % OUT_ROWS, m = e / OUT_ROWS;
      const long n = n_base + r;
      if constexpr (EPI == EPI_SILU) {
        float vg = 0.f, vu = 0.f;
#pragma unroll
        for (int k2 = 0; k2 < KS; ++k2) {
          vg += red[((0 * KS + k2) * 16 + r) * NCOL + m];
          vu += red[((1 * KS + k2) * 16 + r) * NCOL + m];
        }
        const float g16 = rnd<T>(vg), u16 = rnd<T>(vu);
        const float act = rnd<T>(g16 / (1.0f + expf(-g16)));
        Y[long(m) * a.ldy + n] = fromf<T>(act * u16);
      } else {
        const int tl = r / 16, rr = r % 16;
        float v = 0.f;
#pragma unroll
        for (int k2 = 0; k2 < KS; ++k2) v += red[((tl * KS + k2) * 16 + rr) * NCOL + m];
        v = rnd<T>(v);
        if (a.bias) v = rnd<T>(v + tof<T>(reinterpret_cast<const T*>(a.bias)[n]));
        if constexpr (EPI == EPI_RESID) {
          v = v + tof<T>(reinterpret_cast<const T*>(a.res)[long(m) * a.ldres + n]);
          Y[long(m) * a.ldy + n] = fromf<T>(v);
        } else if constexpr (EPI == EPI_STORE) {
          Y[long(m) * a.ldy + n] = fromf<T>(v);
        } else {  // EPI_ARGMAX: keep the rounded logit for the scan below
          if (a.logits) reinterpret_cast<T*>(a.logits)[long(m) * a.N + n] = fromf<T>(v);
          if (a.logits_f32) a.logits_f32[long(m) * a.N + n] = v;
          lg[r * NCOL + m] = v;
        }
      }
    }
    if constexpr (EPI == EPI_ARGMAX) {
      __syncthreads();
      if (tid < M) {
        for (int r = 0; r < OUT_ROWS; ++r) {
          const float v = lg[r * NCOL + tid];
          const int idx = int(n_base + r);
          if (v > best_v || (v == best_v && idx < best_i)) {
            best_v = v;
            best_i = idx;
          }
        }
      }
    }
    __syncthreads();
  }

  if constexpr (EPI == EPI_ARGMAX) {
    if (tid < M) {
      a.part_val[long(tid) * gridDim.x + blockIdx.x] = best_v;
      a.part_idx[long(tid) * gridDim.x + blockIdx.x] = best_i;
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
      const unsigned ticket = atomicAdd(a.counter, 1u);
      s_last = (ticket == gridDim.x - 1) ? 1 : 0;
    }
    __syncthreads();
    if (s_last) {
      __threadfence();
      for (int m = 0; m < M; ++m) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int i = tid; i < int(gridDim.x); i += kThreads) {
          const float v = __ldcg(a.part_val + long(m) * gridDim.x + i);
          const int ix = __ldcg(a.part_idx + long(m) * gridDim.x + i);
          if (v > bv || (v == bv && ix < bi)) {
            bv = v;
            bi = ix;
          }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
          const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
          if (ov > bv || (ov == bv && oi < bi)) {
            bv = ov;
            bi = oi;
          }
        }
        if (lane == 0) {
          s_wsum[warp][0] = bv;
          reinterpret_cast<int*>(s_wmax[warp])[0] = bi;
        }
        __syncthreads();
        if (tid == 0) {
          for (int w = 1; w < kWarps; ++w) {
            const float ov = s_wsum[w][0];
            const int oi = reinterpret_cast<int*>(s_wmax[w])[0];
            if (ov > bv || (ov == bv && oi < bi)) {
              bv = ov;
              bi = oi;
            }
          }
          if (bi == 0x7fffffff) bi = 0;  // all NaN: id 0
          a.out_ids[m] = bi;
          if (a.next_tokens) a.next_tokens[m] = bi;
        }
        __syncthreads();
      }
      if (tid == 0) *a.counter = 0u;
    }
  }
}

struct KernelInfo {
  int max_ctas_per_sm = 1;
};

template <typename T, int BITS, int GS, int NT, int EPI, int TPC>
nmx_status_t launch_one(Ctx* c, const GemvArgs& a, int M) {
  using C = QCfg<BITS, GS>;
  constexpr int NCOL = NT * 8;
  constexpr int KS = kWarps / TPC;
  const int ng = a.K / GS;
  const int colstride = ng * 4 * C::MP + 4;
  const size_t smem = align_up(size_t(M) * colstride * 4, 16) + size_t(ng) * NCOL * sizeof(float2) +
                      size_t(TPC * KS * 16 * NCOL + 16 * TPC * NCOL) * sizeof(float);
  auto kern = qgemv_kernel<T, BITS, GS, NT, EPI, TPC>;
  static std::mutex mu;
  static std::map<int, bool> attr_set;                // device → max smem attribute raised
  static std::map<std::pair<int, size_t>, int> occ;  // (device, smem) → CTAs per SM
  int per_sm = 0;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (!attr_set[c->device]) {
      // raise the kernel's limit once to the largest size any launch uses
      NMX_CUDA_OK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxDynSmem));
      attr_set[c->device] = true;
    }
    auto key = std::make_pair(c->device, smem);
    auto itr = occ.find(key);
    if (itr == occ.end()) {
      NMX_CUDA_OK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem));
      occ[key] = per_sm;
    } else {
      per_sm = itr->second;
    }
  }
  NMX_CHECK(smem <= size_t(kMaxDynSmem), NMX_ERR_UNSUPPORTED, "qgemv: shared-memory staging too large");
  NMX_CHECK(per_sm > 0, NMX_ERR_UNSUPPORTED, "qgemv: configuration does not fit on an SM");
  const int rows_per_tg = (EPI == EPI_SILU) ? 16 : 16 * TPC;
  const int num_tg = a.N / rows_per_tg;
  int grid = std::min(num_tg, per_sm * c->num_sms);
  if (EPI == EPI_ARGMAX) grid = std::min(grid, kArgmaxMaxGridPerSm * c->num_sms);
  GemvArgs b = a;
  b.M = M;
  return launch(c, kern, dim3(grid), dim3(kThreads), smem, b, num_tg);
}

// ---------------------------------------------------------------------------
// Few-row fast path (M <= 8, 4-bit, f16, plain store): the operator-level
// quantized matmul of a handful of rows (the engine's QuantizedLinear call on
// a short prompt, MLX.quantizedMM in BailingHybridModel.swift:213).
//
// A CTA owns one 16-row tile; its eight warps take the tile's 128-k steps
// round-robin, so there is no CTA-wide activation prologue: each lane loads
// the 16 bytes of packed weights of rows g and g+8 it needs per step (words
// 4t..4t+3, k = 32t .. 32t+31 of the step), its two rows' group scale and
// bias, and 64 bytes of activation row g straight into registers, with the
// next step's loads in flight while it computes. Weights are dequantised to
// f16 (q exact, then w = q·s + b rounded once, as MLX's own large-row kernel
// stages them) and fed to mma.sync m16n8k16; the MMA's k order is a
// permutation of the step's 128 k that both operands share: lane t's pair
// (q_i, q_{i+4}) of word j meets activations (x_{8j+i}, x_{8j+i+4}). The
// eight warps' fp32 tiles are summed in warp order through shared memory.
constexpr int kMlxWarps = 8;

__device__ __forceinline__ uint32_t hsub2_u(uint32_t a, uint32_t b) {
  __half2 r = __hsub2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}
__device__ __forceinline__ uint32_t hfma2_u(uint32_t a, __half2 s, __half2 b) {
  __half2 r = __hfma2(*reinterpret_cast<__half2*>(&a), s, b);
  return *reinterpret_cast<uint32_t*>(&r);
}

template <int GS>
__global__ void __launch_bounds__(kMlxWarps * 32, 2) qgemv_mlx4_small_kernel(GemvArgs a) {
  __shared__ float red[kMlxWarps][16][8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int K = a.K, M = a.M, wpr = K / 8, ng = K / GS, steps = K / 128;
  const long r0 = long(blockIdx.x) * 16 + g;
  const uint32_t* w0 = a.w + r0 * wpr + 4 * t;
  const uint32_t* w1 = w0 + 8L * wpr;
  const half* S = static_cast<const half*>(a.s);
  const half* B = static_cast<const half*>(a.b);
  const half* X = static_cast<const half*>(a.x) + long(g < M ? g : 0) * a.ldx + 32 * t;
  const bool has_col = g < M;

  struct Step {
    uint4 wa, wb;      // rows g, g+8: 32 nibbles each
    half sa, ba, sb, bb;
    uint4 x[4];        // x[g][32t .. 32t+31] of the step
  };
  auto load = [&](Step& st, int k) {
    st.wa = *reinterpret_cast<const uint4*>(w0 + k * 16);
    st.wb = *reinterpret_cast<const uint4*>(w1 + k * 16);
    const int G = (k * 128 + 32 * t) / GS;
    st.sa = S[r0 * ng + G];
    st.ba = B[r0 * ng + G];
    st.sb = S[(r0 + 8) * ng + G];
    st.bb = B[(r0 + 8) * ng + G];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      st.x[i] = has_col ? reinterpret_cast<const uint4*>(X + k * 128)[i] : make_uint4(0, 0, 0, 0);
  };
  float d[4] = {0.f, 0.f, 0.f, 0.f};
  auto compute = [&](const Step& st) {
    const uint32_t magic = 0x64006400u;  // f16 1024.0 in both halves
    const __half2 sa2 = __halves2half2(st.sa, st.sa), ba2 = __halves2half2(st.ba, st.ba);
    const __half2 sb2 = __halves2half2(st.sb, st.sb), bb2 = __halves2half2(st.bb, st.bb);
    const uint32_t wa[4] = {st.wa.x, st.wa.y, st.wa.z, st.wa.w};
    const uint32_t wb[4] = {st.wb.x, st.wb.y, st.wb.z, st.wb.w};
    const uint32_t xs[16] = {st.x[0].x, st.x[0].y, st.x[0].z, st.x[0].w, st.x[1].x, st.x[1].y, st.x[1].z, st.x[1].w,
                             st.x[2].x, st.x[2].y, st.x[2].z, st.x[2].w, st.x[3].x, st.x[3].y, st.x[3].z, st.x[3].w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      // word j of each row: pairs (q_i, q_{i+4}), i = 0..3, as f16 weights
      uint32_t A[4], Bw[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        A[i] = hfma2_u(hsub2_u(and_or(wa[j] >> (4 * i), 0x000F000Fu, magic), magic), sa2, ba2);
        Bw[i] = hfma2_u(hsub2_u(and_or(wb[j] >> (4 * i), 0x000F000Fu, magic), magic), sb2, bb2);
      }
      // activations k = 8j .. 8j+7 of the lane's 32: pairs (x_i, x_{i+4})
      const uint32_t X0 = xs[4 * j], X1 = xs[4 * j + 1], X2 = xs[4 * j + 2], X3 = xs[4 * j + 3];
      const uint32_t p0 = __byte_perm(X0, X2, 0x5410), p1 = __byte_perm(X0, X2, 0x7632);
      const uint32_t p2 = __byte_perm(X1, X3, 0x5410), p3 = __byte_perm(X1, X3, 0x7632);
      // two k16 steps: (pairs 0, 1) and (pairs 2, 3)
      mma16816(d, A[0], Bw[0], A[1], Bw[1], p0, p1, d[0], d[1], d[2], d[3]);
      mma16816(d, A[2], Bw[2], A[3], Bw[3], p2, p3, d[0], d[1], d[2], d[3]);
    }
  };
  grid_wait();
  Step cur, nxt;
  int k = warp;
  if (k < steps) load(cur, k);
  for (; k < steps; k += kMlxWarps) {
    if (k + kMlxWarps < steps) load(nxt, k + kMlxWarps);
    compute(cur);
    cur = nxt;
  }
  grid_launch_dependents();
  red[warp][g][2 * t] = d[0];
  red[warp][g][2 * t + 1] = d[1];
  red[warp][g + 8][2 * t] = d[2];
  red[warp][g + 8][2 * t + 1] = d[3];
  __syncthreads();
  for (int e = threadIdx.x; e < 16 * M; e += kMlxWarps * 32) {
    const int r = e % 16, m = e / 16;
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kMlxWarps; ++w) v += red[w][r][m];
    static_cast<half*>(a.y)[long(m) * a.ldy + long(blockIdx.x) * 16 + r] = __float2half_rn(v);
  }
}

bool mlx4_small_ok(const GemvArgs& a, int bits, int gs, nmx_dtype_t dt, int epi) {
  return bits == 4 && (gs == 32 || gs == 64 || gs == 128) && dt == NMX_F16 && epi == EPI_STORE &&
         a.M >= 1 && a.M <= 8 && a.gamma == nullptr && a.bias == nullptr && a.K % 128 == 0 && a.N % 16 == 0 &&
         reinterpret_cast<uintptr_t>(a.x) % 16 == 0 && (a.ldx * 2) % 16 == 0 &&
         reinterpret_cast<uintptr_t>(a.w) % 16 == 0;
}

nmx_status_t launch_mlx4_small(Ctx* c, const GemvArgs& a, int gs) {
  const dim3 grid(a.N / 16), block(kMlxWarps * 32);
  if (gs == 64) return launch(c, qgemv_mlx4_small_kernel<64>, grid, block, 0, a);
  if (gs == 32) return launch(c, qgemv_mlx4_small_kernel<32>, grid, block, 0, a);
  return launch(c, qgemv_mlx4_small_kernel<128>, grid, block, 0, a);
}

template <typename T, int BITS, int GS>
nmx_status_t dispatch_nt(Ctx* c, const GemvArgs& a, int M, int epi) {
  if (M <= 8) {
    switch (epi) {
      case EPI_STORE: return launch_one<T, BITS, GS, 1, EPI_STORE, 1>(c, a, M);
      case EPI_RESID: return launch_one<T, BITS, GS, 1, EPI_RESID, 1>(c, a, M);
      case EPI_SILU: return launch_one<T, BITS, GS, 1, EPI_SILU, 2>(c, a, M);
      case EPI_ARGMAX: return launch_one<T, BITS, GS, 1, EPI_ARGMAX, 1>(c, a, M);
    }
  } else {
    switch (epi) {
      case EPI_STORE: return launch_one<T, BITS, GS, 4, EPI_STORE, 1>(c, a, M);
      case EPI_RESID: return launch_one<T, BITS, GS, 4, EPI_RESID, 1>(c, a, M);
      case EPI_SILU: return launch_one<T, BITS, GS, 4, EPI_SILU, 2>(c, a, M);
      case EPI_ARGMAX: return launch_one<T, BITS, GS, 4, EPI_ARGMAX, 1>(c, a, M);
    }
  }
  NMX_CHECK(false, NMX_ERR_UNSUPPORTED, "qgemv: unknown epilogue");
}

template <typename T>
nmx_status_t dispatch_bits(Ctx* c, const GemvArgs& a, int M, int bits, int gs, int epi) {
  if (bits == 4) {
    if (gs == 64) return dispatch_nt<T, 4, 64>(c, a, M, epi);
    if (gs == 32) return dispatch_nt<T, 4, 32>(c, a, M, epi);
    if (gs == 128) return dispatch_nt<T, 4, 128>(c, a, M, epi);
  } else if (bits == 8) {
    if (gs == 64) return dispatch_nt<T, 8, 64>(c, a, M, epi);
    if (gs == 32) return dispatch_nt<T, 8, 32>(c, a, M, epi);
    if (gs == 128) return dispatch_nt<T, 8, 128>(c, a, M, epi);
  }
  NMX_CHECK(false, NMX_ERR_UNSUPPORTED, "qgemv: bits must be 4 or 8 and group 32, 64 or 128");
}

}  // namespace

int qgemv_max_m(int K, int gs) {
  const size_t budget = 200 * 1024;
  const int ng = K / gs;
  const size_t fixed = size_t(ng) * 32 * sizeof(float2) + size_t(kWarps + 2) * 16 * 32 * sizeof(float) + 64;
  if (fixed >= budget) return 0;
  const size_t per_col = size_t(ng) * gs * 2 + 16;
  int m = int((budget - fixed) / per_col);
  return std::min(m, 32);
}

nmx_status_t qgemv(Ctx* c, const GemvArgs& a, int bits, int gs, nmx_dtype_t dt, int epi) {
  NMX_CHECK(a.M > 0 && a.N > 0 && a.K > 0, NMX_ERR_INVALID, "qgemv: empty shape");
  NMX_CHECK(a.N % 16 == 0, NMX_ERR_UNSUPPORTED, "qgemv: N must be a multiple of 16");
  NMX_CHECK(a.K % gs == 0, NMX_ERR_UNSUPPORTED, "qgemv: K must be a multiple of the group size");
  NMX_CHECK(((a.K * bits / 32) % 4) == 0, NMX_ERR_UNSUPPORTED, "qgemv: packed row must be 16-byte aligned");
  NMX_CHECK(dt == NMX_F16 || dt == NMX_BF16, NMX_ERR_UNSUPPORTED, "qgemv: dtype must be f16 or bf16");
  const int mmax = qgemv_max_m(a.K, gs);
  NMX_CHECK(mmax > 0, NMX_ERR_UNSUPPORTED, "qgemv: K too large for shared-memory staging");
  NMX_CHECK(epi != EPI_ARGMAX || a.M <= std::min(mmax, 32), NMX_ERR_UNSUPPORTED,
            "qgemv: argmax epilogue needs all rows in one launch");
  if (mlx4_small_ok(a, bits, gs, dt, epi)) return launch_mlx4_small(c, a, gs);
  const size_t esz = 2;
  for (int m0 = 0; m0 < a.M; m0 += mmax) {
    const int mc = std::min(mmax, a.M - m0);
    GemvArgs b = a;
    b.x = static_cast<const char*>(a.x) + size_t(m0) * a.ldx * esz;
    b.y = static_cast<char*>(a.y) + size_t(m0) * a.ldy * esz;
    if (a.res) b.res = static_cast<const char*>(a.res) + size_t(m0) * a.ldres * esz;
    nmx_status_t st = (dt == NMX_F16) ? dispatch_bits<half>(c, b, mc, bits, gs, epi)
                                      : dispatch_bits<__nv_bfloat16>(c, b, mc, bits, gs, epi);
    if (st != NMX_OK) return st;
  }
  return NMX_OK;
}

}  // namespace nmx
