// Prefill GEMM on the 5th-generation tensor cores: y[M, N] = x[M, K] ·
// dequant(W)[N, K]ᵀ with W in decode records (4-bit, group 64) and the
// GEMV epilogues (store + bias, + residual, SiLU(gate)·up).
//
// One CTA computes a 128 × 256 tile of the product (for SiLU·up: 128 rows
// of gate and the matching 128 rows of up, one 128-column output tile) over
// K in steps of 64 (one quantization group), through a ring of 3 shared
// stages of {x tile 128 × 64, weight tile 256 × 64} f16, both K-major in the
// 128-byte swizzle:
//   * warp 9 loads the x tile with a TMA tensor copy (box 64 × 128,
//     SWIZZLE_128B; rows past M read as zeros);
//   * warp 10 brings the 16 records of each 128-k block of the weight tile
//     into a ring of 3 raw slots with two 3-d tensor copies of 8 records
//     (mbarrier tx count);
//   * warps 0-7 dequantize the weight tile from the raw records into the
//     same swizzled layout: w = s·q + b rounded to f16 (the precision
//     MLX's own large-M kernel stages its weights in), with the nibble-to-
//     f16 trick (q | 0x6400 = 1024 + q, minus 1024 exactly) and one f16 FMA;
//   * one thread of warp 8 issues tcgen05.mma (kind::f16, M = 128, N = 256,
//     f32 accumulator in 256 TMEM columns) four times per stage and commits
//     each stage back to its producers through an mbarrier;
//   * after the last stage warps 0-7 read TMEM with tcgen05.ld (32x32b;
//     warp w: lanes 32 (w % 4) .. +31, half the columns) and run the
//     epilogue, one output row per thread.
// All mbarrier waits are bounded; a wait that runs out sets bit 0 of *err
// and the CTA skips ahead to its teardown (TMEM is always released).
#include <map>
#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "tc_common.cuh"

namespace nmx {

namespace {

constexpr int kTM = 128;          // rows of x per MMA (MMA M); a CTA takes MT such sub-tiles
constexpr int kTN = 256;          // MMA N: weight rows per CTA
constexpr int kTK = 64;           // k per stage (one group)
constexpr int kRS = 3;            // raw record slots (one 128-k block of the 16 tiles each)
constexpr int kABytes = kTM * kTK * 2;   // 16 KB per x sub-tile
constexpr int kBBytes = kTN * kTK * 2;   // 32 KB
// stage: MT x sub-tiles, then the dequantized weight tile; 3 stages for one
// sub-tile, 2 for two (the shared-memory budget)
template <int MT>
struct TcStages {
  static constexpr int kTS = MT == 1 ? 3 : 2;
  static constexpr int kStageBytes = MT * kABytes + kBBytes;
  static constexpr size_t kSmem = size_t(kTS) * kStageBytes + size_t(kRS) * (16 * tc::kRecPad) + 1024;
};
constexpr int kDW = 8;            // dequant / epilogue warps (one weight row per thread)
constexpr int kGThreads = (kDW + 3) * 32;  // + MMA, x-tile and record-loader warps
constexpr int kWMma = kDW, kWTma = kDW + 1, kWRec = kDW + 2;
constexpr int kRawBytes = 16 * tc::kRecPad;  // the 16 records of one block of the weight tile (two boxes of 8)
constexpr int kRecG = tc::kRecG;
constexpr uint32_t kIDesc = tc::idesc_f16(kTM, kTN);
using tc::mbar_init;
using tc::mbar_arrive;
using tc::mbar_expect_tx;
using tc::mbar_wait;
using tc::sa_;
using tc::smem_desc;
using tc::mma_commit;
using tc::tc_fence_after;
using tc::tc_fence_before;
using tc::tmem_ld32;
__device__ __forceinline__ void mma_f16_tc(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  tc::mma_f16(tmem_d, adesc, bdesc, kIDesc, accumulate);
}

struct GemmArgs {
  const unsigned char* w;   // decode records of the whole matrix
  int M, N_out, K;          // N_out = output columns (gate rows for SiLU)
  long long pair_tiles;     // SiLU: tile offset of the up rows
  const half* bias;
  half* y;
  long ldy;
  const half* res;
  long ldres;
  unsigned* err;
};

template <int EPI, int MT>
__global__ void __launch_bounds__(kGThreads, 1) qgemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_x,
                                                                 const __grid_constant__ CUtensorMap tmap_w,
                                                                 GemmArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // 1024-byte aligned, derived from the shared array itself so that its
  // loads and stores compile to shared-memory (not generic) accesses
  unsigned char* smem = smem_raw + ((1024u - (tc::sa_(smem_raw) & 1023u)) & 1023u);
  constexpr int kTS = TcStages<MT>::kTS, kStageBytes = TcStages<MT>::kStageBytes;
  __shared__ __align__(8) uint64_t full[kTS];
  __shared__ __align__(8) uint64_t empty[kTS];
  __shared__ __align__(8) uint64_t acc_bar;
  __shared__ __align__(8) uint64_t raw_full[kRS];
  __shared__ __align__(8) uint64_t raw_empty[kRS];
  __shared__ uint32_t s_taddr;
  __shared__ int s_fail;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const unsigned lim = wait_polls(a.err);  // polls before a pipeline wait gives up
  const int m0 = blockIdx.x * kTM * MT;
  const int nt = blockIdx.y;  // output tile
  const int KT = a.K / kTK, nb = a.K / 128;

  if (tid == 0) {
    for (int s = 0; s < kTS; ++s) {
      mbar_init(&full[s], 1 + kDW);  // TMA thread (expect_tx) + one arrival per dequant warp
      mbar_init(&empty[s], 1);       // tcgen05.commit
    }
    mbar_init(&acc_bar, 1);
    for (int s = 0; s < kRS; ++s) {
      mbar_init(&raw_full[s], 1);      // record loader (expect_tx)
      mbar_init(&raw_empty[s], kDW);  // the dequant warps, after the block's second stage
    }
    s_fail = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kWMma) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(sa_(&s_taddr)),
                 "r"(kTN * MT)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t taddr = s_taddr;
  grid_wait();  // x (and the residual) come from the previous kernel

  unsigned char* raw = smem + kTS * kStageBytes;
  if (warp == kWRec) {
    // ------------------------------------------- bulk copies: raw record blocks
    if (lane == 0) {
      for (int b = 0; b < nb; ++b) {
        const int rs = b % kRS;
        if (b >= kRS && !mbar_wait(&raw_empty[rs], ((b / kRS) - 1) & 1, lim)) {
          atomicOr(a.err, kErrPipeWait);
          s_fail = 1;
          break;
        }
        mbar_expect_tx(&raw_full[rs], kRawBytes);
        // two tensor copies of 8 consecutive 16-row tiles each
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          long long T0;
          if constexpr (EPI == EPI_SILU)
            T0 = h == 0 ? (long long)nt * 8 : a.pair_tiles + (long long)nt * 8;
          else
            T0 = (long long)nt * 16 + 8 * h;
          tc::load_records(raw + rs * kRawBytes + h * 8 * tc::kRecPad, &tmap_w, b, int(T0), &raw_full[rs]);
        }
      }
    }
  } else if (warp == kWTma) {
    // ---------------------------------------------------------------- TMA: x tiles
    if (lane == 0) {
      for (int kt = 0; kt < KT; ++kt) {
        const int s = kt % kTS;
        if (kt >= kTS && !mbar_wait(&empty[s], ((kt / kTS) - 1) & 1, lim)) {
          atomicOr(a.err, kErrPipeWait);
          s_fail = 1;
          break;
        }
        unsigned char* dst = smem + s * kStageBytes;
        mbar_expect_tx(&full[s], MT * kABytes);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
          asm volatile(
              "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
              "[%4];" ::"r"(sa_(dst + mt * kABytes)),
              "l"(&tmap_x), "r"(kt * kTK), "r"(m0 + mt * kTM), "r"(sa_(&full[s]))
              : "memory");
      }
    }
  } else if (warp == kWMma) {
    // ---------------------------------------------------------------- MMA issue
    if (lane == 0) {
      // one thread issues every MMA: descriptors are computed once and
      // advanced with adds (start addresses in 16-byte units)
      const uint64_t desc0 = smem_desc(smem);
      constexpr uint32_t kStageD = kStageBytes >> 4, kAD = kABytes >> 4;
      for (int kt = 0; kt < KT; ++kt) {
        const int s = kt % kTS;
        if (!mbar_wait(&full[s], (kt / kTS) & 1, lim)) {
          atomicOr(a.err, kErrPipeWait);
          s_fail = 1;
          break;
        }
        tc_fence_after();
        const uint64_t ad = desc0 + uint64_t(s * kStageD), bd = ad + MT * kAD;
        const uint32_t first = kt ? 1u : 0u;
        // the dequantized weight stage serves every x sub-tile
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
          for (int k16 = 0; k16 < kTK / 16; ++k16)
            mma_f16_tc(taddr + uint32_t(mt * kTN), ad + mt * kAD + 2 * k16, bd + 2 * k16, k16 ? 1u : first);
        mma_commit(&empty[s]);
      }
      mma_commit(&acc_bar);
    }
  } else {
    // ----------------------------------------- dequant warps: weight tile rows
    for (int kt = 0; kt < KT; ++kt) {
      const int s = kt % kTS;
      unsigned char* B = smem + s * kStageBytes + MT * kABytes;
      const int blk = kt >> 1, gi = kt & 1, rs = blk % kRS;
      // waits agreed over the warp: its lanes arrive together (warp_arrive)
      bool ok = kt < kTS || mbar_wait(&empty[s], ((kt / kTS) - 1) & 1, lim);
      ok = ok && (gi != 0 || mbar_wait(&raw_full[rs], (blk / kRS) & 1, lim));
      if (!__all_sync(0xffffffffu, ok)) {
        atomicOr(a.err, kErrPipeWait);
        s_fail = 1;
        break;
      }
      const unsigned char* rawb = raw + rs * kRawBytes;
      // warp w fills record halves 4w .. 4w+3 (8 tile rows each): lane 4g+t
      // reads its 16 bytes of the half (words 2t, 2t+1 of both groups of row
      // g: one conflict-free 512-byte sweep per warp) and writes chunks 2t,
      // 2t+1 of tile row 8·(half index) + g (conflict-free in the swizzle)
      {
        const int g = lane >> 2, t = lane & 3;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int hh = warp * 4 + j;  // record hh / 2, rows 8·(hh % 2) ..
          const unsigned char* rec = rawb + (hh >> 1) * tc::kRecPad;
          const int hf = hh & 1;
          const uint4 wv = *reinterpret_cast<const uint4*>(rec + hf * 512 + 16 * lane);
          const __half sc = *reinterpret_cast<const __half*>(rec + 1024 + ((0 * 2 + gi) * 8 + g) * 4 + hf * 2);
          const __half bi = *reinterpret_cast<const __half*>(rec + 1024 + ((1 * 2 + gi) * 8 + g) * 4 + hf * 2);
          const __half2 s2 = __halves2half2(sc, sc);
          const __half2 s16 = __hmul2(s2, __float2half2_rn(0.0625f));
          const __half2 b2 = __halves2half2(bi, bi);
          const int row = hh * 8 + g;
          const uint32_t w0 = gi ? wv.z : wv.x, w1 = gi ? wv.w : wv.y;
          *reinterpret_cast<uint4*>(B + tc::sw128(row, 2 * t)) = tc::dequant_word_chunk(w0, s2, s16, b2);
          *reinterpret_cast<uint4*>(B + tc::sw128(row, 2 * t + 1)) = tc::dequant_word_chunk(w1, s2, s16, b2);
        }
      }
      // generic-proxy writes, read by the tensor core's async proxy
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tc::warp_arrive(&full[s]);
      if (gi == 1) tc::warp_arrive(&raw_empty[rs]);  // the block's records are read
    }

    // ------------------------------------------------------------ epilogue
    if (!s_fail && !mbar_wait(&acc_bar, 0, lim)) {
      atomicOr(a.err, kErrPipeWait);
      s_fail = 1;
    }
    tc_fence_after();
    // warp w reads TMEM lanes 32 (w % 4) .. +31 (its rows) and half the columns
    const int quad = warp & 3, chalf = warp >> 2;
    constexpr int OUT = EPI == EPI_SILU ? 128 : kTN;  // output columns of the tile
    for (int mt = 0; mt < MT; ++mt)
    for (int c0 = chalf * (OUT / 2); c0 < (chalf + 1) * (OUT / 2); c0 += 32) {
      const int m = m0 + mt * kTM + 32 * quad + lane;
      const uint32_t lane_addr = taddr + uint32_t(mt * kTN) + (uint32_t(32 * quad) << 16);
      float v[32], u[32];
      tmem_ld32(lane_addr + c0, v);
      if constexpr (EPI == EPI_SILU) tmem_ld32(lane_addr + 128 + c0, u);
      if (m < a.M && !s_fail) {
        const long n0 = (long)nt * OUT + c0;
        half* yrow = a.y + (long)m * a.ldy + n0;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 out;
          uint32_t* po = reinterpret_cast<uint32_t*>(&out);
          uint4 rv = make_uint4(0, 0, 0, 0);
          if constexpr (EPI == EPI_RESID) rv = *reinterpret_cast<const uint4*>(a.res + (long)m * a.ldres + n0 + 8 * q);
          const half* rh = reinterpret_cast<const half*>(&rv);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float o2[2];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int i = 8 * q + 2 * e + h;
              float val;
              if constexpr (EPI == EPI_SILU) {
                const float g16 = rnd<half>(v[i]), u16 = rnd<half>(u[i]);
                val = rnd<half>(g16 / (1.0f + expf(-g16))) * u16;
              } else {
                val = rnd<half>(v[i]);
                if (a.bias) val = rnd<half>(val + __half2float(a.bias[n0 + i]));
                if constexpr (EPI == EPI_RESID) val += __half2float(rh[2 * e + h]);
              }
              o2[h] = val;
            }
            __half2 hh = __floats2half2_rn(o2[0], o2[1]);
            po[e] = *reinterpret_cast<uint32_t*>(&hh);
          }
          *reinterpret_cast<uint4*>(yrow + 8 * q) = out;
        }
      }
    }
  }

  // ------------------------------------------------------------ teardown
  grid_launch_dependents();
  tc_fence_before();
  __syncthreads();
  if (warp == kWMma) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(kTN * MT) : "memory");
  }
}

template <int EPI, int MT>
nmx_status_t launch_gemm(Ctx* c, const CUtensorMap& tm, const CUtensorMap& tw, const GemmArgs& g, dim3 grid) {
  static std::mutex mu;
  static std::map<int, bool> set;
  const size_t smem = TcStages<MT>::kSmem;
  static_assert(TcStages<MT>::kSmem <= 227 * 1024, "prefill GEMM shared memory");
  {
    std::lock_guard<std::mutex> lk(mu);
    if (!set[c->device]) {
      NMX_CUDA_OK(
          cudaFuncSetAttribute(qgemm_tc_kernel<EPI, MT>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
      set[c->device] = true;
    }
  }
  return launch(c, qgemm_tc_kernel<EPI, MT>, grid, dim3(kGThreads), smem, tm, tw, g);
}
// two x sub-tiles per CTA (each dequantized weight stage feeds both) once
// the second sub-tile holds at least half a tile of rows
template <int EPI>
nmx_status_t launch_gemm_mt(Ctx* c, const CUtensorMap& tm, const CUtensorMap& tw, const GemmArgs& g, int ntiles) {
  if (g.M >= kTM + kTM / 2)
    return launch_gemm<EPI, 2>(c, tm, tw, g, dim3((g.M + 2 * kTM - 1) / (2 * kTM), ntiles));
  return launch_gemm<EPI, 1>(c, tm, tw, g, dim3((g.M + kTM - 1) / kTM, ntiles));
}

}  // namespace

bool qgemm_tc_supported(int N_out, int K, int epi) {
  if (K % 128 != 0 || K <= 0) return false;
  if (epi == EPI_SILU) return N_out % 128 == 0;
  if (epi == EPI_STORE || epi == EPI_RESID) return N_out % kTN == 0;
  return false;
}

nmx_status_t qgemm_tc(Ctx* c, const GemvDLArgs& a, int epi) {
  NMX_CHECK(qgemm_tc_supported(a.N, a.K, epi), NMX_ERR_UNSUPPORTED, "qgemm_tc: shape or epilogue");
  NMX_CHECK(a.gamma == nullptr, NMX_ERR_UNSUPPORTED, "qgemm_tc: normalise x first");
  NMX_CHECK(a.err != nullptr, NMX_ERR_INVALID, "qgemm_tc: no error word");
  NMX_CHECK(reinterpret_cast<uintptr_t>(a.x) % 16 == 0 && (a.ldx * 2) % 16 == 0, NMX_ERR_UNSUPPORTED,
            "qgemm_tc: x must be 16-byte aligned with a 16-byte row pitch");
  NMX_CHECK(reinterpret_cast<uintptr_t>(a.y) % 16 == 0 && (a.ldy * 2) % 16 == 0 &&
                (!a.res || (reinterpret_cast<uintptr_t>(a.res) % 16 == 0 && (a.ldres * 2) % 16 == 0)),
            NMX_ERR_UNSUPPORTED, "qgemm_tc: y / residual must be 16-byte aligned");
  if (a.M == 0) return NMX_OK;
  CUtensorMap tm, tw;
  NMX_TRY(tc::encode_x_map(&tm, a.x, a.ldx, a.M, a.K, kTM));
  const long long rows = epi == EPI_SILU ? (long long)a.pair_tiles * 16 + a.N : a.N;
  NMX_TRY(tc::encode_records_map(&tw, a.w, a.K / 128, rows / 16, 8));
  GemmArgs g;
  g.w = static_cast<const unsigned char*>(a.w);
  g.M = a.M;
  g.N_out = a.N;
  g.K = a.K;
  g.pair_tiles = a.pair_tiles;
  g.bias = static_cast<const half*>(a.bias);
  g.y = static_cast<half*>(a.y);
  g.ldy = a.ldy;
  g.res = static_cast<const half*>(a.res);
  g.ldres = a.ldres;
  g.err = a.err;
  const int ntiles = epi == EPI_SILU ? a.N / 128 : a.N / kTN;
  switch (epi) {
    case EPI_STORE: return launch_gemm_mt<EPI_STORE>(c, tm, tw, g, ntiles);
    case EPI_RESID: return launch_gemm_mt<EPI_RESID>(c, tm, tw, g, ntiles);
    default: return launch_gemm_mt<EPI_SILU>(c, tm, tw, g, ntiles);
  }
}

}  // namespace nmx
