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
//   * warp 10 bulk-copies the 16 records of each 128-k block of the weight
//     tile into a ring of 3 raw slots (cp.async.bulk, mbarrier tx count);
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
#include <cuda.h>
#include <cudaTypedefs.h>

#include <map>
#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "qgemv_common.cuh"

namespace nmx {

namespace {

constexpr int kTM = 128;          // rows of x per CTA (MMA M)
constexpr int kTN = 256;          // MMA N: weight rows per CTA
constexpr int kTK = 64;           // k per stage (one group)
constexpr int kTS = 3;            // stages
constexpr int kRS = 3;            // raw record slots (one 128-k block of the 16 tiles each)
constexpr int kABytes = kTM * kTK * 2;   // 16 KB
constexpr int kBBytes = kTN * kTK * 2;   // 32 KB
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kDW = 8;            // dequant / epilogue warps (one weight row per thread)
constexpr int kGThreads = (kDW + 3) * 32;  // + MMA, x-tile and record-loader warps
constexpr int kWMma = kDW, kWTma = kDW + 1, kWRec = kDW + 2;
constexpr unsigned kGSpin = 1u << 24;
constexpr int kRecG = 1152;
constexpr int kRawBytes = 16 * kRecG;  // the 16 records of one block of the weight tile

__device__ __forceinline__ unsigned sa_(const void* p) { return static_cast<unsigned>(__cvta_generic_to_shared(p)); }
__device__ __forceinline__ void mbar_init(uint64_t* b, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(sa_(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(sa_(b)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(sa_(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_wait(uint64_t* b, unsigned parity) {
  const unsigned a = sa_(b);
  for (unsigned it = 0; it < kGSpin; ++it) {
    unsigned ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(a), "r"(parity)
        : "memory");
    if (ok) return true;
  }
  return false;
}

// K-major operand in the 128-byte swizzle: 8-row groups 1024 B apart (SBO),
// version 1, layout SWIZZLE_128B (2); the start address steps 32 B per k16
__device__ __forceinline__ uint64_t smem_desc(const void* p) {
  const uint64_t a = sa_(p);
  return ((a >> 4) & 0x3FFFull) | (1ull << 16) | (uint64_t(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}
// kind::f16 instruction descriptor: f32 accumulator, f16 A and B, both K-major
constexpr uint32_t kIDesc = (1u << 4) | (uint32_t(kTN >> 3) << 17) | (uint32_t(kTM >> 4) << 24);

__device__ __forceinline__ void mma_f16_tc(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(kIDesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(sa_(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

// 32 consecutive f32 columns of this thread's TMEM lane
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// byte offset of (row, 16-byte chunk) in a K-major 64-wide f16 tile, 128 B swizzle
__device__ __forceinline__ int sw128(int row, int chunk) {
  return (row >> 3) * 1024 + (row & 7) * 128 + ((chunk ^ (row & 7)) << 4);
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

template <int EPI>
__global__ void __launch_bounds__(kGThreads, 1) qgemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_x,
                                                                 GemmArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full[kTS];
  __shared__ __align__(8) uint64_t empty[kTS];
  __shared__ __align__(8) uint64_t acc_bar;
  __shared__ __align__(8) uint64_t raw_full[kRS];
  __shared__ __align__(8) uint64_t raw_empty[kRS];
  __shared__ uint32_t s_taddr;
  __shared__ int s_fail;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int m0 = blockIdx.x * kTM;
  const int nt = blockIdx.y;  // output tile
  const int KT = a.K / kTK, nb = a.K / 128;

  if (tid == 0) {
    for (int s = 0; s < kTS; ++s) {
      mbar_init(&full[s], 1 + kDW * 32);  // TMA thread (expect_tx) + the dequant threads
      mbar_init(&empty[s], 1);       // tcgen05.commit
    }
    mbar_init(&acc_bar, 1);
    for (int s = 0; s < kRS; ++s) {
      mbar_init(&raw_full[s], 1);      // record loader (expect_tx)
      mbar_init(&raw_empty[s], kDW * 32);  // the dequant threads, after the block's second stage
    }
    s_fail = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kWMma) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(sa_(&s_taddr)), "r"(kTN)
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
        if (b >= kRS && !mbar_wait(&raw_empty[rs], ((b / kRS) - 1) & 1)) {
          atomicOr(a.err, 1u);
          s_fail = 1;
          break;
        }
        mbar_expect_tx(&raw_full[rs], kRawBytes);
        for (int i = 0; i < 16; ++i) {
          long long T;  // 16-row tile of the matrix
          if constexpr (EPI == EPI_SILU)
            T = (i < 8) ? (long long)nt * 8 + i : a.pair_tiles + (long long)nt * 8 + (i - 8);
          else
            T = (long long)nt * 16 + i;
          const unsigned char* src = a.w + (T * nb + b) * kRecG;
          asm volatile(
              "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                  sa_(raw + rs * kRawBytes + i * kRecG)),
              "l"(src), "r"(kRecG), "r"(sa_(&raw_full[rs]))
              : "memory");
        }
      }
    }
  } else if (warp == kWTma) {
    // ---------------------------------------------------------------- TMA: x tiles
    if (lane == 0) {
      for (int kt = 0; kt < KT; ++kt) {
        const int s = kt % kTS;
        if (kt >= kTS && !mbar_wait(&empty[s], ((kt / kTS) - 1) & 1)) {
          atomicOr(a.err, 1u);
          s_fail = 1;
          break;
        }
        unsigned char* dst = smem + s * kStageBytes;
        mbar_expect_tx(&full[s], kABytes);
        asm volatile(
            "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
                "r"(sa_(dst)),
            "l"(&tmap_x), "r"(kt * kTK), "r"(m0), "r"(sa_(&full[s]))
            : "memory");
      }
    }
  } else if (warp == kWMma) {
    // ---------------------------------------------------------------- MMA issue
    if (lane == 0) {
      for (int kt = 0; kt < KT; ++kt) {
        const int s = kt % kTS;
        if (!mbar_wait(&full[s], (kt / kTS) & 1)) {
          atomicOr(a.err, 1u);
          s_fail = 1;
          break;
        }
        tc_fence_after();
        unsigned char* A = smem + s * kStageBytes;
        unsigned char* B = A + kABytes;
#pragma unroll
        for (int k16 = 0; k16 < kTK / 16; ++k16)
          mma_f16_tc(taddr, smem_desc(A + 32 * k16), smem_desc(B + 32 * k16), (kt | k16) ? 1u : 0u);
        mma_commit(&empty[s]);
      }
      mma_commit(&acc_bar);
    }
  } else {
    // ----------------------------------------- dequant warps: weight tile rows
    // thread t fills weight row t of the tile
    for (int kt = 0; kt < KT; ++kt) {
      const int s = kt % kTS;
      if (kt >= kTS && !mbar_wait(&empty[s], ((kt / kTS) - 1) & 1)) {
        atomicOr(a.err, 1u);
        s_fail = 1;
        break;
      }
      unsigned char* B = smem + s * kStageBytes + kABytes;
      const int blk = kt >> 1, gi = kt & 1, rs = blk % kRS;
      if (gi == 0 && !mbar_wait(&raw_full[rs], (blk / kRS) & 1)) {
        atomicOr(a.err, 1u);
        s_fail = 1;
        break;
      }
      const unsigned char* rawb = raw + rs * kRawBytes;
      {
        const int r = tid;  // weight row of the tile: record r / 16, row r % 16
        const int g16 = r & 15, half_ = g16 >> 3, g = g16 & 7;
        const unsigned char* rec = rawb + (r >> 4) * kRecG;
        const unsigned char* wb = rec + half_ * 512 + 16 * (4 * g) + 8 * gi;
        // words 2t, 2t+1 of this group sit in lane 4g+t's 16 bytes
        uint2 wv[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) wv[t] = *reinterpret_cast<const uint2*>(wb + 16 * t);
        const __half sc = *reinterpret_cast<const __half*>(rec + 1024 + ((0 * 2 + gi) * 8 + g) * 4 + half_ * 2);
        const __half bi = *reinterpret_cast<const __half*>(rec + 1024 + ((1 * 2 + gi) * 8 + g) * 4 + half_ * 2);
        const __half2 s2 = __halves2half2(sc, sc);
        const __half2 s16 = __hmul2(s2, __float2half2_rn(0.0625f));
        const __half2 b2 = __halves2half2(bi, bi);
        const __half2 k1024 = __float2half2_rn(1024.f);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint32_t word = (j & 1) ? wv[j >> 1].y : wv[j >> 1].x;
          uint32_t P[4];
          dequant_word<4>(word, P);  // (q0,q4), (16q1,16q5), (q2,q6), (16q3,16q7), each + 1024
          __half2 v0 = __hfma2(__hsub2(*reinterpret_cast<__half2*>(&P[0]), k1024), s2, b2);   // w0, w4
          __half2 v1 = __hfma2(__hsub2(*reinterpret_cast<__half2*>(&P[1]), k1024), s16, b2);  // w1, w5
          __half2 v2 = __hfma2(__hsub2(*reinterpret_cast<__half2*>(&P[2]), k1024), s2, b2);   // w2, w6
          __half2 v3 = __hfma2(__hsub2(*reinterpret_cast<__half2*>(&P[3]), k1024), s16, b2);  // w3, w7
          const uint32_t u0 = *reinterpret_cast<uint32_t*>(&v0), u1 = *reinterpret_cast<uint32_t*>(&v1);
          const uint32_t u2 = *reinterpret_cast<uint32_t*>(&v2), u3 = *reinterpret_cast<uint32_t*>(&v3);
          uint4 o;
          o.x = __byte_perm(u0, u1, 0x5410);  // w0, w1
          o.y = __byte_perm(u2, u3, 0x5410);  // w2, w3
          o.z = __byte_perm(u0, u1, 0x7632);  // w4, w5
          o.w = __byte_perm(u2, u3, 0x7632);  // w6, w7
          *reinterpret_cast<uint4*>(B + sw128(r, j)) = o;
        }
      }
      // generic-proxy writes, read by the tensor core's async proxy
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive(&full[s]);
      if (gi == 1) mbar_arrive(&raw_empty[rs]);  // the block's records are read
    }

    // ------------------------------------------------------------ epilogue
    if (!s_fail && !mbar_wait(&acc_bar, 0)) {
      atomicOr(a.err, 1u);
      s_fail = 1;
    }
    tc_fence_after();
    // warp w reads TMEM lanes 32 (w % 4) .. +31 (its rows) and half the columns
    const int quad = warp & 3, chalf = warp >> 2;
    const int m = m0 + 32 * quad + lane;
    const uint32_t lane_addr = taddr + (uint32_t(32 * quad) << 16);
    constexpr int OUT = EPI == EPI_SILU ? 128 : kTN;  // output columns of the tile
    for (int c0 = chalf * (OUT / 2); c0 < (chalf + 1) * (OUT / 2); c0 += 32) {
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
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(kTN) : "memory");
  }
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, []() {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

template <int EPI>
nmx_status_t launch_gemm(Ctx* c, const CUtensorMap& tm, const GemmArgs& g, dim3 grid) {
  static std::mutex mu;
  static std::map<int, bool> set;
  const size_t smem = size_t(kTS) * kStageBytes + size_t(kRS) * kRawBytes + 1024;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (!set[c->device]) {
      NMX_CUDA_OK(cudaFuncSetAttribute(qgemm_tc_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
      set[c->device] = true;
    }
  }
  return launch(c, qgemm_tc_kernel<EPI>, grid, dim3(kGThreads), smem, tm, g);
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
  auto enc = tensor_map_encoder();
  NMX_CHECK(enc != nullptr, NMX_ERR_UNSUPPORTED, "qgemm_tc: no tensor-map encoder in the driver");
  if (a.M == 0) return NMX_OK;
  // x as a [M rows][K cols] f16 tensor; box 64 (k) × 128 (rows), 128-byte swizzle
  CUtensorMap tm;
  const cuuint64_t dims[2] = {cuuint64_t(a.K), cuuint64_t(a.M)};
  const cuuint64_t strides[1] = {cuuint64_t(a.ldx) * 2};
  const cuuint32_t box[2] = {cuuint32_t(kTK), cuuint32_t(kTM)};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(&tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(a.x), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  NMX_CHECK(r == CUDA_SUCCESS, NMX_ERR_CUDA, "qgemm_tc: cuTensorMapEncodeTiled failed (" + std::to_string(int(r)) + ")");
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
  const int mt = (a.M + kTM - 1) / kTM;
  const int ntiles = epi == EPI_SILU ? a.N / 128 : a.N / kTN;
  const dim3 grid(mt, ntiles);
  switch (epi) {
    case EPI_STORE: return launch_gemm<EPI_STORE>(c, tm, g, grid);
    case EPI_RESID: return launch_gemm<EPI_RESID>(c, tm, g, grid);
    default: return launch_gemm<EPI_SILU>(c, tm, g, grid);
  }
}

}  // namespace nmx
