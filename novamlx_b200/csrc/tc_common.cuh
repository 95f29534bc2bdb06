// Shared pieces of the tcgen05 GEMMs over decode records (gemm_tc.cu,
// gemm_tcs.cu): bounded mbarrier waits, shared-memory matrix descriptors in
// the 128-byte swizzle, tcgen05.mma / commit / ld wrappers, the dequantiser
// of one record row into a swizzled f16 tile, and the tensor-map encoder.
#pragma once
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "qgemv_common.cuh"

namespace nmx {
namespace tc {

constexpr int kRecG = 1152;            // bytes of one decode record (16 rows x 128 k)

__device__ __forceinline__ unsigned sa_(const void* p) { return static_cast<unsigned>(__cvta_generic_to_shared(p)); }
__device__ __forceinline__ void mbar_init(uint64_t* b, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(sa_(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(sa_(b)) : "memory");
}
// One arrival for the whole warp (the barrier counts warps): the lanes'
// prior writes are ordered before lane 0's release-arrive by __syncwarp.
// An arrive is a shared-memory atomic, so per-thread arrivals on a hot
// barrier serialise hundreds of atomics per handoff.
__device__ __forceinline__ void warp_arrive(uint64_t* b) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(b);
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(sa_(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try(unsigned a, unsigned parity) {
  unsigned ok;
  asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
               : "=r"(ok)
               : "r"(a), "r"(parity)
               : "memory");
  return ok != 0;
}
// bounded: false after `lim` polls (the context's wait limit)
__device__ __forceinline__ bool mbar_wait(uint64_t* b, unsigned parity, unsigned lim) {
  const unsigned a = sa_(b);
  for (unsigned it = 0; it < lim; ++it)
    if (mbar_try(a, parity)) return true;
  return false;
}
// K-major operand in the 128-byte swizzle: 8-row groups 1024 B apart (SBO),
// version 1, layout SWIZZLE_128B (2); the start address steps 32 B per k16
__device__ __forceinline__ uint64_t smem_desc(const void* p) {
  const uint64_t a = sa_(p);
  return ((a >> 4) & 0x3FFFull) | (1ull << 16) | (uint64_t(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}
// kind::f16 instruction descriptor: f32 accumulator, f16 A and B, both K-major
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N) {
  return (1u << 4) | (uint32_t(N >> 3) << 17) | (uint32_t(M >> 4) << 24);
}

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
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
// 8 consecutive f32 columns of this thread's TMEM lane
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float* v) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

// byte offset of (row, 16-byte chunk) in a K-major 64-wide f16 tile, 128 B swizzle
__device__ __forceinline__ int sw128(int row, int chunk) {
  return (row >> 3) * 1024 + (row & 7) * 128 + ((chunk ^ (row & 7)) << 4);
}

// one 32-bit word (8 nibbles, k 8w .. 8w+7 of a group) as 8 f16 weights
// w = s·q + b in k order (one 16-byte chunk of a K-major tile row)
__device__ __forceinline__ uint4 dequant_word_chunk(uint32_t word, __half2 s2, __half2 s16, __half2 b2) {
  const __half2 k1024 = __float2half2_rn(1024.f);
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
  return o;
}

// Row g16 (0..15) of one decode record, group gi (k 0-63 or 64-127), as 64
// f16 weights w = s·q + b (rounded to f16) into row `row` of a swizzled
// 64-wide tile. Record layout: bytes [0, 512) rows 0-7, [512, 1024) rows
// 8-15, lane 4g+t's 16 bytes holding words (2t, 2t+1) of both groups of row
// g; then (scale | bias, group, row g) half2 pairs (row g, row g+8).
__device__ __forceinline__ void dequant_record_row(const unsigned char* rec, int g16, int gi, unsigned char* tile,
                                                   int row) {
  const int half_ = g16 >> 3, g = g16 & 7;
  const unsigned char* wb = rec + half_ * 512 + 16 * (4 * g) + 8 * gi;
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
    *reinterpret_cast<uint4*>(tile + sw128(row, j)) = o;
  }
}

inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
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

// x as a [rows][K] f16 tensor with row pitch ldx elements; box 64 (k) x
// box_rows, 128-byte swizzle; rows past `rows` read as zeros
inline nmx_status_t encode_x_map(CUtensorMap* tm, const void* x, long ldx, int rows, int K, int box_rows) {
  auto enc = tensor_map_encoder();
  NMX_CHECK(enc != nullptr, NMX_ERR_UNSUPPORTED, "tensor-core GEMM: no tensor-map encoder in the driver");
  const cuuint64_t dims[2] = {cuuint64_t(K), cuuint64_t(rows)};
  const cuuint64_t strides[1] = {cuuint64_t(ldx) * 2};
  const cuuint32_t box[2] = {64u, cuuint32_t(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(x), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  NMX_CHECK(r == CUDA_SUCCESS, NMX_ERR_CUDA,
            "tensor-core GEMM: cuTensorMapEncodeTiled failed (" + std::to_string(int(r)) + ")");
  return NMX_OK;
}

// Decode records as a 3-d tensor of 8-byte words [16-row tiles][K blocks]
// [144 words], so ONE tensor copy brings the records of `box_tiles`
// consecutive tiles at one K block. The box is 146 words wide: each record
// lands kRecPad = 1168 bytes after the previous one (the 16 bytes past a
// record's end read as zeros), which staggers the records over the shared
// memory banks.
constexpr int kRecPad = kRecG + 16;
inline nmx_status_t encode_records_map(CUtensorMap* tm, const void* w, int nb, long long n_tiles16, int box_tiles) {
  auto enc = tensor_map_encoder();
  NMX_CHECK(enc != nullptr, NMX_ERR_UNSUPPORTED, "tensor-core GEMM: no tensor-map encoder in the driver");
  const cuuint64_t dims[3] = {cuuint64_t(kRecG / 8), cuuint64_t(nb), cuuint64_t(n_tiles16)};
  const cuuint64_t strides[2] = {cuuint64_t(kRecG), cuuint64_t(kRecG) * cuuint64_t(nb)};
  const cuuint32_t box[3] = {cuuint32_t(kRecPad / 8), 1u, cuuint32_t(box_tiles)};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, const_cast<void*>(w), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  NMX_CHECK(r == CUDA_SUCCESS, NMX_ERR_CUDA,
            "tensor-core GEMM: records tensor map failed (" + std::to_string(int(r)) + ")");
  return NMX_OK;
}

// tensor copy of `tile0`'s box of records at K block b into shared memory
__device__ __forceinline__ void load_records(void* dst, const CUtensorMap* tm, int b, int tile0, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
          "r"(sa_(dst)),
      "l"(tm), "r"(0), "r"(b), "r"(tile0), "r"(sa_(bar))
      : "memory");
}

}  // namespace tc
}  // namespace nmx
