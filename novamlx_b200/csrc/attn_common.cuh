// Device helpers shared by the decode attention kernels: cp.async, ldmatrix,
// the f16 m16n8k16 MMA, the XOR-swizzled [16][D] f16 tile layout and RoPE of
// one pair.
#pragma once

#include "common.cuh"

namespace nmx {
namespace {

__device__ __forceinline__ void cp_async16a(void* smem_dst, const void* gsrc) {
  const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem_dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t* r, const void* p) {
  const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(s));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t* r, const void* p) {
  const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(s));
}
__device__ __forceinline__ void ldsm_x2(uint32_t* r, const void* p) {
  const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];\n" : "=r"(r[0]), "=r"(r[1]) : "r"(s));
}

__device__ __forceinline__ void mma_f16(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// The same MMA when rows 8-15 of A are zero (a1 = a3 = 0): only the
// accumulators of rows 0-7 (d[0], d[1]) are kept; rows 8-15 read zeros and
// their results are dropped, so they hold no registers across calls.
__device__ __forceinline__ void mma_f16_top(float* d, uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
  float x2, x3;
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%11,%12,%13};\n"
      : "=f"(d[0]), "=f"(d[1]), "=f"(x2), "=f"(x3)
      : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1), "f"(d[0]), "f"(d[1]), "f"(0.f), "f"(0.f));
  (void)x2;
  (void)x3;
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// byte offset of (row, 16-byte chunk) in a swizzled [16][D] f16 tile
template <int D>
__device__ __forceinline__ int swz(int row, int chunk) {
  return row * (D * 2) + ((chunk ^ (row & 7)) << 4);
}

__device__ __forceinline__ void rope2(float a, float b, float ang, float& ra, float& rb) {
  float sn, cs;
  sincosf(ang, &sn, &cs);
  ra = a * cs - b * sn;
  rb = b * cs + a * sn;
}

// ---------------------------------------------------------------------------
// Quantized KV pages (the kvBits path): page records as kv_page_bytes
// (kernels.h) describes them.

// One K or V row held by a warp (lane l: values d = l * VPL .. + VPL - 1),
// quantized in groups of gs: scale = (max - min) / (2^bits - 1) and bias =
// min in fp32 for the codes, stored as f16; the row's codes, scales and
// biases go to slot `tok` of the page record `rec`, and v returns the
// dequantized values (q * s + b with the f16 scale and bias, one rounding).
template <int D>
__device__ __forceinline__ void quantize_row_warp(float* v, int bits, int gs, unsigned char* rec, int tok) {
  constexpr int VPL = D / 32;
  const int lane = threadIdx.x & 31;
  const int lpg = gs / VPL;  // lanes per group: a power of two <= 32
  float mn = v[0], mx = v[0];
#pragma unroll
  for (int i = 1; i < VPL; ++i) {
    mn = fminf(mn, v[i]);
    mx = fmaxf(mx, v[i]);
  }
  for (int o = lpg / 2; o > 0; o >>= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  const float nbins = float((1 << bits) - 1);
  const float scale = (mx - mn) / nbins, bias = mn;
  const half s16 = __float2half_rn(scale), b16 = __float2half_rn(bias);
  uint32_t packed = 0;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    float q = 0.f;
    if (scale > 0.f) q = fminf(fmaxf(rintf((v[i] - bias) / scale), 0.f), nbins);
    packed |= uint32_t(q) << (i * bits);
    v[i] = __half2float(__hfma(__float2half_rn(q), s16, b16));
  }
  // a 32-bit word holds the codes of lpw consecutive lanes
  const int lpw = 32 / (bits * VPL);
  uint32_t word = packed;
  for (int o = 1; o < lpw; o <<= 1) {
    const uint32_t other = __shfl_down_sync(0xffffffffu, word, o);
    if ((lane & (2 * o - 1)) == 0) word |= other << (o * bits * VPL);
  }
  const int rowbytes = D * bits / 8, ng = D / gs;
  if ((lane % lpw) == 0) reinterpret_cast<uint32_t*>(rec + tok * rowbytes)[lane / lpw] = word;
  if ((lane % lpg) == 0) {
    half* sc = reinterpret_cast<half*>(rec + 16 * rowbytes);
    sc[tok * ng + lane / lpg] = s16;
    sc[16 * ng + tok * ng + lane / lpg] = b16;
  }
}

// 8 f16 values w = s * q + b (k order) from one 32-bit word of 4-bit codes
__device__ __forceinline__ uint4 dq4_chunk(uint32_t w, __half2 s2, __half2 b2) {
  const uint32_t magic = 0x64006400u;  // f16 1024.0 in both halves
  const __half2 k1024 = __float2half2_rn(1024.f);
  uint32_t p[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t t;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;\n" : "=r"(t) : "r"(w >> (4 * i)), "r"(0x000F000Fu), "r"(magic));
    __half2 h = __hfma2(__hsub2(*reinterpret_cast<__half2*>(&t), k1024), s2, b2);  // (w_i, w_{i+4})
    p[i] = *reinterpret_cast<uint32_t*>(&h);
  }
  return make_uint4(__byte_perm(p[0], p[1], 0x5410), __byte_perm(p[2], p[3], 0x5410),
                    __byte_perm(p[0], p[1], 0x7632), __byte_perm(p[2], p[3], 0x7632));
}
// 8 f16 values from two 32-bit words of 8-bit codes
__device__ __forceinline__ uint4 dq8_chunk(uint2 w, __half2 s2, __half2 b2) {
  const __half2 k1024 = __float2half2_rn(1024.f);
  uint32_t r[4];
  const uint32_t src[2] = {w.x, w.y};
#pragma unroll
  for (int j = 0; j < 2; ++j) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      uint32_t t = __byte_perm(src[j], 0x64646464u, e ? 0x7362 : 0x5140);  // 1024 + byte, two of them
      __half2 h = __hfma2(__hsub2(*reinterpret_cast<__half2*>(&t), k1024), s2, b2);
      r[2 * j + e] = *reinterpret_cast<uint32_t*>(&h);
    }
  }
  return make_uint4(r[0], r[1], r[2], r[3]);
}

// One page record dequantized into a swizzled [16][D] f16 tile by the
// threads i0, i0 + stride, ... (a warp: lane, 32; a CTA: tid, blockDim).
template <int D>
__device__ __forceinline__ void dequant_page(const unsigned char* rec, int bits, int gs, unsigned char* tile, int i0,
                                             int stride) {
  constexpr int CH = D / 8;
  const int rowbytes = D * bits / 8, ng = D / gs;
  const half* sc = reinterpret_cast<const half*>(rec + 16 * rowbytes);
  const half* bi = sc + 16 * ng;
#pragma unroll 4
  for (int i = i0; i < 16 * CH; i += stride) {
    const int r = i / CH, c = i % CH;
    const int g = (8 * c) / gs;
    const __half2 s2 = __half2half2(sc[r * ng + g]), b2 = __half2half2(bi[r * ng + g]);
    const uint4 o = bits == 4 ? dq4_chunk(*reinterpret_cast<const uint32_t*>(rec + r * rowbytes + 4 * c), s2, b2)
                              : dq8_chunk(*reinterpret_cast<const uint2*>(rec + r * rowbytes + 8 * c), s2, b2);
    *reinterpret_cast<uint4*>(tile + swz<D>(r, c)) = o;
  }
}

}  // namespace
}  // namespace nmx
