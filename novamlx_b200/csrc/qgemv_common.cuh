// Device helpers shared by the quantized GEMV kernels (MLX layout and
// decode-record layout): the m16n8k16 MMA, the LOP3/PRMT dequantisation of
// packed words into f16 pairs, and the per-lane pair order of the
// activations staged in shared memory.
#pragma once

#include "common.cuh"

namespace nmx {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

template <int BITS, int GS>
struct QCfg {
  static constexpr int WPG = GS * BITS / 32;  // packed words per row per group
  static constexpr int WPT = WPG / 4;         // words per lane per row per group
  static constexpr int NMMA = GS / 16;        // m16n8k16 MMAs per group
  static constexpr int MP = GS / 8;           // f16x2 pairs per lane per group
  // groups per pipeline batch: 64 B of packed weights per lane in flight
  static constexpr int BATCH = WPT >= 8 ? 1 : 8 / WPT;
};

__device__ __forceinline__ void mma16816(float* d, uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1, float c0, float c1,
                                         float c2, float c3) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%10,%11,%12,%13};\n"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c0), "f"(c1), "f"(c2),
        "f"(c3));
}

// k offsets (within the group) and type of pair p of lane t.
// 4-bit: word j = p/4, e = p%4 → values (e, e+4) of the word; odd e are the
//        high nibbles of their bytes (pre-scaled by 1/16).
// 8-bit: word j = p/2, e = p%2 → values (2e, 2e+1) of the word.
template <int BITS, int GS>
__device__ __forceinline__ void pair_k(int t, int p, int& k0, int& k1, bool& hi) {
  constexpr int base_t = GS / 4;  // k values per lane per group
  if constexpr (BITS == 4) {
    const int j = p >> 2, e = p & 3;
    k0 = t * base_t + 8 * j + e;
    k1 = k0 + 4;
    hi = (e & 1) != 0;
  } else {
    const int j = p >> 1, e = p & 1;
    k0 = t * base_t + 4 * j + 2 * e;
    k1 = k0 + 1;
    hi = false;
  }
}

template <int WPT>
struct WordVec {
  uint32_t v[WPT];
};

template <int WPT>
__device__ __forceinline__ void load_words(WordVec<WPT>& out, const uint32_t* p) {
  if constexpr (WPT == 1) {
    out.v[0] = __ldg(p);
  } else if constexpr (WPT == 2) {
    uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
    out.v[0] = u.x;
    out.v[1] = u.y;
  } else if constexpr (WPT == 4) {
    uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
    out.v[0] = u.x;
    out.v[1] = u.y;
    out.v[2] = u.z;
    out.v[3] = u.w;
  } else {
    static_assert(WPT == 8, "unsupported words per lane");
    uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
    uint4 w = __ldg(reinterpret_cast<const uint4*>(p) + 1);
    out.v[0] = u.x; out.v[1] = u.y; out.v[2] = u.z; out.v[3] = u.w;
    out.v[4] = w.x; out.v[5] = w.y; out.v[6] = w.z; out.v[7] = w.w;
  }
}

// f16x2 A-operand pairs of one packed word (see pair_k for the order).
// (a & b) | c in one LOP3 (truth table 0xEA)
__device__ __forceinline__ uint32_t and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;\n" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}

template <int BITS>
__device__ __forceinline__ void dequant_word(uint32_t w, uint32_t* P) {
  if constexpr (BITS == 4) {
    const uint32_t magic = 0x64006400u;          // f16 1024.0 in both halves
    P[0] = and_or(w, 0x000F000Fu, magic);        // 1024 + q0,      1024 + q4
    P[1] = and_or(w, 0x00F000F0u, magic);        // 1024 + 16 q1,   1024 + 16 q5
    const uint32_t w8 = w >> 8;
    P[2] = and_or(w8, 0x000F000Fu, magic);       // q2, q6
    P[3] = and_or(w8, 0x00F000F0u, magic);       // 16 q3, 16 q7
  } else {
    P[0] = __byte_perm(w, 0x64646464u, 0x5140);  // 1024 + b0, 1024 + b1
    P[1] = __byte_perm(w, 0x64646464u, 0x7362);  // 1024 + b2, 1024 + b3
  }
}

}  // namespace
}  // namespace nmx
