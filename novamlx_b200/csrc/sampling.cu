// Sampling beyond greedy, on the device: CompiledSampler's temperature /
// top-p categorical (Sources/NovaMLXEngine/CompiledSampler.swift:17-49) and
// the logprob helper of FusedBatchScheduler (computeRawLogprobs,
// FusedBatchScheduler.swift:900-941), one CTA per row of logits.
//
//   lp = logSoftmax(logits) (f32);
//   temperature 0: argmax (lowest id on ties);
//   0 < top_p < 1: the reference keeps, in ascending order of lp, the
//     entries whose inclusive cumulative probability exceeds 1 - top_p, i.e.
//     the tokens whose strictly-higher mass is below top_p. Here: a binary
//     search over the order-preserving integer keys of lp finds the largest
//     key whose strictly-higher mass reaches top_p; tokens above it are kept
//     (all of a tie group at the boundary are kept);
//   categorical over lp / temperature of the kept tokens by the Gumbel-max
//     rule: argmax(lp / T - log(-log(u))), u from a counter-based hash of
//     (seed, counter, row, token) — reproducible for the same arguments, and
//     the same distribution as MLX's categorical (not the same stream: MLX's
//     generator is its own);
//   logprob of the chosen id, and the top_k (<= 32) largest lp with their
//     ids in descending order, from the unfiltered, untempered lp as the
//     reference computes them.
#include <cfloat>

#include "common.cuh"
#include "kernels.h"

namespace nmx {

namespace {

constexpr int kSThreadsS = 512;
constexpr int kMaxTopK = 32;

template <typename T>
__device__ __forceinline__ float ld_l(const void* p, long i);
template <>
__device__ __forceinline__ float ld_l<half>(const void* p, long i) {
  return __half2float(reinterpret_cast<const half*>(p)[i]);
}
template <>
__device__ __forceinline__ float ld_l<__nv_bfloat16>(const void* p, long i) {
  return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
}
template <>
__device__ __forceinline__ float ld_l<float>(const void* p, long i) {
  return reinterpret_cast<const float*>(p)[i];
}

// order-preserving map of a float to an unsigned key
__device__ __forceinline__ unsigned fkey(float v) {
  const unsigned u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// 64-bit mix (splitmix64 finaliser) → uniform in (0, 1)
__device__ __forceinline__ float uniform01(unsigned long long seed, unsigned long long counter, int row, int v) {
  unsigned long long z = seed ^ (counter * 0x9E3779B97F4A7C15ull) ^ ((unsigned long long)row << 40) ^
                         (unsigned long long)(unsigned)v;
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  z ^= z >> 31;
  return (float((z >> 40) & 0xFFFFFFull) + 0.5f) * (1.0f / 16777216.0f);
}

__device__ __forceinline__ float block_sum(float v, float* sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.f;
  for (int w = 0; w < int(blockDim.x >> 5); ++w) t += sh[w];
  return t;
}
__device__ __forceinline__ float block_max(float v, float* sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = -INFINITY;
  for (int w = 0; w < int(blockDim.x >> 5); ++w) t = fmaxf(t, sh[w]);
  return t;
}
// (value, id) maximum, lowest id on ties
__device__ __forceinline__ bool better(float v, int i, float bv, int bi) { return v > bv || (v == bv && i < bi); }
__device__ __forceinline__ void block_argmax(float& bv, int& bi, float* shv, int* shi) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(ov, oi, bv, bi)) {
      bv = ov;
      bi = oi;
    }
  }
  __syncthreads();
  if ((threadIdx.x & 31) == 0) {
    shv[threadIdx.x >> 5] = bv;
    shi[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  bv = -INFINITY;
  bi = 0x7fffffff;
  for (int w = 0; w < int(blockDim.x >> 5); ++w)
    if (better(shv[w], shi[w], bv, bi)) {
      bv = shv[w];
      bi = shi[w];
    }
}

template <typename T>
__global__ void __launch_bounds__(kSThreadsS) sample_kernel(const void* logits, int V, float temperature, float top_p,
                                                            unsigned long long seed, unsigned long long counter,
                                                            int* out_ids, float* out_lp, int top_k, int* top_ids,
                                                            float* top_lp) {
  __shared__ float shf[32];
  __shared__ int shi[32];
  __shared__ int s_sel[kMaxTopK];
  grid_wait();
  const int row = blockIdx.x;
  const long base = long(row) * V;
  // log-softmax constants
  float m = -INFINITY;
  for (int v = threadIdx.x; v < V; v += blockDim.x) m = fmaxf(m, ld_l<T>(logits, base + v));
  m = block_max(m, shf);
  float s = 0.f;
  for (int v = threadIdx.x; v < V; v += blockDim.x) s += expf(ld_l<T>(logits, base + v) - m);
  s = block_sum(s, shf);
  const float lse = m + logf(s);

  int chosen;
  if (temperature <= 0.f) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int v = threadIdx.x; v < V; v += blockDim.x) {
      const float x = ld_l<T>(logits, base + v);
      if (better(x, v, bv, bi)) {
        bv = x;
        bi = v;
      }
    }
    block_argmax(bv, bi, shf, shi);
    chosen = bi == 0x7fffffff ? 0 : bi;
  } else {
    // nucleus boundary: the largest key whose strictly-higher mass >= top_p
    bool have_cut = false;
    unsigned cut = 0u;
    if (top_p > 0.f && top_p < 1.f) {
      // the largest key k with P(k): mass of lp with key > k >= top_p (P is
      // true at k = 0, every finite lp having a larger key, and monotone)
      unsigned lo = 0u, hi = 0xFFFFFFFFu;
      for (int it = 0; it < 32 && lo < hi; ++it) {
        const unsigned mid = unsigned((static_cast<unsigned long long>(lo) + hi + 1ull) / 2ull);
        float mass = 0.f;
        for (int v = threadIdx.x; v < V; v += blockDim.x) {
          const float lp = ld_l<T>(logits, base + v) - lse;
          if (fkey(lp) > mid) mass += expf(lp);
        }
        mass = block_sum(mass, shf);
        if (mass >= top_p) lo = mid;
        else hi = mid - 1u;
      }
      float mass0 = 0.f;  // confirm P(lo)
      for (int v = threadIdx.x; v < V; v += blockDim.x) {
        const float lp = ld_l<T>(logits, base + v) - lse;
        if (fkey(lp) > lo) mass0 += expf(lp);
      }
      mass0 = block_sum(mass0, shf);
      have_cut = mass0 >= top_p;
      cut = lo;
    }
    const float inv_t = 1.0f / temperature;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int v = threadIdx.x; v < V; v += blockDim.x) {
      const float lp = ld_l<T>(logits, base + v) - lse;
      if (have_cut && fkey(lp) <= cut) continue;
      const float g = -logf(-logf(uniform01(seed, counter, row, v)));
      const float sc = lp * inv_t + g;
      if (better(sc, v, bv, bi)) {
        bv = sc;
        bi = v;
      }
    }
    block_argmax(bv, bi, shf, shi);
    chosen = bi == 0x7fffffff ? 0 : bi;
  }
  if (threadIdx.x == 0) {
    out_ids[row] = chosen;
    if (out_lp) out_lp[row] = ld_l<T>(logits, base + chosen) - lse;
  }
  // top_k logprobs, descending (k passes of a masked argmax)
  for (int j = 0; j < top_k; ++j) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int v = threadIdx.x; v < V; v += blockDim.x) {
      bool taken = false;
      for (int q = 0; q < j; ++q) taken |= (s_sel[q] == v);
      if (taken) continue;
      const float x = ld_l<T>(logits, base + v);
      if (better(x, v, bv, bi)) {
        bv = x;
        bi = v;
      }
    }
    block_argmax(bv, bi, shf, shi);
    if (threadIdx.x == 0) {
      s_sel[j] = bi;
      top_ids[long(row) * top_k + j] = bi;
      top_lp[long(row) * top_k + j] = bv - lse;
    }
    __syncthreads();
  }
  grid_launch_dependents();
}

}  // namespace

nmx_status_t sample_rows(Ctx* c, const void* logits, nmx_dtype_t dt, int rows, int V, float temperature, float top_p,
                         unsigned long long seed, unsigned long long counter, int* out_ids, float* out_lp, int top_k,
                         int* top_ids, float* top_lp) {
  NMX_CHECK(V > 0 && rows >= 0, NMX_ERR_INVALID, "sample: empty vocabulary");
  NMX_CHECK(top_k >= 0 && top_k <= kMaxTopK && top_k <= V, NMX_ERR_INVALID, "sample: top_k must be in [0, 32]");
  NMX_CHECK(top_k == 0 || (top_ids && top_lp), NMX_ERR_INVALID, "sample: top_k outputs missing");
  NMX_CHECK(temperature >= 0.f, NMX_ERR_INVALID, "sample: negative temperature");
  if (rows == 0) return NMX_OK;
#define NMX_SAMPLE(T)                                                                                            \
  return launch(c, sample_kernel<T>, dim3(rows), dim3(kSThreadsS), 0, logits, V, temperature, top_p, seed, counter, \
                out_ids, out_lp, top_k, top_ids, top_lp)
  if (dt == NMX_F16) NMX_SAMPLE(half);
  if (dt == NMX_BF16) NMX_SAMPLE(__nv_bfloat16);
  if (dt == NMX_F32) NMX_SAMPLE(float);
#undef NMX_SAMPLE
  NMX_CHECK(false, NMX_ERR_UNSUPPORTED, "sample: logits must be f16, bf16 or f32");
}

}  // namespace nmx
