// Small device ops around the hot path: RMSNorm, embedding gather, greedy
// sampling (plain and frequency-penalised), MLX-affine quantize/dequantize,
// seeded weight generation, KV block copies and the decode-loop bookkeeping.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace nmx {

namespace {

template <typename T>
__global__ void rmsnorm_kernel(const T* x, long ldx, const T* g, int H, float eps, T* y, long ldy) {
  __shared__ float s_red[32];
  grid_wait();
  const int row = blockIdx.x;
  const T* xr = x + long(row) * ldx;
  float ss = 0.f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    const float v = tof<T>(xr[i]);
    ss = fmaf(v, v, ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < blockDim.x / 32 ? s_red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (threadIdx.x == 0) s_red[0] = v;
  }
  __syncthreads();
  const float inv = 1.0f / sqrtf(s_red[0] / float(H) + eps);
  grid_launch_dependents();
  for (int i = threadIdx.x; i < H; i += blockDim.x)
    y[long(row) * ldy + i] = fromf<T>(tof<T>(xr[i]) * inv * tof<T>(g[i]));
}

// One row per CTA, 8 values per 16-byte load: every thread issues all its
// loads of x and g at once, so a row costs one round trip instead of a loop
// of dependent loads. Rows need H % 8 == 0 and 16-byte aligned pitches
// (rmsnorm() checks).
template <typename T, int CPT>
__global__ void rmsnorm_vec_kernel(const T* x, long ldx, const T* g, int H, float eps, T* y, long ldy) {
  __shared__ float s_red[32];
  const int H8 = H / 8, row = blockIdx.x;
  uint4 gv[CPT], xv[CPT];
  grid_wait();
  const uint4* xr = reinterpret_cast<const uint4*>(x + long(row) * ldx);
#pragma unroll
  for (int j = 0; j < CPT; ++j) {
    const int c = threadIdx.x + j * blockDim.x;
    if (c < H8) {
      xv[j] = xr[c];
      gv[j] = reinterpret_cast<const uint4*>(g)[c];
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < CPT; ++j) {
    const int c = threadIdx.x + j * blockDim.x;
    if (c < H8) {
      const T* e = reinterpret_cast<const T*>(&xv[j]);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float v = tof<T>(e[k]);
        ss = fmaf(v, v, ss);
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < blockDim.x / 32 ? s_red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (threadIdx.x == 0) s_red[0] = v;
  }
  __syncthreads();
  const float inv = 1.0f / sqrtf(s_red[0] / float(H) + eps);
  grid_launch_dependents();
  uint4* yr = reinterpret_cast<uint4*>(y + long(row) * ldy);
#pragma unroll
  for (int j = 0; j < CPT; ++j) {
    const int c = threadIdx.x + j * blockDim.x;
    if (c < H8) {
      const T* e = reinterpret_cast<const T*>(&xv[j]);
      const T* w = reinterpret_cast<const T*>(&gv[j]);
      uint4 o;
      T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
      for (int k = 0; k < 8; ++k) oe[k] = fromf<T>(tof<T>(e[k]) * inv * tof<T>(w[k]));
      yr[c] = o;
    }
  }
}

__global__ void embed_kernel(const uint4* table, const int* ids, int T, int H8, uint4* out) {
  grid_wait();
  const long n = long(T) * H8;
  for (long i = blockIdx.x * long(blockDim.x) + threadIdx.x; i < n; i += long(gridDim.x) * blockDim.x) {
    const long t = i / H8, c = i % H8;
    out[i] = table[long(ids[t]) * H8 + c];
  }
  grid_launch_dependents();
}

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}

template <typename T>
__device__ __forceinline__ float ld_logit(const void* p, long i) {
  return tof<T>(reinterpret_cast<const T*>(p)[i]);
}
template <>
__device__ __forceinline__ float ld_logit<float>(const void* p, long i) {
  return reinterpret_cast<const float*>(p)[i];
}

// penalised = 1: subtract penalty × (occurrences of the id in recent[row]).
template <typename T, bool PEN>
__global__ void argmax_kernel(const void* logits, int V, int* out, const int* recent,
                              const int* n_recent, int max_recent, float penalty) {
  __shared__ float s_v[32];
  __shared__ int s_i[32];
  __shared__ int s_ids[256];
  __shared__ int s_n;
  grid_wait();
  const int row = blockIdx.x;
  if (PEN) {
    if (threadIdx.x == 0) {
      int n = min(n_recent[row], min(max_recent, 256));
      for (int i = 0; i < n; ++i) s_ids[i] = recent[long(row) * max_recent + i];
      // insertion sort (n <= 256, one thread)
      for (int i = 1; i < n; ++i) {
        const int v = s_ids[i];
        int j = i - 1;
        while (j >= 0 && s_ids[j] > v) {
          s_ids[j + 1] = s_ids[j];
          --j;
        }
        s_ids[j + 1] = v;
      }
      s_n = n;
    }
    __syncthreads();
  }
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  int v0 = 0;  // first id of the scalar loop
  if constexpr (!PEN && sizeof(T) == 2) {
    // 16-bit logits, rows on 16-byte boundaries: eight ids per load
    const uint4* rp = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(logits) + long(row) * V);
    if (V % 8 == 0 && (reinterpret_cast<uintptr_t>(rp) & 15) == 0) {
      for (int v8 = threadIdx.x; v8 < V / 8; v8 += blockDim.x) {
        const uint4 w = rp[v8];
        const T* h = reinterpret_cast<const T*>(&w);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float x = tof<T>(h[j]);
          if (better(x, 8 * v8 + j, bv, bi)) {
            bv = x;
            bi = 8 * v8 + j;
          }
        }
      }
      v0 = V;
    }
  }
  for (int v = v0 + threadIdx.x; v < V; v += blockDim.x) {
    float x = ld_logit<T>(logits, long(row) * V + v);
    if (PEN) {
      // count occurrences by binary search for the first and last match
      int lo = 0, hi = s_n;
      while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (s_ids[mid] < v) lo = mid + 1; else hi = mid;
      }
      int cnt = 0;
      while (lo + cnt < s_n && s_ids[lo + cnt] == v) ++cnt;
      x = x - float(cnt) * penalty;
    }
    if (better(x, v, bv, bi)) {
      bv = x;
      bi = v;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(ov, oi, bv, bi)) {
      bv = ov;
      bi = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    s_v[threadIdx.x >> 5] = bv;
    s_i[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < int(blockDim.x / 32); ++w)
      if (better(s_v[w], s_i[w], bv, bi)) {
        bv = s_v[w];
        bi = s_i[w];
      }
    out[row] = bi == 0x7fffffff ? 0 : bi;
  }
  grid_launch_dependents();
}

// One thread per (row, group): min/max, fp32 scale/bias, round-half-even
// codes, packing low bits first. Identical rule to the oracle.
template <typename T, bool RANDOM>
__global__ void quantize_kernel(const float* w, int N, int K, int bits, int gs, uint32_t* wq, T* s,
                                T* b, uint64_t seed, uint64_t sid, float stdv);

__device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

// N(0,1) from the counter (seed, stream, index): Box-Muller on two 24-bit uniforms.
__device__ __forceinline__ float normal_at(uint64_t seed, uint64_t sid, uint64_t idx) {
  const uint64_t h = splitmix64(seed ^ splitmix64(sid * 0xD1B54A32D192ED03ull + idx));
  const float u1 = (float((h >> 40) & 0xFFFFFFu) + 1.0f) * (1.0f / 16777216.0f);
  const float u2 = float((h >> 16) & 0xFFFFFFu) * (1.0f / 16777216.0f);
  return sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
}

template <typename T, bool RANDOM>
__global__ void quantize_kernel(const float* w, int N, int K, int bits, int gs, uint32_t* wq, T* s,
                                T* b, uint64_t seed, uint64_t sid, float stdv) {
  grid_wait();
  const int ng = K / gs, vpw = 32 / bits, nbins = (1 << bits) - 1;
  const long total = long(N) * ng;
  float buf[128];
  for (long it = blockIdx.x * long(blockDim.x) + threadIdx.x; it < total; it += long(gridDim.x) * blockDim.x) {
    const long n = it / ng;
    const int g = int(it % ng);
    const long base = n * K + long(g) * gs;
    float mn = INFINITY, mx = -INFINITY;
    for (int i = 0; i < gs; ++i) {
      const float v = RANDOM ? stdv * normal_at(seed, sid, uint64_t(base + i)) : w[base + i];
      buf[i] = v;
      mn = fminf(mn, v);
      mx = fmaxf(mx, v);
    }
    const float scale = __fdiv_rn(mx - mn, float(nbins));
    const float bias = mn;
    s[it] = fromf<T>(scale);
    b[it] = fromf<T>(bias);
    uint32_t* dst = wq + (n * K + long(g) * gs) / vpw;
    for (int i = 0; i < gs; i += vpw) {
      uint32_t word = 0;
      for (int j = 0; j < vpw; ++j) {
        uint32_t q = 0;
        if (scale > 0.f) {
          float r = rintf(__fdiv_rn(buf[i + j] - bias, scale));
          r = fminf(fmaxf(r, 0.f), float(nbins));
          q = uint32_t(r);
        }
        word |= q << (j * bits);
      }
      dst[i / vpw] = word;
    }
  }
  grid_launch_dependents();
}

template <typename T>
__global__ void dequantize_kernel(const uint32_t* wq, const T* s, const T* b, int N, int K, int bits,
                                  int gs, float* w) {
  grid_wait();
  const long total = long(N) * K;
  const int vpw = 32 / bits, ng = K / gs;
  const uint32_t mask = (1u << bits) - 1u;
  for (long i = blockIdx.x * long(blockDim.x) + threadIdx.x; i < total; i += long(gridDim.x) * blockDim.x) {
    const long n = i / K;
    const int k = int(i % K);
    const uint32_t q = (wq[n * (K / vpw) + k / vpw] >> ((k % vpw) * bits)) & mask;
    w[i] = fmaf(float(q), tof<T>(s[n * ng + k / gs]), tof<T>(b[n * ng + k / gs]));
  }
  grid_launch_dependents();
}

template <typename T>
__global__ void random_fill_kernel(uint64_t seed, uint64_t sid, float stdv, float mean, long n, T* out) {
  grid_wait();
  for (long i = blockIdx.x * long(blockDim.x) + threadIdx.x; i < n; i += long(gridDim.x) * blockDim.x)
    out[i] = fromf<T>(mean + stdv * normal_at(seed, sid, uint64_t(i)));
  grid_launch_dependents();
}

template <typename T>
__global__ void fill_kernel(long n, float v, T* out) {
  grid_wait();
  for (long i = blockIdx.x * long(blockDim.x) + threadIdx.x; i < n; i += long(gridDim.x) * blockDim.x)
    out[i] = fromf<T>(v);
  grid_launch_dependents();
}

__global__ void copy_blocks_kernel(char* base, long layer_stride, long half_stride, long block_bytes,
                                   const int* src, const int* dst) {
  grid_wait();
  const int pair = blockIdx.x, part = blockIdx.y;  // part = layer * 2 + (0: K, 1: V)
  const long off = long(part / 2) * layer_stride + long(part % 2) * half_stride;
  const uint4* s4 = reinterpret_cast<const uint4*>(base + off + long(src[pair]) * block_bytes);
  uint4* d4 = reinterpret_cast<uint4*>(base + off + long(dst[pair]) * block_bytes);
  for (long i = threadIdx.x; i < block_bytes / 16; i += blockDim.x) d4[i] = s4[i];
  grid_launch_dependents();
}

__global__ void advance_kernel(int* pos, const int* tok, int B, int* hist, int hist_cap, int* step) {
  grid_wait();
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    const int st = *step;
    const bool room = hist && (long(st) + 1) * B <= long(hist_cap);
    for (int b = 0; b < B; ++b) {
      if (room) hist[long(st) * B + b] = tok[b];
      pos[b] += 1;
    }
    *step = st + 1;
  }
  grid_launch_dependents();
}

__global__ void seq_rows_kernel(const int* lens, int B, int* seq, int* pos) {
  grid_wait();
  for (int b = blockIdx.x * blockDim.x + threadIdx.x; b < B; b += gridDim.x * blockDim.x) {
    seq[b] = b;
    pos[b] = lens[b] - 1;
  }
  grid_launch_dependents();
}

inline int grid_for(long n, int threads, int num_sms) {
  long g = (n + threads - 1) / threads;
  return int(std::max<long>(1, std::min<long>(g, long(num_sms) * 16)));
}

}  // namespace

nmx_status_t rmsnorm(Ctx* c, const void* x, long ldx, const void* g, int M, int H, float eps,
                     nmx_dtype_t dt, void* y, long ldy) {
  if (M == 0) return NMX_OK;
  const bool vec = H % 8 == 0 && (ldx * 2) % 16 == 0 && (ldy * 2) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(x) % 16 == 0 && reinterpret_cast<uintptr_t>(y) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(g) % 16 == 0 && H / 8 <= 2 * 1024;
  if (vec && (dt == NMX_F16 || dt == NMX_BF16)) {
    const int H8 = H / 8;
    const int threads = std::min(1024, (H8 + 31) / 32 * 32);
    const bool two = H8 > threads;
    if (dt == NMX_F16)
      return two ? launch(c, rmsnorm_vec_kernel<half, 2>, dim3(M), dim3(threads), 0, (const half*)x, ldx,
                          (const half*)g, H, eps, (half*)y, ldy)
                 : launch(c, rmsnorm_vec_kernel<half, 1>, dim3(M), dim3(threads), 0, (const half*)x, ldx,
                          (const half*)g, H, eps, (half*)y, ldy);
    return two ? launch(c, rmsnorm_vec_kernel<__nv_bfloat16, 2>, dim3(M), dim3(threads), 0,
                        (const __nv_bfloat16*)x, ldx, (const __nv_bfloat16*)g, H, eps, (__nv_bfloat16*)y, ldy)
               : launch(c, rmsnorm_vec_kernel<__nv_bfloat16, 1>, dim3(M), dim3(threads), 0,
                        (const __nv_bfloat16*)x, ldx, (const __nv_bfloat16*)g, H, eps, (__nv_bfloat16*)y, ldy);
  }
  if (dt == NMX_F16)
    return launch(c, rmsnorm_kernel<half>, dim3(M), dim3(256), 0, (const half*)x, ldx, (const half*)g,
                  H, eps, (half*)y, ldy);
  if (dt == NMX_BF16)
    return launch(c, rmsnorm_kernel<__nv_bfloat16>, dim3(M), dim3(256), 0, (const __nv_bfloat16*)x,
                  ldx, (const __nv_bfloat16*)g, H, eps, (__nv_bfloat16*)y, ldy);
  NMX_CHECK(false, NMX_ERR_UNSUPPORTED, "rmsnorm: dtype must be f16 or bf16");
}

nmx_status_t embed_rows(Ctx* c, const void* table, const int* ids, int T, int H, void* out) {
  NMX_CHECK(H % 8 == 0, NMX_ERR_UNSUPPORTED, "embedding: hidden must be a multiple of 8");
  if (T == 0) return NMX_OK;
  const long n = long(T) * (H / 8);
  return launch(c, embed_kernel, dim3(grid_for(n, 256, c->num_sms)), dim3(256), 0,
                (const uint4*)table, ids, T, H / 8, (uint4*)out);
}

nmx_status_t argmax_rows(Ctx* c, const void* logits, int M, int V, nmx_dtype_t dt, int* out) {
  if (M == 0) return NMX_OK;
  NMX_CHECK(V > 0, NMX_ERR_INVALID, "argmax: empty vocabulary");
  if (dt == NMX_F16)
    return launch(c, argmax_kernel<half, false>, dim3(M), dim3(1024), 0, logits, V, out,
                  (const int*)nullptr, (const int*)nullptr, 0, 0.f);
  if (dt == NMX_BF16)
    return launch(c, argmax_kernel<__nv_bfloat16, false>, dim3(M), dim3(1024), 0, logits, V, out,
                  (const int*)nullptr, (const int*)nullptr, 0, 0.f);
  if (dt == NMX_F32)
    return launch(c, argmax_kernel<float, false>, dim3(M), dim3(1024), 0, logits, V, out,
                  (const int*)nullptr, (const int*)nullptr, 0, 0.f);
  NMX_CHECK(false, NMX_ERR_UNSUPPORTED, "argmax: dtype must be f16, bf16 or f32");
}

nmx_status_t penalized_argmax(Ctx* c, const void* logits, int M, int V, nmx_dtype_t dt,
                              const int* recent, const int* n_recent, int max_recent,
                              float penalty, int* out) {
  if (M == 0) return NMX_OK;
  NMX_CHECK(max_recent <= 256, NMX_ERR_UNSUPPORTED, "penalized argmax: at most 256 recent ids");
  if (dt == NMX_F16)
    return launch(c, argmax_kernel<half, true>, dim3(M), dim3(1024), 0, logits, V, out, recent,
                  n_recent, max_recent, penalty);
  if (dt == NMX_BF16)
    return launch(c, argmax_kernel<__nv_bfloat16, true>, dim3(M), dim3(1024), 0, logits, V, out,
                  recent, n_recent, max_recent, penalty);
  if (dt == NMX_F32)
    return launch(c, argmax_kernel<float, true>, dim3(M), dim3(1024), 0, logits, V, out, recent,
                  n_recent, max_recent, penalty);
  NMX_CHECK(false, NMX_ERR_UNSUPPORTED, "penalized argmax: dtype must be f16, bf16 or f32");
}

static nmx_status_t check_quant(int N, int K, int bits, int gs) {
  NMX_CHECK(N >= 0 && K > 0, NMX_ERR_INVALID, "quantize: bad shape");
  NMX_CHECK(bits == 4 || bits == 8, NMX_ERR_UNSUPPORTED, "quantize: bits must be 4 or 8");
  NMX_CHECK(gs == 32 || gs == 64 || gs == 128, NMX_ERR_UNSUPPORTED, "quantize: group must be 32/64/128");
  NMX_CHECK(K % gs == 0, NMX_ERR_UNSUPPORTED, "quantize: K must be a multiple of the group size");
  return NMX_OK;
}

template <typename T, bool RANDOM>
static nmx_status_t quant_t(Ctx* c, const float* w, int N, int K, int bits, int gs, uint32_t* wq, void* s,
                            void* b, uint64_t seed, uint64_t sid, float stdv) {
  const long groups = long(N) * (K / gs);
  if (groups == 0) return NMX_OK;
  return launch(c, quantize_kernel<T, RANDOM>, dim3(grid_for(groups, 128, c->num_sms)), dim3(128), 0, w,
                N, K, bits, gs, wq, (T*)s, (T*)b, seed, sid, stdv);
}

nmx_status_t quantize(Ctx* c, const float* w, int N, int K, int bits, int gs, nmx_dtype_t sdt,
                      uint32_t* wq, void* s, void* b) {
  NMX_TRY(check_quant(N, K, bits, gs));
  if (sdt == NMX_F16) return quant_t<half, false>(c, w, N, K, bits, gs, wq, s, b, 0, 0, 0.f);
  if (sdt == NMX_BF16) return quant_t<__nv_bfloat16, false>(c, w, N, K, bits, gs, wq, s, b, 0, 0, 0.f);
  NMX_CHECK(false, NMX_ERR_UNSUPPORTED, "quantize: scale dtype must be f16 or bf16");
}

nmx_status_t random_quantized(Ctx* c, uint64_t seed, uint64_t sid, float stdv, int N, int K, int bits,
                              int gs, nmx_dtype_t sdt, uint32_t* wq, void* s, void* b) {
  NMX_TRY(check_quant(N, K, bits, gs));
  if (sdt == NMX_F16) return quant_t<half, true>(c, nullptr, N, K, bits, gs, wq, s, b, seed, sid, stdv);
  if (sdt == NMX_BF16)
    return quant_t<__nv_bfloat16, true>(c, nullptr, N, K, bits, gs, wq, s, b, seed, sid, stdv);
  NMX_CHECK(false, NMX_ERR_UNSUPPORTED, "quantize: scale dtype must be f16 or bf16");
}

nmx_status_t dequantize(Ctx* c, const uint32_t* wq, const void* s, const void* b, int N, int K, int bits,
                        int gs, nmx_dtype_t sdt, float* w) {
  NMX_TRY(check_quant(N, K, bits, gs));
  const long n = long(N) * K;
  if (n == 0) return NMX_OK;
  if (sdt == NMX_F16)
    return launch(c, dequantize_kernel<half>, dim3(grid_for(n, 256, c->num_sms)), dim3(256), 0, wq,
                  (const half*)s, (const half*)b, N, K, bits, gs, w);
  if (sdt == NMX_BF16)
    return launch(c, dequantize_kernel<__nv_bfloat16>, dim3(grid_for(n, 256, c->num_sms)), dim3(256), 0,
                  wq, (const __nv_bfloat16*)s, (const __nv_bfloat16*)b, N, K, bits, gs, w);
  NMX_CHECK(false, NMX_ERR_UNSUPPORTED, "dequantize: scale dtype must be f16 or bf16");
}

nmx_status_t random_fill(Ctx* c, uint64_t seed, uint64_t sid, float stdv, float mean, size_t n,
                         nmx_dtype_t dt, void* out) {
  if (n == 0) return NMX_OK;
  const int grid = grid_for(long(n), 256, c->num_sms);
  if (dt == NMX_F16)
    return launch(c, random_fill_kernel<half>, dim3(grid), dim3(256), 0, seed, sid, stdv, mean, long(n),
                  (half*)out);
  if (dt == NMX_BF16)
    return launch(c, random_fill_kernel<__nv_bfloat16>, dim3(grid), dim3(256), 0, seed, sid, stdv, mean,
                  long(n), (__nv_bfloat16*)out);
  NMX_CHECK(false, NMX_ERR_UNSUPPORTED, "random fill: dtype must be f16 or bf16");
}

nmx_status_t fill_value(Ctx* c, size_t n, float v, nmx_dtype_t dt, void* out) {
  if (n == 0) return NMX_OK;
  const int grid = grid_for(long(n), 256, c->num_sms);
  if (dt == NMX_F16) return launch(c, fill_kernel<half>, dim3(grid), dim3(256), 0, long(n), v, (half*)out);
  if (dt == NMX_BF16)
    return launch(c, fill_kernel<__nv_bfloat16>, dim3(grid), dim3(256), 0, long(n), v, (__nv_bfloat16*)out);
  NMX_CHECK(false, NMX_ERR_UNSUPPORTED, "fill: dtype must be f16 or bf16");
}

nmx_status_t copy_kv_blocks(Ctx* c, void* base, long layer_stride_bytes, int layers, long block_bytes,
                            const int* src, const int* dst, int n) {
  if (n == 0) return NMX_OK;
  NMX_CHECK(block_bytes % 16 == 0, NMX_ERR_INVALID, "kv copy: block bytes must be 16-aligned");
  return launch(c, copy_blocks_kernel, dim3(n, layers * 2), dim3(256), 0, (char*)base, layer_stride_bytes,
                layer_stride_bytes / 2, block_bytes, src, dst);
}

nmx_status_t seq_rows_from_lens(Ctx* c, const int* lens, int B, int* seq, int* pos) {
  return launch(c, seq_rows_kernel, dim3((B + 255) / 256), dim3(256), 0, lens, B, seq, pos);
}

nmx_status_t decode_advance(Ctx* c, int* pos, const int* tok, int B, int* history, int hist_cap, int* step) {
  return launch(c, advance_kernel, dim3(1), dim3(32), 0, pos, tok, B, history, hist_cap, step);
}

}  // namespace nmx
