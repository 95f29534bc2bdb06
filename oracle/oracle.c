/*
 * oracle.c — CPU restatement of NovaMLX's decode/prefill hot-path arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the checker for the CUDA library and
 * the timed CPU baseline; nothing in the product links or calls it. Only
 * tests/, __graft_entry__.smoke() and bench.py's CPU legs load liboracle.so.
 *
 * What it restates, and from where:
 *   - MLX-affine quantize / dequantize / quantized matmul (transpose = true).
 *     The arithmetic lives in ml-explore/mlx-swift 0.31.3 (pinned at
 *     DEVELOPMENT.md:47 and PATCHES.md:98 of the reference; not vendored in
 *     the reference tree). Call sites: Sources/NovaMLXEngine/Models/
 *     BailingHybridModel.swift:179 (quantized), :213 (quantizedMM), :816
 *     (dequantized), :812-815 (group-size relation K/(32/bits) words, K/gs
 *     groups). Nibble order and dequant formula are pinned by the
 *     reference's own kernel: FusedQuantizedSDPA.swift:77-81,95-99
 *     (word = d / values_per_word; shift = (d % values_per_word) * bits;
 *     ((w >> shift) & mask) * s + b). The quantization rule is the one the
 *     workload definition states: scale = (max-min)/(2^bits-1), bias = min,
 *     q = clamp(round_half_even((w-bias)/scale)), fp16 scale/bias.
 *   - Single-query attention over affine-quantized K/V:
 *     Sources/NovaMLXEngine/FusedQuantizedSDPA.swift:17-135 (GQA head map
 *     :45, causal rule :70, online softmax :84-101, sum==0 guard :125).
 *   - Llama / Qwen2 forward (mlx-swift-lm 2.31.3, not vendored): embed →
 *     L × [RMSNorm → q,k,v (+bias) → RoPE (non-traditional, rotate-half) →
 *     SDPA (GQA, causal, scale 1/sqrt(head_dim)) → o → +res → RMSNorm →
 *     gate,up → silu(gate)*up → down → +res] → RMSNorm → lm_head. Values are
 *     rounded to the activation dtype at the points MLX materialises arrays
 *     (after every linear, bias add, RoPE, attention, residual add, norm,
 *     silu and gating multiply). RoPE frequencies follow Llama-3.1's
 *     "llama3" scaling when rope_factor > 0.
 *   - Quantized KV cache (the kvBits path: TurboQuantService.
 *     applyToGenerateParameters, Sources/NovaMLXEngine/TurboQuantCache.swift:
 *     78-104, which turns on mlx-swift-lm's quantized KV cache): with
 *     kv_bits > 0 every appended K row (after RoPE) and V row is quantized by
 *     the rule above in groups of kv_gs along head_dim and stored
 *     dequantized (w = q * s + b with the f16 scale and bias); attention
 *     then reads those values.
 *   - Greedy sampling: argmax, lowest index on ties
 *     (Sources/NovaMLXEngine/CompiledSampler.swift:24-27) and the frequency
 *     penalty (Sources/NovaMLXEngine/FusedBatchScheduler.swift:1218-1227).
 *
 * Parity status: the integer parts (packing, nibble order, quantization
 * codes, block indexing, argmax ids) are pinned by known-answer vectors
 * derived from the reference source (tests/golden). The floating-point
 * parts are parity UNPINNED against MLX itself: the reference ships no
 * numeric golden tensors and MLX cannot run in this environment, so this
 * restatement is the contract, checked by two independent implementations
 * (this file and tests/oracle_np.py).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define EXPORT __attribute__((visibility("default")))

/* ---------------------------------------------------------------- dtypes */
/* dt: 0 = f16, 1 = bf16, 2 = f32 (argmax only). */

static float h2f(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1fu;
  uint32_t mant = h & 0x3ffu;
  uint32_t x;
  if (exp == 0) {
    float v = ldexpf((float)mant, -24);
    return (h & 0x8000u) ? -v : v;
  } else if (exp == 31) {
    x = sign | 0x7f800000u | (mant << 13);
  } else {
    x = sign | ((exp + 112u) << 23) | (mant << 13);
  }
  float f;
  memcpy(&f, &x, 4);
  return f;
}

static uint16_t f2h(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t mant = x & 0x7fffffu;
  int exp = (int)((x >> 23) & 0xffu);
  if (exp == 0xff) return (uint16_t)(sign | 0x7c00u | (mant ? 0x200u : 0u));
  int e = exp - 127 + 15;
  if (e >= 31) return (uint16_t)(sign | 0x7c00u);
  if (e <= 0) {
    if (exp == 0) return (uint16_t)sign; /* fp32 subnormal → 0 */
    uint32_t m = mant | 0x800000u;
    int shift = 14 - e;
    if (shift > 24) return (uint16_t)sign;
    uint32_t h = m >> shift;
    uint32_t rem = m & ((1u << shift) - 1u);
    uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (h & 1u))) h++;
    return (uint16_t)(sign | h);
  }
  uint32_t h = ((uint32_t)e << 10) | (mant >> 13);
  uint32_t rem = mant & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
  return (uint16_t)(sign | h);
}

static float bf2f(uint16_t b) {
  uint32_t x = (uint32_t)b << 16;
  float f;
  memcpy(&f, &x, 4);
  return f;
}

static uint16_t f2bf(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  if ((x & 0x7f800000u) == 0x7f800000u && (x & 0x7fffffu)) return (uint16_t)((x >> 16) | 0x40u);
  x += 0x7fffu + ((x >> 16) & 1u);
  return (uint16_t)(x >> 16);
}

/* f16 → f32 through a table built from h2f (same values, faster). */
static float g_h2f_table[65536];
static int g_h2f_ready = 0;
static void h2f_table_init(void) {
  if (g_h2f_ready) return;
  for (uint32_t i = 0; i < 65536u; ++i) g_h2f_table[i] = h2f((uint16_t)i);
  g_h2f_ready = 1;
}
__attribute__((constructor)) static void oracle_init(void) { h2f_table_init(); }

static inline float ldv(const uint16_t* p, size_t i, int dt) {
  return dt == 1 ? bf2f(p[i]) : g_h2f_table[p[i]];
}
static inline uint16_t stv(float v, int dt) { return dt == 1 ? f2bf(v) : f2h(v); }
static inline float rnd(float v, int dt) { return ldv((uint16_t[]){stv(v, dt)}, 0, dt); }

EXPORT float oracle_h2f(uint16_t h) { return h2f(h); }
EXPORT uint16_t oracle_f2h(float f) { return f2h(f); }
EXPORT float oracle_bf2f(uint16_t h) { return bf2f(h); }
EXPORT uint16_t oracle_f2bf(float f) { return f2bf(f); }

EXPORT void oracle_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

EXPORT int oracle_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* ------------------------------------------------------- quantization */

/* Affine quantization along K; see the file header for the rule. */
EXPORT void oracle_quantize(const float* w, int N, int K, int bits, int gs, int sdt, uint32_t* wq,
                            uint16_t* s, uint16_t* b) {
  const int vpw = 32 / bits;
  const int nbins = (1 << bits) - 1;
  const int ng = K / gs;
  const int wpr = K / vpw;
#pragma omp parallel for schedule(static)
  for (int n = 0; n < N; ++n) {
    for (int g = 0; g < ng; ++g) {
      const float* src = w + (size_t)n * K + (size_t)g * gs;
      float mn = src[0], mx = src[0];
      for (int i = 1; i < gs; ++i) {
        mn = src[i] < mn ? src[i] : mn;
        mx = src[i] > mx ? src[i] : mx;
      }
      float scale = (mx - mn) / (float)nbins;
      float bias = mn;
      s[(size_t)n * ng + g] = stv(scale, sdt);
      b[(size_t)n * ng + g] = stv(bias, sdt);
      for (int i = 0; i < gs; i += vpw) {
        uint32_t word = 0;
        for (int j = 0; j < vpw; ++j) {
          uint32_t q = 0;
          if (scale > 0.0f) {
            float r = rintf((src[i + j] - bias) / scale);
            r = r < 0.0f ? 0.0f : (r > (float)nbins ? (float)nbins : r);
            q = (uint32_t)r;
          }
          word |= q << (j * bits);
        }
        wq[(size_t)n * wpr + (size_t)(g * gs + i) / vpw] = word;
      }
    }
  }
}

/* Unpack value k of a packed row (FusedQuantizedSDPA.swift:79-81). */
static inline uint32_t unpack(const uint32_t* row, int k, int bits) {
  const int vpw = 32 / bits;
  return (row[k / vpw] >> ((k % vpw) * bits)) & ((1u << bits) - 1u);
}

EXPORT void oracle_unpack(const uint32_t* wq, int N, int K, int bits, uint8_t* q) {
  const int wpr = K * bits / 32;
  for (int n = 0; n < N; ++n)
    for (int k = 0; k < K; ++k) q[(size_t)n * K + k] = (uint8_t)unpack(wq + (size_t)n * wpr, k, bits);
}

EXPORT void oracle_dequantize(const uint32_t* wq, const uint16_t* s, const uint16_t* b, int N, int K,
                              int bits, int gs, int sdt, float* w) {
  const int wpr = K * bits / 32;
  const int ng = K / gs;
#pragma omp parallel for schedule(static)
  for (int n = 0; n < N; ++n)
    for (int k = 0; k < K; ++k) {
      float sc = ldv(s, (size_t)n * ng + k / gs, sdt);
      float bi = ldv(b, (size_t)n * ng + k / gs, sdt);
      w[(size_t)n * K + k] = fmaf((float)unpack(wq + (size_t)n * wpr, k, bits), sc, bi);
    }
}

/* y[m,n] = Σ_k x[m,k]·(q·s+b), fp32 accumulation (per group, then across
 * groups), rounded to dt. x is [M,K] in dt. Parallel over n. */
static void qmm_f32(const float* xf, const uint32_t* wq, const uint16_t* s, const uint16_t* b, int M,
                    int N, int K, int bits, int gs, int dt, float* yf) {
  const int wpr = K * bits / 32;
  const int ng = K / gs;
  const int vpw = 32 / bits;
  const uint32_t mask = (1u << bits) - 1u;
#pragma omp parallel
  {
    float wbuf[256];
    float accm[64];
#pragma omp for schedule(static)
    for (int n = 0; n < N; ++n) {
      const uint32_t* row = wq + (size_t)n * wpr;
      for (int m0 = 0; m0 < M; m0 += 64) {
        int mc = M - m0 < 64 ? M - m0 : 64;
        for (int m = 0; m < mc; ++m) accm[m] = 0.0f;
        for (int g = 0; g < ng; ++g) {
          float sc = ldv(s, (size_t)n * ng + g, dt), bi = ldv(b, (size_t)n * ng + g, dt);
          for (int i = 0; i < gs; ++i) {
            int k = g * gs + i;
            wbuf[i] = fmaf((float)((row[k / vpw] >> ((k % vpw) * bits)) & mask), sc, bi);
          }
          for (int m = 0; m < mc; ++m) {
            const float* xr = xf + (size_t)(m0 + m) * K + (size_t)g * gs;
            float part = 0.0f;
            for (int i = 0; i < gs; ++i) part += xr[i] * wbuf[i];
            accm[m] += part;
          }
        }
        for (int m = 0; m < mc; ++m) yf[(size_t)(m0 + m) * N + n] = accm[m];
      }
    }
  }
}

EXPORT void oracle_qmatmul(const uint16_t* x, const uint32_t* wq, const uint16_t* s, const uint16_t* b,
                           int M, int N, int K, int bits, int gs, int dt, uint16_t* y) {
  float* xf = (float*)malloc(sizeof(float) * (size_t)M * K);
  float* yf = (float*)malloc(sizeof(float) * (size_t)M * N);
  for (size_t i = 0; i < (size_t)M * K; ++i) xf[i] = ldv(x, i, dt);
  qmm_f32(xf, wq, s, b, M, N, K, bits, gs, dt, yf);
  for (size_t i = 0; i < (size_t)M * N; ++i) y[i] = stv(yf[i], dt);
  free(xf);
  free(yf);
}

/* ------------------------------------------------------------ small ops */

EXPORT void oracle_rmsnorm(const uint16_t* x, const uint16_t* g, int M, int H, float eps, int dt,
                           uint16_t* y) {
  for (int m = 0; m < M; ++m) {
    float ss = 0.0f;
    for (int i = 0; i < H; ++i) {
      float v = ldv(x, (size_t)m * H + i, dt);
      ss += v * v;
    }
    float inv = 1.0f / sqrtf(ss / (float)H + eps);
    for (int i = 0; i < H; ++i)
      y[(size_t)m * H + i] = stv(ldv(x, (size_t)m * H + i, dt) * inv * ldv(g, i, dt), dt);
  }
}

/* RoPE inverse frequencies, D/2 of them, in double then rounded to float.
 * With factor > 0 applies Llama-3.1's "llama3" rescaling (wavelength bands
 * split at orig/low and orig/high; linear blend in between). */
EXPORT void oracle_rope_inv_freq(int D, float theta, float factor, float low, float high, int orig,
                                 float* inv_freq) {
  for (int i = 0; i < D / 2; ++i) {
    double f = 1.0 / pow((double)theta, (2.0 * i) / (double)D);
    if (factor > 0.0f) {
      double low_wl = (double)orig / (double)low;
      double high_wl = (double)orig / (double)high;
      double wl = 2.0 * M_PI / f;
      if (wl < high_wl) {
        /* unchanged */
      } else if (wl > low_wl) {
        f = f / (double)factor;
      } else {
        double smooth = ((double)orig / wl - (double)low) / ((double)high - (double)low);
        f = (1.0 - smooth) * f / (double)factor + smooth * f;
      }
    }
    inv_freq[i] = (float)f;
  }
}

/* In place on x[T, H, D] (rotate-half form): for i < D/2, angle =
 * pos[t]*inv_freq[i] (fp32), (a, b) = (x[i], x[i+D/2]) →
 * (a cos - b sin, b cos + a sin). */
EXPORT void oracle_rope(uint16_t* x, int T, int H, int D, const int32_t* pos, const float* inv_freq,
                        int dt) {
  const int half = D / 2;
  for (int t = 0; t < T; ++t)
    for (int h = 0; h < H; ++h) {
      uint16_t* r = x + ((size_t)t * H + h) * D;
      for (int i = 0; i < half; ++i) {
        float ang = (float)pos[t] * inv_freq[i];
        float c = cosf(ang), sn = sinf(ang);
        float a = ldv(r, i, dt), bb = ldv(r, i + half, dt);
        r[i] = stv(a * c - bb * sn, dt);
        r[i + half] = stv(bb * c + a * sn, dt);
      }
    }
}

/* Causal GQA attention. q [T, Hq, D] at positions q_start.., k/v [S, Hkv, D]
 * holding positions 0..S-1. Query t sees keys j <= q_start + t. */
EXPORT void oracle_attention(const uint16_t* q, const uint16_t* k, const uint16_t* v, int T, int Hq,
                             int Hkv, int D, int S, int q_start, float scale, int dt, uint16_t* out) {
  const int rep = Hq / Hkv;
#pragma omp parallel for collapse(2) schedule(static)
  for (int t = 0; t < T; ++t)
    for (int hq = 0; hq < Hq; ++hq) {
      const int hk = hq / rep;
      int last = q_start + t;
      if (last > S - 1) last = S - 1;
      float* sc = (float*)malloc(sizeof(float) * (size_t)(last + 1));
      float* o = (float*)calloc((size_t)D, sizeof(float));
      float mx = -INFINITY;
      for (int j = 0; j <= last; ++j) {
        float acc = 0.0f;
        for (int d = 0; d < D; ++d)
          acc += ldv(q, ((size_t)t * Hq + hq) * D + d, dt) * ldv(k, ((size_t)j * Hkv + hk) * D + d, dt);
        sc[j] = acc * scale;
        mx = sc[j] > mx ? sc[j] : mx;
      }
      float l = 0.0f;
      for (int j = 0; j <= last; ++j) {
        float p = expf(sc[j] - mx);
        l += p;
        for (int d = 0; d < D; ++d) o[d] += p * ldv(v, ((size_t)j * Hkv + hk) * D + d, dt);
      }
      for (int d = 0; d < D; ++d) out[((size_t)t * Hq + hq) * D + d] = stv(o[d] / l, dt);
      free(sc);
      free(o);
    }
}

/* The reference's quantized-KV vector kernel (FusedQuantizedSDPA.swift:17-135),
 * restated per query row. q [BH, L, D]; k_w/v_w [BHkv, N, D*bits/32];
 * scales/biases [BHkv, N, D/gs]. Out [BH, L, D] in dt. */
EXPORT void oracle_quantized_sdpa(const uint16_t* q, const uint32_t* kw, const uint16_t* ks,
                                  const uint16_t* kb, const uint32_t* vw, const uint16_t* vs,
                                  const uint16_t* vb, int BH, int gqa, int N, int L, int D,
                                  float scale, int gs, int bits, int dt, uint16_t* out) {
  const int wstride = D * bits / 32;
  const int sstride = D / gs;
  for (int bh = 0; bh < BH; ++bh) {
    const int kvh = bh / gqa; /* :45 */
    for (int l = 0; l < L; ++l) {
      float* qv = (float*)malloc(sizeof(float) * (size_t)D);
      float* o = (float*)calloc((size_t)D, sizeof(float));
      for (int d = 0; d < D; ++d) qv[d] = scale * ldv(q, ((size_t)bh * L + l) * D + d, dt);
      float mx = -1e30f, sum = 0.0f;
      for (int i = 0; i < N; ++i) {
        if (!(i <= N - L + l)) continue; /* :70 */
        const uint32_t* kr = kw + ((size_t)kvh * N + i) * wstride;
        const uint32_t* vr = vw + ((size_t)kvh * N + i) * wstride;
        float score = 0.0f;
        for (int d = 0; d < D; ++d) {
          size_t si = ((size_t)kvh * N + i) * sstride + d / gs;
          score += qv[d] * ((float)unpack(kr, d, bits) * ldv(ks, si, dt) + ldv(kb, si, dt));
        }
        float nm = score > mx ? score : mx;
        float factor = expf(mx - nm);
        float e = expf(score - nm);
        mx = nm;
        sum = sum * factor + e;
        for (int d = 0; d < D; ++d) {
          size_t si = ((size_t)kvh * N + i) * sstride + d / gs;
          float dv = (float)unpack(vr, d, bits) * ldv(vs, si, dt) + ldv(vb, si, dt);
          o[d] = o[d] * factor + e * dv;
        }
      }
      for (int d = 0; d < D; ++d)
        out[((size_t)bh * L + l) * D + d] = stv(sum == 0.0f ? o[d] : o[d] / sum, dt); /* :125 */
      free(qv);
      free(o);
    }
  }
}

static inline float ld_any(const void* p, size_t i, int dt) {
  if (dt == 2) return ((const float*)p)[i];
  return ldv((const uint16_t*)p, i, dt);
}

/* argmax, lowest index on ties; NaN never wins. */
EXPORT void oracle_argmax(const void* logits, int M, int V, int dt, int32_t* out) {
  for (int m = 0; m < M; ++m) {
    int best = 0;
    float bv = -INFINITY;
    for (int v = 0; v < V; ++v) {
      float x = ld_any(logits, (size_t)m * V + v, dt);
      if (x > bv) {
        bv = x;
        best = v;
      }
    }
    out[m] = best;
  }
}

/* logits - penalty*histogram(recent) → argmax (FusedBatchScheduler.swift:1218-1227).
 * The subtraction is done in fp32 on the fp32 value of each logit. */
EXPORT void oracle_penalized_argmax(const void* logits, int M, int V, int dt, const int32_t* recent,
                                    const int32_t* n_recent, int max_recent, float penalty,
                                    int32_t* out) {
  float* row = (float*)malloc(sizeof(float) * (size_t)V);
  for (int m = 0; m < M; ++m) {
    for (int v = 0; v < V; ++v) row[v] = ld_any(logits, (size_t)m * V + v, dt);
    float* hist = (float*)calloc((size_t)V, sizeof(float));
    for (int i = 0; i < n_recent[m]; ++i) {
      int id = recent[(size_t)m * max_recent + i];
      if (id >= 0 && id < V) hist[id] += 1.0f;
    }
    int best = 0;
    float bv = -INFINITY;
    for (int v = 0; v < V; ++v) {
      float x = row[v] - hist[v] * penalty;
      if (x > bv) {
        bv = x;
        best = v;
      }
    }
    out[m] = best;
    free(hist);
  }
  free(row);
}

/* The same causal GQA attention as oracle_attention, reading K/V straight
 * from a [Hkv, max_ctx, D] cache (one sequence). */
static void attn_cache(const uint16_t* q, const uint16_t* KC, const uint16_t* VC, int max_ctx, int T,
                       int Hq, int Hkv, int D, int q_start, float scale, int dt, uint16_t* out) {
  const int rep = Hq / Hkv;
#pragma omp parallel for collapse(2) schedule(static)
  for (int t = 0; t < T; ++t)
    for (int hq = 0; hq < Hq; ++hq) {
      const int hk = hq / rep;
      const int last = q_start + t;
      float* sc = (float*)malloc(sizeof(float) * (size_t)(last + 1));
      float* o = (float*)calloc((size_t)D, sizeof(float));
      float* qf = (float*)malloc(sizeof(float) * (size_t)D);
      float* kv = (float*)malloc(sizeof(float) * (size_t)D);
      for (int d = 0; d < D; ++d) qf[d] = ldv(q, ((size_t)t * Hq + hq) * D + d, dt);
      float mx = -INFINITY;
      for (int j = 0; j <= last; ++j) {
        const uint16_t* kr = KC + ((size_t)hk * max_ctx + j) * D;
        for (int d = 0; d < D; ++d) kv[d] = ldv(kr, d, dt);
        float acc = 0.0f;
        for (int d = 0; d < D; ++d) acc += qf[d] * kv[d];
        sc[j] = acc * scale;
        mx = sc[j] > mx ? sc[j] : mx;
      }
      float l = 0.0f;
      for (int j = 0; j <= last; ++j) {
        float p = expf(sc[j] - mx);
        l += p;
        const uint16_t* vr = VC + ((size_t)hk * max_ctx + j) * D;
        for (int d = 0; d < D; ++d) kv[d] = ldv(vr, d, dt);
        for (int d = 0; d < D; ++d) o[d] += p * kv[d];
      }
      for (int d = 0; d < D; ++d) out[((size_t)t * Hq + hq) * D + d] = stv(o[d] / l, dt);
      free(sc); free(o); free(qf); free(kv);
    }
}

/* ------------------------------------------------------------ the model */

typedef struct {
  int vocab, hidden, n_layers, n_heads, n_kv_heads, head_dim, ffn, bits, gs, dt, qkv_bias, tie;
  float eps;
  const float* inv_freq;      /* [head_dim/2] */
  const uint16_t* embed;      /* [V, H] */
  const uint16_t* final_norm; /* [H] */
  const uint32_t* lm_w;       /* [V, H*bits/32] (ignored when tie) */
  const uint16_t* lm_s;
  const uint16_t* lm_b;
  const uint16_t* attn_norm; /* [L, H] */
  const uint16_t* mlp_norm;  /* [L, H] */
  const uint32_t *q_w, *k_w, *v_w, *o_w, *g_w, *u_w, *d_w;
  const uint16_t *q_s, *k_s, *v_s, *o_s, *g_s, *u_s, *d_s;
  const uint16_t *q_b, *k_b, *v_b, *o_b, *g_b, *u_b, *d_b;
  const uint16_t *q_bias, *k_bias, *v_bias; /* [L, n] or NULL */
  int kv_bits, kv_gs;                        /* quantized KV cache (0: f16 cache) */
} oracle_model_t;

/* One cached K or V row quantized and dequantized in place: groups of gs
 * along the row, scale = (max-min)/(2^bits-1) and bias = min in fp32 for
 * the codes, the row rebuilt from the codes with the f16 scale and bias. */
static void qdq_row(uint16_t* row, int D, int bits, int gs, int dt) {
  const int nbins = (1 << bits) - 1;
  for (int g = 0; g < D / gs; ++g) {
    uint16_t* r = row + (size_t)g * gs;
    float mn = ldv(r, 0, dt), mx = mn;
    for (int i = 1; i < gs; ++i) {
      const float v = ldv(r, i, dt);
      mn = v < mn ? v : mn;
      mx = v > mx ? v : mx;
    }
    const float scale = (mx - mn) / (float)nbins, bias = mn;
    const float s16 = rnd(scale, dt), b16 = rnd(bias, dt);
    for (int i = 0; i < gs; ++i) {
      float q = 0.0f;
      if (scale > 0.0f) {
        q = rintf((ldv(r, i, dt) - bias) / scale);
        q = q < 0.0f ? 0.0f : (q > (float)nbins ? (float)nbins : q);
      }
      r[i] = stv(fmaf(q, s16, b16), dt);
    }
  }
}

static void linear(const oracle_model_t* m, const float* x, int T, const uint32_t* w, const uint16_t* s,
                   const uint16_t* b, int N, int K, const uint16_t* bias, float* y) {
  qmm_f32(x, w, s, b, T, N, K, m->bits, m->gs, m->dt, y);
  for (size_t i = 0; i < (size_t)T * N; ++i) {
    float v = rnd(y[i], m->dt);
    if (bias) v = rnd(v + ldv(bias, i % (size_t)N, m->dt), m->dt);
    y[i] = v;
  }
}

static void rmsnorm_f(const float* x, const uint16_t* g, int T, int H, float eps, int dt, float* y) {
  for (int t = 0; t < T; ++t) {
    float ss = 0.0f;
    for (int i = 0; i < H; ++i) ss += x[(size_t)t * H + i] * x[(size_t)t * H + i];
    float inv = 1.0f / sqrtf(ss / (float)H + eps);
    for (int i = 0; i < H; ++i) y[(size_t)t * H + i] = rnd(x[(size_t)t * H + i] * inv * ldv(g, i, dt), dt);
  }
}

/* One forward over T tokens of one sequence starting at start_pos.
 * kcache/vcache: [L, Hkv, max_ctx, D] in dt (the KVCacheSimple layout);
 * positions < start_pos must already be filled. logits: fp32 [T, V] when
 * all_logits, else [V] for the last token. */
EXPORT int oracle_forward(const oracle_model_t* m, uint16_t* kcache, uint16_t* vcache, int max_ctx,
                          const int32_t* tokens, int T, int start_pos, float* logits, int all_logits) {
  const int H = m->hidden, L = m->n_layers, Hq = m->n_heads, Hkv = m->n_kv_heads, D = m->head_dim;
  const int F = m->ffn, V = m->vocab, dt = m->dt;
  const int Nq = Hq * D, Nkv = Hkv * D;
  const size_t wpr_h = (size_t)H * m->bits / 32, wpr_q = (size_t)Nq * m->bits / 32;
  const size_t wpr_f = (size_t)F * m->bits / 32;
  const size_t ng_h = (size_t)H / m->gs, ng_q = (size_t)Nq / m->gs, ng_f = (size_t)F / m->gs;
  if (start_pos + T > max_ctx) return -1;

  float* h = (float*)malloc(sizeof(float) * (size_t)T * H);
  float* xn = (float*)malloc(sizeof(float) * (size_t)T * H);
  float* q = (float*)malloc(sizeof(float) * (size_t)T * Nq);
  float* kk = (float*)malloc(sizeof(float) * (size_t)T * Nkv);
  float* vv = (float*)malloc(sizeof(float) * (size_t)T * Nkv);
  float* att = (float*)malloc(sizeof(float) * (size_t)T * Nq);
  float* tmp = (float*)malloc(sizeof(float) * (size_t)T * (H > F ? H : F));
  float* gg = (float*)malloc(sizeof(float) * (size_t)T * F);
  float* uu = (float*)malloc(sizeof(float) * (size_t)T * F);
  uint16_t* q16 = (uint16_t*)malloc(2 * (size_t)T * Nq);
  uint16_t* k16 = (uint16_t*)malloc(2 * (size_t)T * Nkv);
  uint16_t* o16 = (uint16_t*)malloc(2 * (size_t)T * Nq);
  int32_t* pos = (int32_t*)malloc(sizeof(int32_t) * (size_t)T);
  for (int t = 0; t < T; ++t) pos[t] = start_pos + t;

  for (int t = 0; t < T; ++t)
    for (int i = 0; i < H; ++i) h[(size_t)t * H + i] = ldv(m->embed, (size_t)tokens[t] * H + i, dt);

  for (int l = 0; l < L; ++l) {
    rmsnorm_f(h, m->attn_norm + (size_t)l * H, T, H, m->eps, dt, xn);
    linear(m, xn, T, m->q_w + (size_t)l * Nq * wpr_h, m->q_s + (size_t)l * Nq * ng_h,
           m->q_b + (size_t)l * Nq * ng_h, Nq, H, m->q_bias ? m->q_bias + (size_t)l * Nq : NULL, q);
    linear(m, xn, T, m->k_w + (size_t)l * Nkv * wpr_h, m->k_s + (size_t)l * Nkv * ng_h,
           m->k_b + (size_t)l * Nkv * ng_h, Nkv, H, m->k_bias ? m->k_bias + (size_t)l * Nkv : NULL, kk);
    linear(m, xn, T, m->v_w + (size_t)l * Nkv * wpr_h, m->v_s + (size_t)l * Nkv * ng_h,
           m->v_b + (size_t)l * Nkv * ng_h, Nkv, H, m->v_bias ? m->v_bias + (size_t)l * Nkv : NULL, vv);
    for (size_t i = 0; i < (size_t)T * Nq; ++i) q16[i] = stv(q[i], dt);
    for (size_t i = 0; i < (size_t)T * Nkv; ++i) k16[i] = stv(kk[i], dt);
    oracle_rope(q16, T, Hq, D, pos, m->inv_freq, dt);
    oracle_rope(k16, T, Hkv, D, pos, m->inv_freq, dt);
    /* append to the cache ([Hkv, max_ctx, D]) */
    uint16_t* KC = kcache + (size_t)l * Hkv * max_ctx * D;
    uint16_t* VC = vcache + (size_t)l * Hkv * max_ctx * D;
    for (int t = 0; t < T; ++t)
      for (int hk = 0; hk < Hkv; ++hk) {
        uint16_t* kr = KC + ((size_t)hk * max_ctx + pos[t]) * D;
        uint16_t* vr = VC + ((size_t)hk * max_ctx + pos[t]) * D;
        for (int d = 0; d < D; ++d) {
          kr[d] = k16[((size_t)t * Hkv + hk) * D + d];
          vr[d] = stv(vv[((size_t)t * Hkv + hk) * D + d], dt);
        }
        if (m->kv_bits > 0) {
          qdq_row(kr, D, m->kv_bits, m->kv_gs, dt);
          qdq_row(vr, D, m->kv_bits, m->kv_gs, dt);
        }
      }
    attn_cache(q16, KC, VC, max_ctx, T, Hq, Hkv, D, start_pos, 1.0f / sqrtf((float)D), dt, o16);
    for (size_t i = 0; i < (size_t)T * Nq; ++i) att[i] = ldv(o16, i, dt);
    linear(m, att, T, m->o_w + (size_t)l * H * wpr_q, m->o_s + (size_t)l * H * ng_q,
           m->o_b + (size_t)l * H * ng_q, H, Nq, NULL, tmp);
    for (size_t i = 0; i < (size_t)T * H; ++i) h[i] = rnd(h[i] + tmp[i], dt);

    rmsnorm_f(h, m->mlp_norm + (size_t)l * H, T, H, m->eps, dt, xn);
    linear(m, xn, T, m->g_w + (size_t)l * F * wpr_h, m->g_s + (size_t)l * F * ng_h,
           m->g_b + (size_t)l * F * ng_h, F, H, NULL, gg);
    linear(m, xn, T, m->u_w + (size_t)l * F * wpr_h, m->u_s + (size_t)l * F * ng_h,
           m->u_b + (size_t)l * F * ng_h, F, H, NULL, uu);
    for (size_t i = 0; i < (size_t)T * F; ++i) {
      float g = gg[i];
      float a = rnd(g / (1.0f + expf(-g)), dt);
      gg[i] = rnd(a * uu[i], dt);
    }
    linear(m, gg, T, m->d_w + (size_t)l * H * wpr_f, m->d_s + (size_t)l * H * ng_f,
           m->d_b + (size_t)l * H * ng_f, H, F, NULL, tmp);
    for (size_t i = 0; i < (size_t)T * H; ++i) h[i] = rnd(h[i] + tmp[i], dt);
  }

  const int t0 = all_logits ? 0 : T - 1;
  const int nt = T - t0;
  rmsnorm_f(h + (size_t)t0 * H, m->final_norm, nt, H, m->eps, dt, xn);
  if (m->tie) {
    /* tied embeddings are not quantized here: logits = xn · embedᵀ */
#pragma omp parallel for schedule(static)
    for (int v = 0; v < V; ++v)
      for (int t = 0; t < nt; ++t) {
        float acc = 0.0f;
        for (int i = 0; i < H; ++i) acc += xn[(size_t)t * H + i] * ldv(m->embed, (size_t)v * H + i, dt);
        logits[(size_t)t * V + v] = rnd(acc, dt);
      }
  } else {
    qmm_f32(xn, m->lm_w, m->lm_s, m->lm_b, nt, V, H, m->bits, m->gs, dt, logits);
    for (size_t i = 0; i < (size_t)nt * V; ++i) logits[i] = rnd(logits[i], dt);
  }

  free(h); free(xn); free(q); free(kk); free(vv); free(att); free(tmp); free(gg); free(uu);
  free(q16); free(k16); free(o16); free(pos);
  return 0;
}
