// Internal kernel-launch interface of libnovamlx_cuda (host side).
#pragma once

#include "common.cuh"

namespace nmx {

enum Epi { EPI_STORE = 0, EPI_RESID = 1, EPI_SILU = 2, EPI_ARGMAX = 3 };
// The argmax epilogue uses at most this many CTAs per SM; its partial
// buffers hold 32 rows × kArgmaxMaxGridPerSm × SMs entries.
constexpr int kArgmaxMaxGridPerSm = 4;

// y[M, N] = epilogue( norm?(x)[M, K] · dequant(W)[rows, K]^T )
struct GemvArgs {
  const void* x = nullptr;  // [M, K] activations (dtype)
  long ldx = 0;
  const void* gamma = nullptr;  // RMSNorm weight [K]; null → x used as is
  float eps = 1e-5f;
  const uint32_t* w = nullptr;  // packed [rows, K*bits/32]
  const void* s = nullptr;      // [rows, K/gs]
  const void* b = nullptr;
  // weights are not written by any kernel of this stream's step: the first
  // k-batch may be requested before griddepcontrol.wait (model forward only)
  bool weights_static = false;
  int N = 0, K = 0, M = 0;
  long pair_off = 0;            // EPI_SILU: up rows start at this row index
  const void* bias = nullptr;   // [N] added after rounding (qkv bias)
  void* y = nullptr;            // [M, ldy]
  long ldy = 0;
  const void* res = nullptr;    // EPI_RESID: y = rnd(res + rnd(acc)); may alias y
  long ldres = 0;
  // EPI_ARGMAX
  void* logits = nullptr;       // optional [M, N] rounded logits in dtype
  float* logits_f32 = nullptr;  // optional [M, N] fp32 copy of the rounded logits
  float* part_val = nullptr;    // [M, grid] scratch
  int* part_idx = nullptr;
  unsigned* counter = nullptr;  // zero on entry, left zero on exit
  int* out_ids = nullptr;       // [M]
  int* next_tokens = nullptr;   // optional second copy of out_ids
};

// Launch the quantized GEMV; M rows are processed in chunks the kernel's
// shared-memory staging can hold. EPI_ARGMAX requires M <= 32 (one chunk).
nmx_status_t qgemv(Ctx* c, const GemvArgs& a, int bits, int gs, nmx_dtype_t dt, int epi);
// Largest M one qgemv launch handles for this K (0 when K is too large).
int qgemv_max_m(int K, int gs);

// Decode GEMV over decode records (4-bit g64, f16): see qgemv_dl.cu.
struct GemvDLArgs {
  const void* x = nullptr;  // [M, K] f16
  long ldx = 0;
  const void* gamma = nullptr;
  float eps = 1e-5f;
  const void* w = nullptr;  // decode records of the whole matrix
  int N = 0, K = 0, M = 0;  // N = output columns (gate rows for EPI_SILU)
  int n_tg = 0;             // set by qgemv_dl
  long pair_tiles = 0;      // EPI_SILU: tile offset of the up rows
  const void* bias = nullptr;
  void* y = nullptr;
  long ldy = 0;
  const void* res = nullptr;
  long ldres = 0;
  float* logits_f32 = nullptr;        // EPI_ARGMAX: optional [M, N]
  unsigned long long* keys = nullptr; // EPI_ARGMAX: [32] packed (value, index), zero between launches
  unsigned* done = nullptr;           // EPI_ARGMAX: finished tile groups, zero between launches
  int* out_ids = nullptr;
  int* next_tokens = nullptr;
  float* partials = nullptr;          // split tile groups' partial sums
  size_t partials_cap = 0;            // floats
  int max_contrib = 0;                // slot stride (set per launch)
  unsigned* counters = nullptr;       // [n_tg], zero between launches
  int ctas_per_sm = 2;
  // the records are never written on this stream while the launch may be in
  // flight (model weights): the weight stream may start before the
  // programmatic-launch wait
  bool weights_static = false;
  unsigned* err = nullptr;            // device word: bit 0 = a bounded wait ran out
  // tensor parallelism (qgemm_tcs, residual epilogue): the communicator
  // (Comm*) and partial region whose exchange the GEMM fuses; y = res +
  // sum over ranks of x · W_rankᵀ
  void* comm = nullptr;
  int comm_region = 0;
};
bool qgemv_dl_supported(int bits, int gs, nmx_dtype_t dt, int N, int K);
int qgemv_dl_max_m(int K, int epi);
// floats of partial-sum scratch one launch of this shape may need
size_t qgemv_dl_partials_floats(int N_out, int K, int epi, int num_sms, int ctas_per_sm);
nmx_status_t qgemv_dl(Ctx* c, const GemvDLArgs& a, int epi);
// tensor-core (tcgen05) GEMM over decode records for many rows (prefill):
// store / residual / SiLU·up epilogues, no RMSNorm prologue (normalise x
// first); N_out % 256 (SiLU: % 128) and K % 128
bool qgemm_tc_supported(int N_out, int K, int epi);
nmx_status_t qgemm_tc(Ctx* c, const GemvDLArgs& a, int epi);
constexpr int kGemmMinRows = 64;  // qgemv_dl hands row counts from here on to qgemm_tc
// tensor-core GEMM for decode batches (weights as the MMA's 128 rows,
// activation rows as its N, K split over the SMs): 1..128 rows, N_out % 128,
// K % 128; store / residual / SiLU·up epilogues, no RMSNorm prologue
constexpr int kTcsMinRows = 9;    // qgemv_dl hands kTcsMinRows..kTcsMaxRows rows to qgemm_tcs
constexpr int kTcsMaxRows = 112;  // the decode GEMM's shared-memory budget: x tiles of <= 112 rows
bool qgemm_tcs_supported(int M, int N_out, int K, int epi);
// floats of partial-sum scratch (partials) and counters one launch needs
size_t qgemm_tcs_partials_floats(int M, int N_out, int K, int epi, int num_sms);
int qgemm_tcs_groups(int M, int N_out, int K, int epi, int num_sms);
nmx_status_t qgemm_tcs(Ctx* c, const GemvDLArgs& a, int epi);
// 1..8 activation rows (qgemv_dl dispatches here when the staging fits)
bool qgemv_small_fits(int M, int N_out, int K, int epi, int num_sms);
size_t qgemv_small_partials_floats(int N_out, int K, int epi, int num_sms);
nmx_status_t qgemv_small(Ctx* c, const GemvDLArgs& a, int epi);
// MLX-layout parts (mask 1 = words, 2 = scales, 4 = biases) of rows
// [row0, row0 + rows) to decode records, and back.
nmx_status_t repack_to_records(Ctx* c, const uint32_t* wq, const void* s, const void* b, int rows, int K,
                               long row0, void* rec, int part_mask);
nmx_status_t unpack_from_records(Ctx* c, const void* rec, int rows, int K, long row0, uint32_t* wq, void* s,
                                 void* b, int part_mask);

// ---- attention
// A KV page record: one (block, kv head) of K or V for 16 tokens. f16 pages
// (bits = 0): [16][D] f16. Quantized pages: codes [16][D * bits / 32] u32
// (MLX packing, low bits first along d), then scales [16][D / gs] and biases
// [16][D / gs] f16 — MLX-affine quantization in groups of gs along head_dim.
__host__ __device__ constexpr int kv_page_bytes(int D, int bits, int gs) {
  return bits == 0 ? 16 * D * 2 : 16 * (D * bits / 8 + 2 * (D / gs) * 2);
}

struct AttnArgs {
  const void* q = nullptr;     // FUSED: qkv rows [T, ldq] (pre-RoPE q|k|v); else q [T, Hq*D] roped
  long ldq = 0;
  void* k_cache = nullptr;     // [NB][Hkv][BT][D]
  void* v_cache = nullptr;
  const int* block_tables = nullptr;  // [n_seqs][max_blocks]
  int max_blocks = 0;
  const int* tok_seq = nullptr;  // [T] sequence index of each query row
  const int* tok_pos = nullptr;  // [T] absolute position of each query row
  const float* inv_freq = nullptr;  // [D/2] (FUSED only)
  void* out = nullptr;         // [T, Hq*D]
  int T = 0, Hq = 0, Hkv = 0, D = 0, BT = 16;
  int splits = 1;
  float scale = 1.0f;
  // the pages are not written by the kernel before this one on the stream
  // (true in the decode step): the K/V stream may start before its wait
  bool kv_static = false;
  // prefill: blocks of the pool (tensor-map extent), the leading items that
  // go to the tensor-core kernel, and the error word of bounded waits
  int pool_blocks = 0;
  int prefill_tc_items = 0;
  unsigned* err = nullptr;
  // quantized pages (kv_page_bytes): code width 4 / 8 and group along the
  // head dim; 0 = f16 pages
  int kv_bits = 0, kv_gs = 0;
};

// fused = 1: apply RoPE to q and append the row's own k/v (one query row per
// sequence, decode); fused = 0: q is already roped and K/V already appended.
// The splits of one (row, kv head) are one thread-block cluster and combine
// through distributed shared memory: no global scratch beyond the row
// descriptors. At most kMaxDecodeRows rows (the grid's z extent).
constexpr int kMaxDecodeSplits = 16;
constexpr long kMaxDecodeRows = 65535;
nmx_status_t paged_attention(Ctx* c, const AttnArgs& a, bool fused);
// key splits per (row, kv head): enough CTAs for two per SM, at most one
// cluster, and no thin last wave. A CTA keeps only a few pages in flight, so
// a last wave that fills under half of the SMs' CTA slots streams its pages
// well below HBM speed (at 4 kv heads × 32 rows, 3 splits made 384 CTAs for
// 296 slots: 0.84 of HBM; 2 splits, one wave, reach the roofline). Fewer
// splits are taken until the grid fits one wave or its last wave is at
// least half full.
inline int decode_attn_splits(int num_sms, long rows, int Hkv) {
  const long units = rows * long(Hkv > 0 ? Hkv : 1);
  const long slots = 2L * num_sms;
  long s = (slots + units - 1) / units;
  s = s < 1 ? 1 : (s > kMaxDecodeSplits ? kMaxDecodeSplits : s);
  while (s > 1) {
    const long ctas = units * s, last = ctas % slots;
    if (ctas <= slots || last == 0 || 2 * last >= slots) break;
    --s;
  }
  return int(s);
}
// prefill chunks / mixed batches: query blocks of up to 16 rows of one
// sequence (attention_prefill.cu). prefill_items cuts the batch's rows
// (row_seq: sequence of each row, rows of a sequence consecutive) into
// items (first row, rows); at most T items.
// Items for head layout (D, rep): with the tensor-core kernel, up to
// 128 / rep positions each, those too small for it (at most 16 positions and
// fewer than 64 tile rows) last and cut to at most 16 positions; *n_tc = the
// leading items for the tensor-core kernel. Without it, items of <= 16 rows.
int prefill_items(const int32_t* row_seq, int T, int D, int rep, int2* items_host, int* n_tc);
bool prefill_tc_supported(int D, int rep);
// attention_prefill_tc.cu: the leading items on tcgen05 (see there)
nmx_status_t paged_prefill_attention_tc(Ctx* c, const AttnArgs& a, const int2* items, int n_items);
nmx_status_t paged_prefill_attention(Ctx* c, const AttnArgs& a, const int2* items, int n_items);
// the tensor-core implementation behind paged_attention (attention_mma.cu)
nmx_status_t paged_attention_mma(Ctx* c, const AttnArgs& a, bool fused);

// RoPE q and k of T new tokens in place in qkv [T, ldq] and write k/v to the
// pages at each token's position.
nmx_status_t rope_append(Ctx* c, void* qkv, long ldq, int T, int Hq, int Hkv, int D,
                         const int* tok_seq, const int* tok_pos, const int* block_tables,
                         int max_blocks, int BT, void* k_cache, void* v_cache,
                         const float* inv_freq, void* q_out, long ldqo, int kv_bits = 0, int kv_gs = 0);

nmx_status_t quantized_sdpa(Ctx* c, const void* q, const uint32_t* kw, const void* ks,
                            const void* kb, const uint32_t* vw, const void* vs, const void* vb,
                            int BH, int gqa, int N, int L, int D, float scale, int gs, int bits,
                            nmx_dtype_t dt, void* out);

// ---- small ops
nmx_status_t rmsnorm(Ctx* c, const void* x, long ldx, const void* g, int M, int H, float eps,
                     nmx_dtype_t dt, void* y, long ldy);
nmx_status_t embed_rows(Ctx* c, const void* table, const int* ids, int T, int H, void* out);
nmx_status_t argmax_rows(Ctx* c, const void* logits, int M, int V, nmx_dtype_t dt, int* out);
// temperature / top-p categorical per row, chosen-id logprob, top_k logprobs (sampling.cu)
nmx_status_t sample_rows(Ctx* c, const void* logits, nmx_dtype_t dt, int rows, int V, float temperature, float top_p,
                         unsigned long long seed, unsigned long long counter, int* out_ids, float* out_lp, int top_k,
                         int* top_ids, float* top_lp);
nmx_status_t penalized_argmax(Ctx* c, const void* logits, int M, int V, nmx_dtype_t dt,
                              const int* recent, const int* n_recent, int max_recent,
                              float penalty, int* out);
nmx_status_t quantize(Ctx* c, const float* w, int N, int K, int bits, int gs, nmx_dtype_t sdt,
                      uint32_t* wq, void* s, void* b);
nmx_status_t dequantize(Ctx* c, const uint32_t* wq, const void* s, const void* b, int N, int K,
                        int bits, int gs, nmx_dtype_t sdt, float* w);
// generate N(0, std) for rows [N, K] from (seed, stream_id) and quantize in one pass
nmx_status_t random_quantized(Ctx* c, uint64_t seed, uint64_t stream_id, float std, int N, int K,
                              int bits, int gs, nmx_dtype_t sdt, uint32_t* wq, void* s, void* b);
nmx_status_t random_fill(Ctx* c, uint64_t seed, uint64_t stream_id, float std, float mean,
                         size_t n, nmx_dtype_t dt, void* out);
nmx_status_t fill_value(Ctx* c, size_t n, float v, nmx_dtype_t dt, void* out);
nmx_status_t copy_kv_blocks(Ctx* c, void* base, long layer_stride_bytes, int layers,
                            long block_bytes, const int* src, const int* dst, int n);
// seq[b] = b, pos[b] = lens[b] - 1 (one query row per sequence)
nmx_status_t seq_rows_from_lens(Ctx* c, const int* lens, int B, int* seq, int* pos);
// decode bookkeeping after a step: pos[b] += 1; history[step * B + b] = tok[b]
// while (step + 1) * B <= hist_cap; step++
nmx_status_t decode_advance(Ctx* c, int* pos, const int* tok, int B, int* history, int hist_cap, int* step);

}  // namespace nmx
