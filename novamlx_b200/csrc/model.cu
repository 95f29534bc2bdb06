// Llama / Qwen2 model runtime behind nmx_model_* / nmx_forward /
// nmx_decode_greedy: weight storage, the paged KV pool, and the two forward
// schedules.
//
//   prefill / mixed batch (any token count):
//     embed → L × [qkv GEMV (RMSNorm prologue, bias) → RoPE + KV append →
//     paged attention → o GEMV (+residual) → gate/up GEMV (RMSNorm prologue,
//     SiLU·up epilogue) → down GEMV (+residual)] → gather last rows →
//     lm_head GEMV (final RMSNorm prologue, argmax epilogue)
//   decode batch (one new token per sequence):
//     the same, but RoPE + KV append run inside the attention kernel and the
//     whole step (embed … argmax, plus the position/token advance) is one
//     CUDA graph per batch size, replayed per token; kernels are chained
//     with programmatic dependent launch so each GEMV's weight stream starts
//     before its predecessor finishes.
//
// Mirrors the engine's per-step call `context.model(tokens, cache:)`
// (Sources/NovaMLXEngine/FusedBatchScheduler.swift:677,817,1215,1259) with
// the batched-decode shape of Sources/NovaMLXEngine/BatchScheduler.swift:162-258
// (one forward for the whole batch), with KV in pages instead of padded,
// stacked per-sequence caches (Sources/NovaMLXEngine/FusedBatchDecode.swift:95-147).
#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "common.cuh"
#include "kernels.h"
#include "model.h"

namespace nmx {

namespace {

constexpr int kBT = 16;             // tokens per KV block
constexpr int kBlockCap = 4096;     // block-table columns per sequence (65,536 tokens)
constexpr int kHistCap = 1 << 16;   // decode-loop id history entries

size_t dsize(nmx_dtype_t dt) { return dt == NMX_F32 || dt == NMX_U32 || dt == NMX_I32 ? 4 : 2; }

}  // namespace

static nmx_status_t alloc_dev(void** p, size_t bytes) {
  cudaError_t e = cudaMalloc(p, bytes);
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error("cudaMalloc(" + std::to_string(bytes) + " B): " + cudaGetErrorString(e));
    return NMX_ERR_OOM;
  }
  return NMX_OK;
}

static void rope_table(const nmx_model_cfg& c, std::vector<float>& out) {
  const int D = c.head_dim;
  out.resize(D / 2);
  for (int i = 0; i < D / 2; ++i) {
    double f = 1.0 / std::pow(double(c.rope_theta), (2.0 * i) / double(D));
    if (c.rope_factor > 0.0f) {
      const double low_wl = double(c.rope_original_max_pos) / double(c.rope_low_freq_factor);
      const double high_wl = double(c.rope_original_max_pos) / double(c.rope_high_freq_factor);
      const double wl = 2.0 * M_PI / f;
      if (wl < high_wl) {
      } else if (wl > low_wl) {
        f = f / double(c.rope_factor);
      } else {
        const double smooth = (double(c.rope_original_max_pos) / wl - double(c.rope_low_freq_factor)) /
                              (double(c.rope_high_freq_factor) - double(c.rope_low_freq_factor));
        f = (1.0 - smooth) * f / double(c.rope_factor) + smooth * f;
      }
    }
    out[i] = float(f);
  }
}

nmx_status_t Model::create(Ctx* c, const nmx_model_cfg& cfg, Model** out) {
  NMX_CHECK(cfg.hidden > 0 && cfg.n_layers > 0 && cfg.n_heads > 0 && cfg.n_kv_heads > 0 &&
                cfg.head_dim > 0 && cfg.ffn > 0 && cfg.vocab > 0,
            NMX_ERR_INVALID, "model: every dimension must be positive");
  NMX_CHECK(cfg.bits == 4 || cfg.bits == 8, NMX_ERR_UNSUPPORTED, "model: bits must be 4 or 8");
  NMX_CHECK(cfg.group_size == 32 || cfg.group_size == 64 || cfg.group_size == 128, NMX_ERR_UNSUPPORTED,
            "model: group size must be 32, 64 or 128");
  NMX_CHECK(cfg.dtype == NMX_F16, NMX_ERR_UNSUPPORTED, "model: activation dtype must be f16 (KV pages are f16)");
  NMX_CHECK(cfg.tie_embeddings == 0, NMX_ERR_UNSUPPORTED, "model: tied embeddings are not supported");
  NMX_CHECK(cfg.head_dim == 64 || cfg.head_dim == 128, NMX_ERR_UNSUPPORTED, "model: head_dim must be 64 or 128");
  NMX_CHECK(cfg.n_heads % cfg.n_kv_heads == 0 && cfg.n_heads / cfg.n_kv_heads <= 8, NMX_ERR_UNSUPPORTED,
            "model: q heads per kv head must divide and be <= 8");
  const int gs = cfg.group_size;
  const int Nq = cfg.n_heads * cfg.head_dim, Nkv = cfg.n_kv_heads * cfg.head_dim;
  NMX_CHECK(cfg.hidden % gs == 0 && Nq % gs == 0 && cfg.ffn % gs == 0, NMX_ERR_UNSUPPORTED,
            "model: hidden, q width and ffn must be multiples of the group size");
  NMX_CHECK(cfg.hidden % 16 == 0 && Nkv % 16 == 0 && cfg.ffn % 16 == 0 && cfg.vocab % 16 == 0,
            NMX_ERR_UNSUPPORTED, "model: output widths must be multiples of 16");
  NMX_CHECK(qgemv_max_m(cfg.ffn, gs) > 0 && qgemv_max_m(cfg.hidden, gs) > 0, NMX_ERR_UNSUPPORTED,
            "model: reduction width too large");

  auto* m = new Model();
  m->ctx = c;
  m->cfg = cfg;
  m->dt = nmx_dtype_t(cfg.dtype);
  m->max_batch = cfg.max_batch > 0 ? cfg.max_batch : 1;
  m->max_tokens = cfg.max_tokens > 0 ? cfg.max_tokens : 2048;
  if (m->max_tokens < m->max_batch) m->max_tokens = m->max_batch;
  m->Nq = Nq;
  m->Nkv = Nkv;
  m->Nqkv = Nq + 2 * Nkv;

  // ---- weights: one allocation, 256-byte aligned slices
  const int H = cfg.hidden, F = cfg.ffn, V = cfg.vocab, L = cfg.n_layers;
  const size_t es = 2;
  std::vector<std::pair<void**, size_t>> slices;
  size_t total = 0;
  auto plan = [&](void** p, size_t bytes) { slices.push_back({p, bytes}); total += align_up(bytes, 256); };
  std::vector<Lin*> lins;
  auto plan_lin = [&](Lin& l, int N, int K) {
    l.N = N;
    l.K = K;
    l.dl = qgemv_dl_supported(cfg.bits, gs, nmx_dtype_t(cfg.dtype), N, K);
    l.bytes = size_t(N) * K * cfg.bits / 8 + 2 * size_t(N) * (K / gs) * es;
    plan(reinterpret_cast<void**>(&l.w), l.bytes);  // words | scales | biases, or decode records
    lins.push_back(&l);
  };
  m->layers.resize(L);
  plan(&m->embed, size_t(V) * H * es);
  plan(&m->final_norm, size_t(H) * es);
  plan_lin(m->lm, V, H);
  for (auto& ly : m->layers) {
    plan(&ly.attn_norm, size_t(H) * es);
    plan(&ly.mlp_norm, size_t(H) * es);
    plan_lin(ly.qkv, m->Nqkv, H);
    if (cfg.qkv_bias) plan(&ly.qkv_bias, size_t(m->Nqkv) * es);
    plan_lin(ly.o, H, Nq);
    plan_lin(ly.gu, 2 * F, H);
    plan_lin(ly.down, H, F);
  }
  nmx_status_t st = alloc_dev(reinterpret_cast<void**>(&m->wbase), total);
  if (st != NMX_OK) {
    delete m;
    return st;
  }
  m->wbytes = total;
  size_t off = 0;
  for (auto& s : slices) {
    *s.first = m->wbase + off;
    off += align_up(s.second, 256);
  }
  for (Lin* l : lins) {
    if (l->dl) continue;
    char* base = reinterpret_cast<char*>(l->w);
    const size_t wb = size_t(l->N) * l->K * cfg.bits / 8, sb = size_t(l->N) * (l->K / gs) * es;
    l->s = base + wb;
    l->b = base + wb + sb;
  }
  // byte counts: everything one decode step reads once
  m->step_bytes = 0;
  auto lin_bytes = [&](const Lin& l) {
    return uint64_t(l.N) * l.K * cfg.bits / 8 + 2ull * l.N * (l.K / gs) * es;
  };
  m->step_bytes += lin_bytes(m->lm) + uint64_t(H) * es * (1 + 2 * L) + uint64_t(H) * es /*embed row*/;
  for (auto& ly : m->layers) {
    m->step_bytes += lin_bytes(ly.qkv) + lin_bytes(ly.o) + lin_bytes(ly.gu) + lin_bytes(ly.down);
    if (cfg.qkv_bias) m->step_bytes += uint64_t(m->Nqkv) * es;
  }

  // ---- workspace
  const int T = m->max_tokens, B = std::max(m->max_batch, 1);
  const int rows_logits = std::max(B, std::min(T, 256));
  struct WS {
    void** p;
    size_t bytes;
  };
  std::vector<WS> ws = {
      {&m->h, size_t(T) * H * es},
      {&m->qkv, size_t(T) * m->Nqkv * es},
      {&m->q_roped, size_t(T) * Nq * es},
      {&m->attn, size_t(T) * Nq * es},
      {&m->act, size_t(T) * F * es},
      {&m->xn, size_t(T) * H * es},
      {&m->last_h, size_t(rows_logits) * H * es},
      {reinterpret_cast<void**>(&m->logits_f32), size_t(rows_logits) * V * 4},
      {reinterpret_cast<void**>(&m->am_val), size_t(32) * kArgmaxMaxGridPerSm * c->num_sms * 4},
      {reinterpret_cast<void**>(&m->am_idx), size_t(32) * kArgmaxMaxGridPerSm * c->num_sms * 4},
      {reinterpret_cast<void**>(&m->am_counter), 256},
      {reinterpret_cast<void**>(&m->tok_ids), size_t(T) * 4},
      {reinterpret_cast<void**>(&m->tok_seq), size_t(T) * 4},
      {reinterpret_cast<void**>(&m->tok_pos), size_t(T) * 4},
      {reinterpret_cast<void**>(&m->last_rows), size_t(rows_logits) * 4},
      {reinterpret_cast<void**>(&m->pf_items), size_t(T) * 8},
      {reinterpret_cast<void**>(&m->out_ids), size_t(rows_logits) * 4},
      {reinterpret_cast<void**>(&m->block_tables), size_t(B) * kBlockCap * 4},
      {reinterpret_cast<void**>(&m->hist), size_t(kHistCap) * 4},
      {reinterpret_cast<void**>(&m->step), 256},
      {reinterpret_cast<void**>(&m->inv_freq), size_t(cfg.head_dim / 2) * 4},
      {reinterpret_cast<void**>(&m->dl_partials), 0},
      {reinterpret_cast<void**>(&m->dl_counters), 0},
      {reinterpret_cast<void**>(&m->dl_keys), 32 * 8},
      {reinterpret_cast<void**>(&m->dl_done), 256},
  };
  {
    size_t pf = 0, ntg = 1;
    auto need = [&](const Lin& l, bool paired) {
      if (!l.dl) return;
      const int n_out = paired ? l.N / 2 : l.N;
      const int epi = paired ? EPI_SILU : EPI_STORE;
      pf = std::max(pf, qgemv_dl_partials_floats(n_out, l.K, epi, c->num_sms, m->dl_ctas_per_sm));
      // decode batches and short prefill chunks on the tensor-core decode GEMM
      const int rows_max = std::min(kTcsMaxRows, std::max(m->max_batch, m->max_tokens));
      for (int rows = 16; rows < rows_max + 16; rows += 16)
        pf = std::max(pf, qgemm_tcs_partials_floats(std::min(rows, rows_max), n_out, l.K, epi, c->num_sms));
      ntg = std::max(ntg, size_t(n_out / 16));
    };
    need(m->lm, false);
    for (const auto& ly : m->layers) {
      need(ly.qkv, false);
      need(ly.o, false);
      need(ly.gu, true);
      need(ly.down, false);
    }
    m->dl_partials_cap = pf;
    for (auto& w : ws) {
      if (w.p == reinterpret_cast<void**>(&m->dl_partials)) w.bytes = std::max<size_t>(pf, 1) * 4;
      if (w.p == reinterpret_cast<void**>(&m->dl_counters)) w.bytes = ntg * 4;
    }
  }
  size_t wtot = 0;
  for (auto& w : ws) wtot += align_up(w.bytes, 256);
  st = alloc_dev(reinterpret_cast<void**>(&m->wsbase), wtot);
  if (st != NMX_OK) {
    cudaFree(m->wbase);
    delete m;
    return st;
  }
  size_t o2 = 0;
  for (auto& w : ws) {
    *w.p = m->wsbase + o2;
    o2 += align_up(w.bytes, 256);
  }
  m->rows_logits = rows_logits;
  cudaError_t e = cudaMemsetAsync(m->wsbase, 0, wtot, c->stream);
  std::vector<float> inv;
  rope_table(cfg, inv);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(m->inv_freq, inv.data(), inv.size() * 4, cudaMemcpyHostToDevice, c->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
  // pinned staging for per-call step descriptors
  m->pinned_bytes = size_t(T) * 3 * 4 + size_t(B) * kBlockCap * 4 + size_t(rows_logits) * 4 + size_t(T) * 8 + 4096;
  if (e == cudaSuccess) e = cudaMallocHost(reinterpret_cast<void**>(&m->pinned), m->pinned_bytes);
  if (e != cudaSuccess) {
    set_error(std::string("model workspace: ") + cudaGetErrorString(e));
    cudaFree(m->wbase);
    cudaFree(m->wsbase);
    delete m;
    return NMX_ERR_CUDA;
  }
  *out = m;
  return NMX_OK;
}

Model::~Model() {
  for (auto& g : graphs) {
    if (g.second.exec) cudaGraphExecDestroy(g.second.exec);
  }
  if (pinned) cudaFreeHost(pinned);
  if (wsbase) cudaFree(wsbase);
  if (wbase) cudaFree(wbase);
}

nmx_status_t Model::init_random(uint64_t seed, float stdv) {
  Ctx* c = ctx;
  const int H = cfg.hidden, F = cfg.ffn, V = cfg.vocab;
  const int bits = cfg.bits, gs = cfg.group_size;
  uint64_t sid = 1;
  // decode-record linears are generated in MLX layout into a scratch slice
  // and repacked; the scratch holds the largest slice (the lm_head)
  size_t tmp_bytes = lm.bytes;
  for (const auto& ly : layers)
    for (const Lin* l : {&ly.qkv, &ly.o, &ly.gu, &ly.down}) tmp_bytes = std::max(tmp_bytes, l->bytes);
  char* tmp = nullptr;
  NMX_TRY(alloc_dev(reinterpret_cast<void**>(&tmp), tmp_bytes));
  struct TmpFree {
    char* p;
    ~TmpFree() { cudaFree(p); }
  } tmp_free{tmp};
  auto rq = [&](Lin& l, long row0, int rows) -> nmx_status_t {
    const size_t wpr = size_t(l.K) * bits / 32, ng = size_t(l.K) / gs;
    if (!l.dl)
      return random_quantized(c, seed, sid++, stdv, rows, l.K, bits, gs, dt, l.w + row0 * wpr,
                              static_cast<char*>(l.s) + row0 * ng * 2, static_cast<char*>(l.b) + row0 * ng * 2);
    uint32_t* tw = reinterpret_cast<uint32_t*>(tmp);
    char* ts = tmp + size_t(rows) * wpr * 4;
    char* tb = ts + size_t(rows) * ng * 2;
    NMX_TRY(random_quantized(c, seed, sid++, stdv, rows, l.K, bits, gs, dt, tw, ts, tb));
    NMX_TRY(repack_to_records(c, tw, ts, tb, rows, l.K, row0, l.w, 7));
    return cudaStreamSynchronize(c->stream) == cudaSuccess ? NMX_OK : NMX_ERR_CUDA;
  };
  NMX_TRY(random_fill(c, seed, sid++, stdv, 0.f, size_t(V) * H, dt, embed));
  NMX_TRY(fill_value(c, H, 1.0f, dt, final_norm));
  NMX_TRY(rq(lm, 0, V));
  for (auto& ly : layers) {
    NMX_TRY(fill_value(c, H, 1.0f, dt, ly.attn_norm));
    NMX_TRY(fill_value(c, H, 1.0f, dt, ly.mlp_norm));
    NMX_TRY(rq(ly.qkv, 0, Nq));
    NMX_TRY(rq(ly.qkv, Nq, Nkv));
    NMX_TRY(rq(ly.qkv, Nq + Nkv, Nkv));
    if (cfg.qkv_bias) NMX_TRY(random_fill(c, seed, sid++, stdv, 0.f, size_t(Nqkv), dt, ly.qkv_bias));
    NMX_TRY(rq(ly.o, 0, H));
    NMX_TRY(rq(ly.gu, 0, F));
    NMX_TRY(rq(ly.gu, F, F));
    NMX_TRY(rq(ly.down, 0, H));
  }
  NMX_CUDA_OK(cudaStreamSynchronize(c->stream));
  weights_ready = true;
  return NMX_OK;
}

// Resolve an MLX safetensors name to a device region (+ expected shape).
nmx_status_t Model::resolve(const std::string& name, char** dst, size_t* bytes,
                            std::vector<int64_t>* shape, nmx_dtype_t* dtype) {
  const int H = cfg.hidden, F = cfg.ffn, V = cfg.vocab, gs = cfg.group_size, bits = cfg.bits;
  rs_lin = nullptr;
  auto lin_part = [&](Lin& l, long row0, int rows, const std::string& part) -> nmx_status_t {
    const size_t wpr = size_t(l.K) * bits / 32, ng = size_t(l.K) / gs;
    if (l.dl) {  // the part lives scattered inside decode records
      rs_lin = &l;
      rs_row0 = row0;
      rs_rows = rows;
      rs_mask = part == "weight" ? 1 : part == "scales" ? 2 : part == "biases" ? 4 : 0;
      NMX_CHECK(rs_mask != 0, NMX_ERR_NOT_FOUND, "unknown tensor part: " + part);
    }
    if (part == "weight") {
      *dst = reinterpret_cast<char*>(l.w + row0 * wpr);
      *bytes = size_t(rows) * wpr * 4;
      *shape = {rows, int64_t(wpr)};
      *dtype = NMX_U32;
    } else if (part == "scales" || part == "biases") {
      char* base = static_cast<char*>(part == "scales" ? l.s : l.b);
      *dst = base + row0 * ng * 2;
      *bytes = size_t(rows) * ng * 2;
      *shape = {rows, int64_t(ng)};
      *dtype = dt;
    } else {
      set_error("unknown tensor part: " + part);
      return NMX_ERR_NOT_FOUND;
    }
    return NMX_OK;
  };
  auto vec = [&](void* p, int n) {
    *dst = static_cast<char*>(p);
    *bytes = size_t(n) * 2;
    *shape = {n};
    *dtype = dt;
    return NMX_OK;
  };
  if (name == "model.embed_tokens.weight") {
    *dst = static_cast<char*>(embed);
    *bytes = size_t(V) * H * 2;
    *shape = {V, H};
    *dtype = dt;
    return NMX_OK;
  }
  if (name == "model.norm.weight") return vec(final_norm, H);
  if (name.rfind("lm_head.", 0) == 0) return lin_part(lm, 0, V, name.substr(8));
  const std::string pre = "model.layers.";
  if (name.rfind(pre, 0) == 0) {
    size_t p = pre.size();
    size_t dot = name.find('.', p);
    if (dot == std::string::npos) return NMX_ERR_NOT_FOUND;
    const int li = std::atoi(name.substr(p, dot - p).c_str());
    NMX_CHECK(li >= 0 && li < cfg.n_layers, NMX_ERR_NOT_FOUND, "layer index out of range: " + name);
    LayerW& ly = layers[li];
    const std::string rest = name.substr(dot + 1);
    if (rest == "input_layernorm.weight") return vec(ly.attn_norm, H);
    if (rest == "post_attention_layernorm.weight") return vec(ly.mlp_norm, H);
    struct Map {
      const char* prefix;
      Lin* lin;
      long row0;
      int rows;
    };
    const Map maps[] = {
        {"self_attn.q_proj.", &ly.qkv, 0, Nq},       {"self_attn.k_proj.", &ly.qkv, Nq, Nkv},
        {"self_attn.v_proj.", &ly.qkv, Nq + Nkv, Nkv}, {"self_attn.o_proj.", &ly.o, 0, H},
        {"mlp.gate_proj.", &ly.gu, 0, F},            {"mlp.up_proj.", &ly.gu, F, F},
        {"mlp.down_proj.", &ly.down, 0, H},
    };
    for (const auto& mp : maps) {
      const std::string pf = mp.prefix;
      if (rest.rfind(pf, 0) == 0) {
        const std::string part = rest.substr(pf.size());
        if (part == "bias") {
          NMX_CHECK(cfg.qkv_bias && mp.lin == &ly.qkv, NMX_ERR_NOT_FOUND, "model has no bias: " + name);
          *dst = static_cast<char*>(ly.qkv_bias) + mp.row0 * 2;
          *bytes = size_t(mp.rows) * 2;
          *shape = {mp.rows};
          *dtype = dt;
          return NMX_OK;
        }
        return lin_part(*mp.lin, mp.row0, mp.rows, part);
      }
    }
  }
  set_error("unknown tensor: " + name);
  return NMX_ERR_NOT_FOUND;
}

nmx_status_t Model::load_tensor(const std::string& name, const void* host, nmx_dtype_t dtype,
                                const int64_t* shape, int ndim) {
  char* dst = nullptr;
  size_t bytes = 0;
  std::vector<int64_t> exp;
  nmx_dtype_t edt;
  NMX_TRY(resolve(name, &dst, &bytes, &exp, &edt));
  NMX_CHECK(dtype == edt, NMX_ERR_INVALID, "tensor " + name + ": wrong dtype");
  NMX_CHECK(ndim == int(exp.size()), NMX_ERR_INVALID, "tensor " + name + ": wrong rank");
  for (int i = 0; i < ndim; ++i)
    NMX_CHECK(shape[i] == exp[i], NMX_ERR_INVALID,
              "tensor " + name + ": dim " + std::to_string(i) + " is " + std::to_string(shape[i]) +
                  ", expected " + std::to_string(exp[i]));
  if (rs_lin) {
    Lin* l = rs_lin;
    const long row0 = rs_row0;
    const int rows = rs_rows, mask = rs_mask;
    void* tmp = nullptr;
    NMX_TRY(alloc_dev(&tmp, bytes));
    // copy and repack are ordered on the model's stream (a pageable copy on
    // another stream may still be in flight when the call returns)
    cudaError_t e = cudaMemcpyAsync(tmp, host, bytes, cudaMemcpyHostToDevice, ctx->stream);
    nmx_status_t st = NMX_OK;
    if (e == cudaSuccess)
      st = repack_to_records(ctx, mask == 1 ? static_cast<uint32_t*>(tmp) : nullptr, mask == 2 ? tmp : nullptr,
                             mask == 4 ? tmp : nullptr, rows, l->K, row0, l->w, mask);
    if (e == cudaSuccess && st == NMX_OK) e = cudaStreamSynchronize(ctx->stream);
    cudaFree(tmp);
    NMX_CUDA_OK(e);
    NMX_TRY(st);
  } else {
    NMX_CUDA_OK(cudaMemcpyAsync(dst, host, bytes, cudaMemcpyHostToDevice, ctx->stream));
    NMX_CUDA_OK(cudaStreamSynchronize(ctx->stream));
  }
  loaded_any = true;
  return NMX_OK;
}

nmx_status_t Model::get_tensor(const std::string& name, void* host, size_t host_bytes) {
  char* src = nullptr;
  size_t bytes = 0;
  std::vector<int64_t> exp;
  nmx_dtype_t edt;
  NMX_TRY(resolve(name, &src, &bytes, &exp, &edt));
  NMX_CHECK(host_bytes >= bytes, NMX_ERR_INVALID, "tensor " + name + ": host buffer too small");
  NMX_CUDA_OK(cudaStreamSynchronize(ctx->stream));
  if (rs_lin) {
    void* tmp = nullptr;
    NMX_TRY(alloc_dev(&tmp, bytes));
    const int mask = rs_mask;
    nmx_status_t st = unpack_from_records(ctx, rs_lin->w, rs_rows, rs_lin->K, rs_row0,
                                          mask == 1 ? static_cast<uint32_t*>(tmp) : nullptr,
                                          mask == 2 ? tmp : nullptr, mask == 4 ? tmp : nullptr, mask);
    cudaError_t e = cudaSuccess;
    if (st == NMX_OK) e = cudaMemcpyAsync(host, tmp, bytes, cudaMemcpyDeviceToHost, ctx->stream);
    if (st == NMX_OK && e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    cudaFree(tmp);
    NMX_TRY(st);
    NMX_CUDA_OK(e);
    return NMX_OK;
  }
  NMX_CUDA_OK(cudaMemcpyAsync(host, src, bytes, cudaMemcpyDeviceToHost, ctx->stream));
  NMX_CUDA_OK(cudaStreamSynchronize(ctx->stream));
  return NMX_OK;
}

// ------------------------------------------------------------------ KV pool

nmx_status_t KvPool::create(Model* m, int block_tokens, int num_blocks, KvPool** out, int kv_bits, int kv_gs) {
  NMX_CHECK(block_tokens == kBT, NMX_ERR_UNSUPPORTED, "kv pool: block size must be 16 tokens");
  NMX_CHECK(num_blocks > 0, NMX_ERR_INVALID, "kv pool: num_blocks must be positive");
  const int D = m->cfg.head_dim;
  NMX_CHECK(kv_bits == 0 || ((kv_bits == 4 || kv_bits == 8) && (kv_gs == 32 || kv_gs == 64) &&
                             (D == 64 || D == 128)),
            NMX_ERR_UNSUPPORTED, "kv pool: quantized pages need 4 or 8 bits, group 32 or 64, head_dim 64 or 128");
  auto* p = new KvPool();
  p->model = m;
  p->num_blocks = num_blocks;
  p->kv_bits = kv_bits;
  p->kv_gs = kv_bits ? kv_gs : 0;
  p->block_bytes = size_t(m->cfg.n_kv_heads) * size_t(kv_page_bytes(D, kv_bits, kv_gs));
  p->layer_stride = 2 * p->block_bytes * size_t(num_blocks);
  const size_t total = p->layer_stride * m->cfg.n_layers;
  nmx_status_t st = alloc_dev(reinterpret_cast<void**>(&p->base), total);
  if (st != NMX_OK) {
    delete p;
    return st;
  }
  cudaError_t e = cudaMemsetAsync(p->base, 0, total, m->ctx->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(m->ctx->stream);
  if (e != cudaSuccess) {
    set_error(std::string("kv pool: ") + cudaGetErrorString(e));
    cudaFree(p->base);
    delete p;
    return NMX_ERR_CUDA;
  }
  *out = p;
  return NMX_OK;
}

KvPool::~KvPool() {
  if (base) cudaFree(base);
}

// ------------------------------------------------------------------ forward

nmx_status_t Model::linear(const Lin& l, const void* x, long ldx, const void* gamma, int M, int N_out,
                           long pair_off_rows, const void* bias, void* y, long ldy, const void* res, long ldres,
                           int epi, float* logits_f32, int* ids, int* next_tokens) {
  const bool tc_prefill = l.dl && M > kTcsMaxRows && qgemm_tc_supported(N_out, l.K, epi);
  const bool tc_batch = l.dl && !tc_prefill && M >= kTcsMinRows && qgemm_tcs_supported(M, N_out, l.K, epi);
  if (tc_prefill || tc_batch || (l.dl && M >= kGemmMinRows && qgemm_tc_supported(N_out, l.K, epi))) {
    // decode batches and prefill: the tensor-core GEMMs, after the RMSNorm
    // they have no prologue for
    if (gamma) {
      NMX_TRY(rmsnorm(ctx, x, ldx, gamma, M, l.K, cfg.rms_eps, NMX_F16, xn, l.K));
      x = xn;
      ldx = l.K;
    }
    GemvDLArgs a;
    a.x = x; a.ldx = ldx; a.w = l.w; a.N = N_out; a.K = l.K; a.M = M; a.pair_tiles = pair_off_rows / 16;
    a.bias = bias; a.y = y; a.ldy = ldy; a.res = res; a.ldres = ldres;
    a.err = ctx->dev_err;
    a.weights_static = true;
    if (tc_batch) {
      a.partials = dl_partials; a.partials_cap = dl_partials_cap; a.counters = dl_counters;
      return qgemm_tcs(ctx, a, epi);
    }
    return qgemm_tc(ctx, a, epi);
  }
  if (l.dl) {
    GemvDLArgs a;
    a.x = x; a.ldx = ldx; a.gamma = gamma; a.eps = cfg.rms_eps; a.w = l.w;
    a.N = N_out; a.K = l.K; a.M = M; a.pair_tiles = pair_off_rows / 16;
    a.bias = bias; a.y = y; a.ldy = ldy; a.res = res; a.ldres = ldres;
    a.logits_f32 = logits_f32; a.keys = dl_keys; a.done = dl_done; a.out_ids = ids; a.next_tokens = next_tokens;
    a.partials = dl_partials; a.partials_cap = dl_partials_cap; a.counters = dl_counters;
    a.ctas_per_sm = dl_ctas_per_sm;
    a.weights_static = true;
    a.err = ctx->dev_err;
    return qgemv_dl(ctx, a, epi);
  }
  GemvArgs a;
  a.weights_static = true;
  a.x = x; a.ldx = ldx; a.gamma = gamma; a.eps = cfg.rms_eps;
  a.w = l.w; a.s = l.s; a.b = l.b; a.N = N_out; a.K = l.K; a.M = M; a.pair_off = pair_off_rows;
  a.bias = bias; a.y = y; a.ldy = ldy; a.res = res; a.ldres = ldres;
  a.logits_f32 = logits_f32; a.part_val = am_val; a.part_idx = am_idx; a.counter = am_counter;
  a.out_ids = ids; a.next_tokens = next_tokens;
  return qgemv(ctx, a, cfg.bits, cfg.group_size, dt, epi);
}

// o_proj / down_proj: h += x · Wᵀ. Under tensor parallelism this rank's
// partial (its K shard) goes to the communicator's region and the exchange
// kernel writes h = h + Σ_ranks partial on every rank.
nmx_status_t Model::block_out(const Lin& l, const void* x, long ldx, int M, int region) {
  const int H = cfg.hidden;
  if (!comm) return linear(l, x, ldx, nullptr, M, H, 0, nullptr, h, H, h, H, EPI_RESID);
  if (fused_exchange && l.dl && M >= kTcsMinRows && M <= kTcsMaxRows && qgemm_tcs_supported(M, H, l.K, EPI_RESID)) {
    // one kernel: the decode-batch GEMM joins the ranks' partials in its
    // epilogue, tile group by tile group, over peer memory
    GemvDLArgs a;
    a.x = x; a.ldx = ldx; a.w = l.w; a.N = H; a.K = l.K; a.M = M;
    a.y = h; a.ldy = H; a.res = h; a.ldres = H;
    a.partials = dl_partials; a.partials_cap = dl_partials_cap; a.counters = dl_counters;
    a.weights_static = true;
    a.err = ctx->dev_err;
    a.comm = comm;
    a.comm_region = region;
    return qgemm_tcs(ctx, a, EPI_RESID);
  }
  NMX_TRY(linear(l, x, ldx, nullptr, M, H, 0, nullptr, comm_region(comm, region), H, nullptr, 0, EPI_STORE));
  return comm_allreduce_resid(comm, region, M, H, h, H, h, H, ctx->dev_err);
}

nmx_status_t Model::run_layers_decode(KvPool* pool, int B) {
  Ctx* c = ctx;
  const nmx_model_cfg& cf = cfg;
  const int H = cf.hidden, F = cf.ffn, bits = cf.bits, gs = cf.group_size;
  const int splits = decode_attn_splits(c->num_sms, B, cf.n_kv_heads);
  NMX_TRY(embed_rows(c, embed, tok_ids, B, H, h));
  for (int l = 0; l < cf.n_layers; ++l) {
    LayerW& ly = layers[l];
    NMX_TRY(linear(ly.qkv, h, H, ly.attn_norm, B, Nqkv, 0, ly.qkv_bias, qkv, Nqkv, nullptr, 0, EPI_STORE));

    AttnArgs at;
    at.q = qkv; at.ldq = Nqkv;
    at.k_cache = pool->k_layer(l); at.v_cache = pool->v_layer(l);
    at.block_tables = block_tables; at.max_blocks = kBlockCap;
    at.tok_seq = tok_seq; at.tok_pos = tok_pos; at.inv_freq = inv_freq;
    at.out = attn;
    at.T = B; at.Hq = cf.n_heads; at.Hkv = cf.n_kv_heads; at.D = cf.head_dim; at.BT = kBT;
    at.splits = splits; at.scale = 1.0f / std::sqrt(float(cf.head_dim));
    at.kv_static = true;
    at.kv_bits = pool->kv_bits; at.kv_gs = pool->kv_gs;
    NMX_TRY(paged_attention(c, at, true));

    NMX_TRY(block_out(ly.o, attn, Nq, B, 0));

    NMX_TRY(linear(ly.gu, h, H, ly.mlp_norm, B, F, F, nullptr, act, F, nullptr, 0, EPI_SILU));

    NMX_TRY(block_out(ly.down, act, F, B, 1));
  }
  return NMX_OK;
}

nmx_status_t Model::run_layers_prefill(KvPool* pool, int T) {
  Ctx* c = ctx;
  const nmx_model_cfg& cf = cfg;
  const int H = cf.hidden, F = cf.ffn, bits = cf.bits, gs = cf.group_size;
  NMX_TRY(embed_rows(c, embed, tok_ids, T, H, h));
  for (int l = 0; l < cf.n_layers; ++l) {
    LayerW& ly = layers[l];
    NMX_TRY(linear(ly.qkv, h, H, ly.attn_norm, T, Nqkv, 0, ly.qkv_bias, qkv, Nqkv, nullptr, 0, EPI_STORE));
    NMX_TRY(rope_append(c, qkv, Nqkv, T, cf.n_heads, cf.n_kv_heads, cf.head_dim, tok_seq, tok_pos,
                        block_tables, kBlockCap, kBT, pool->k_layer(l), pool->v_layer(l), inv_freq,
                        q_roped, Nq, pool->kv_bits, pool->kv_gs));
    AttnArgs at;
    at.q = q_roped; at.ldq = Nq;
    at.k_cache = pool->k_layer(l); at.v_cache = pool->v_layer(l);
    at.block_tables = block_tables; at.max_blocks = kBlockCap;
    at.tok_seq = tok_seq; at.tok_pos = tok_pos; at.out = attn;
    at.T = T; at.Hq = cf.n_heads; at.Hkv = cf.n_kv_heads; at.D = cf.head_dim; at.BT = kBT;
    at.splits = 1; at.scale = 1.0f / std::sqrt(float(cf.head_dim));
    at.pool_blocks = pool->num_blocks; at.prefill_tc_items = n_pf_tc; at.err = c->dev_err;
    at.kv_bits = pool->kv_bits; at.kv_gs = pool->kv_gs;
    NMX_TRY(paged_prefill_attention(c, at, pf_items, n_pf_items));

    NMX_TRY(block_out(ly.o, attn, Nq, T, 0));

    NMX_TRY(linear(ly.gu, h, H, ly.mlp_norm, T, F, F, nullptr, act, F, nullptr, 0, EPI_SILU));

    NMX_TRY(block_out(ly.down, act, F, T, 1));
  }
  return NMX_OK;
}

// lm_head over `rows` hidden rows (already gathered into x), argmax into
// out_ids[0:rows], optional fp32 logits; chunks of 32 rows.
nmx_status_t Model::run_head(const void* x, int rows, bool want_logits, int* next_tokens) {
  Ctx* c = ctx;
  const int H = cfg.hidden, V = cfg.vocab;
  if (!want_logits && lm.dl && rows >= kTcsMinRows && qgemm_tcs_supported(std::min(rows, kTcsMaxRows), V, H, EPI_STORE)) {
    // many rows (a decode batch, a verify block): f16 logits from the
    // tensor-core decode GEMM (one pass over the head's weights per 128
    // rows) into the logits scratch, then a row-wise argmax over them (the
    // GEMV argmax epilogue's rule: f16-rounded values, lowest id on ties)
    half* lg = reinterpret_cast<half*>(logits_f32);
    for (int r0 = 0; r0 < rows; r0 += kTcsMaxRows) {
      const int rc = std::min(kTcsMaxRows, rows - r0);
      NMX_TRY(linear(lm, static_cast<const char*>(x) + size_t(r0) * H * 2, H, final_norm, rc, V, 0, nullptr,
                     lg + size_t(r0) * V, V, nullptr, 0, EPI_STORE));
      NMX_TRY(argmax_rows(c, lg + size_t(r0) * V, rc, V, NMX_F16, out_ids + r0));
      if (next_tokens)
        NMX_CUDA_OK(cudaMemcpyAsync(next_tokens + r0, out_ids + r0, size_t(rc) * 4, cudaMemcpyDeviceToDevice,
                                    c->stream));
    }
    return NMX_OK;
  }
  const int chunk = lm.dl ? std::min(32, qgemv_dl_max_m(H, EPI_ARGMAX)) : 32;
  for (int r0 = 0; r0 < rows; r0 += chunk) {
    const int rc = std::min(chunk, rows - r0);
    NMX_TRY(linear(lm, static_cast<const char*>(x) + size_t(r0) * H * 2, H, final_norm, rc, V, 0, nullptr, nullptr,
                   V, nullptr, 0, EPI_ARGMAX, want_logits ? logits_f32 + size_t(r0) * V : nullptr, out_ids + r0,
                   next_tokens ? next_tokens + r0 : nullptr));
  }
  return NMX_OK;
}

nmx_status_t Model::decode_step_body(KvPool* pool, int B) {
  NMX_TRY(run_layers_decode(pool, B));
  NMX_TRY(run_head(h, B, false, tok_ids));
  return decode_advance(ctx, tok_pos, out_ids, B, hist, kHistCap, step);
}

nmx_status_t Model::run_decode_graph(KvPool* pool, int B) {
  Ctx* c = ctx;
  auto key = std::make_pair(B, static_cast<const void*>(pool));
  auto it = graphs.find(key);
  if (it == graphs.end()) {
    // first use of this shape: run once eagerly (sets kernel attributes), then capture
    NMX_TRY(decode_step_body(pool, B));
    NMX_CUDA_OK(cudaStreamSynchronize(c->stream));
    GraphEntry ge;
    cudaGraph_t g = nullptr;
    NMX_CUDA_OK(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
    const uint64_t before = c->launches;
    nmx_status_t st = decode_step_body(pool, B);
    cudaError_t e = cudaStreamEndCapture(c->stream, &g);
    c->launches = before;
    if (st != NMX_OK) {
      if (g) cudaGraphDestroy(g);
      return st;
    }
    NMX_CUDA_OK(e);
    size_t n = 0;
    NMX_CUDA_OK(cudaGraphGetNodes(g, nullptr, &n));
    ge.nodes = n;
    e = cudaGraphInstantiate(&ge.exec, g, 0);
    cudaGraphDestroy(g);
    NMX_CUDA_OK(e);
    graphs[key] = ge;
    // the eager run above already advanced one step; undo nothing — callers
    // upload positions and tokens before every launch they depend on.
    return NMX_OK;
  }
  NMX_CUDA_OK(cudaGraphLaunch(it->second.exec, c->stream));
  c->launches += it->second.nodes;
  return NMX_OK;
}

nmx_status_t Model::upload_batch(const nmx_seq_t* seqs, int n, int* T_out, bool* decode_out, bool tc_items) {
  NMX_CHECK(n > 0 && seqs, NMX_ERR_INVALID, "forward: empty batch");
  NMX_CHECK(n <= max_batch, NMX_ERR_INVALID, "forward: more sequences than max_batch");
  int T = 0;
  bool decode = true;
  for (int i = 0; i < n; ++i) {
    const nmx_seq_t& s = seqs[i];
    NMX_CHECK(s.n_new_tokens > 0 && s.token_ids && s.start_pos >= 0, NMX_ERR_INVALID,
              "forward: every sequence needs at least one new token");
    NMX_CHECK(s.block_table && s.n_blocks > 0 && s.n_blocks <= kBlockCap, NMX_ERR_INVALID,
              "forward: bad block table");
    NMX_CHECK(long(s.start_pos) + s.n_new_tokens <= long(s.n_blocks) * kBT, NMX_ERR_INVALID,
              "forward: block table does not cover the new tokens");
    T += s.n_new_tokens;
    if (s.n_new_tokens != 1) decode = false;
  }
  NMX_CHECK(T <= max_tokens, NMX_ERR_INVALID, "forward: more tokens than max_tokens");
  int32_t* ids = reinterpret_cast<int32_t*>(pinned);
  int32_t* sq = ids + T;
  int32_t* ps = sq + T;
  int32_t* last = ps + T;
  int32_t* tbl = last + n;
  int t = 0;
  for (int i = 0; i < n; ++i) {
    const nmx_seq_t& s = seqs[i];
    for (int j = 0; j < s.n_new_tokens; ++j, ++t) {
      NMX_CHECK(s.token_ids[j] >= 0 && s.token_ids[j] < cfg.vocab, NMX_ERR_INVALID, "forward: token id out of range");
      ids[t] = s.token_ids[j];
      sq[t] = i;
      ps[t] = s.start_pos + j;
    }
    last[i] = t - 1;
    for (int b = 0; b < s.n_blocks; ++b) {
      NMX_CHECK(s.block_table[b] >= 0 && s.block_table[b] < pool_blocks_hint, NMX_ERR_INVALID,
                "forward: block id out of range");
      tbl[size_t(i) * kBlockCap + b] = s.block_table[b];
    }
  }
  Ctx* c = ctx;
  NMX_CUDA_OK(cudaMemcpyAsync(tok_ids, ids, size_t(T) * 4, cudaMemcpyHostToDevice, c->stream));
  NMX_CUDA_OK(cudaMemcpyAsync(tok_seq, sq, size_t(T) * 4, cudaMemcpyHostToDevice, c->stream));
  NMX_CUDA_OK(cudaMemcpyAsync(tok_pos, ps, size_t(T) * 4, cudaMemcpyHostToDevice, c->stream));
  NMX_CUDA_OK(cudaMemcpyAsync(last_rows, last, size_t(n) * 4, cudaMemcpyHostToDevice, c->stream));
  // all tables in one strided copy of the widest table's columns
  int nb_max = 0;
  for (int i = 0; i < n; ++i) nb_max = std::max(nb_max, seqs[i].n_blocks);
  NMX_CUDA_OK(cudaMemcpy2DAsync(block_tables, size_t(kBlockCap) * 4, tbl, size_t(kBlockCap) * 4, size_t(nb_max) * 4,
                                size_t(n), cudaMemcpyHostToDevice, c->stream));
  h2d_bytes_last = size_t(T) * 12 + size_t(n) * 4 + size_t(n) * nb_max * 4;
  n_pf_items = 0;
  n_pf_tc = 0;
  if (!decode) {
    int2* items = reinterpret_cast<int2*>(tbl + size_t(max_batch) * kBlockCap);
    // quantized pages go through the small-item kernel only
    n_pf_items = prefill_items(sq, T, tc_items ? cfg.head_dim : 0, cfg.n_heads / cfg.n_kv_heads, items, &n_pf_tc);
    NMX_CUDA_OK(cudaMemcpyAsync(pf_items, items, size_t(n_pf_items) * 8, cudaMemcpyHostToDevice, c->stream));
    h2d_bytes_last += size_t(n_pf_items) * 8;
  }
  *T_out = T;
  *decode_out = decode;
  return NMX_OK;
}

nmx_status_t Model::forward(KvPool* pool, const nmx_seq_t* seqs, int n, nmx_out_mode_t mode, void* out_host) {
  NMX_CHECK(weights_ready || loaded_any, NMX_ERR_STATE, "forward: weights not initialised");
  NMX_CHECK(pool && pool->model == this, NMX_ERR_INVALID, "forward: pool belongs to another model");
  NMX_CHECK(out_host, NMX_ERR_INVALID, "forward: null output");
  Ctx* c = ctx;
  pool_blocks_hint = pool->num_blocks;
  int T = 0;
  bool decode = false;
  NMX_TRY(upload_batch(seqs, n, &T, &decode, pool->kv_bits == 0));
  const bool all = (mode == NMX_OUT_ARGMAX_ALL || mode == NMX_OUT_LOGITS_ALL);
  const bool logits = (mode == NMX_OUT_LOGITS_LAST || mode == NMX_OUT_LOGITS_ALL);
  const int rows = all ? T : n;
  NMX_CHECK(rows <= rows_logits, NMX_ERR_UNSUPPORTED, "forward: too many output rows for all-position mode");
  int out_rows = rows;
  if (decode && !all && !logits) {
    NMX_TRY(run_decode_graph(pool, n));
  } else if (decode) {
    NMX_TRY(run_layers_decode(pool, n));
    NMX_TRY(run_head(h, n, logits, nullptr));
  } else {
    NMX_TRY(run_layers_prefill(pool, T));
    if (all) {
      NMX_TRY(run_head(h, T, logits, nullptr));
    } else {
      NMX_TRY(embed_rows(c, h, last_rows, n, cfg.hidden, last_h));
      NMX_TRY(run_head(last_h, n, logits, nullptr));
    }
  }
  if (logits) {
    NMX_CUDA_OK(cudaMemcpyAsync(out_host, logits_f32, size_t(out_rows) * cfg.vocab * 4, cudaMemcpyDeviceToHost,
                                c->stream));
  } else {
    NMX_CUDA_OK(cudaMemcpyAsync(out_host, out_ids, size_t(out_rows) * 4, cudaMemcpyDeviceToHost, c->stream));
  }
  return finish_step();
}

// read the device error word with the step's results, then wait for both
nmx_status_t Model::finish_step() {
  unsigned* perr = reinterpret_cast<unsigned*>(pinned + pinned_bytes - 4);
  *perr = 0u;
  NMX_CUDA_OK(cudaMemcpyAsync(perr, ctx->dev_err, 4, cudaMemcpyDeviceToHost, ctx->stream));
  NMX_CUDA_OK(cudaStreamSynchronize(ctx->stream));
  if (*perr != 0u) return ctx_check_device_error(ctx);
  return NMX_OK;
}

nmx_status_t Model::decode_greedy(KvPool* pool, const int32_t* first, const int32_t* start,
                                  const int32_t* tables, int max_blocks_in, int n, int steps,
                                  int32_t* out_host) {
  NMX_CHECK(weights_ready || loaded_any, NMX_ERR_STATE, "decode: weights not initialised");
  NMX_CHECK(n > 0 && n <= max_batch, NMX_ERR_INVALID, "decode: batch must be in [1, max_batch]");
  NMX_CHECK(steps >= 0 && size_t(steps) * n <= size_t(kHistCap), NMX_ERR_INVALID, "decode: too many steps");
  NMX_CHECK(max_blocks_in > 0 && max_blocks_in <= kBlockCap, NMX_ERR_INVALID, "decode: bad block table width");
  Ctx* c = ctx;
  pool_blocks_hint = pool->num_blocks;
  int32_t* ids = reinterpret_cast<int32_t*>(pinned);
  int32_t* sq = ids + n;
  int32_t* ps = sq + n;
  int32_t* zero = ps + n;
  for (int i = 0; i < n; ++i) {
    NMX_CHECK(first[i] >= 0 && first[i] < cfg.vocab, NMX_ERR_INVALID, "decode: token id out of range");
    NMX_CHECK(long(start[i]) + steps <= long(max_blocks_in) * kBT, NMX_ERR_INVALID,
              "decode: block table does not cover the decoded positions");
    ids[i] = first[i];
    sq[i] = i;
    ps[i] = start[i];
  }
  for (long i = 0; i < long(n) * max_blocks_in; ++i)
    NMX_CHECK(tables[i] >= 0 && tables[i] < pool->num_blocks, NMX_ERR_INVALID, "decode: block id out of range");
  zero[0] = 0;
  NMX_CUDA_OK(cudaMemcpyAsync(tok_ids, ids, size_t(n) * 4, cudaMemcpyHostToDevice, c->stream));
  NMX_CUDA_OK(cudaMemcpyAsync(tok_seq, sq, size_t(n) * 4, cudaMemcpyHostToDevice, c->stream));
  for (int i = 0; i < n; ++i)
    NMX_CUDA_OK(cudaMemcpy2DAsync(block_tables + size_t(i) * kBlockCap, 4, tables + size_t(i) * max_blocks_in, 4,
                                  4, max_blocks_in, cudaMemcpyHostToDevice, c->stream));
  // graph capture happens outside the timed steps: build it first if needed
  auto key = std::make_pair(n, static_cast<const void*>(pool));
  if (graphs.find(key) == graphs.end()) {
    NMX_CUDA_OK(cudaMemcpyAsync(tok_pos, ps, size_t(n) * 4, cudaMemcpyHostToDevice, c->stream));
    NMX_TRY(run_decode_graph(pool, n));  // eager step + capture; positions re-uploaded below
    NMX_CUDA_OK(cudaMemcpyAsync(tok_ids, ids, size_t(n) * 4, cudaMemcpyHostToDevice, c->stream));
  }
  NMX_CUDA_OK(cudaMemcpyAsync(tok_pos, ps, size_t(n) * 4, cudaMemcpyHostToDevice, c->stream));
  NMX_CUDA_OK(cudaMemcpyAsync(step, zero, 4, cudaMemcpyHostToDevice, c->stream));
  for (int s = 0; s < steps; ++s) NMX_TRY(run_decode_graph(pool, n));
  if (out_host && steps > 0)
    NMX_CUDA_OK(cudaMemcpyAsync(out_host, hist, size_t(steps) * n * 4, cudaMemcpyDeviceToHost, c->stream));
  return finish_step();
}

}  // namespace nmx
