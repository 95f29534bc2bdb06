// extern "C" entry points of libnovamlx_cuda (declared in include/nmx.h):
// argument validation, per-thread error strings, handle lifetimes.
#include <cstring>
#include <string>

#include "common.cuh"
#include "kernels.h"
#include "model.h"

namespace nmx {

static thread_local std::string g_err;
void set_error(const std::string& msg) { g_err = msg; }
const char* get_error() { return g_err.c_str(); }
void clear_error() { g_err.clear(); }

nmx_status_t ctx_workspace(Ctx* c, size_t bytes, void** out) {
  if (bytes > c->ws_bytes) {
    if (c->ws) {
      NMX_CUDA_OK(cudaStreamSynchronize(c->stream));
      cudaFree(c->ws);
      c->ws = nullptr;
      c->ws_bytes = 0;
    }
    cudaError_t e = cudaMalloc(&c->ws, bytes);
    if (e != cudaSuccess) {
      cudaGetLastError();
      set_error(std::string("workspace: ") + cudaGetErrorString(e));
      return NMX_ERR_OOM;
    }
    c->ws_bytes = bytes;
  }
  *out = c->ws;
  return NMX_OK;
}

nmx_status_t ctx_check_device_error(Ctx* c) {
  unsigned v = 0;
  NMX_CUDA_OK(cudaMemcpy(&v, c->dev_err, sizeof(v), cudaMemcpyDeviceToHost));
  if (v != 0) {
    NMX_CUDA_OK(cudaMemset(c->dev_err, 0, sizeof(v)));
    std::string what;
    if (v & kErrPeerWait) what += " a peer rank's exchange flag;";
    if (v & kErrPipeWait) what += " a tensor-core GEMM pipeline barrier;";
    if (v & kErrShareWait) what += " the K shares of a split GEMM;";
    set_error("a bounded device wait ran out (device error word " + std::to_string(v) + ":" + what +
              ") results of the work since the last check are not valid");
    return NMX_ERR_TIMEOUT;
  }
  return NMX_OK;
}

nmx_status_t ctx_counters(Ctx* c, size_t n, unsigned** out) {
  if (n > c->n_counters) {
    if (c->counters) {
      NMX_CUDA_OK(cudaStreamSynchronize(c->stream));
      cudaFree(c->counters);
      c->counters = nullptr;
      c->n_counters = 0;
    }
    cudaError_t e = cudaMalloc(reinterpret_cast<void**>(&c->counters), n * sizeof(unsigned));
    if (e != cudaSuccess) {
      cudaGetLastError();
      set_error(std::string("counters: ") + cudaGetErrorString(e));
      return NMX_ERR_OOM;
    }
    NMX_CUDA_OK(cudaMemsetAsync(c->counters, 0, n * sizeof(unsigned), c->stream));
    c->n_counters = n;
  }
  *out = c->counters;
  return NMX_OK;
}

}  // namespace nmx

using namespace nmx;

#define API_BEGIN clear_error();
#define REQUIRE(p, what) NMX_CHECK((p) != nullptr, NMX_ERR_INVALID, std::string("null ") + what)

extern "C" {

NMX_API const char* nmx_last_error(void) { return get_error(); }
NMX_API const char* nmx_version(void) { return "novamlx-b200 0.1 (sm_100a)"; }

NMX_API nmx_status_t nmx_ctx_create(int device, nmx_ctx_t* out) {
  API_BEGIN;
  REQUIRE(out, "output handle");
  int n = 0;
  NMX_CUDA_OK(cudaGetDeviceCount(&n));
  NMX_CHECK(device >= 0 && device < n, NMX_ERR_INVALID, "nmx_ctx_create: no such device");
  NMX_CUDA_OK(cudaSetDevice(device));
  cudaDeviceProp prop;
  NMX_CUDA_OK(cudaGetDeviceProperties(&prop, device));
  NMX_CHECK(prop.major >= 10, NMX_ERR_UNSUPPORTED,
            std::string("nmx_ctx_create: needs an sm_100 device, found ") + prop.name);
  auto* h = new nmx_ctx_s();
  h->c.device = device;
  h->c.num_sms = prop.multiProcessorCount;
  cudaError_t e = cudaStreamCreateWithFlags(&h->c.stream, cudaStreamNonBlocking);
  if (e != cudaSuccess) {
    delete h;
    set_error(std::string("stream: ") + cudaGetErrorString(e));
    return NMX_ERR_CUDA;
  }
  h->c.owns_stream = true;
  e = cudaMalloc(reinterpret_cast<void**>(&h->c.dev_err), 256);
  if (e == cudaSuccess) e = cudaMemset(h->c.dev_err, 0, 256);
  if (e == cudaSuccess) e = cudaMemcpy(h->c.dev_err + 1, &kDefaultWaitPolls, 4, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    cudaGetLastError();
    if (h->c.dev_err) cudaFree(h->c.dev_err);
    cudaStreamDestroy(h->c.stream);
    delete h;
    set_error(std::string("error word: ") + cudaGetErrorString(e));
    return NMX_ERR_CUDA;
  }
  *out = h;
  return NMX_OK;
}

static void ctx_release(nmx_ctx_t ctx) {
  if (--ctx->refs > 0) return;
  cudaSetDevice(ctx->c.device);
  if (ctx->c.stream) cudaStreamSynchronize(ctx->c.stream);
  if (ctx->c.ws) cudaFree(ctx->c.ws);
  if (ctx->c.counters) cudaFree(ctx->c.counters);
  if (ctx->c.dev_err) cudaFree(ctx->c.dev_err);
  if (ctx->c.owns_stream && ctx->c.stream) cudaStreamDestroy(ctx->c.stream);
  delete ctx;
}

static void model_release(nmx_model_t model) {
  if (--model->refs > 0) return;
  cudaStreamSynchronize(model->m->ctx->stream);
  delete model->m;
  nmx_ctx_s* ctx = model->ctx;
  delete model;
  ctx_release(ctx);
}

NMX_API nmx_status_t nmx_ctx_destroy(nmx_ctx_t ctx) {
  API_BEGIN;
  if (!ctx) return NMX_OK;
  ctx_release(ctx);
  return NMX_OK;
}

NMX_API nmx_status_t nmx_ctx_set_stream(nmx_ctx_t ctx, void* stream) {
  API_BEGIN;
  REQUIRE(ctx, "context");
  if (ctx->c.owns_stream && ctx->c.stream) {
    cudaStreamSynchronize(ctx->c.stream);
    cudaStreamDestroy(ctx->c.stream);
  }
  ctx->c.stream = static_cast<cudaStream_t>(stream);
  ctx->c.owns_stream = false;
  return NMX_OK;
}

NMX_API void* nmx_ctx_stream(nmx_ctx_t ctx) { return ctx ? static_cast<void*>(ctx->c.stream) : nullptr; }

NMX_API nmx_status_t nmx_ctx_synchronize(nmx_ctx_t ctx) {
  API_BEGIN;
  REQUIRE(ctx, "context");
  NMX_CUDA_OK(cudaStreamSynchronize(ctx->c.stream));
  return ctx_check_device_error(&ctx->c);
}

NMX_API nmx_status_t nmx_ctx_set_wait_limit(nmx_ctx_t ctx, uint32_t polls) {
  API_BEGIN;
  REQUIRE(ctx, "context");
  // the value travels with the stream, so kernels already queued keep theirs
  static thread_local uint32_t v;
  v = polls == 0 ? kDefaultWaitPolls : polls;
  NMX_CUDA_OK(cudaMemcpyAsync(ctx->c.dev_err + 1, &v, 4, cudaMemcpyHostToDevice, ctx->c.stream));
  NMX_CUDA_OK(cudaStreamSynchronize(ctx->c.stream));
  return NMX_OK;
}

NMX_API uint64_t nmx_ctx_kernel_launches(nmx_ctx_t ctx) { return ctx ? ctx->c.launches : 0; }

// ---------------------------------------------------------------- op level

static nmx_status_t check_dt16(nmx_dtype_t dt, const char* who) {
  NMX_CHECK(dt == NMX_F16 || dt == NMX_BF16, NMX_ERR_UNSUPPORTED, std::string(who) + ": dtype must be f16 or bf16");
  return NMX_OK;
}

NMX_API nmx_status_t nmx_op_qmatmul(nmx_ctx_t ctx, const void* x, const uint32_t* w, const void* scales,
                                    const void* biases, int M, int N, int K, int bits, int group_size,
                                    int transpose, nmx_dtype_t dtype, void* y) {
  API_BEGIN;
  REQUIRE(ctx, "context");
  NMX_CHECK(M >= 0 && N >= 0 && K >= 0, NMX_ERR_INVALID, "nmx_op_qmatmul: negative size");
  if (M == 0 || N == 0) return NMX_OK;
  REQUIRE(x, "x");
  REQUIRE(w, "w");
  REQUIRE(scales, "scales");
  REQUIRE(biases, "biases");
  REQUIRE(y, "y");
  NMX_CHECK(transpose == 1, NMX_ERR_UNSUPPORTED, "nmx_op_qmatmul: only transpose = true is built");
  NMX_TRY(check_dt16(dtype, "nmx_op_qmatmul"));
  NMX_CHECK(reinterpret_cast<uintptr_t>(w) % 16 == 0, NMX_ERR_INVALID, "nmx_op_qmatmul: w must be 16-byte aligned");
  GemvArgs a;
  a.x = x; a.ldx = K; a.w = w; a.s = scales; a.b = biases; a.N = N; a.K = K; a.M = M; a.y = y; a.ldy = N;
  return qgemv(&ctx->c, a, bits, group_size, dtype, EPI_STORE);
}

NMX_API nmx_status_t nmx_op_pack_records(nmx_ctx_t ctx, const uint32_t* wq, const void* scales, const void* biases,
                                         int N, int K, void* records) {
  API_BEGIN;
  REQUIRE(ctx, "context");
  if (N == 0) return NMX_OK;
  REQUIRE(wq, "wq");
  REQUIRE(scales, "scales");
  REQUIRE(biases, "biases");
  REQUIRE(records, "records");
  NMX_CHECK(N % 16 == 0 && K % 128 == 0, NMX_ERR_UNSUPPORTED, "nmx_op_pack_records: N % 16, K % 128");
  NMX_CHECK(reinterpret_cast<uintptr_t>(records) % 16 == 0, NMX_ERR_INVALID, "records must be 16-byte aligned");
  return repack_to_records(&ctx->c, wq, scales, biases, N, K, 0, records, 7);
}

NMX_API nmx_status_t nmx_op_qmatmul_records(nmx_ctx_t ctx, const void* x, const void* records, int M, int N, int K,
                                            void* y) {
  API_BEGIN;
  REQUIRE(ctx, "context");
  if (M == 0 || N == 0) return NMX_OK;
  REQUIRE(x, "x");
  REQUIRE(records, "records");
  REQUIRE(y, "y");
  NMX_CHECK(qgemv_dl_supported(4, 64, NMX_F16, N, K), NMX_ERR_UNSUPPORTED, "nmx_op_qmatmul_records: needs N % 16 == 0, K % 128 == 0, (N/16)*(K/128) >= 8");
  NMX_CHECK(reinterpret_cast<uintptr_t>(records) % 16 == 0, NMX_ERR_INVALID, "records must be 16-byte aligned");
  Ctx* c = &ctx->c;
  GemvDLArgs a;
  const size_t pf = std::max(qgemv_dl_partials_floats(N, K, EPI_STORE, c->num_sms, a.ctas_per_sm),
                             qgemm_tcs_partials_floats(std::min(M, kTcsMaxRows), N, K, EPI_STORE, c->num_sms));
  void* ws = nullptr;
  NMX_TRY(ctx_workspace(c, pf * 4 + 256, &ws));
  unsigned* ctr = nullptr;
  NMX_TRY(ctx_counters(c, size_t(N / 16), &ctr));
  a.x = x; a.ldx = K; a.w = records; a.N = N; a.K = K; a.M = M; a.y = y; a.ldy = N;
  a.partials = static_cast<float*>(ws); a.partials_cap = pf; a.counters = ctr; a.err = c->dev_err;
  return qgemv_dl(c, a, EPI_STORE);
}

NMX_API nmx_status_t nmx_op_quantize(nmx_ctx_t ctx, const float* w, int N, int K, int bits, int group_size,
                                     nmx_dtype_t sdtype, uint32_t* wq, void* scales, void* biases) {
  API_BEGIN;
  REQUIRE(ctx, "context");
  if (N == 0) return NMX_OK;
  REQUIRE(w, "w");
  REQUIRE(wq, "wq");
  REQUIRE(scales, "scales");
  REQUIRE(biases, "biases");
  return quantize(&ctx->c, w, N, K, bits, group_size, sdtype, wq, scales, biases);
}

NMX_API nmx_status_t nmx_op_dequantize(nmx_ctx_t ctx, const uint32_t* wq, const void* scales, const void* biases,
                                       int N, int K, int bits, int group_size, nmx_dtype_t sdtype, float* w) {
  API_BEGIN;
  REQUIRE(ctx, "context");
  if (N == 0) return NMX_OK;
  REQUIRE(wq, "wq");
  REQUIRE(scales, "scales");
  REQUIRE(biases, "biases");
  REQUIRE(w, "w");
  return dequantize(&ctx->c, wq, scales, biases, N, K, bits, group_size, sdtype, w);
}

NMX_API nmx_status_t nmx_op_rmsnorm(nmx_ctx_t ctx, const void* x, const void* gamma, int M, int H, float eps,
                                    nmx_dtype_t dtype, void* y) {
  API_BEGIN;
  REQUIRE(ctx, "context");
  if (M == 0) return NMX_OK;
  REQUIRE(x, "x");
  REQUIRE(gamma, "gamma");
  REQUIRE(y, "y");
  NMX_CHECK(H > 0, NMX_ERR_INVALID, "nmx_op_rmsnorm: H must be positive");
  return rmsnorm(&ctx->c, x, H, gamma, M, H, eps, dtype, y, H);
}

NMX_API nmx_status_t nmx_op_argmax(nmx_ctx_t ctx, const void* logits, int M, int V, nmx_dtype_t dtype,
                                   int32_t* out) {
  API_BEGIN;
  REQUIRE(ctx, "context");
  if (M == 0) return NMX_OK;
  REQUIRE(logits, "logits");
  REQUIRE(out, "out");
  return argmax_rows(&ctx->c, logits, M, V, dtype, out);
}

NMX_API nmx_status_t nmx_op_sample(nmx_ctx_t ctx, const void* logits, int M, int V, nmx_dtype_t dtype,
                                   float temperature, float top_p, uint64_t seed, uint64_t counter, int32_t* out_ids,
                                   float* out_logprob, int top_k, int32_t* out_top_ids, float* out_top_logprobs) {
  API_BEGIN;
  REQUIRE(ctx, "context");
  if (M == 0) return NMX_OK;
  REQUIRE(logits, "logits");
  REQUIRE(out_ids, "out_ids");
  return sample_rows(&ctx->c, logits, dtype, M, V, temperature, top_p, seed, counter, out_ids, out_logprob, top_k,
                     out_top_ids, out_top_logprobs);
}

NMX_API nmx_status_t nmx_op_penalized_argmax(nmx_ctx_t ctx, const void* logits, int M, int V, nmx_dtype_t dtype,
                                             const int32_t* recent, const int32_t* n_recent, int max_recent,
                                             float penalty, int32_t* out) {
  API_BEGIN;
  REQUIRE(ctx, "context");
  if (M == 0) return NMX_OK;
  REQUIRE(logits, "logits");
  REQUIRE(recent, "recent");
  REQUIRE(n_recent, "n_recent");
  REQUIRE(out, "out");
  return penalized_argmax(&ctx->c, logits, M, V, dtype, recent, n_recent, max_recent, penalty, out);
}

NMX_API nmx_status_t nmx_op_attn_quantized_decode(nmx_ctx_t ctx, const void* q, const uint32_t* k_w,
                                                  const void* k_s, const void* k_b, const uint32_t* v_w,
                                                  const void* v_s, const void* v_b, int B, int Hq, int Hkv,
                                                  int N, int L, int D, float scale, int group_size, int bits,
                                                  int allow_multi_query, nmx_dtype_t dtype, void* out) {
  API_BEGIN;
  REQUIRE(ctx, "context");
  // the reference kernel's guards (FusedQuantizedSDPA.swift:179-188)
  NMX_CHECK(L == 1 || allow_multi_query, NMX_ERR_UNSUPPORTED, "quantized sdpa: L must be 1");
  NMX_CHECK(D == 64 || D == 96 || D == 128 || D == 256, NMX_ERR_UNSUPPORTED, "quantized sdpa: D not supported");
  NMX_CHECK(bits == 4 || bits == 8, NMX_ERR_UNSUPPORTED, "quantized sdpa: bits must be 4 or 8");
  NMX_CHECK(group_size > 0 && D % group_size == 0, NMX_ERR_UNSUPPORTED, "quantized sdpa: D % group_size != 0");
  NMX_CHECK(k_b && v_b, NMX_ERR_UNSUPPORTED, "quantized sdpa: biases are required");
  NMX_CHECK(Hkv > 0 && Hq % Hkv == 0, NMX_ERR_INVALID, "quantized sdpa: Hq must be a multiple of Hkv");
  NMX_CHECK(N >= 0 && L >= 1 && B >= 0, NMX_ERR_INVALID, "quantized sdpa: bad sizes");
  REQUIRE(q, "q");
  REQUIRE(k_w, "k_w");
  REQUIRE(k_s, "k_s");
  REQUIRE(v_w, "v_w");
  REQUIRE(v_s, "v_s");
  REQUIRE(out, "out");
  NMX_TRY(check_dt16(dtype, "quantized sdpa"));
  return quantized_sdpa(&ctx->c, q, k_w, k_s, k_b, v_w, v_s, v_b, B * Hq, Hq / Hkv, N, L, D, scale, group_size,
                        bits, dtype, out);
}

NMX_API nmx_status_t nmx_op_attn_paged_decode(nmx_ctx_t ctx, const void* q, const void* k_cache,
                                              const void* v_cache, const int32_t* block_tables,
                                              const int32_t* seq_lens, int B, int Hq, int Hkv, int D,
                                              int block_tokens, int max_blocks, float scale, void* out) {
  API_BEGIN;
  REQUIRE(ctx, "context");
  if (B == 0) return NMX_OK;
  REQUIRE(q, "q");
  REQUIRE(k_cache, "k_cache");
  REQUIRE(v_cache, "v_cache");
  REQUIRE(block_tables, "block_tables");
  REQUIRE(seq_lens, "seq_lens");
  REQUIRE(out, "out");
  NMX_CHECK(Hkv > 0 && Hq % Hkv == 0, NMX_ERR_INVALID, "paged decode: Hq must be a multiple of Hkv");
  NMX_CHECK(B > 0 && B <= kMaxDecodeRows, NMX_ERR_UNSUPPORTED,
            "paged decode: at most " + std::to_string(kMaxDecodeRows) + " rows per call");
  Ctx* c = &ctx->c;
  const int S = decode_attn_splits(c->num_sms, B, Hkv);
  // workspace: the row descriptors tok_seq[B], tok_pos[B]
  void* ws = nullptr;
  NMX_TRY(ctx_workspace(c, size_t(B) * 8, &ws));
  int* tok_seq = static_cast<int*>(ws);
  int* tok_pos = tok_seq + B;
  NMX_TRY(seq_rows_from_lens(c, seq_lens, B, tok_seq, tok_pos));
  AttnArgs a;
  a.q = q; a.ldq = long(Hq) * D; a.k_cache = const_cast<void*>(k_cache); a.v_cache = const_cast<void*>(v_cache);
  a.block_tables = block_tables; a.max_blocks = max_blocks; a.tok_seq = tok_seq; a.tok_pos = tok_pos;
  a.out = out;
  a.T = B; a.Hq = Hq; a.Hkv = Hkv; a.D = D; a.BT = block_tokens; a.splits = S; a.scale = scale;
  return paged_attention(c, a, false);
}

// ------------------------------------------------------------- model level

NMX_API nmx_status_t nmx_model_create(nmx_ctx_t ctx, const nmx_model_cfg* cfg, nmx_model_t* out) {
  API_BEGIN;
  REQUIRE(ctx, "context");
  REQUIRE(cfg, "config");
  REQUIRE(out, "output handle");
  NMX_CUDA_OK(cudaSetDevice(ctx->c.device));
  Model* m = nullptr;
  NMX_TRY(Model::create(&ctx->c, *cfg, &m));
  ctx->refs++;
  *out = new nmx_model_s{m, ctx};
  return NMX_OK;
}

NMX_API nmx_status_t nmx_model_destroy(nmx_model_t model) {
  API_BEGIN;
  if (!model) return NMX_OK;
  model_release(model);
  return NMX_OK;
}

NMX_API nmx_status_t nmx_model_init_random(nmx_model_t model, uint64_t seed, float stdv) {
  API_BEGIN;
  REQUIRE(model, "model");
  return model->m->init_random(seed, stdv);
}

NMX_API nmx_status_t nmx_model_load_tensor(nmx_model_t model, const char* name, const void* host,
                                           nmx_dtype_t dtype, const int64_t* shape, int ndim) {
  API_BEGIN;
  REQUIRE(model, "model");
  REQUIRE(name, "name");
  REQUIRE(host, "host data");
  REQUIRE(shape, "shape");
  return model->m->load_tensor(name, host, dtype, shape, ndim);
}

NMX_API nmx_status_t nmx_model_get_tensor(nmx_model_t model, const char* name, void* host, size_t host_bytes) {
  API_BEGIN;
  REQUIRE(model, "model");
  REQUIRE(name, "name");
  REQUIRE(host, "host buffer");
  return model->m->get_tensor(name, host, host_bytes);
}

NMX_API uint64_t nmx_model_weight_bytes(nmx_model_t model) { return model ? model->m->wbytes : 0; }
NMX_API uint64_t nmx_model_step_weight_bytes(nmx_model_t model) { return model ? model->m->step_bytes : 0; }

NMX_API nmx_status_t nmx_kv_pool_create(nmx_model_t model, int block_tokens, int num_blocks, nmx_kv_pool_t* out) {
  API_BEGIN;
  REQUIRE(model, "model");
  REQUIRE(out, "output handle");
  KvPool* p = nullptr;
  NMX_TRY(KvPool::create(model->m, block_tokens, num_blocks, &p));
  model->refs++;
  *out = new nmx_kv_pool_s{p, model};
  return NMX_OK;
}

NMX_API nmx_status_t nmx_kv_pool_create_quantized(nmx_model_t model, int block_tokens, int num_blocks, int kv_bits,
                                                  int kv_group_size, nmx_kv_pool_t* out) {
  API_BEGIN;
  REQUIRE(model, "model");
  REQUIRE(out, "output handle");
  NMX_CHECK(kv_bits == 4 || kv_bits == 8, NMX_ERR_UNSUPPORTED, "quantized kv pool: bits must be 4 or 8");
  KvPool* p = nullptr;
  NMX_TRY(KvPool::create(model->m, block_tokens, num_blocks, &p, kv_bits, kv_group_size));
  model->refs++;
  *out = new nmx_kv_pool_s{p, model};
  return NMX_OK;
}

NMX_API uint64_t nmx_kv_pool_bytes_per_token(nmx_kv_pool_t pool) {
  if (!pool) return 0;
  const KvPool* p = pool->p;
  return uint64_t(p->block_bytes) * 2 * uint64_t(p->model->cfg.n_layers) / 16;
}

NMX_API nmx_status_t nmx_kv_pool_destroy(nmx_kv_pool_t pool) {
  API_BEGIN;
  if (!pool) return NMX_OK;
  cudaStreamSynchronize(pool->p->model->ctx->stream);
  pool->p->model->graphs_drop_pool(pool->p);
  delete pool->p;
  nmx_model_s* model = pool->model;
  delete pool;
  model_release(model);
  return NMX_OK;
}

NMX_API nmx_status_t nmx_kv_copy_blocks(nmx_kv_pool_t pool, const int32_t* src, const int32_t* dst, int n) {
  API_BEGIN;
  REQUIRE(pool, "pool");
  if (n == 0) return NMX_OK;
  REQUIRE(src, "src");
  REQUIRE(dst, "dst");
  KvPool* p = pool->p;
  Ctx* c = p->model->ctx;
  for (int i = 0; i < n; ++i)
    NMX_CHECK(src[i] >= 0 && src[i] < p->num_blocks && dst[i] >= 0 && dst[i] < p->num_blocks,
              NMX_ERR_INVALID, "kv copy: block id out of range");
  void* ws = nullptr;
  NMX_TRY(ctx_workspace(c, size_t(n) * 8, &ws));
  int* d_src = static_cast<int*>(ws);
  NMX_CUDA_OK(cudaMemcpyAsync(d_src, src, size_t(n) * 4, cudaMemcpyHostToDevice, c->stream));
  NMX_CUDA_OK(cudaMemcpyAsync(d_src + n, dst, size_t(n) * 4, cudaMemcpyHostToDevice, c->stream));
  NMX_TRY(copy_kv_blocks(c, p->base, long(p->layer_stride), p->model->cfg.n_layers, long(p->block_bytes), d_src,
                         d_src + n, n));
  NMX_CUDA_OK(cudaStreamSynchronize(c->stream));
  return NMX_OK;
}

static nmx_status_t kv_host_copy(nmx_kv_pool_t pool, const int32_t* ids, int n, void* host, bool to_host) {
  KvPool* p = pool->p;
  Ctx* c = p->model->ctx;
  const int L = p->model->cfg.n_layers;
  for (int i = 0; i < n; ++i)
    NMX_CHECK(ids[i] >= 0 && ids[i] < p->num_blocks, NMX_ERR_INVALID, "kv host copy: block id out of range");
  NMX_CUDA_OK(cudaStreamSynchronize(c->stream));
  char* hb = static_cast<char*>(host);
  for (int i = 0; i < n; ++i)
    for (int l = 0; l < L; ++l)
      for (int kv = 0; kv < 2; ++kv) {
        char* d = static_cast<char*>(kv == 0 ? p->k_layer(l) : p->v_layer(l)) + size_t(ids[i]) * p->block_bytes;
        char* h = hb + ((size_t(i) * L + l) * 2 + kv) * p->block_bytes;
        if (to_host) {
          NMX_CUDA_OK(cudaMemcpyAsync(h, d, p->block_bytes, cudaMemcpyDeviceToHost, c->stream));
        } else {
          NMX_CUDA_OK(cudaMemcpyAsync(d, h, p->block_bytes, cudaMemcpyHostToDevice, c->stream));
        }
      }
  NMX_CUDA_OK(cudaStreamSynchronize(c->stream));
  return NMX_OK;
}

NMX_API nmx_status_t nmx_kv_read_blocks(nmx_kv_pool_t pool, const int32_t* ids, int n, void* host) {
  API_BEGIN;
  REQUIRE(pool, "pool");
  if (n == 0) return NMX_OK;
  REQUIRE(ids, "ids");
  REQUIRE(host, "host buffer");
  return kv_host_copy(pool, ids, n, host, true);
}

NMX_API nmx_status_t nmx_kv_write_blocks(nmx_kv_pool_t pool, const int32_t* ids, int n, const void* host) {
  API_BEGIN;
  REQUIRE(pool, "pool");
  if (n == 0) return NMX_OK;
  REQUIRE(ids, "ids");
  REQUIRE(host, "host buffer");
  return kv_host_copy(pool, ids, n, const_cast<void*>(host), false);
}

NMX_API nmx_status_t nmx_kv_pool_layer_ptrs(nmx_kv_pool_t pool, int layer, void** k, void** v) {
  API_BEGIN;
  REQUIRE(pool, "pool");
  NMX_CHECK(layer >= 0 && layer < pool->p->model->cfg.n_layers, NMX_ERR_INVALID, "kv pool: layer out of range");
  if (k) *k = pool->p->k_layer(layer);
  if (v) *v = pool->p->v_layer(layer);
  return NMX_OK;
}

NMX_API int nmx_kv_pool_num_blocks(nmx_kv_pool_t pool) { return pool ? pool->p->num_blocks : 0; }

NMX_API nmx_status_t nmx_kv_pool_fill_random(nmx_kv_pool_t pool, uint64_t seed, float std) {
  API_BEGIN;
  REQUIRE(pool, "pool");
  KvPool* p = pool->p;
  Ctx* c = p->model->ctx;
  const size_t halves = p->layer_stride * size_t(p->model->cfg.n_layers) / 2;
  NMX_TRY(random_fill(c, seed, 0x6b76ull, std, 0.f, halves, NMX_F16, p->base));
  NMX_CUDA_OK(cudaStreamSynchronize(c->stream));
  return NMX_OK;
}

NMX_API uint64_t nmx_kv_bytes_per_token(nmx_model_t model) {
  if (!model) return 0;
  const auto& c = model->m->cfg;
  return 2ull * c.n_layers * c.n_kv_heads * c.head_dim * 2ull;
}

NMX_API nmx_status_t nmx_forward(nmx_model_t model, nmx_kv_pool_t pool, const nmx_seq_t* seqs, int n_seqs,
                                 nmx_out_mode_t mode, void* out_host) {
  API_BEGIN;
  REQUIRE(model, "model");
  REQUIRE(pool, "pool");
  REQUIRE(seqs, "seqs");
  NMX_CUDA_OK(cudaSetDevice(model->m->ctx->device));
  return model->m->forward(pool->p, seqs, n_seqs, mode, out_host);
}

NMX_API nmx_status_t nmx_decode_greedy(nmx_model_t model, nmx_kv_pool_t pool, const int32_t* first_tokens,
                                       const int32_t* start_pos, const int32_t* block_tables, int max_blocks,
                                       int n_seqs, int n_steps, int32_t* out_ids_host) {
  API_BEGIN;
  REQUIRE(model, "model");
  REQUIRE(pool, "pool");
  REQUIRE(first_tokens, "first_tokens");
  REQUIRE(start_pos, "start_pos");
  REQUIRE(block_tables, "block_tables");
  NMX_CUDA_OK(cudaSetDevice(model->m->ctx->device));
  return model->m->decode_greedy(pool->p, first_tokens, start_pos, block_tables, max_blocks, n_seqs, n_steps,
                                 out_ids_host);
}

}  // extern "C"
