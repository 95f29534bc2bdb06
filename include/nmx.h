/*
 * nmx.h — C ABI of libnovamlx_cuda.so, the sm_100a (B200) implementation of
 * NovaMLX's decode/prefill hot path: MLX-affine group-quantized matmul
 * (4/8-bit, uint32-packed, fp16/bf16 per-group scales and biases), attention
 * over a paged, prefix-shared KV cache, and the Llama/Qwen2 block around them.
 *
 * Conventions
 *   - Every entry point returns nmx_status_t. On failure the message is kept
 *     per thread and read with nmx_last_error(). There is no CPU fallback:
 *     an unsupported shape returns NMX_ERR_UNSUPPORTED and the caller decides,
 *     which is the contract of the reference's attention hook (a nil return
 *     means "use the stock path"), Sources/NovaMLXEngine/FusedQuantizedSDPA.swift:179-188.
 *   - Op-level entry points ("nmx_op_*") take DEVICE pointers and run on the
 *     context's stream (stream-ordered, no implicit synchronisation).
 *     Model-level entry points take HOST pointers, which are borrowed for the
 *     duration of the call; the library owns every device allocation behind
 *     an opaque handle.
 *   - One model handle is not re-entrant (the reference serialises its model
 *     behind `mlxContainer.perform`, Sources/NovaMLXEngine/FusedBatchScheduler.swift:631-634).
 *     Different contexts may be used from different threads.
 *   - Packed weight layout (identical to MLX's): W u32[N, K*bits/32], value k
 *     of row n sits in word k/(32/bits) at bit offset (k%(32/bits))*bits, low
 *     bits first; scales/biases [N, K/group]; dequant = q*scale + bias
 *     (Sources/NovaMLXEngine/FusedQuantizedSDPA.swift:77-81,95-99).
 */
#ifndef NMX_H
#define NMX_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NMX_API __attribute__((visibility("default")))

typedef enum {
  NMX_OK = 0,
  NMX_ERR_INVALID = 1,     /* bad argument (null pointer, negative size, ...) */
  NMX_ERR_UNSUPPORTED = 2, /* shape/bits/group/dtype combination not built    */
  NMX_ERR_CUDA = 3,        /* CUDA runtime or kernel error                    */
  NMX_ERR_OOM = 4,         /* device allocation failed or KV pool exhausted   */
  NMX_ERR_TIMEOUT = 5,     /* a bounded device-side wait ran out              */
  NMX_ERR_STATE = 6,       /* call made in the wrong state (e.g. no weights)  */
  NMX_ERR_NOT_FOUND = 7    /* unknown tensor name / request id                */
} nmx_status_t;

typedef enum {
  NMX_F16 = 0,
  NMX_BF16 = 1,
  NMX_F32 = 2,
  NMX_U32 = 3,
  NMX_I32 = 4
} nmx_dtype_t;

/* ------------------------------------------------------------------------ */
/* Library / context                                                         */
/* ------------------------------------------------------------------------ */

/* Message of the last failed call on this thread ("" if none). */
NMX_API const char* nmx_last_error(void);
NMX_API const char* nmx_version(void);

typedef struct nmx_ctx_s* nmx_ctx_t;

/* Bind a CUDA device and create one non-blocking stream. Replaces the
 * implicit MLX default device/stream the engine uses
 * (Sources/NovaMLXEngine/MLXEngine.swift:654 loadModel → mlx-swift). */
NMX_API nmx_status_t nmx_ctx_create(int device, nmx_ctx_t* out);
NMX_API nmx_status_t nmx_ctx_destroy(nmx_ctx_t ctx);
/* Use an external cudaStream_t (passed as void*) instead of the owned one. */
NMX_API nmx_status_t nmx_ctx_set_stream(nmx_ctx_t ctx, void* cuda_stream);
NMX_API void* nmx_ctx_stream(nmx_ctx_t ctx);
/* Waits for the context's stream; NMX_ERR_TIMEOUT if a kernel gave up a
 * bounded device-side wait since the last check (the error is then cleared
 * and the results of that work are not valid). */
NMX_API nmx_status_t nmx_ctx_synchronize(nmx_ctx_t ctx);
/* Polls a device-side wait makes before it gives up and reports
 * NMX_ERR_TIMEOUT (peer-rank exchange flags, the pipeline barriers of the
 * tensor-core GEMMs, the K shares of a split GEMM); 0 restores the default
 * (2^24 polls, seconds). Every wait is bounded, so a rank that never
 * publishes, or a fault elsewhere, ends the kernel instead of holding the
 * GPU. Takes effect for kernels launched after the call (stream order). No
 * counterpart in the reference, whose MLX calls have no device waits. */
NMX_API nmx_status_t nmx_ctx_set_wait_limit(nmx_ctx_t ctx, uint32_t polls);
/* Number of kernels this library launched on the context so far (graph
 * replays count every node). Used by benchmarks to report launches. */
NMX_API uint64_t nmx_ctx_kernel_launches(nmx_ctx_t ctx);

/* ------------------------------------------------------------------------ */
/* Op level (device pointers)                                                */
/* ------------------------------------------------------------------------ */

/* y[M,N] = x[M,K] · dequant(W)[N,K]^T   (transpose = 1, the only layout MLX's
 * QuantizedLinear uses). fp32 accumulation, output rounded to `dtype`.
 * Replaces MLX.quantizedMM(x, w, scales:, biases:, transpose: true,
 * groupSize:, bits:) — Sources/NovaMLXEngine/Models/BailingHybridModel.swift:213.
 * bits ∈ {4, 8}; group_size ∈ {32, 64, 128}; dtype ∈ {NMX_F16, NMX_BF16}
 * (x, scales, biases and y share it); N % 16 == 0, K % group_size == 0. */
NMX_API nmx_status_t nmx_op_qmatmul(nmx_ctx_t ctx, const void* x, const uint32_t* w,
                                    const void* scales, const void* biases, int M, int N,
                                    int K, int bits, int group_size, int transpose,
                                    nmx_dtype_t dtype, void* y);

/* Repack an MLX-layout 4-bit group-64 fp16 linear (wq u32[N, K/8], scales
 * and biases f16[N, K/64]) into decode records: 1152-byte records of 16 rows
 * x 128 k (packed words in MMA-fragment order, then the 2x16 scales and
 * biases), the layout the model streams in its decode GEMV. `records` holds
 * N*K*9/16 bytes (the same bytes as the three MLX arrays). N % 16 == 0,
 * K % 128 == 0. Same operator as MLX.quantizedMM's weights
 * (Sources/NovaMLXEngine/Models/BailingHybridModel.swift:213), stored for
 * streaming. */
NMX_API nmx_status_t nmx_op_pack_records(nmx_ctx_t ctx, const uint32_t* wq, const void* scales,
                                         const void* biases, int N, int K, void* records);
/* y[M,N] = x[M,K] · dequant(W)^T for W held as decode records (see
 * nmx_op_pack_records); fp16 in/out, fp32 accumulation. Same arithmetic as
 * nmx_op_qmatmul on the MLX-layout weights. */
NMX_API nmx_status_t nmx_op_qmatmul_records(nmx_ctx_t ctx, const void* x, const void* records, int M,
                                            int N, int K, void* y);

/* Affine quantization of fp32 W[N,K] along K: per group, scale =
 * (max-min)/(2^bits-1), bias = min, q = clamp(rint((w-bias)/scale), 0,
 * 2^bits-1) computed with the fp32 scale/bias, which are then stored in
 * `sdtype`. A constant group stores scale 0 and q = 0. Replaces
 * MLX.quantized(w, groupSize:, bits:) —
 * Sources/NovaMLXEngine/Models/BailingHybridModel.swift:179. */
NMX_API nmx_status_t nmx_op_quantize(nmx_ctx_t ctx, const float* w, int N, int K, int bits,
                                     int group_size, nmx_dtype_t sdtype, uint32_t* wq,
                                     void* scales, void* biases);

/* w[N,K] (fp32) = dequant(wq, scales, biases). Replaces MLX.dequantized —
 * Sources/NovaMLXEngine/Models/BailingHybridModel.swift:816. */
NMX_API nmx_status_t nmx_op_dequantize(nmx_ctx_t ctx, const uint32_t* wq, const void* scales,
                                       const void* biases, int N, int K, int bits,
                                       int group_size, nmx_dtype_t sdtype, float* w);

/* y[M,H] = x * rsqrt(mean(x^2) + eps) * gamma, fp32 math, output in dtype.
 * Replaces MLXFast.rmsNorm — Sources/NovaMLXEngine/Models/BailingHybridModel.swift:244. */
NMX_API nmx_status_t nmx_op_rmsnorm(nmx_ctx_t ctx, const void* x, const void* gamma, int M,
                                    int H, float eps, nmx_dtype_t dtype, void* y);

/* out[m] = argmax_v logits[m, v] (lowest index on ties), logits in dtype
 * (f16/bf16/f32). Replaces CompiledSampler's greedy argMax —
 * Sources/NovaMLXEngine/CompiledSampler.swift:24-27. */
NMX_API nmx_status_t nmx_op_argmax(nmx_ctx_t ctx, const void* logits, int M, int V,
                                   nmx_dtype_t dtype, int32_t* out);

/* Sampling beyond greedy, per row of logits (dtype f16/bf16/f32), all
 * outputs in device memory: temperature 0 → argmax; otherwise categorical
 * over logSoftmax(logits) / temperature, restricted to the top-p nucleus when
 * 0 < top_p < 1 (the tokens whose strictly-higher probability mass is below
 * top_p, as CompiledSampler keeps them, Sources/NovaMLXEngine/CompiledSampler.swift:28-49).
 * Draws are a function of (seed, counter, row, token): the same arguments
 * give the same ids. out_logprob (may be NULL): the chosen id's logprob;
 * top_k (0..32) largest logprobs and their ids, descending — the data of
 * computeRawLogprobs, FusedBatchScheduler.swift:900-941. */
NMX_API nmx_status_t nmx_op_sample(nmx_ctx_t ctx, const void* logits, int M, int V, nmx_dtype_t dtype,
                                   float temperature, float top_p, uint64_t seed, uint64_t counter,
                                   int32_t* out_ids, float* out_logprob, int top_k, int32_t* out_top_ids,
                                   float* out_top_logprobs);

/* Greedy next id with the engine's frequency penalty applied first:
 * logits[m] - penalty * histogram(recent[m, 0:n_recent[m]]) →
 * argmax. recent is int32[M, max_recent]. Mirrors
 * Sources/NovaMLXEngine/FusedBatchScheduler.swift:1218-1227,1231. */
NMX_API nmx_status_t nmx_op_penalized_argmax(nmx_ctx_t ctx, const void* logits, int M, int V,
                                             nmx_dtype_t dtype, const int32_t* recent,
                                             const int32_t* n_recent, int max_recent,
                                             float penalty, int32_t* out);

/* Single-query attention over an affine-quantized KV cache: the semantics of
 * the reference's only GPU kernel, sdpa_quantized_vector_{D}_{gs}_{bits}
 * (Sources/NovaMLXEngine/FusedQuantizedSDPA.swift:7-250). Shapes:
 *   q       [B*Hq, L, D]     dtype (f16/bf16)
 *   k_w,v_w [B*Hkv, N, D*bits/32]  u32
 *   k_s,k_b,v_s,v_b [B*Hkv, N, D/group]  dtype
 *   out     [B*Hq, L, D]     dtype (written in `dtype`, not always half —
 *           the reference casts to half at :131 whatever the query dtype)
 * Key i is used by query position l iff i <= N - L + l (:70). Guards as the
 * reference: D ∈ {64,96,128,256}, bits ∈ {4,8}, D % group == 0, L == 1
 * unless allow_multi_query is set. Violations return NMX_ERR_UNSUPPORTED. */
NMX_API nmx_status_t nmx_op_attn_quantized_decode(
    nmx_ctx_t ctx, const void* q, const uint32_t* k_w, const void* k_s, const void* k_b,
    const uint32_t* v_w, const void* v_s, const void* v_b, int B, int Hq, int Hkv, int N,
    int L, int D, float scale, int group_size, int bits, int allow_multi_query,
    nmx_dtype_t dtype, void* out);

/* Decode attention over the paged KV pool of a model (one new token per
 * sequence, GQA). q [B, Hq, D] f16; k_cache/v_cache are the pool's layer
 * views returned by nmx_kv_pool_layer_ptrs; block_tables int32[B, max_blocks];
 * seq_lens int32[B] (keys 0..seq_lens-1 are attended). out [B, Hq, D] f16.
 * At most 65535 rows per call (NMX_ERR_UNSUPPORTED beyond).
 * Replaces MLXFast.scaledDotProductAttention over KVCacheSimple for L == 1
 * (call sites Sources/NovaMLXEngine/FusedBatchScheduler.swift:1215 via
 * mlx-swift-lm AttentionUtils). */
NMX_API nmx_status_t nmx_op_attn_paged_decode(nmx_ctx_t ctx, const void* q, const void* k_cache,
                                              const void* v_cache, const int32_t* block_tables,
                                              const int32_t* seq_lens, int B, int Hq, int Hkv,
                                              int D, int block_tokens, int max_blocks,
                                              float scale, void* out);

/* The same decode attention as nmx_op_attn_paged_decode, for callers that
 * cannot allocate device memory (a host that reserves its whole device
 * budget up front and admits work against it, or one that cannot afford the
 * device synchronisation cudaMalloc/cudaFree may cause). Its only scratch,
 * the per-row descriptors (8 bytes per row), lives in a fixed 256 KiB array
 * inside the library, held on every GPU that loads it until exit; it never
 * allocates. At most 32768 rows per call: larger batches return
 * NMX_ERR_UNSUPPORTED before anything is launched. Same key splits and the
 * same bits as nmx_op_attn_paged_decode. The first call on a device looks up
 * that array's address with the device current; make it before any stream
 * capture. Calls share the array: calls that overlap on the GPU race. No
 * counterpart in the reference. */
NMX_API nmx_status_t nmx_op_attn_paged_decode_noalloc(nmx_ctx_t ctx, const void* q,
                                                      const void* k_cache, const void* v_cache,
                                                      const int32_t* block_tables,
                                                      const int32_t* seq_lens, int B, int Hq,
                                                      int Hkv, int D, int block_tokens,
                                                      int max_blocks, float scale, void* out);

/* ------------------------------------------------------------------------ */
/* Model level                                                               */
/* ------------------------------------------------------------------------ */

typedef struct nmx_model_s* nmx_model_t;
typedef struct nmx_kv_pool_s* nmx_kv_pool_t;

/* Llama / Qwen2 architecture description (the fields mlx-swift-lm reads from
 * config.json). dtype is the activation/scale dtype (NMX_F16 or NMX_BF16). */
typedef struct {
  int vocab;
  int hidden;
  int n_layers;
  int n_heads;
  int n_kv_heads;
  int head_dim;
  int ffn;
  int bits;         /* 4 or 8 */
  int group_size;   /* 32, 64 or 128 */
  int dtype;        /* nmx_dtype_t */
  int qkv_bias;     /* 1 for Qwen2 */
  int tie_embeddings;
  float rms_eps;
  float rope_theta;
  /* Llama-3.1 "llama3" RoPE scaling; factor <= 0 disables it. */
  float rope_factor;
  float rope_low_freq_factor;
  float rope_high_freq_factor;
  int rope_original_max_pos;
  int max_batch;    /* largest decode batch the model will be asked to run */
  int max_tokens;   /* largest token count of one forward (prefill chunk) */
} nmx_model_cfg;

/* Create a model on a context; weights are allocated but uninitialised.
 * Replaces MLXEngine.loadModel → LLMModelFactory.loadContainer
 * (Sources/NovaMLXEngine/MLXEngine.swift:654,727). */
NMX_API nmx_status_t nmx_model_create(nmx_ctx_t ctx, const nmx_model_cfg* cfg, nmx_model_t* out);
NMX_API nmx_status_t nmx_model_destroy(nmx_model_t model);

/* Fill every weight on the device from a counter-based N(0, std) generator
 * (seeded), quantizing each linear layer with nmx_op_quantize's rule;
 * embeddings are N(0, std) in dtype, norm weights are 1. */
NMX_API nmx_status_t nmx_model_init_random(nmx_model_t model, uint64_t seed, float std);

/* Copy one tensor from host memory, using MLX safetensors names:
 *   model.embed_tokens.weight, model.norm.weight, lm_head.{weight,scales,biases},
 *   model.layers.{i}.input_layernorm.weight, .post_attention_layernorm.weight,
 *   model.layers.{i}.self_attn.{q,k,v,o}_proj.{weight,scales,biases},
 *   model.layers.{i}.self_attn.{q,k,v}_proj.bias (qkv_bias models),
 *   model.layers.{i}.mlp.{gate,up,down}_proj.{weight,scales,biases}.
 * `weight` of a linear is u32 packed; the rest are in the model dtype.
 * The pre-quantized loader path of PATCHES.md:21-40 (no requantisation).
 * shape/ndim are checked against the expected shape. */
NMX_API nmx_status_t nmx_model_load_tensor(nmx_model_t model, const char* name,
                                           const void* host, nmx_dtype_t dtype,
                                           const int64_t* shape, int ndim);
/* Copy one tensor back to host memory (same names). */
NMX_API nmx_status_t nmx_model_get_tensor(nmx_model_t model, const char* name, void* host,
                                          size_t host_bytes);
/* Bytes of all weights on the device, counted once (packed + scales + biases
 * of every linear, plus embeddings and norms). */
NMX_API uint64_t nmx_model_weight_bytes(nmx_model_t model);
/* Bytes the weights of one decode step read (every linear once, one
 * embedding row, norms). */
NMX_API uint64_t nmx_model_step_weight_bytes(nmx_model_t model);

/* Paged KV pool: num_blocks blocks of block_tokens tokens, fp16 K and V for
 * every layer. Layout per layer: [num_blocks][Hkv][block_tokens][head_dim]
 * for K, the same for V. Block ids are what block tables hold. Replaces the
 * contiguous KVCacheSimple per sequence plus the dedup-only PagedBlockPool
 * (Sources/NovaMLXPrefixCache/PagedBlockPool.swift:108-139). */
NMX_API nmx_status_t nmx_kv_pool_create(nmx_model_t model, int block_tokens, int num_blocks,
                                        nmx_kv_pool_t* out);
/* A paged KV pool whose pages hold MLX-affine quantized K and V: kv_bits 4
 * or 8, groups of kv_group_size (32 or 64) along head_dim (64 or 128). Page
 * record of one (block, kv head) of K or of V: codes [block_tokens]
 * [head_dim * kv_bits / 32] u32 (low bits first), then scales and biases
 * [block_tokens][head_dim / kv_group_size] f16. Appended rows are quantized
 * on write (scale = (max - min) / (2^bits - 1), bias = min); attention reads
 * the dequantized values. The kvBits path of the reference:
 * TurboQuantService.applyToGenerateParameters
 * (Sources/NovaMLXEngine/TurboQuantCache.swift:78-104) turns on
 * mlx-swift-lm's quantized KV cache. Prefill attention over such pages runs
 * on the small-item kernel; nmx_kv_read_blocks / nmx_kv_write_blocks move
 * the raw page records (host layout [n][layers][2][Hkv * record bytes]). */
NMX_API nmx_status_t nmx_kv_pool_create_quantized(nmx_model_t model, int block_tokens, int num_blocks,
                                                  int kv_bits, int kv_group_size, nmx_kv_pool_t* out);
/* KV bytes one token occupies in this pool over all layers (f16 or
 * quantized pages): the budget figure of effectiveBytesPerToken
 * (Sources/NovaMLXEngine/MLXEngine.swift:1368-1386). */
NMX_API uint64_t nmx_kv_pool_bytes_per_token(nmx_kv_pool_t pool);
NMX_API nmx_status_t nmx_kv_pool_destroy(nmx_kv_pool_t pool);
/* Copy whole blocks src[i] → dst[i] in every layer (copy-on-write of a shared
 * partial block, and the device side of forkBlockTable,
 * Sources/NovaMLXPrefixCache/PagedBlockPool.swift:246). */
NMX_API nmx_status_t nmx_kv_copy_blocks(nmx_kv_pool_t pool, const int32_t* src,
                                        const int32_t* dst, int n);
/* Copy whole blocks between the pool and HOST memory, every layer:
 * host layout [n][layers][2 (K, V)][Hkv][block_tokens][head_dim] fp16.
 * The device side of the SSD prefix-block store (SSDCacheStore.saveBlock /
 * loadBlock, Sources/NovaMLXPrefixCache/SSDCacheStore.swift:194-269) and of
 * CacheBlockExtractor (Sources/NovaMLXPrefixCache/CacheBlockExtractor.swift:7-143). */
NMX_API nmx_status_t nmx_kv_read_blocks(nmx_kv_pool_t pool, const int32_t* ids, int n, void* host);
NMX_API nmx_status_t nmx_kv_write_blocks(nmx_kv_pool_t pool, const int32_t* ids, int n, const void* host);
/* Device pointers of layer `layer`'s K and V pages (for op-level tests). */
NMX_API nmx_status_t nmx_kv_pool_layer_ptrs(nmx_kv_pool_t pool, int layer, void** k, void** v);
NMX_API int nmx_kv_pool_num_blocks(nmx_kv_pool_t pool);
/* Fill every page of every layer (K and V) with seeded N(0, std) values: a
 * KV cache of a given context without running its prefill (benchmark and
 * test set-up). No counterpart in the reference. */
NMX_API nmx_status_t nmx_kv_pool_fill_random(nmx_kv_pool_t pool, uint64_t seed, float std);
/* KV bytes one token occupies over all layers: 2 * layers * Hkv * head_dim * 2,
 * the engine's kvMemoryBytesPerToken (Sources/NovaMLXEngine/MLXEngine.swift:833). */
NMX_API uint64_t nmx_kv_bytes_per_token(nmx_model_t model);

/* One sequence's slice of a forward: n_new_tokens tokens starting at absolute
 * position start_pos (the tokens before it are already in the sequence's
 * pages), with its block table (host int32[n_blocks]). */
typedef struct {
  int n_new_tokens;
  const int32_t* token_ids;
  int start_pos;
  const int32_t* block_table;
  int n_blocks;
} nmx_seq_t;

typedef enum {
  NMX_OUT_ARGMAX_LAST = 0, /* argmax of the last position of every sequence */
  NMX_OUT_LOGITS_LAST = 1, /* fp32 logits of the last position [n_seqs, vocab] */
  NMX_OUT_ARGMAX_ALL = 2,  /* argmax of every position (speculative verify) */
  NMX_OUT_LOGITS_ALL = 3   /* fp32 logits of every position [total_tokens, vocab] */
} nmx_out_mode_t;

/* One forward over a packed, variable-length batch mixing prefill chunks and
 * single-token decodes: appends every new token's K/V to the pages, attends
 * causally over the sequence's pages, and returns argmax ids (int32) or fp32
 * logits into HOST memory. One host synchronisation per call. Replaces
 * `context.model(tokens, cache:)` as called from
 * Sources/NovaMLXEngine/FusedBatchScheduler.swift:677,817,1215,1259 and
 * Sources/NovaMLXEngine/BatchScheduler.swift:213. Decode-only batches of a
 * shape seen before replay a captured CUDA graph. */
NMX_API nmx_status_t nmx_forward(nmx_model_t model, nmx_kv_pool_t pool, const nmx_seq_t* seqs,
                                 int n_seqs, nmx_out_mode_t mode, void* out_host);

/* Greedy decode of n_steps tokens for n_seqs sequences entirely on the
 * device: step t feeds the argmax of step t-1 back as the next input (the
 * TokenIterator loop of mlx-swift-lm, as driven at
 * Sources/NovaMLXEngine/FusedBatchScheduler.swift:1148-1245), with no host
 * round trip between steps. first_tokens[s] is the input of step 0 at
 * position start_pos[s]; block tables must already cover
 * start_pos + n_steps tokens. out_ids_host int32[n_steps, n_seqs] (may be
 * NULL, then ids stay on the device). */
NMX_API nmx_status_t nmx_decode_greedy(nmx_model_t model, nmx_kv_pool_t pool,
                                       const int32_t* first_tokens, const int32_t* start_pos,
                                       const int32_t* block_tables, int max_blocks, int n_seqs,
                                       int n_steps, int32_t* out_ids_host);

/* ------------------------------------------------------------------------ */
/* Prefix cache (host side, integer exact)                                   */
/* ------------------------------------------------------------------------ */

/* SHA-1 chain hash of one block: SHA1(model_name? ‖ (parent or "NovaMLX-root")
 * ‖ int64 count ‖ int32 tokens...). Mirrors BlockHasher.computeBlockHash,
 * Sources/NovaMLXPrefixCache/BlockHasher.swift:7-27. parent may be NULL. */
NMX_API void nmx_block_hash(const uint8_t* parent20, const int32_t* tokens, int n_tokens,
                            const char* model_name, uint8_t out20[20]);
/* computeChainHashes (:29-53): writes floor(n/block) hashes, returns count. */
NMX_API int nmx_chain_hashes(const int32_t* tokens, int n_tokens, int block_size,
                             const char* model_name, uint8_t* out20xN, int max_hashes);

typedef struct nmx_block_pool_s* nmx_block_pool_t;
/* Ref-counted block pool with a FIFO free list and a hash → block map, the
 * semantics of PagedBlockPool (Sources/NovaMLXPrefixCache/PagedBlockPool.swift:108-291):
 * block 0 is the reserved null block; the pool grows by up to 256 blocks
 * when the free list is empty, up to max_blocks. */
NMX_API nmx_status_t nmx_block_pool_create(int block_size, int max_blocks, int initial_blocks,
                                           const char* model_name, nmx_block_pool_t* out);
NMX_API void nmx_block_pool_destroy(nmx_block_pool_t pool);
/* allocateBlock (:141-156): returns the block id, or -1 when exhausted. */
NMX_API int nmx_block_pool_allocate(nmx_block_pool_t pool);
/* freeBlock / incrementRef (:158-180). */
NMX_API void nmx_block_pool_free(nmx_block_pool_t pool, int block_id);
NMX_API void nmx_block_pool_incref(nmx_block_pool_t pool, int block_id);
NMX_API int nmx_block_pool_refcount(nmx_block_pool_t pool, int block_id);
/* registerBlock (:209-220): hash (parent, tokens) and index the block. */
NMX_API void nmx_block_pool_register(nmx_block_pool_t pool, int block_id,
                                     const uint8_t* parent20, const int32_t* tokens,
                                     int n_tokens);
/* findSharedPrefix (:182-207): longest chain of full cached blocks; writes
 * up to max_ids block ids, returns the matched count, *remaining = tokens
 * not covered. */
NMX_API int nmx_block_pool_find_prefix(nmx_block_pool_t pool, const int32_t* tokens,
                                       int n_tokens, int32_t* out_ids, int max_ids,
                                       int* remaining);
/* getStats (:257-263): total, allocated (excluding the null block), free, shared. */
NMX_API void nmx_block_pool_stats(nmx_block_pool_t pool, int* total, int* allocated, int* free_,
                                  int* shared);
/* clear (:265-279). */
NMX_API void nmx_block_pool_clear(nmx_block_pool_t pool);
/* Request block tables kept by the pool (createBlockTable :231-237,
 * deleteBlockTable :239-244 frees every listed block once, forkBlockTable
 * :246-253 increments every listed block's refcount). A table is a list of
 * block ids held by the pool under the request id. */
NMX_API nmx_status_t nmx_block_pool_table_create(nmx_block_pool_t pool, const char* request_id);
NMX_API nmx_status_t nmx_block_pool_table_append(nmx_block_pool_t pool, const char* request_id,
                                                 int block_id);
/* Returns the table length (-1 if unknown) and copies up to max_ids ids. */
NMX_API int nmx_block_pool_table_get(nmx_block_pool_t pool, const char* request_id, int32_t* out_ids,
                                     int max_ids);
NMX_API nmx_status_t nmx_block_pool_table_delete(nmx_block_pool_t pool, const char* request_id);
NMX_API nmx_status_t nmx_block_pool_table_fork(nmx_block_pool_t pool, const char* src_request_id,
                                               const char* new_request_id);

/* ------------------------------------------------------------------------ */
/* Memory budget (MemoryBudgetTracker, Sources/NovaMLXEngine/MemoryBudgetTracker.swift):
 * available = limit - weights - committed; canAdmit (:57-80) accepts
 * estimated_tokens * bytes_per_token <= available * (100 - headroom) / 100;
 * reserve / release per sequence id. */
typedef struct nmx_budget_s* nmx_budget_t;
NMX_API nmx_status_t nmx_budget_create(uint64_t limit_bytes, int headroom_percent, nmx_budget_t* out);
NMX_API void nmx_budget_destroy(nmx_budget_t budget);
NMX_API void nmx_budget_add_weights(nmx_budget_t budget, uint64_t bytes);
NMX_API int nmx_budget_can_admit(nmx_budget_t budget, uint64_t estimated_tokens, uint64_t bytes_per_token);
NMX_API void nmx_budget_reserve(nmx_budget_t budget, int64_t seq_id, uint64_t estimated_tokens,
                                uint64_t bytes_per_token);
NMX_API void nmx_budget_release(nmx_budget_t budget, int64_t seq_id);
NMX_API uint64_t nmx_budget_available(nmx_budget_t budget);

/* Continuous batching (FusedBatchScheduler's engine-step loop,
 * Sources/NovaMLXEngine/FusedBatchScheduler.swift:281-1575): requests wait
 * in submission order; a step admits what the concurrency limit
 * (optimalConcurrency :264-277: sequences of 4096 tokens in 90% of the
 * available budget, at most max_concurrent) and the budget (canAdmit,
 * prompt + max_new_tokens tokens) allow, reusing cached prefix blocks, then
 * runs ONE nmx_forward over every running sequence: a prefill chunk of up to
 * prefill_chunk tokens for sequences still in their prompt, one decode token
 * for the others, at most max_step_tokens tokens. When the page pool runs
 * out, the newest other sequence is preempted (:502; its state becomes
 * NMX_REQ_PREEMPTED and it must be submitted again). Greedy ids; a request
 * ends after max_new_tokens ids or its eos id. The pool's blocks are the
 * scheduler's to hand out; destroy the scheduler before the pool. */
typedef struct {
  int max_batch;           /* sequences per step (<= the model's max_batch) */
  int max_step_tokens;     /* tokens per step (<= the model's max_tokens) */
  int prefill_chunk;       /* prompt tokens per sequence per step (the reference: 512) */
  int max_concurrent;      /* hard limit on running sequences */
  int headroom_percent;    /* budget headroom (the reference: 10) */
  uint64_t kv_budget_bytes; /* 0: the whole pool */
  const char* model_name;  /* prefix-cache hash namespace (may be NULL) */
} nmx_sched_cfg;
enum { NMX_REQ_WAITING = 0, NMX_REQ_PREFILL = 1, NMX_REQ_DECODE = 2, NMX_REQ_DONE = 3, NMX_REQ_PREEMPTED = 4 };
typedef struct {
  uint64_t steps, generated, finished, preemptions, prefix_hit_tokens, tokens_in_steps;
  int running, waiting;
  int blocks_in_use;        /* distinct pool blocks held (shared prefix blocks once) */
  uint64_t logical_blocks;  /* blocks summed over running sequences' tables */
  uint64_t kv_available_bytes;
} nmx_sched_stats_t;
typedef struct nmx_sched_s* nmx_sched_t;
NMX_API nmx_status_t nmx_sched_create(nmx_model_t model, nmx_kv_pool_t pool, const nmx_sched_cfg* cfg,
                                      nmx_sched_t* out);
NMX_API void nmx_sched_destroy(nmx_sched_t sched);
NMX_API nmx_status_t nmx_sched_submit(nmx_sched_t sched, const int32_t* prompt, int n_tokens,
                                      int max_new_tokens, int eos_id, int64_t* out_request_id);
/* One engine step; *n_generated = ids produced by it. */
NMX_API nmx_status_t nmx_sched_step(nmx_sched_t sched, int* n_generated);
/* The request's ids so far (up to max_tokens copied) and its NMX_REQ_* state. */
NMX_API nmx_status_t nmx_sched_poll(nmx_sched_t sched, int64_t request_id, int32_t* out_tokens,
                                    int max_tokens, int* n_tokens, int* state);
NMX_API nmx_status_t nmx_sched_stats(nmx_sched_t sched, nmx_sched_stats_t* out);

/* ------------------------------------------------------------------------ */
/* safetensors files: checkpoints and the SSD prefix-block store. */
typedef struct nmx_safetensors_s* nmx_safetensors_t;
/* Header checks of SafetensorsHeader.swift:12-31 (length > 0, < 16 MiB),
 * plus every entry's dtype / shape / offsets. */
NMX_API nmx_status_t nmx_safetensors_open(const char* path, nmx_safetensors_t* out);
NMX_API void nmx_safetensors_close(nmx_safetensors_t st);
NMX_API int nmx_safetensors_count(nmx_safetensors_t st);
/* name (NUL-terminated, name_cap bytes), dtype ("F16", "U32", ... in 8
 * bytes), shape (up to 8 dims), ndim, data bytes of tensor i. */
NMX_API nmx_status_t nmx_safetensors_info(nmx_safetensors_t st, int i, char* name, int name_cap, char* dtype,
                                          int64_t* shape, int* ndim, uint64_t* nbytes);
/* __metadata__[key] into out (truncated to cap - 1); returns its length, -1 if absent. */
NMX_API int nmx_safetensors_metadata(nmx_safetensors_t st, const char* key, char* out, int cap);
NMX_API nmx_status_t nmx_safetensors_read(nmx_safetensors_t st, const char* name, void* host, uint64_t host_bytes);
NMX_API nmx_status_t nmx_safetensors_write(const char* path, int n, const char* const* names,
                                           const char* const* dtypes, const int64_t* const* shapes, const int* ndims,
                                           const void* const* data, int n_meta, const char* const* meta_keys,
                                           const char* const* meta_values);
/* Every tensor of an MLX checkpoint file the model has a slot for
 * (nmx_model_load_tensor names; others are counted in n_skipped). With
 * tp_size > 1, this rank's shard of q/k/v/gate/up rows and o/down K columns
 * (the model must be the rank's local configuration). */
NMX_API nmx_status_t nmx_model_load_safetensors(nmx_model_t model, const char* path, int tp_rank, int tp_size,
                                                int* n_loaded, int* n_skipped);
/* SSD prefix-block store, SSDCacheStore's file format
 * (Sources/NovaMLXPrefixCache/SSDCacheStore.swift:132-135,194-269): the
 * block's pages of every layer as tensors "i.0" (keys) and "i.1" (values),
 * shape [1, kv heads, block tokens, head dim], in
 * cache_dir/<first hex digit>/<hex of hash20>.safetensors with metadata
 * block_hash, token_count, num_layers, model_name, created_at,
 * layer_cache_types; load checks the layer count and the shapes. */
NMX_API nmx_status_t nmx_ssd_save_block(nmx_kv_pool_t pool, int block_id, const uint8_t hash20[20], int token_count,
                                        const char* model_name, const char* cache_dir);
NMX_API nmx_status_t nmx_ssd_load_block(nmx_kv_pool_t pool, const uint8_t hash20[20], const char* cache_dir,
                                        int block_id, int* token_count);

/* ------------------------------------------------------------------------ */
/* Tensor parallelism (one process per GPU). Each rank creates the model of
 * its shard: n_heads / t and n_kv_heads / t heads, ffn / t, and loads the
 * matching rows of q/k/v/gate/up (and q/k/v biases) and the matching K
 * columns (words, scales, biases) of o_proj / down_proj; embeddings, norms
 * and the LM head are replicated. A communicator joins the ranks' block
 * outputs: after o_proj and after down_proj every rank computes
 * h = h + sum over ranks of the partial products, by one kernel reading the
 * peers' partials over NVLink (CUDA IPC, plain peer loads and stores, no
 * collective library). Setup: nmx_comm_create on every rank, exchange the
 * NMX_IPC_HANDLE_BYTES handles (any host rendezvous), nmx_comm_connect with
 * all of them in rank order, nmx_model_set_comm. Every rank must then run the
 * same sequence of forwards. Replaces the sharded model the north star's
 * 32B/70B configurations call for (no counterpart in the single-device
 * reference engine). */
#define NMX_IPC_HANDLE_BYTES 64
typedef struct nmx_comm_s* nmx_comm_t;
/* region_bytes: at least max_tokens x hidden x 2 of the models it serves */
NMX_API nmx_status_t nmx_comm_create(nmx_ctx_t ctx, int rank, int world, size_t region_bytes, nmx_comm_t* out);
NMX_API nmx_status_t nmx_comm_ipc_handle(nmx_comm_t comm, void* out_handle);
NMX_API nmx_status_t nmx_comm_connect(nmx_comm_t comm, const void* handles /* world x NMX_IPC_HANDLE_BYTES */);
NMX_API void nmx_comm_destroy(nmx_comm_t comm);
/* NULL detaches. Clears the model's captured decode graphs. */
NMX_API nmx_status_t nmx_model_set_comm(nmx_model_t model, nmx_comm_t comm);
/* 1: decode batches (9..128 rows) join the ranks' o_proj / down_proj
 * partials inside the GEMM's epilogue, tile group by tile group; 0 (the
 * default) runs the GEMM and the exchange kernel separately (same
 * arithmetic, same bits). */
NMX_API nmx_status_t nmx_model_set_exchange_fusion(nmx_model_t model, int enable);
/* out[rows, cols] = res + sum over ranks of every rank's partial (f16, rank
 * order); every rank calls it with its own partial. */
NMX_API nmx_status_t nmx_op_allreduce_resid(nmx_comm_t comm, const void* partial, int rows, int cols, const void* res,
                                            void* out);

/* ------------------------------------------------------------------------ */
/* Speculative decoding. */

/* N-gram draft source (NGramSpeculator, Sources/NovaMLXEngine/CompiledSampler.swift:60-204,
 * and SpeculativeDecoder's acceptance count, :206-250): continuations of the
 * last ngram_size tokens, up to max_draft distinct ones per n-gram, offered
 * once the n-gram has min_hits hits; the cache is cut to max_cache_size / 2
 * entries (fewest hits first, older first on ties) when it outgrows the cap. */
typedef struct nmx_ngram_s* nmx_ngram_t;
NMX_API nmx_status_t nmx_ngram_create(int ngram_size, int max_draft, int min_hits, int max_cache_size,
                                      nmx_ngram_t* out);
NMX_API void nmx_ngram_destroy(nmx_ngram_t ngram);
NMX_API void nmx_ngram_record_token(nmx_ngram_t ngram, int32_t token);
NMX_API void nmx_ngram_record_tokens(nmx_ngram_t ngram, const int32_t* tokens, int n_tokens);
/* Drafts for the context's last n-gram (context NULL: the recorded token
 * buffer); returns how many were written (0 .. min(max_draft, max_drafts)). */
NMX_API int nmx_ngram_speculate(nmx_ngram_t ngram, const int32_t* context, int n_context, int32_t* out_drafts,
                                int max_drafts);
/* recordAccepted: record the tokens and count n_tokens proposed, accepted accepted. */
NMX_API void nmx_ngram_record_accepted(nmx_ngram_t ngram, const int32_t* tokens, int n_tokens, int accepted);
NMX_API void nmx_ngram_stats(nmx_ngram_t ngram, int* cache_size, long long* total_hits, int* buffer_size,
                             double* acceptance_rate);

/* Verification of drafted tokens (FusedBatchScheduler.swift:1247-1300): ONE
 * forward over [last_token] + drafts of every sequence (its K/V appended at
 * start_pos ..), the greedy id at every position, then per sequence:
 *   NMX_VERIFY_NGRAM:  the reference's n-gram rule as written — tokens =
 *     [g0, g1, ..., g_p] up to and including the first p >= 1 with
 *     g_p != drafts[p-1]; accepted = the number of matches;
 *   NMX_VERIFY_PREFIX: draft-model verification — accepted = the longest
 *     prefix with drafts[i] == g_i; tokens = drafts[0..accepted) + [g_accepted].
 * out_tokens is [n_seqs][max n_drafts + 1]; out_counts[i] tokens of row i are
 * valid. The pages past the kept positions are simply overwritten later
 * (the cache "trim"). */
typedef enum { NMX_VERIFY_NGRAM = 0, NMX_VERIFY_PREFIX = 1 } nmx_verify_rule_t;
typedef struct {
  int32_t last_token;
  const int32_t* drafts;
  int n_drafts;
  int start_pos;                /* position of last_token */
  const int32_t* block_table;
  int n_blocks;
} nmx_spec_seq_t;
NMX_API nmx_status_t nmx_spec_verify(nmx_model_t model, nmx_kv_pool_t pool, const nmx_spec_seq_t* seqs, int n_seqs,
                                     nmx_verify_rule_t rule, int32_t* out_tokens, int* out_counts,
                                     int* out_accepted);

#ifdef __cplusplus
}
#endif
#endif /* NMX_H */
