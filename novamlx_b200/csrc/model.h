// Model and KV-pool objects behind the nmx_model_t / nmx_kv_pool_t handles.
#pragma once

#include <map>
#include <string>
#include <utility>
#include <vector>

#include "common.cuh"
#include "kernels.h"

namespace nmx {

struct Lin {
  uint32_t* w = nullptr;  // packed [N, K*bits/32], or the decode records when dl
  void* s = nullptr;      // [N, K/gs] (MLX layout only)
  void* b = nullptr;
  int N = 0, K = 0;
  bool dl = false;        // stored as decode records (see qgemv_dl.cu)
  size_t bytes = 0;       // words + scales + biases
};

struct LayerW {
  void* attn_norm = nullptr;
  void* mlp_norm = nullptr;
  Lin qkv;                  // rows: q | k | v
  void* qkv_bias = nullptr;
  Lin o;
  Lin gu;                   // rows: gate | up
  Lin down;
};

struct GraphEntry {
  cudaGraphExec_t exec = nullptr;
  size_t nodes = 0;
};

struct KvPool;

struct Comm;

struct Model {
  Ctx* ctx = nullptr;
  nmx_model_cfg cfg{};
  nmx_dtype_t dt = NMX_F16;
  int max_batch = 1, max_tokens = 1, rows_logits = 1;
  int Nq = 0, Nkv = 0, Nqkv = 0;
  char* wbase = nullptr;
  size_t wbytes = 0;
  uint64_t step_bytes = 0;
  void* embed = nullptr;
  void* final_norm = nullptr;
  Lin lm;
  std::vector<LayerW> layers;
  bool weights_ready = false, loaded_any = false;

  // workspace
  char* wsbase = nullptr;
  void *h = nullptr, *qkv = nullptr, *q_roped = nullptr, *attn = nullptr, *act = nullptr, *last_h = nullptr;
  void* xn = nullptr;  // RMSNorm output for the tensor-core GEMM (prefill)
  float* logits_f32 = nullptr;
  float* am_val = nullptr;
  int* am_idx = nullptr;
  unsigned* am_counter = nullptr;
  int *tok_ids = nullptr, *tok_seq = nullptr, *tok_pos = nullptr, *last_rows = nullptr, *out_ids = nullptr;
  int2* pf_items = nullptr;  // prefill attention work items of the current batch
  int n_pf_items = 0;
  int n_pf_tc = 0;  // leading items for the tensor-core prefill attention
  int *block_tables = nullptr, *hist = nullptr, *step = nullptr;
  float* inv_freq = nullptr;
  char* pinned = nullptr;
  size_t pinned_bytes = 0;
  int pool_blocks_hint = 0;
  size_t h2d_bytes_last = 0;
  std::map<std::pair<int, const void*>, GraphEntry> graphs;
  void graphs_clear() {
    for (auto& g : graphs)
      if (g.second.exec) cudaGraphExecDestroy(g.second.exec);
    graphs.clear();
  }
  // the decode graphs captured over `pool` (its pages and page format are
  // baked in): dropped when the pool goes, since a later pool may get the
  // same host address
  void graphs_drop_pool(const void* pool) {
    for (auto it = graphs.begin(); it != graphs.end();) {
      if (it->first.second == pool) {
        if (it->second.exec) cudaGraphExecDestroy(it->second.exec);
        it = graphs.erase(it);
      } else {
        ++it;
      }
    }
  }

  // set by resolve() when the named part lives inside decode records
  Lin* rs_lin = nullptr;
  long rs_row0 = 0;
  int rs_rows = 0, rs_mask = 0;

  static nmx_status_t create(Ctx* c, const nmx_model_cfg& cfg, Model** out);
  ~Model();
  nmx_status_t init_random(uint64_t seed, float stdv);
  nmx_status_t resolve(const std::string& name, char** dst, size_t* bytes, std::vector<int64_t>* shape,
                       nmx_dtype_t* dtype);
  nmx_status_t load_tensor(const std::string& name, const void* host, nmx_dtype_t dtype, const int64_t* shape,
                           int ndim);
  nmx_status_t get_tensor(const std::string& name, void* host, size_t host_bytes);

  // partial-sum scratch and counters of the decode-record GEMV
  float* dl_partials = nullptr;
  size_t dl_partials_cap = 0;
  unsigned* dl_counters = nullptr;
  unsigned long long* dl_keys = nullptr;
  unsigned* dl_done = nullptr;
  int dl_ctas_per_sm = 2;

  // y = epilogue(norm?(x) · W^T) through whichever GEMV the layout calls for
  nmx_status_t linear(const Lin& l, const void* x, long ldx, const void* gamma, int M, int N_out,
                      long pair_off_rows, const void* bias, void* y, long ldy, const void* res, long ldres,
                      int epi, float* logits_f32 = nullptr, int* ids = nullptr, int* next_tokens = nullptr);
  nmx_status_t block_out(const Lin& l, const void* x, long ldx, int M, int region);
  nmx_status_t run_layers_decode(KvPool* pool, int B);
  nmx_status_t run_layers_prefill(KvPool* pool, int T);
  nmx_status_t run_head(const void* x, int rows, bool want_logits, int* next_tokens);
  nmx_status_t decode_step_body(KvPool* pool, int B);
  nmx_status_t run_decode_graph(KvPool* pool, int B);
  nmx_status_t upload_batch(const nmx_seq_t* seqs, int n, int* T_out, bool* decode_out, bool tc_items = true);
  nmx_status_t forward(KvPool* pool, const nmx_seq_t* seqs, int n, nmx_out_mode_t mode, void* out_host);
  nmx_status_t finish_step();
  // tensor parallelism: this rank's shard of every linear; o/down partials
  // are exchanged and summed (with the residual) through the communicator
  Comm* comm = nullptr;
  nmx_comm_s* comm_handle = nullptr;
  bool fused_exchange = false;  // decode batches: the GEMM epilogue does the exchange (nmx_model_set_exchange_fusion)

  nmx_status_t decode_greedy(KvPool* pool, const int32_t* first, const int32_t* start, const int32_t* tables,
                             int max_blocks, int n, int steps, int32_t* out_host);
};

struct Comm;
size_t comm_region_bytes(const Comm* c);
void* comm_region(Comm* c, int r);
// out = res + sum over ranks (rank order) of every rank's region r rows
nmx_status_t comm_allreduce_resid(Comm* cm, int region, int rows, int cols, const void* res, long ldres, void* out,
                                  long ldo, unsigned* err);

struct KvPool {
  Model* model = nullptr;
  // [L][K|V][num_blocks][Hkv][BT][D] f16, or for a quantized pool
  // [L][K|V][num_blocks][Hkv] page records (codes, scales, biases of 16
  // tokens; kv_page_bytes in attn_common.cuh)
  char* base = nullptr;
  int num_blocks = 0;
  int kv_bits = 0, kv_gs = 0;  // 0: f16 pages
  size_t block_bytes = 0;   // one block of K (or V) of one layer
  size_t layer_stride = 0;  // bytes per layer (K and V)
  static nmx_status_t create(Model* m, int block_tokens, int num_blocks, KvPool** out, int kv_bits = 0,
                             int kv_gs = 0);
  ~KvPool();
  void* k_layer(int l) const { return base + size_t(l) * layer_stride; }
  void* v_layer(int l) const { return base + size_t(l) * layer_stride + layer_stride / 2; }
};

}  // namespace nmx

// Handles are reference counted: a model keeps its context alive and a pool
// keeps its model alive, so destroying handles in any order is safe.
struct nmx_ctx_s {
  nmx::Ctx c;
  int refs = 1;
};
struct nmx_model_s {
  nmx::Model* m;
  nmx_ctx_s* ctx;
  int refs = 1;
};
struct nmx_kv_pool_s {
  nmx::KvPool* p;
  nmx_model_s* model;
};
