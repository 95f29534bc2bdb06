// Continuous batching over the paged KV pool: the engine-step loop of
// Sources/NovaMLXEngine/FusedBatchScheduler.swift (submit :281, admission
// canAdmitAndReserve :456, optimalConcurrency :264-277, preemption of the
// newest sequence :502, chunked prefill :539-789, decode step :1148-1575),
// with the budget rules of Sources/NovaMLXEngine/MemoryBudgetTracker.swift
// (canAdmit :57-80, reserve / release) and the prefix cache of
// Sources/NovaMLXPrefixCache/PagedBlockPool.swift (shared full blocks).
//
// Where the reference runs one M = 1 forward per sequence per step
// (FusedBatchScheduler.swift:1198-1245), one step here is ONE batched forward
// (nmx_forward) over every running sequence: prefill chunks of newly admitted
// sequences and one decode token of each running sequence, each with its own
// block table into the shared pool.
//
// Block ids come from a PagedBlockPool (nmx_block_pool_*) whose ids index the
// device KV pool directly; a request holds one reference on every block of
// its table. A prompt's full blocks are registered under their chained SHA-1
// hash once its prefill has written them, so a later prompt with the same
// prefix reuses them (at most floor((n-1)/16) blocks: the last prompt token is
// always computed, which also yields the first generated id).
#include <algorithm>
#include <cstring>
#include <deque>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"
#include "model.h"

namespace {

// ------------------------------------------------------- budget tracker
struct Budget {
  uint64_t limit = 0;       // bytes the tracker may hand out
  uint64_t weights = 0;     // weights registered against the limit
  uint64_t committed = 0;   // KV bytes reserved by admitted sequences
  int headroom = 10;        // percent kept free
  std::map<int64_t, uint64_t> seqs;
  uint64_t available() const { return limit >= weights + committed ? limit - weights - committed : 0; }
  bool can_admit(uint64_t tokens, uint64_t bytes_per_token) const {
    const uint64_t usable = available() * uint64_t(100 - headroom) / 100;
    return tokens * bytes_per_token <= usable;
  }
  void reserve(int64_t id, uint64_t tokens, uint64_t bytes_per_token) {
    const uint64_t b = tokens * bytes_per_token;
    seqs[id] = b;
    committed += b;
  }
  void release(int64_t id) {
    auto it = seqs.find(id);
    if (it == seqs.end()) return;
    committed -= std::min(committed, it->second);
    seqs.erase(it);
  }
};

}  // namespace

struct nmx_budget_s {
  Budget b;
  std::mutex mu;
};

enum { REQ_WAITING = 0, REQ_PREFILL = 1, REQ_DECODE = 2, REQ_DONE = 3, REQ_PREEMPTED = 4 };

struct SchedRequest {
  int64_t id = 0;
  std::vector<int32_t> prompt;
  int max_new = 0;
  int eos = -1;
  std::vector<int32_t> out;
  std::vector<int32_t> blocks;  // pool block ids, one reference each
  int n_cached = 0;             // tokens whose K/V are in the pages
  int hit_blocks = 0;           // blocks reused from the prefix cache
  std::string first_hash;       // chained hash of the first full prompt block ("" if none)
  bool registered = false;      // the prompt's full blocks are in the cache
  int state = REQ_WAITING;
  uint64_t admitted = 0;
};

struct nmx_sched_s {
  nmx_model_t model = nullptr;
  nmx_kv_pool_t kv = nullptr;
  nmx_block_pool_t bp = nullptr;
  nmx_sched_cfg cfg{};
  std::string model_name;
  Budget budget;
  uint64_t bytes_per_token = 0;
  int block = 16;
  std::map<int64_t, std::unique_ptr<SchedRequest>> all;
  std::deque<SchedRequest*> waiting;
  std::vector<SchedRequest*> running;
  int64_t next_id = 1;
  uint64_t admit_counter = 0;
  nmx_sched_stats_t stats{};
  std::mutex mu;
};

namespace {

using nmx::set_error;

int blocks_for(int tokens, int bs) { return (tokens + bs - 1) / bs; }

void free_blocks(nmx_sched_s* s, SchedRequest* r) {
  for (int b : r->blocks) nmx_block_pool_free(s->bp, b);
  r->blocks.clear();
}

void finish(nmx_sched_s* s, SchedRequest* r, int state) {
  free_blocks(s, r);
  s->budget.release(r->id);
  r->state = state;
  s->running.erase(std::remove(s->running.begin(), s->running.end(), r), s->running.end());
  if (state == REQ_DONE) s->stats.finished++;
  if (state == REQ_PREEMPTED) s->stats.preemptions++;
}

// optimalConcurrency (FusedBatchScheduler.swift:264-277): sequences of 4096
// tokens that fit 90% of the available budget, at least 1, at most the limit
int optimal_concurrency(const nmx_sched_s* s) {
  const uint64_t usable = s->budget.available() * 90 / 100;
  const uint64_t per_seq = uint64_t(4096) * s->bytes_per_token;
  if (per_seq == 0) return s->cfg.max_concurrent;
  const uint64_t fit = usable / per_seq;
  return int(std::max<uint64_t>(1, std::min<uint64_t>(fit, uint64_t(s->cfg.max_concurrent))));
}

// the most recently admitted running sequence (preemptNewest, :502)
SchedRequest* newest_running(nmx_sched_s* s) {
  SchedRequest* v = nullptr;
  for (SchedRequest* r : s->running)
    if (!v || r->admitted > v->admitted) v = r;
  return v;
}

// blocks so that positions [0, upto) have a page; while the pool is
// exhausted the newest running sequence is preempted; false when that is r
// itself (the caller preempts it)
bool ensure_blocks(nmx_sched_s* s, SchedRequest* r, int upto) {
  const int need = blocks_for(upto, s->block);
  while (int(r->blocks.size()) < need) {
    const int b = nmx_block_pool_allocate(s->bp);
    if (b >= 0) {
      r->blocks.push_back(b);
      continue;
    }
    SchedRequest* v = newest_running(s);
    if (!v || v == r) return false;
    finish(s, v, REQ_PREEMPTED);
  }
  return true;
}

// a running sequence is still computing a prompt that starts with the same
// block: admitting this one now would compute the shared prefix twice
bool prefix_in_flight(const nmx_sched_s* s, const SchedRequest* r) {
  if (r->first_hash.empty()) return false;
  for (const SchedRequest* o : s->running)
    if (!o->registered && o->first_hash == r->first_hash) return true;
  return false;
}

// admit waiting requests in submission order while concurrency and budget
// allow; a request whose prefix another sequence is still computing waits
// for it (later requests may go first)
void admit(nmx_sched_s* s) {
  for (auto it = s->waiting.begin(); it != s->waiting.end();) {
    const int limit = std::min(s->cfg.max_batch, optimal_concurrency(s));
    if (int(s->running.size()) >= limit) break;
    SchedRequest* r = *it;
    if (prefix_in_flight(s, r)) {
      ++it;
      continue;
    }
    const uint64_t est = uint64_t(r->prompt.size()) + uint64_t(r->max_new);
    if (!s->budget.can_admit(est, s->bytes_per_token)) break;
    it = s->waiting.erase(it);
    s->budget.reserve(r->id, est, s->bytes_per_token);
    // prefix-cache hit: full blocks of the prompt except the one holding its
    // last token, which is always recomputed
    const int n = int(r->prompt.size());
    const int max_hit = (n - 1) / s->block;
    std::vector<int32_t> ids(size_t(max_hit) + 1);
    int rem = 0;
    int hit = max_hit > 0 ? nmx_block_pool_find_prefix(s->bp, r->prompt.data(), max_hit * s->block, ids.data(),
                                                       max_hit, &rem)
                          : 0;
    hit = std::min(hit, max_hit);
    for (int i = 0; i < hit; ++i) {
      nmx_block_pool_incref(s->bp, ids[i]);
      r->blocks.push_back(ids[i]);
    }
    r->hit_blocks = hit;
    r->n_cached = hit * s->block;
    s->stats.prefix_hit_tokens += uint64_t(hit) * s->block;
    r->state = REQ_PREFILL;
    r->admitted = ++s->admit_counter;
    s->running.push_back(r);
  }
}

// register the prompt's full blocks that this request computed
void register_prompt_blocks(nmx_sched_s* s, SchedRequest* r) {
  const int full = int(r->prompt.size()) / s->block;
  uint8_t parent[20], h[20];
  bool has_parent = false;
  for (int i = 0; i < full && i < int(r->blocks.size()); ++i) {
    const int32_t* toks = r->prompt.data() + size_t(i) * s->block;
    if (i >= r->hit_blocks) nmx_block_pool_register(s->bp, r->blocks[i], has_parent ? parent : nullptr, toks, s->block);
    nmx_block_hash(has_parent ? parent : nullptr, toks, s->block, s->cfg.model_name, h);
    memcpy(parent, h, 20);
    has_parent = true;
  }
  r->registered = true;
}

}  // namespace

extern "C" {

NMX_API nmx_status_t nmx_budget_create(uint64_t limit_bytes, int headroom_percent, nmx_budget_t* out) {
  nmx::clear_error();
  NMX_CHECK(out != nullptr, NMX_ERR_INVALID, "null output");
  NMX_CHECK(headroom_percent >= 0 && headroom_percent < 100, NMX_ERR_INVALID, "headroom must be in [0, 100)");
  auto* b = new nmx_budget_s();
  b->b.limit = limit_bytes;
  b->b.headroom = headroom_percent;
  *out = b;
  return NMX_OK;
}
NMX_API void nmx_budget_destroy(nmx_budget_t b) { delete b; }
NMX_API void nmx_budget_add_weights(nmx_budget_t b, uint64_t bytes) {
  if (!b) return;
  std::lock_guard<std::mutex> lk(b->mu);
  b->b.weights += bytes;
}
NMX_API int nmx_budget_can_admit(nmx_budget_t b, uint64_t estimated_tokens, uint64_t bytes_per_token) {
  if (!b) return 0;
  std::lock_guard<std::mutex> lk(b->mu);
  return b->b.can_admit(estimated_tokens, bytes_per_token) ? 1 : 0;
}
NMX_API void nmx_budget_reserve(nmx_budget_t b, int64_t seq_id, uint64_t estimated_tokens, uint64_t bytes_per_token) {
  if (!b) return;
  std::lock_guard<std::mutex> lk(b->mu);
  b->b.reserve(seq_id, estimated_tokens, bytes_per_token);
}
NMX_API void nmx_budget_release(nmx_budget_t b, int64_t seq_id) {
  if (!b) return;
  std::lock_guard<std::mutex> lk(b->mu);
  b->b.release(seq_id);
}
NMX_API uint64_t nmx_budget_available(nmx_budget_t b) {
  if (!b) return 0;
  std::lock_guard<std::mutex> lk(b->mu);
  return b->b.available();
}

NMX_API nmx_status_t nmx_sched_create(nmx_model_t model, nmx_kv_pool_t pool, const nmx_sched_cfg* cfg,
                                      nmx_sched_t* out) {
  nmx::clear_error();
  NMX_CHECK(model && pool && cfg && out, NMX_ERR_INVALID, "nmx_sched_create: null argument");
  nmx::Model* m = model->m;
  NMX_CHECK(cfg->max_batch >= 1 && cfg->max_batch <= m->max_batch, NMX_ERR_INVALID,
            "nmx_sched_create: max_batch must be in [1, the model's max_batch]");
  NMX_CHECK(cfg->max_step_tokens >= cfg->max_batch && cfg->max_step_tokens <= m->max_tokens, NMX_ERR_INVALID,
            "nmx_sched_create: max_step_tokens must be in [max_batch, the model's max_tokens]");
  NMX_CHECK(cfg->prefill_chunk >= 1, NMX_ERR_INVALID, "nmx_sched_create: prefill_chunk must be positive");
  NMX_CHECK(cfg->max_concurrent >= 1, NMX_ERR_INVALID, "nmx_sched_create: max_concurrent must be positive");
  NMX_CHECK(cfg->headroom_percent >= 0 && cfg->headroom_percent < 100, NMX_ERR_INVALID,
            "nmx_sched_create: headroom must be in [0, 100)");
  auto* s = new nmx_sched_s();
  s->model = model;
  s->kv = pool;
  s->cfg = *cfg;
  s->model_name = cfg->model_name ? cfg->model_name : "";
  s->cfg.model_name = s->model_name.c_str();
  s->block = 16;
  s->bytes_per_token = nmx_kv_bytes_per_token(model);
  const int nblocks = pool->p->num_blocks;
  // block 0 is the pool's reserved null block; every other block is usable
  nmx_status_t st = nmx_block_pool_create(s->block, nblocks, nblocks, s->cfg.model_name, &s->bp);
  if (st != NMX_OK) {
    delete s;
    return st;
  }
  s->budget.limit = cfg->kv_budget_bytes ? cfg->kv_budget_bytes
                                         : uint64_t(nblocks - 1) * uint64_t(s->block) * s->bytes_per_token;
  s->budget.headroom = cfg->headroom_percent;
  model->refs++;
  *out = s;
  return NMX_OK;
}

NMX_API void nmx_sched_destroy(nmx_sched_t s) {
  if (!s) return;
  if (s->bp) nmx_block_pool_destroy(s->bp);
  nmx_model_destroy(s->model);  // drops the reference taken at creation
  delete s;
}

NMX_API nmx_status_t nmx_sched_submit(nmx_sched_t s, const int32_t* prompt, int n_tokens, int max_new_tokens,
                                      int eos_id, int64_t* out_id) {
  nmx::clear_error();
  NMX_CHECK(s && prompt && out_id, NMX_ERR_INVALID, "nmx_sched_submit: null argument");
  NMX_CHECK(n_tokens >= 1 && max_new_tokens >= 1, NMX_ERR_INVALID,
            "nmx_sched_submit: need at least one prompt token and one new token");
  nmx::Model* m = s->model->m;
  for (int i = 0; i < n_tokens; ++i)
    NMX_CHECK(prompt[i] >= 0 && prompt[i] < m->cfg.vocab, NMX_ERR_INVALID, "nmx_sched_submit: token id out of range");
  NMX_CHECK(blocks_for(n_tokens + max_new_tokens, s->block) <= s->kv->p->num_blocks - 1, NMX_ERR_INVALID,
            "nmx_sched_submit: the request needs more pages than the pool holds");
  std::lock_guard<std::mutex> lk(s->mu);
  auto r = std::make_unique<SchedRequest>();
  r->id = s->next_id++;
  r->prompt.assign(prompt, prompt + n_tokens);
  r->max_new = max_new_tokens;
  r->eos = eos_id;
  if (n_tokens > s->block) {
    uint8_t h[20];
    nmx_block_hash(nullptr, prompt, s->block, s->cfg.model_name, h);
    r->first_hash.assign(reinterpret_cast<const char*>(h), 20);
  }
  s->waiting.push_back(r.get());
  *out_id = r->id;
  s->all[r->id] = std::move(r);
  return NMX_OK;
}

NMX_API nmx_status_t nmx_sched_step(nmx_sched_t s, int* n_generated) {
  nmx::clear_error();
  NMX_CHECK(s != nullptr, NMX_ERR_INVALID, "null scheduler");
  std::lock_guard<std::mutex> lk(s->mu);
  if (n_generated) *n_generated = 0;
  admit(s);
  if (s->running.empty()) return NMX_OK;

  // build the batch in admission order: prefill chunks, then decode tokens
  struct Slot {
    SchedRequest* r;
    int start, n;
    std::vector<int32_t> toks;
  };
  std::vector<Slot> slots;
  int budget = s->cfg.max_step_tokens;
  std::vector<SchedRequest*> order = s->running;
  std::sort(order.begin(), order.end(), [](const SchedRequest* a, const SchedRequest* b) {
    return a->admitted < b->admitted;
  });
  for (SchedRequest* r : order) {
    if (r->state != REQ_PREFILL && r->state != REQ_DECODE) continue;  // preempted while building
    if (int(slots.size()) >= s->cfg.max_batch || budget <= 0) break;
    Slot sl;
    sl.r = r;
    if (r->state == REQ_PREFILL) {
      const int left = int(r->prompt.size()) - r->n_cached;
      sl.n = std::min({left, s->cfg.prefill_chunk, budget});
      sl.start = r->n_cached;
      sl.toks.assign(r->prompt.begin() + sl.start, r->prompt.begin() + sl.start + sl.n);
    } else {
      sl.n = 1;
      sl.start = r->n_cached;
      sl.toks.assign(1, r->out.back());
    }
    if (!ensure_blocks(s, r, sl.start + sl.n)) {
      // r is the newest sequence left: it gives way
      finish(s, r, REQ_PREEMPTED);
      continue;
    }
    budget -= sl.n;
    slots.push_back(std::move(sl));
  }
  // sequences preempted after they were placed leave the batch
  slots.erase(std::remove_if(slots.begin(), slots.end(),
                             [](const Slot& x) { return x.r->state == REQ_PREEMPTED; }),
              slots.end());
  if (slots.empty()) return NMX_OK;

  std::vector<nmx_seq_t> seqs(slots.size());
  for (size_t i = 0; i < slots.size(); ++i) {
    seqs[i].n_new_tokens = slots[i].n;
    seqs[i].token_ids = slots[i].toks.data();
    seqs[i].start_pos = slots[i].start;
    seqs[i].block_table = slots[i].r->blocks.data();
    seqs[i].n_blocks = int(slots[i].r->blocks.size());
  }
  std::vector<int32_t> ids(slots.size());
  NMX_TRY(nmx_forward(s->model, s->kv, seqs.data(), int(seqs.size()), NMX_OUT_ARGMAX_LAST, ids.data()));
  s->stats.steps++;
  for (const Slot& x : slots) s->stats.tokens_in_steps += uint64_t(x.n);

  int gen = 0;
  for (size_t i = 0; i < slots.size(); ++i) {
    SchedRequest* r = slots[i].r;
    r->n_cached += slots[i].n;
    if (r->state == REQ_PREFILL) {
      if (r->n_cached < int(r->prompt.size())) continue;  // more prompt chunks to go
      register_prompt_blocks(s, r);
      r->state = REQ_DECODE;
    }
    r->out.push_back(ids[i]);
    ++gen;
    s->stats.generated++;
    if (int(r->out.size()) >= r->max_new || ids[i] == r->eos) finish(s, r, REQ_DONE);
  }
  if (n_generated) *n_generated = gen;
  return NMX_OK;
}

NMX_API nmx_status_t nmx_sched_poll(nmx_sched_t s, int64_t request_id, int32_t* out_tokens, int max_tokens,
                                    int* n_tokens, int* state) {
  nmx::clear_error();
  NMX_CHECK(s != nullptr, NMX_ERR_INVALID, "null scheduler");
  std::lock_guard<std::mutex> lk(s->mu);
  auto it = s->all.find(request_id);
  NMX_CHECK(it != s->all.end(), NMX_ERR_INVALID, "nmx_sched_poll: unknown request");
  const SchedRequest* r = it->second.get();
  if (n_tokens) *n_tokens = int(r->out.size());
  if (state) *state = r->state;
  if (out_tokens)
    for (int i = 0; i < int(r->out.size()) && i < max_tokens; ++i) out_tokens[i] = r->out[i];
  return NMX_OK;
}

NMX_API nmx_status_t nmx_sched_stats(nmx_sched_t s, nmx_sched_stats_t* out) {
  nmx::clear_error();
  NMX_CHECK(s && out, NMX_ERR_INVALID, "null argument");
  std::lock_guard<std::mutex> lk(s->mu);
  nmx_sched_stats_t st = s->stats;
  st.running = int(s->running.size());
  st.waiting = int(s->waiting.size());
  int total = 0, allocated = 0, free_ = 0, shared = 0;
  nmx_block_pool_stats(s->bp, &total, &allocated, &free_, &shared);
  st.blocks_in_use = allocated;
  uint64_t logical = 0;
  for (const SchedRequest* r : s->running) logical += r->blocks.size();
  st.logical_blocks = logical;
  st.kv_available_bytes = s->budget.available();
  *out = st;
  return NMX_OK;
}

}  // extern "C"
