// Speculative decoding on the host side of the C ABI:
//   * nmx_ngram_*: the n-gram draft source of
//     Sources/NovaMLXEngine/CompiledSampler.swift:60-204 (NGramSpeculator:
//     a map from the last n tokens to up to max_draft distinct continuations
//     with a hit count; record(token) / record(tokens) update it from a
//     bounded token buffer; speculate returns the continuations of the
//     context's last n-gram once it has min_hits hits; the cache is cut to
//     half its cap, fewest hits first, when it outgrows the cap) and the
//     acceptance bookkeeping of SpeculativeDecoder (:206-250);
//   * nmx_spec_verify: one batched forward of [last] + drafts per sequence
//     with the greedy id at every position (nmx_forward, NMX_OUT_ARGMAX_ALL),
//     then the acceptance rule per sequence:
//       NMX_VERIFY_NGRAM  — FusedBatchScheduler.swift:1247-1300 as written:
//         out = [g0]; for p = 1..D: out += g_p; stop after the first p with
//         g_p != draft[p-1]; accepted = matches;
//       NMX_VERIFY_PREFIX — greedy draft-model verification: accepted = the
//         longest prefix with draft[i] == g_i; out = draft[0..a) + [g_a].
//     "Trimming" the rejected positions (the reference's cache.trim of
//     n_drafts - accepted entries) is the caller's: under both rules the
//     sequence's next position is start_pos + 1 + accepted, and the pages
//     past it are overwritten by later steps.
#include <algorithm>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"
#include "model.h"

namespace {

struct NGram {
  int n = 4, max_draft = 5, min_hits = 1, max_cache = 65536;
  struct Entry {
    std::vector<int32_t> cont;
    long long hits = 0;
    unsigned long long order = 0;  // insertion order: deterministic eviction among equal hit counts
  };
  std::map<std::vector<int32_t>, Entry> cache;
  std::vector<int32_t> buf;
  unsigned long long next_order = 0;
  unsigned long long proposed = 0, accepted = 0;
  std::mutex mu;

  size_t buf_cap() const { return size_t(n + max_draft + 10); }
  void trim_buffer() {
    if (buf.size() > buf_cap()) buf.erase(buf.begin(), buf.end() - long(buf_cap()));
  }
  void add(size_t start) {
    std::vector<int32_t> key(buf.begin() + long(start), buf.begin() + long(start) + n);
    const int32_t c = buf[start + size_t(n)];
    auto it = cache.find(key);
    if (it == cache.end()) {
      Entry e;
      e.cont.push_back(c);
      e.hits = 1;
      e.order = next_order++;
      cache.emplace(std::move(key), std::move(e));
    } else {
      it->second.hits += 1;
      if (int(it->second.cont.size()) < max_draft &&
          std::find(it->second.cont.begin(), it->second.cont.end(), c) == it->second.cont.end())
        it->second.cont.push_back(c);
    }
  }
  void evict() {
    if (int(cache.size()) <= max_cache) return;
    std::vector<std::pair<std::pair<long long, unsigned long long>, const std::vector<int32_t>*>> v;
    v.reserve(cache.size());
    for (const auto& kv : cache) v.push_back({{kv.second.hits, kv.second.order}, &kv.first});
    std::sort(v.begin(), v.end(), [](const auto& a, const auto& b) { return a.first < b.first; });
    const size_t remove = cache.size() - size_t(max_cache / 2);
    std::vector<std::vector<int32_t>> keys;
    for (size_t i = 0; i < remove; ++i) keys.push_back(*v[i].second);
    for (const auto& k : keys) cache.erase(k);
  }
  // record(token:) (:103-111) / updateCache (:136-156)
  void record_token(int32_t t) {
    buf.push_back(t);
    trim_buffer();
    if (int(buf.size()) > n) add(buf.size() - size_t(n) - 1);
    evict();
  }
  // record(tokens:) (:113-134)
  void record_tokens(const int32_t* t, int count) {
    buf.insert(buf.end(), t, t + count);
    trim_buffer();
    for (int i = 0; i < count; ++i) {
      const long start = long(buf.size()) - n - 1 - i;
      if (long(buf.size()) >= n + 1 + i && start >= 0) add(size_t(start));
    }
    evict();
  }
  // speculate(context:) (:172-184); speculate() uses the token buffer
  int speculate(const int32_t* ctx, int count, int32_t* out, int max_out) {
    if (count < n) return 0;
    std::vector<int32_t> key(ctx + count - n, ctx + count);
    auto it = cache.find(key);
    if (it == cache.end() || it->second.hits < min_hits) return 0;
    const int k = std::min({int(it->second.cont.size()), max_draft, max_out});
    for (int i = 0; i < k; ++i) out[i] = it->second.cont[size_t(i)];
    return k;
  }
};

}  // namespace

struct nmx_ngram_s {
  NGram g;
};

extern "C" {

NMX_API nmx_status_t nmx_ngram_create(int ngram_size, int max_draft, int min_hits, int max_cache_size,
                                      nmx_ngram_t* out) {
  nmx::clear_error();
  NMX_CHECK(out != nullptr, NMX_ERR_INVALID, "null output");
  NMX_CHECK(ngram_size >= 1 && max_draft >= 1 && min_hits >= 1 && max_cache_size >= 1, NMX_ERR_INVALID,
            "nmx_ngram_create: sizes must be positive");
  auto* s = new nmx_ngram_s();
  s->g.n = ngram_size;
  s->g.max_draft = max_draft;
  s->g.min_hits = min_hits;
  s->g.max_cache = max_cache_size;
  *out = s;
  return NMX_OK;
}

NMX_API void nmx_ngram_destroy(nmx_ngram_t s) { delete s; }

NMX_API void nmx_ngram_record_token(nmx_ngram_t s, int32_t token) {
  if (!s) return;
  std::lock_guard<std::mutex> lk(s->g.mu);
  s->g.record_token(token);
}

NMX_API void nmx_ngram_record_tokens(nmx_ngram_t s, const int32_t* tokens, int n_tokens) {
  if (!s || !tokens || n_tokens <= 0) return;
  std::lock_guard<std::mutex> lk(s->g.mu);
  s->g.record_tokens(tokens, n_tokens);
}

NMX_API int nmx_ngram_speculate(nmx_ngram_t s, const int32_t* context, int n_context, int32_t* out_drafts,
                                int max_drafts) {
  if (!s || !out_drafts || max_drafts <= 0) return 0;
  std::lock_guard<std::mutex> lk(s->g.mu);
  if (!context) return s->g.speculate(s->g.buf.data(), int(s->g.buf.size()), out_drafts, max_drafts);
  return s->g.speculate(context, n_context, out_drafts, max_drafts);
}

NMX_API void nmx_ngram_record_accepted(nmx_ngram_t s, const int32_t* tokens, int n_tokens, int accepted) {
  if (!s) return;
  std::lock_guard<std::mutex> lk(s->g.mu);
  if (tokens && n_tokens > 0) s->g.record_tokens(tokens, n_tokens);
  s->g.proposed += uint64_t(std::max(n_tokens, 0));
  s->g.accepted += uint64_t(std::max(accepted, 0));
}

NMX_API void nmx_ngram_stats(nmx_ngram_t s, int* cache_size, long long* total_hits, int* buffer_size,
                             double* acceptance_rate) {
  if (!s) return;
  std::lock_guard<std::mutex> lk(s->g.mu);
  long long hits = 0;
  for (const auto& kv : s->g.cache) hits += kv.second.hits;
  if (cache_size) *cache_size = int(s->g.cache.size());
  if (total_hits) *total_hits = hits;
  if (buffer_size) *buffer_size = int(s->g.buf.size());
  if (acceptance_rate) *acceptance_rate = s->g.proposed ? double(s->g.accepted) / double(s->g.proposed) : 0.0;
}

NMX_API nmx_status_t nmx_spec_verify(nmx_model_t model, nmx_kv_pool_t pool, const nmx_spec_seq_t* seqs, int n_seqs,
                                     nmx_verify_rule_t rule, int32_t* out_tokens, int* out_counts,
                                     int* out_accepted) {
  nmx::clear_error();
  NMX_CHECK(model && pool && seqs && n_seqs > 0 && out_tokens && out_counts && out_accepted, NMX_ERR_INVALID,
            "nmx_spec_verify: null argument");
  NMX_CHECK(rule == NMX_VERIFY_NGRAM || rule == NMX_VERIFY_PREFIX, NMX_ERR_INVALID, "nmx_spec_verify: unknown rule");
  int total = 0, max_d = 0;
  for (int i = 0; i < n_seqs; ++i) {
    NMX_CHECK(seqs[i].n_drafts >= 0 && (seqs[i].n_drafts == 0 || seqs[i].drafts), NMX_ERR_INVALID,
              "nmx_spec_verify: bad drafts");
    total += 1 + seqs[i].n_drafts;
    max_d = std::max(max_d, seqs[i].n_drafts);
  }
  // one row per position: [last] + drafts
  std::vector<int32_t> toks(static_cast<size_t>(total));
  std::vector<nmx_seq_t> fs(static_cast<size_t>(n_seqs));
  int o = 0;
  for (int i = 0; i < n_seqs; ++i) {
    toks[size_t(o)] = seqs[i].last_token;
    for (int d = 0; d < seqs[i].n_drafts; ++d) toks[size_t(o + 1 + d)] = seqs[i].drafts[d];
    fs[size_t(i)].n_new_tokens = 1 + seqs[i].n_drafts;
    fs[size_t(i)].token_ids = toks.data() + o;
    fs[size_t(i)].start_pos = seqs[i].start_pos;
    fs[size_t(i)].block_table = seqs[i].block_table;
    fs[size_t(i)].n_blocks = seqs[i].n_blocks;
    o += 1 + seqs[i].n_drafts;
  }
  std::vector<int32_t> g(static_cast<size_t>(total));
  NMX_TRY(nmx_forward(model, pool, fs.data(), n_seqs, NMX_OUT_ARGMAX_ALL, g.data()));
  o = 0;
  for (int i = 0; i < n_seqs; ++i) {
    const int D = seqs[i].n_drafts;
    const int32_t* gi = g.data() + o;
    const int32_t* dr = seqs[i].drafts;
    int32_t* out = out_tokens + size_t(i) * size_t(max_d + 1);
    int cnt = 0, acc = 0;
    if (rule == NMX_VERIFY_NGRAM) {
      out[cnt++] = gi[0];
      for (int p = 1; p <= D; ++p) {
        out[cnt++] = gi[p];
        if (gi[p] == dr[p - 1]) {
          ++acc;
        } else {
          break;
        }
      }
    } else {
      while (acc < D && dr[acc] == gi[acc]) out[cnt++] = dr[acc++];
      out[cnt++] = gi[acc];
    }
    out_counts[i] = cnt;
    out_accepted[i] = acc;
    o += 1 + D;
  }
  return NMX_OK;
}

}  // extern "C"
