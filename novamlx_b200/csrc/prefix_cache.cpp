// Host-side prefix cache: SHA-1 chained block hashes and the ref-counted
// block pool whose ids index the device KV pages.
//
// Semantics follow the reference's NovaMLXPrefixCache:
//   BlockHasher.computeBlockHash / computeChainHashes
//     (Sources/NovaMLXPrefixCache/BlockHasher.swift:7-53): SHA-1 over
//     model name (when non-empty) ‖ parent digest or "NovaMLX-root" ‖
//     Int64 token count ‖ Int32 tokens, all little-endian.
//   PagedBlockPool (Sources/NovaMLXPrefixCache/PagedBlockPool.swift:108-291):
//     FIFO free list (FreeBlockQueue, :4-82), hash → block map, block 0 is
//     the reserved null block, growth by up to 256 blocks when the free list
//     is empty, refcounts, request block tables with fork/delete.
// One quirk is kept on purpose: freeing a block removes its hash from the
// map but leaves the hash on the block, and re-allocating that block removes
// the hash from the map again (:146-149, :169-172), which can drop a newer
// block registered under the same hash.
#include <stdint.h>
#include <string.h>

#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/nmx.h"

namespace {

// ---------------------------------------------------------------- SHA-1
// FIPS 180-4 SHA-1, written from the standard's description.
struct Sha1 {
  uint32_t h[5] = {0x67452301u, 0xEFCDAB89u, 0x98BADCFEu, 0x10325476u, 0xC3D2E1F0u};
  uint8_t buf[64];
  size_t nbuf = 0;
  uint64_t total = 0;

  static uint32_t rol(uint32_t x, int n) { return (x << n) | (x >> (32 - n)); }

  void block(const uint8_t* p) {
    uint32_t w[80];
    for (int i = 0; i < 16; ++i)
      w[i] = (uint32_t(p[4 * i]) << 24) | (uint32_t(p[4 * i + 1]) << 16) | (uint32_t(p[4 * i + 2]) << 8) |
             uint32_t(p[4 * i + 3]);
    for (int i = 16; i < 80; ++i) w[i] = rol(w[i - 3] ^ w[i - 8] ^ w[i - 14] ^ w[i - 16], 1);
    uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4];
    for (int i = 0; i < 80; ++i) {
      uint32_t f, k;
      if (i < 20) {
        f = (b & c) | (~b & d);
        k = 0x5A827999u;
      } else if (i < 40) {
        f = b ^ c ^ d;
        k = 0x6ED9EBA1u;
      } else if (i < 60) {
        f = (b & c) | (b & d) | (c & d);
        k = 0x8F1BBCDCu;
      } else {
        f = b ^ c ^ d;
        k = 0xCA62C1D6u;
      }
      const uint32_t t = rol(a, 5) + f + e + k + w[i];
      e = d;
      d = c;
      c = rol(b, 30);
      b = a;
      a = t;
    }
    h[0] += a;
    h[1] += b;
    h[2] += c;
    h[3] += d;
    h[4] += e;
  }

  void update(const void* data, size_t n) {
    const uint8_t* p = static_cast<const uint8_t*>(data);
    total += n;
    while (n > 0) {
      const size_t take = (64 - nbuf) < n ? (64 - nbuf) : n;
      memcpy(buf + nbuf, p, take);
      nbuf += take;
      p += take;
      n -= take;
      if (nbuf == 64) {
        block(buf);
        nbuf = 0;
      }
    }
  }

  void finish(uint8_t out[20]) {
    const uint64_t bits = total * 8;
    const uint8_t one = 0x80, zero = 0;
    update(&one, 1);
    while (nbuf != 56) update(&zero, 1);
    uint8_t len[8];
    for (int i = 0; i < 8; ++i) len[i] = uint8_t(bits >> (56 - 8 * i));
    update(len, 8);
    for (int i = 0; i < 5; ++i) {
      out[4 * i] = uint8_t(h[i] >> 24);
      out[4 * i + 1] = uint8_t(h[i] >> 16);
      out[4 * i + 2] = uint8_t(h[i] >> 8);
      out[4 * i + 3] = uint8_t(h[i]);
    }
  }
};

void block_hash(const uint8_t* parent, const int32_t* tokens, int n, const char* model, uint8_t out[20]) {
  Sha1 s;
  if (model && model[0]) s.update(model, strlen(model));
  if (parent) {
    s.update(parent, 20);
  } else {
    static const char root[] = "NovaMLX-root";
    s.update(root, sizeof(root) - 1);
  }
  const int64_t count = n;  // Swift Int: 8 bytes, little-endian
  uint8_t cb[8];
  for (int i = 0; i < 8; ++i) cb[i] = uint8_t(uint64_t(count) >> (8 * i));
  s.update(cb, 8);
  for (int i = 0; i < n; ++i) {
    const uint32_t t = uint32_t(tokens[i]);
    const uint8_t tb[4] = {uint8_t(t), uint8_t(t >> 8), uint8_t(t >> 16), uint8_t(t >> 24)};
    s.update(tb, 4);
  }
  s.finish(out);
}

struct Block {
  int id = 0;
  int ref = 0;
  bool has_hash = false;
  std::string hash;  // 20 raw bytes
  int token_count = 0;
  bool is_null = false;
  int prev = -1, next = -1;  // free-list links (-1: none; kHead / kTail sentinels)
  bool in_free = false;
};

constexpr int kHead = -2, kTail = -3;

}  // namespace

struct nmx_block_pool_s {
  int block_size = 64;
  int max_blocks = 4096;
  int initial_blocks = 256;
  std::string model;
  std::vector<Block> blocks;
  int head_next = kTail, tail_prev = kHead;
  int num_free = 0;
  int current = 0;
  std::unordered_map<std::string, int> hash_map;
  std::unordered_map<int, bool> allocated;  // id → present
  std::unordered_map<std::string, std::vector<int>> tables;
  std::mutex mu;

  // ---- FreeBlockQueue (PagedBlockPool.swift:4-82)
  void fq_reset(int n) {
    head_next = kTail;
    tail_prev = kHead;
    num_free = 0;
    for (int i = 0; i < n; ++i) fq_append(i);
  }
  void link_next(int from, int to) {
    if (from == kHead) head_next = to; else blocks[from].next = to;
  }
  void link_prev(int of, int to) {
    if (of == kTail) tail_prev = to; else blocks[of].prev = to;
  }
  int fq_pop_left() {
    const int b = head_next;
    if (b == kTail) return -1;
    const int nx = blocks[b].next;
    link_next(kHead, nx);
    link_prev(nx, kHead);
    blocks[b].prev = blocks[b].next = -1;
    blocks[b].in_free = false;
    --num_free;
    return b;
  }
  void fq_append(int b) {
    const int last = tail_prev;
    link_next(last, b);
    blocks[b].prev = last;
    blocks[b].next = kTail;
    tail_prev = b;
    blocks[b].in_free = true;
    ++num_free;
  }

  void reset() {
    const int count = initial_blocks < max_blocks ? initial_blocks : max_blocks;
    current = count;
    blocks.assign(count, Block());
    for (int i = 0; i < count; ++i) blocks[i].id = i;
    fq_reset(count);
    hash_map.clear();
    tables.clear();
    allocated.clear();
    const int nb = fq_pop_left();
    if (nb >= 0) {
      blocks[nb].is_null = true;
      blocks[nb].ref = 1;
      allocated[nb] = true;
    }
  }

  int grow(int additional) {
    const int avail = max_blocks - current;
    const int n = additional < avail ? additional : avail;
    if (n <= 0) return 0;
    const int start = current;
    for (int i = 0; i < n; ++i) {
      Block b;
      b.id = start + i;
      blocks.push_back(b);
    }
    for (int i = 0; i < n; ++i) fq_append(start + i);
    current += n;
    return n;
  }

  void free_unlocked(int id) {
    auto it = allocated.find(id);
    if (it == allocated.end()) return;
    Block& b = blocks[id];
    if (b.is_null) return;
    b.ref -= 1;
    if (b.ref <= 0) {
      if (b.has_hash) hash_map.erase(b.hash);
      allocated.erase(id);
      fq_append(id);
    }
  }
  void incref_unlocked(int id) {
    if (allocated.find(id) == allocated.end()) return;
    blocks[id].ref += 1;
  }
};

extern "C" {

NMX_API void nmx_block_hash(const uint8_t* parent20, const int32_t* tokens, int n_tokens, const char* model_name,
                            uint8_t out20[20]) {
  block_hash(parent20, tokens, n_tokens < 0 ? 0 : n_tokens, model_name, out20);
}

NMX_API int nmx_chain_hashes(const int32_t* tokens, int n_tokens, int block_size, const char* model_name,
                             uint8_t* out20xN, int max_hashes) {
  if (block_size <= 0 || n_tokens < 0) return 0;
  const int full = n_tokens / block_size;
  int written = 0;
  const uint8_t* parent = nullptr;
  for (int i = 0; i < full && written < max_hashes; ++i) {
    block_hash(parent, tokens + size_t(i) * block_size, block_size, model_name, out20xN + size_t(written) * 20);
    parent = out20xN + size_t(written) * 20;
    ++written;
  }
  return written;
}

NMX_API nmx_status_t nmx_block_pool_create(int block_size, int max_blocks, int initial_blocks, const char* model_name,
                                           nmx_block_pool_t* out) {
  if (!out || block_size <= 0 || max_blocks <= 0 || initial_blocks <= 0) return NMX_ERR_INVALID;
  auto* p = new nmx_block_pool_s();
  p->block_size = block_size;
  p->max_blocks = max_blocks;
  p->initial_blocks = initial_blocks < max_blocks ? initial_blocks : max_blocks;
  p->model = model_name ? model_name : "";
  p->reset();
  *out = p;
  return NMX_OK;
}

NMX_API void nmx_block_pool_destroy(nmx_block_pool_t pool) { delete pool; }

NMX_API int nmx_block_pool_allocate(nmx_block_pool_t p) {
  if (!p) return -1;
  std::lock_guard<std::mutex> lk(p->mu);
  if (p->num_free == 0) p->grow(256 < p->max_blocks - p->current ? 256 : p->max_blocks - p->current);
  const int id = p->fq_pop_left();
  if (id < 0) return -1;
  Block& b = p->blocks[id];
  if (b.has_hash) {
    p->hash_map.erase(b.hash);
    b.has_hash = false;
    b.hash.clear();
  }
  b.ref = 1;
  p->allocated[id] = true;
  return id;
}

NMX_API void nmx_block_pool_free(nmx_block_pool_t p, int id) {
  if (!p) return;
  std::lock_guard<std::mutex> lk(p->mu);
  p->free_unlocked(id);
}

NMX_API void nmx_block_pool_incref(nmx_block_pool_t p, int id) {
  if (!p) return;
  std::lock_guard<std::mutex> lk(p->mu);
  p->incref_unlocked(id);
}

NMX_API int nmx_block_pool_refcount(nmx_block_pool_t p, int id) {
  if (!p) return -1;
  std::lock_guard<std::mutex> lk(p->mu);
  if (id < 0 || id >= int(p->blocks.size())) return -1;
  return p->blocks[id].ref;
}

NMX_API void nmx_block_pool_register(nmx_block_pool_t p, int id, const uint8_t* parent20, const int32_t* tokens,
                                     int n_tokens) {
  if (!p || id < 0) return;
  std::lock_guard<std::mutex> lk(p->mu);
  if (id >= int(p->blocks.size())) return;
  uint8_t h[20];
  block_hash(parent20, tokens, n_tokens, p->model.c_str(), h);
  Block& b = p->blocks[id];
  b.hash.assign(reinterpret_cast<const char*>(h), 20);
  b.has_hash = true;
  b.token_count = n_tokens;
  p->hash_map[b.hash] = id;
}

NMX_API int nmx_block_pool_find_prefix(nmx_block_pool_t p, const int32_t* tokens, int n_tokens, int32_t* out_ids,
                                       int max_ids, int* remaining) {
  if (!p) return 0;
  std::lock_guard<std::mutex> lk(p->mu);
  const int full = n_tokens / p->block_size;
  int matched = 0;
  uint8_t parent[20];
  bool has_parent = false;
  for (int i = 0; i < full; ++i) {
    uint8_t h[20];
    block_hash(has_parent ? parent : nullptr, tokens + size_t(i) * p->block_size, p->block_size, p->model.c_str(), h);
    auto it = p->hash_map.find(std::string(reinterpret_cast<const char*>(h), 20));
    if (it == p->hash_map.end()) break;
    if (out_ids && matched < max_ids) out_ids[matched] = it->second;
    ++matched;
    memcpy(parent, h, 20);
    has_parent = true;
  }
  if (remaining) *remaining = n_tokens - matched * p->block_size;
  return matched;
}

NMX_API void nmx_block_pool_stats(nmx_block_pool_t p, int* total, int* allocated, int* free_, int* shared) {
  if (!p) return;
  std::lock_guard<std::mutex> lk(p->mu);
  int sh = 0;
  for (const auto& kv : p->allocated)
    if (p->blocks[kv.first].ref > 1) ++sh;
  if (total) *total = p->current;
  if (allocated) *allocated = int(p->allocated.size()) - 1;
  if (free_) *free_ = p->num_free;
  if (shared) *shared = sh;
}

NMX_API void nmx_block_pool_clear(nmx_block_pool_t p) {
  if (!p) return;
  std::lock_guard<std::mutex> lk(p->mu);
  p->reset();
}

NMX_API nmx_status_t nmx_block_pool_table_create(nmx_block_pool_t p, const char* request_id) {
  if (!p || !request_id) return NMX_ERR_INVALID;
  std::lock_guard<std::mutex> lk(p->mu);
  p->tables[request_id] = {};
  return NMX_OK;
}

NMX_API nmx_status_t nmx_block_pool_table_append(nmx_block_pool_t p, const char* request_id, int block_id) {
  if (!p || !request_id) return NMX_ERR_INVALID;
  std::lock_guard<std::mutex> lk(p->mu);
  auto it = p->tables.find(request_id);
  if (it == p->tables.end()) return NMX_ERR_NOT_FOUND;
  it->second.push_back(block_id);
  return NMX_OK;
}

NMX_API int nmx_block_pool_table_get(nmx_block_pool_t p, const char* request_id, int32_t* out_ids, int max_ids) {
  if (!p || !request_id) return -1;
  std::lock_guard<std::mutex> lk(p->mu);
  auto it = p->tables.find(request_id);
  if (it == p->tables.end()) return -1;
  const int n = int(it->second.size());
  for (int i = 0; i < n && i < max_ids; ++i) out_ids[i] = it->second[i];
  return n;
}

NMX_API nmx_status_t nmx_block_pool_table_delete(nmx_block_pool_t p, const char* request_id) {
  if (!p || !request_id) return NMX_ERR_INVALID;
  std::lock_guard<std::mutex> lk(p->mu);
  auto it = p->tables.find(request_id);
  if (it == p->tables.end()) return NMX_OK;
  const std::vector<int> ids = it->second;
  p->tables.erase(it);
  for (int id : ids) p->free_unlocked(id);
  return NMX_OK;
}

NMX_API nmx_status_t nmx_block_pool_table_fork(nmx_block_pool_t p, const char* src_request_id,
                                               const char* new_request_id) {
  if (!p || !src_request_id || !new_request_id) return NMX_ERR_INVALID;
  std::lock_guard<std::mutex> lk(p->mu);
  auto it = p->tables.find(src_request_id);
  if (it == p->tables.end()) return NMX_ERR_NOT_FOUND;
  const std::vector<int> ids = it->second;
  for (int id : ids) p->incref_unlocked(id);
  p->tables[new_request_id] = ids;
  return NMX_OK;
}

}  // extern "C"
