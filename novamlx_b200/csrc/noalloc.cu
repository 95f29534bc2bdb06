// Paged decode attention for callers that cannot allocate device memory.
//
// nmx_op_attn_paged_decode needs scratch for its split-KV partial sums, its
// per-(sequence, kv head) tickets and its query-row descriptors, and takes it
// from a context workspace that grows with cudaMalloc. Some hosts cannot let
// a library call allocate: an engine that reserves its whole device budget at
// start-up and admits work against it (as NovaMLX does with its memory-budget
// tracker) must not see memory appear behind its back, and cudaMalloc /
// cudaFree can synchronise the device and stall the host's other streams.
// This variant uses a fixed, file-scope device array instead and never
// allocates.
//
// The array (kNoAllocScratchBytes) lives in every GPU that loads the library
// until the process exits. Host code cannot use its name as a device address;
// its address is looked up once per device with cudaGetSymbolAddress, on the
// first call made on that device (with that device current) — make that
// first call before any stream capture. All calls share the array and it
// keeps the last call's contents: the tickets are cleared on every call, and
// calls that overlap on the GPU (other streams, other threads) race on it.
#include <map>
#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "model.h"

namespace nmx {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;  // 8 MiB
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_mu;
std::map<int, unsigned char*> g_addr;  // device → address of g_noalloc_scratch

nmx_status_t scratch_address(int device, unsigned char** out) {
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_addr.find(device);
  if (it != g_addr.end()) {
    *out = it->second;
    return NMX_OK;
  }
  int prev = 0;
  NMX_CUDA_OK(cudaGetDevice(&prev));
  if (prev != device) NMX_CUDA_OK(cudaSetDevice(device));
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (prev != device) cudaSetDevice(prev);
  if (e != cudaSuccess || p == nullptr) {
    set_error(std::string("no-alloc scratch: cudaGetSymbolAddress failed: ") + cudaGetErrorString(e));
    return NMX_ERR_CUDA;
  }
  g_addr[device] = static_cast<unsigned char*>(p);
  *out = static_cast<unsigned char*>(p);
  return NMX_OK;
}

struct Carve {
  size_t counters, rows, ml, o, total;
};

// scratch layout for B rows, Hq/Hkv heads, head dim D and S splits
Carve carve(long B, long Hq, long Hkv, long D, int S) {
  Carve c;
  c.counters = 0;
  c.rows = align_up(size_t(B * Hkv) * 4, 256);
  c.ml = c.rows + align_up(size_t(B) * 8, 256);
  const size_t n_ml = S > 1 ? size_t(B * Hq) * S * 2 : 0;
  c.o = c.ml + align_up(n_ml * 4, 256);
  const size_t n_o = S > 1 ? size_t(B * Hq) * S * D : 0;
  c.total = c.o + n_o * 4;
  return c;
}

}  // namespace
}  // namespace nmx

using namespace nmx;

extern "C" NMX_API nmx_status_t nmx_op_attn_paged_decode_noalloc(
    nmx_ctx_t ctx, const void* q, const void* k_cache, const void* v_cache, const int32_t* block_tables,
    const int32_t* seq_lens, int B, int Hq, int Hkv, int D, int block_tokens, int max_blocks, float scale,
    void* out) {
  clear_error();
  NMX_CHECK(ctx != nullptr, NMX_ERR_INVALID, "null context");
  if (B == 0) return NMX_OK;
  NMX_CHECK(B > 0, NMX_ERR_INVALID, "paged decode (no-alloc): B must be positive");
  NMX_CHECK(q && k_cache && v_cache && block_tables && seq_lens && out, NMX_ERR_INVALID,
            "paged decode (no-alloc): null pointer");
  NMX_CHECK(Hkv > 0 && Hq > 0 && Hq % Hkv == 0, NMX_ERR_INVALID,
            "paged decode (no-alloc): Hq must be a multiple of Hkv");
  Ctx* c = &ctx->c;
  // as many key splits as the allocating entry point uses, fewer if they do
  // not fit; one split needs only the tickets and row descriptors
  int S = std::max(1, std::min(32, (2 * c->num_sms + B * Hkv - 1) / (B * Hkv)));
  while (S > 1 && carve(B, Hq, Hkv, D, S).total > kNoAllocScratchBytes) --S;
  const Carve cv = carve(B, Hq, Hkv, D, S);
  NMX_CHECK(cv.total <= kNoAllocScratchBytes, NMX_ERR_UNSUPPORTED,
            "paged decode (no-alloc): batch needs " + std::to_string(cv.total) +
                " bytes of scratch, more than the fixed " + std::to_string(kNoAllocScratchBytes));
  unsigned char* base = nullptr;
  NMX_TRY(scratch_address(c->device, &base));
  unsigned* ctr = reinterpret_cast<unsigned*>(base + cv.counters);
  int* tok_seq = reinterpret_cast<int*>(base + cv.rows);
  int* tok_pos = tok_seq + B;
  // the array keeps the previous call's contents: tickets must start at zero
  NMX_CUDA_OK(cudaMemsetAsync(ctr, 0, size_t(B) * Hkv * 4, c->stream));
  NMX_TRY(seq_rows_from_lens(c, seq_lens, B, tok_seq, tok_pos));
  AttnArgs a;
  a.q = q; a.ldq = long(Hq) * D; a.k_cache = const_cast<void*>(k_cache); a.v_cache = const_cast<void*>(v_cache);
  a.block_tables = block_tables; a.max_blocks = max_blocks; a.tok_seq = tok_seq; a.tok_pos = tok_pos;
  a.out = out; a.part_o = reinterpret_cast<float*>(base + cv.o); a.part_ml = reinterpret_cast<float*>(base + cv.ml);
  a.counters = ctr;
  a.T = B; a.Hq = Hq; a.Hkv = Hkv; a.D = D; a.BT = block_tokens; a.splits = S; a.scale = scale;
  return paged_attention(c, a, false);
}
