// Paged decode attention for callers that cannot allocate device memory.
//
// nmx_op_attn_paged_decode needs a little scratch, the per-row descriptors
// (sequence index and position of each query row) that the kernel reads, and
// takes it from a context workspace that grows with cudaMalloc. Some hosts
// cannot let a library call allocate: an engine that reserves its whole
// device budget at start-up and admits work against it (as NovaMLX does with
// its memory-budget tracker) must not see memory appear behind its back, and
// cudaMalloc / cudaFree can synchronise the device and stall the host's other
// streams. This variant keeps the descriptors in a fixed, file-scope device
// array instead and never allocates. The attention kernel itself needs no
// other scratch: the key splits of a (row, kv head) combine through the
// distributed shared memory of their thread-block cluster.
//
// The array (kNoAllocScratchBytes, 8 bytes per query row: at most
// kNoAllocMaxRows rows) lives in every GPU that loads the library until the
// process exits. Host code cannot use its name as a device address; its
// address is looked up once per device with cudaGetSymbolAddress, on the
// first call made on that device (with that device current) — make that
// first call before any stream capture. All calls share the array and it
// keeps the last call's contents: every call rewrites the descriptors of its
// rows before the kernel reads them, and calls that overlap on the GPU (other
// streams, other threads) race on it.
#include <map>
#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "model.h"

namespace nmx {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(256) << 10;  // 256 KiB
constexpr long kNoAllocMaxRows = long(kNoAllocScratchBytes / 8);  // tok_seq + tok_pos per row
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
  NMX_CHECK(long(B) <= kNoAllocMaxRows, NMX_ERR_UNSUPPORTED,
            "paged decode (no-alloc): " + std::to_string(B) + " rows need " + std::to_string(long(B) * 8) +
                " bytes of scratch, more than the fixed " + std::to_string(kNoAllocScratchBytes) + " (at most " +
                std::to_string(kNoAllocMaxRows) + " rows per call)");
  Ctx* c = &ctx->c;
  // the same key splits as the allocating entry point, so the same bits
  const int S = decode_attn_splits(c->num_sms, B, Hkv);
  unsigned char* base = nullptr;
  NMX_TRY(scratch_address(c->device, &base));
  int* tok_seq = reinterpret_cast<int*>(base);
  int* tok_pos = tok_seq + B;
  NMX_TRY(seq_rows_from_lens(c, seq_lens, B, tok_seq, tok_pos));
  AttnArgs a;
  a.q = q; a.ldq = long(Hq) * D; a.k_cache = const_cast<void*>(k_cache); a.v_cache = const_cast<void*>(v_cache);
  a.block_tables = block_tables; a.max_blocks = max_blocks; a.tok_seq = tok_seq; a.tok_pos = tok_pos;
  a.out = out;
  a.T = B; a.Hq = Hq; a.Hkv = Hkv; a.D = D; a.BT = block_tokens; a.splits = S; a.scale = scale;
  return paged_attention(c, a, false);
}
