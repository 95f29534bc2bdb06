// Tensor-parallel communicator state shared by the exchange kernel
// (comm.cu) and the GEMM that fuses the exchange into its epilogue
// (gemm_tcs.cu).
#pragma once
#include "common.cuh"

struct nmx_ctx_s;

namespace nmx {

constexpr int kMaxRanks = 8;
constexpr int kMaxTileFlags = 1024;  // flag slots per source rank for fused exchanges

struct Comm {
  Ctx* ctx = nullptr;
  nmx_ctx_s* owner = nullptr;  // reference held on the context
  int rank = 0, world = 1;
  size_t region_bytes = 0;
  unsigned char* arena = nullptr;       // this rank's arena
  unsigned char* peer[kMaxRanks] = {};  // every rank's arena as mapped here
  bool connected = false;
  // arena layout: partial regions R0 / R1, the exchange kernel's flags
  // [rank], the shared epoch word, the exchange kernel's CTA ticket, the
  // fused exchanges' flags [source rank][slot] and their CTA ticket
  size_t off_r[2] = {0, 0}, off_flags = 0, off_epoch = 0, off_ticket = 0, off_tflags = 0, off_tticket = 0,
         bytes = 0;
};

// What a GEMM epilogue needs to join its partial with the other ranks'.
struct ExchangeArgs {
  const half* part[kMaxRanks] = {};         // region r on every rank
  unsigned* peer_tflags[kMaxRanks] = {};    // &tflags[this rank][0] in every rank's arena
  unsigned* my_tflags = nullptr;            // tflags[0][0] here; [q][slot] at q * kMaxTileFlags + slot
  unsigned* epoch = nullptr;                // shared epoch word (read at start, advanced by the last CTA)
  unsigned* ticket = nullptr;
  half* part_local = nullptr;               // this rank's region r
  int world = 1, rank = 0;
};

nmx_status_t comm_exchange_args(Comm* c, int region, ExchangeArgs* out);

}  // namespace nmx
