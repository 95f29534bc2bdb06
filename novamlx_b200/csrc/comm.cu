// Tensor-parallel exchange: the one all-reduce per block half of a
// column/row-sharded Llama/Qwen block (q/k/v/gate/up sharded by output rows,
// o/down by K), done by our own kernel over peer memory instead of a
// collective library call.
//
// Every rank (one process per GPU) allocates one device arena: two partial
// regions (R0 for o_proj, R1 for down_proj, each max_rows × hidden f16), a
// flag word per peer, an epoch word and a CTA ticket. The arenas' CUDA IPC
// handles are exchanged by the host (any rendezvous: torch.distributed,
// MPI, a file) and opened on every rank, so each rank holds a device pointer
// into every peer's arena over NVLink.
//
// allreduce_resid_kernel (one launch per block half, after the GEMV that
// wrote this rank's partial into its region with the store epilogue):
//   1. after the programmatic-launch wait (the partial is complete), CTA 0
//      publishes epoch e = old + 1 to every peer's flag slot for this rank
//      (one system-scope fence, then plain stores over NVLink: a release
//      store per peer serialised a fence per peer);
//   2. every CTA waits (bounded) until all peers' flags in its own arena
//      reach e (relaxed polls, then one acquire load of each flag orders its
//      reads after them);
//   3. each thread sums the partials of ranks 0..t-1 (peer loads, fixed rank
//      order, f32) plus the residual and writes the new hidden row — the
//      same bits on every rank;
//   4. the last CTA (ticket) stores e as the arena's epoch.
// Two regions suffice: a rank writes R0 again only in the next layer, after
// it passed the down_proj exchange, which every peer entered only after
// finishing its reads of R0. Epochs only grow, so flags never need resetting.
// A wait that runs out (after the context's poll limit) sets kErrPeerWait in
// *err and skips the sum; the host reads it with the step's results and
// reports NMX_ERR_TIMEOUT. Only plain loads and stores touch peer memory.
#include <cstring>
#include <vector>

#include "comm.h"
#include "common.cuh"
#include "kernels.h"
#include "model.h"

namespace nmx {

namespace {

constexpr int kARThreads = 256;

struct ARArgs {
  const half* part[kMaxRanks];      // the region on every rank (this rank's included)
  unsigned* peer_flag[kMaxRanks];   // &flags[rank] in every rank's arena
  unsigned* my_flags;               // flags[0..world) in this rank's arena
  unsigned* epoch;                  // this rank's epoch word
  unsigned* ticket;                 // this rank's CTA ticket
  const half* res;                  // residual rows (may alias out)
  long ldres;
  half* out;
  long ldo;
  int rows, cols, world, rank;
  unsigned* err;
};

__device__ __forceinline__ void st_relaxed_sys(unsigned* p, unsigned v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_relaxed_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(kARThreads) allreduce_resid_kernel(ARArgs a) {
  __shared__ unsigned s_e;
  __shared__ int s_ok;
  grid_wait();  // this rank's partial (previous kernel) is complete
  if (threadIdx.x == 0) {
    const unsigned e = *reinterpret_cast<volatile unsigned*>(a.epoch) + 1u;
    s_e = e;
    if (blockIdx.x == 0) {
      // one system-scope fence orders the partial (and everything this rank
      // wrote before) ahead of the flags, then plain stores publish them
      fence_acq_rel_sys();
      for (int q = 0; q < a.world; ++q) st_relaxed_sys(a.peer_flag[q], e);
    }
    int ok = 1;
    const unsigned lim = wait_polls(a.err);
    for (int q = 0; q < a.world && ok; ++q) {
      unsigned it = 0;
      while ((int)(ld_relaxed_sys(a.my_flags + q) - e) < 0) {
        if (++it >= lim) {
          ok = 0;
          atomicOr(a.err, kErrPeerWait);
          break;
        }
      }
      // an acquire load of the flag once it is seen: the peer's partial,
      // written before its release of the flag, is visible to this thread,
      // and to the CTA's other threads after the barrier below
      if (ok) (void)ld_acquire_sys(a.my_flags + q);
    }
    s_ok = ok;
  }
  __syncthreads();
  if (s_ok) {
    // every rank's partial is published: sum in rank order, add the residual
    const int c8 = a.cols / 8;
    const long total = (long)a.rows * c8;
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
      const int r = int(i / c8), c = int(i % c8) * 8;
      // all ranks' 16-byte pieces in flight at once, then the sum in rank order
      uint4 v[kMaxRanks];
#pragma unroll
      for (int q = 0; q < kMaxRanks; ++q)
        if (q < a.world) v[q] = __ldcv(reinterpret_cast<const uint4*>(a.part[q] + (long)r * a.cols + c));
      float acc[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.f;
#pragma unroll
      for (int q = 0; q < kMaxRanks; ++q) {
        if (q >= a.world) break;
        const half* h = reinterpret_cast<const half*>(&v[q]);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] += __half2float(h[j]);
      }
      const uint4 rv = *reinterpret_cast<const uint4*>(a.res + (long)r * a.ldres + c);
      const half* rh = reinterpret_cast<const half*>(&rv);
      uint4 o;
      half* oh = reinterpret_cast<half*>(&o);
#pragma unroll
      for (int j = 0; j < 8; ++j) oh[j] = __float2half_rn(__half2float(rh[j]) + rnd<half>(acc[j]));
      *reinterpret_cast<uint4*>(a.out + (long)r * a.ldo + c) = o;
    }
  }
  // the last CTA records the epoch for the next exchange
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(a.ticket, 1u) == gridDim.x - 1) {
      *a.ticket = 0u;
      *a.epoch = s_e;
    }
  }
  grid_launch_dependents();
}

}  // namespace

size_t comm_region_bytes(const Comm* c) { return c->region_bytes; }
void* comm_region(Comm* c, int r) { return c->arena + c->off_r[r]; }

nmx_status_t comm_exchange_args(Comm* c, int region, ExchangeArgs* out) {
  NMX_CHECK(c && c->connected, NMX_ERR_STATE, "exchange: communicator not connected");
  ExchangeArgs x;
  for (int q = 0; q < c->world; ++q) {
    x.part[q] = reinterpret_cast<const half*>(c->peer[q] + c->off_r[region]);
    x.peer_tflags[q] = reinterpret_cast<unsigned*>(c->peer[q] + c->off_tflags) + size_t(c->rank) * kMaxTileFlags;
  }
  x.my_tflags = reinterpret_cast<unsigned*>(c->arena + c->off_tflags);
  x.epoch = reinterpret_cast<unsigned*>(c->arena + c->off_epoch);
  x.ticket = reinterpret_cast<unsigned*>(c->arena + c->off_tticket);
  x.part_local = reinterpret_cast<half*>(c->arena + c->off_r[region]);
  x.world = c->world;
  x.rank = c->rank;
  *out = x;
  return NMX_OK;
}

nmx_status_t comm_allreduce_resid(Comm* cm, int region, int rows, int cols, const void* res, long ldres, void* out,
                                  long ldo, unsigned* err) {
  NMX_CHECK(cm && cm->connected, NMX_ERR_STATE, "allreduce: communicator not connected");
  NMX_CHECK(region == 0 || region == 1, NMX_ERR_INVALID, "allreduce: region must be 0 or 1");
  NMX_CHECK(cols % 8 == 0 && size_t(rows) * cols * 2 <= cm->region_bytes, NMX_ERR_INVALID,
            "allreduce: rows x cols do not fit the region");
  NMX_CHECK(reinterpret_cast<uintptr_t>(res) % 16 == 0 && reinterpret_cast<uintptr_t>(out) % 16 == 0 &&
                ldres % 8 == 0 && ldo % 8 == 0,
            NMX_ERR_INVALID, "allreduce: residual / output must be 16-byte aligned");
  if (rows == 0) return NMX_OK;
  ARArgs a;
  for (int q = 0; q < cm->world; ++q) {
    a.part[q] = reinterpret_cast<const half*>(cm->peer[q] + cm->off_r[region]);
    a.peer_flag[q] = reinterpret_cast<unsigned*>(cm->peer[q] + cm->off_flags) + cm->rank;
  }
  a.my_flags = reinterpret_cast<unsigned*>(cm->arena + cm->off_flags);
  a.epoch = reinterpret_cast<unsigned*>(cm->arena + cm->off_epoch);
  a.ticket = reinterpret_cast<unsigned*>(cm->arena + cm->off_ticket);
  a.res = static_cast<const half*>(res);
  a.ldres = ldres;
  a.out = static_cast<half*>(out);
  a.ldo = ldo;
  a.rows = rows;
  a.cols = cols;
  a.world = cm->world;
  a.rank = cm->rank;
  a.err = err;
  const long items = (long)rows * (cols / 8);
  const int grid = int(std::max<long>(1, std::min<long>((items + kARThreads - 1) / kARThreads, cm->ctx->num_sms)));
  return launch(cm->ctx, allreduce_resid_kernel, dim3(grid), dim3(kARThreads), 0, a);
}

}  // namespace nmx

struct nmx_comm_s {
  nmx::Comm c;
};

namespace {
size_t align_up256(size_t v) { return (v + 255) & ~size_t(255); }
}  // namespace

extern "C" {

NMX_API nmx_status_t nmx_comm_create(nmx_ctx_t ctx, int rank, int world, size_t region_bytes, nmx_comm_t* out) {
  nmx::clear_error();
  NMX_CHECK(ctx && out, NMX_ERR_INVALID, "nmx_comm_create: null argument");
  NMX_CHECK(world >= 1 && world <= nmx::kMaxRanks && rank >= 0 && rank < world, NMX_ERR_INVALID,
            "nmx_comm_create: rank / world out of range (at most 8 ranks)");
  NMX_CHECK(region_bytes > 0, NMX_ERR_INVALID, "nmx_comm_create: empty region");
  auto* s = new nmx_comm_s();
  nmx::Comm& c = s->c;
  c.ctx = &ctx->c;
  c.owner = ctx;
  c.rank = rank;
  c.world = world;
  c.region_bytes = align_up256(region_bytes);
  c.off_r[0] = 0;
  c.off_r[1] = c.region_bytes;
  c.off_flags = 2 * c.region_bytes;
  c.off_epoch = c.off_flags + 256;
  c.off_ticket = c.off_epoch + 256;
  c.off_tflags = c.off_ticket + 256;
  c.off_tticket = c.off_tflags + size_t(nmx::kMaxRanks) * nmx::kMaxTileFlags * 4;
  c.bytes = c.off_tticket + 256;
  cudaError_t e = cudaSetDevice(c.ctx->device);
  if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&c.arena), c.bytes);
  if (e == cudaSuccess) e = cudaMemset(c.arena, 0, c.bytes);
  if (e != cudaSuccess) {
    if (c.arena) cudaFree(c.arena);
    delete s;
    nmx::set_error(std::string("nmx_comm_create: ") + cudaGetErrorString(e));
    return NMX_ERR_CUDA;
  }
  c.peer[rank] = c.arena;
  ctx->refs++;
  *out = s;
  return NMX_OK;
}

NMX_API nmx_status_t nmx_comm_ipc_handle(nmx_comm_t comm, void* out_handle) {
  nmx::clear_error();
  NMX_CHECK(comm && out_handle, NMX_ERR_INVALID, "nmx_comm_ipc_handle: null argument");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, comm->c.arena);
  NMX_CHECK(e == cudaSuccess, NMX_ERR_CUDA, std::string("cudaIpcGetMemHandle: ") + cudaGetErrorString(e));
  std::memcpy(out_handle, &h, sizeof(h));
  return NMX_OK;
}

NMX_API nmx_status_t nmx_comm_connect(nmx_comm_t comm, const void* handles) {
  nmx::clear_error();
  NMX_CHECK(comm && handles, NMX_ERR_INVALID, "nmx_comm_connect: null argument");
  nmx::Comm& c = comm->c;
  NMX_CHECK(!c.connected, NMX_ERR_STATE, "nmx_comm_connect: already connected");
  cudaSetDevice(c.ctx->device);
  for (int q = 0; q < c.world; ++q) {
    if (q == c.rank) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, static_cast<const unsigned char*>(handles) + size_t(q) * NMX_IPC_HANDLE_BYTES, sizeof(h));
    void* p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int r = 0; r < q; ++r)
        if (r != c.rank && c.peer[r]) {
          cudaIpcCloseMemHandle(c.peer[r]);
          c.peer[r] = nullptr;
        }
      nmx::set_error(std::string("cudaIpcOpenMemHandle: ") + cudaGetErrorString(e));
      return NMX_ERR_CUDA;
    }
    c.peer[q] = static_cast<unsigned char*>(p);
  }
  c.connected = true;
  return NMX_OK;
}

NMX_API void nmx_comm_destroy(nmx_comm_t comm) {
  if (!comm) return;
  nmx::Comm& c = comm->c;
  cudaSetDevice(c.ctx->device);
  cudaStreamSynchronize(c.ctx->stream);
  for (int q = 0; q < c.world; ++q)
    if (q != c.rank && c.peer[q]) cudaIpcCloseMemHandle(c.peer[q]);
  if (c.arena) cudaFree(c.arena);
  nmx_ctx_destroy(c.owner);  // drops the reference taken at creation
  delete comm;
}

NMX_API nmx_status_t nmx_op_allreduce_resid(nmx_comm_t comm, const void* partial, int rows, int cols, const void* res,
                                            void* out) {
  nmx::clear_error();
  NMX_CHECK(comm && partial && res && out, NMX_ERR_INVALID, "nmx_op_allreduce_resid: null argument");
  nmx::Comm& c = comm->c;
  NMX_CHECK(size_t(rows) * cols * 2 <= c.region_bytes, NMX_ERR_INVALID, "nmx_op_allreduce_resid: too large");
  if (rows == 0) return NMX_OK;
  NMX_CUDA_OK(cudaMemcpyAsync(nmx::comm_region(&c, 0), partial, size_t(rows) * cols * 2, cudaMemcpyDeviceToDevice,
                              c.ctx->stream));
  return nmx::comm_allreduce_resid(&c, 0, rows, cols, res, cols, out, cols, c.ctx->dev_err);
}

NMX_API nmx_status_t nmx_model_set_comm(nmx_model_t model, nmx_comm_t comm) {
  nmx::clear_error();
  NMX_CHECK(model != nullptr, NMX_ERR_INVALID, "nmx_model_set_comm: null model");
  nmx::Model* m = model->m;
  if (!comm) {
    m->comm = nullptr;
    m->comm_handle = nullptr;
    m->graphs_clear();
    return NMX_OK;
  }
  nmx::Comm& c = comm->c;
  NMX_CHECK(c.connected, NMX_ERR_STATE, "nmx_model_set_comm: connect the communicator first");
  NMX_CHECK(c.ctx == m->ctx, NMX_ERR_INVALID, "nmx_model_set_comm: communicator of another context");
  NMX_CHECK(c.region_bytes >= size_t(m->max_tokens) * m->cfg.hidden * 2, NMX_ERR_INVALID,
            "nmx_model_set_comm: regions must hold max_tokens x hidden f16");
  NMX_CHECK(m->cfg.hidden % 8 == 0, NMX_ERR_UNSUPPORTED, "nmx_model_set_comm: hidden must be a multiple of 8");
  m->comm = &c;
  m->comm_handle = comm;
  m->graphs_clear();  // captured steps have no exchange
  return NMX_OK;
}

NMX_API nmx_status_t nmx_model_set_exchange_fusion(nmx_model_t model, int enable) {
  nmx::clear_error();
  NMX_CHECK(model != nullptr, NMX_ERR_INVALID, "nmx_model_set_exchange_fusion: null model");
  model->m->fused_exchange = enable != 0;
  model->m->graphs_clear();
  return NMX_OK;
}

}  // extern "C"
