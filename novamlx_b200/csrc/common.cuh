// Shared device/host helpers for libnovamlx_cuda (sm_100a only).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/nmx.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "libnovamlx_cuda is built for sm_100a only"
#endif

namespace nmx {

// ----------------------------------------------------------------- errors
void set_error(const std::string& msg);
const char* get_error();
void clear_error();

struct Status {
  nmx_status_t code;
};

#define NMX_CUDA_OK(expr)                                                               \
  do {                                                                                  \
    cudaError_t _e = (expr);                                                            \
    if (_e != cudaSuccess) {                                                            \
      ::nmx::set_error(std::string(#expr) + ": " + cudaGetErrorString(_e) + " at " +    \
                       __FILE__ + ":" + std::to_string(__LINE__));                      \
      return NMX_ERR_CUDA;                                                              \
    }                                                                                   \
  } while (0)

#define NMX_CHECK(cond, code, msg)        \
  do {                                    \
    if (!(cond)) {                        \
      ::nmx::set_error(std::string(msg)); \
      return (code);                      \
    }                                     \
  } while (0)

#define NMX_TRY(expr)                \
  do {                               \
    nmx_status_t _s = (expr);        \
    if (_s != NMX_OK) return _s;     \
  } while (0)

// --------------------------------------------------------------- contexts
struct Ctx {
  int device = 0;
  cudaStream_t stream = nullptr;
  bool owns_stream = false;
  int num_sms = 148;
  uint64_t launches = 0;
  // growable device workspace for op-level entry points
  void* ws = nullptr;
  size_t ws_bytes = 0;
  unsigned* counters = nullptr;  // zeroed, reset by kernels after use
  size_t n_counters = 0;
  // device words: [0] error bits that kernels set when a bounded wait runs
  // out (read and cleared with each step's results and by
  // nmx_ctx_synchronize); [1] the number of polls a wait makes before it
  // gives up (nmx_ctx_set_wait_limit)
  unsigned* dev_err = nullptr;
};

// error bits of the device word: which kind of bounded wait ran out
constexpr unsigned kErrPeerWait = 1u;   // a peer rank's exchange flag (tensor parallelism)
constexpr unsigned kErrPipeWait = 2u;   // a pipeline barrier inside a tensor-core GEMM
constexpr unsigned kErrShareWait = 4u;  // the K shares of a split GEMM tile group
constexpr unsigned kDefaultWaitPolls = 1u << 24;
// the poll limit the host set for this context (one load per kernel)
__device__ __forceinline__ unsigned wait_polls(const unsigned* err) {
  return reinterpret_cast<const volatile unsigned*>(err)[1];
}

nmx_status_t ctx_workspace(Ctx* c, size_t bytes, void** out);
// after the stream has drained: NMX_ERR_TIMEOUT if a kernel reported a wait
// that ran out (the word is cleared)
nmx_status_t ctx_check_device_error(Ctx* c);
nmx_status_t ctx_counters(Ctx* c, size_t n, unsigned** out);

// ---------------------------------------------------------- dtype traits
template <typename T>
struct DT;
template <>
struct DT<half> {
  static __device__ __forceinline__ float to_f(half v) { return __half2float(v); }
  static __device__ __forceinline__ half from_f(float v) { return __float2half_rn(v); }
};
template <>
struct DT<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};

template <typename T>
__device__ __forceinline__ float tof(T v) {
  return DT<T>::to_f(v);
}
template <typename T>
__device__ __forceinline__ T fromf(float v) {
  return DT<T>::from_f(v);
}
// round through the storage type, as an MLX array materialisation does
template <typename T>
__device__ __forceinline__ float rnd(float v) {
  return tof<T>(fromf<T>(v));
}

// ------------------------------------------------ programmatic dependent launch
// Every kernel calls grid_wait() before it reads data written by the previous
// kernel on the stream and before it writes anything; loads of immutable data
// (weights) may be issued before it.
__device__ __forceinline__ void grid_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Launch with the programmatic-stream-serialisation attribute so the next
// kernel's prologue overlaps this kernel's tail. Works under stream capture.
template <typename... KArgs, typename... Args>
nmx_status_t launch(Ctx* c, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                    Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = c->stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
  if (e != cudaSuccess) {
    set_error(std::string("kernel launch: ") + cudaGetErrorString(e));
    return NMX_ERR_CUDA;
  }
  c->launches++;
  return NMX_OK;
}

// As launch, with CTAs grouped in clusters of cluster_x along x (1 = none).
template <typename... KArgs, typename... Args>
nmx_status_t launch_cluster(Ctx* c, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, unsigned cluster_x,
                            Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = c->stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = cluster_x;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = cluster_x > 1 ? 2 : 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
  if (e != cudaSuccess) {
    set_error(std::string("kernel launch (cluster ") + std::to_string(cluster_x) + "): " + cudaGetErrorString(e));
    return NMX_ERR_CUDA;
  }
  c->launches++;
  return NMX_OK;
}

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

}  // namespace nmx
