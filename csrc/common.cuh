// Shared device helpers for the k8v4 sm_100a kernel library.
#pragma once
#include <atomic>
#include <cstdint>
#include <cstdlib>
#include <utility>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#ifndef K8V4_HOST_DEVICE
#define K8V4_HOST_DEVICE __host__ __device__
#endif

namespace k8v4 {

// Error codes written into the library's device status word when a kernel
// gives up instead of waiting forever (bounded waits) or rejects its inputs.
enum : int {
  kOk = 0,
  kErrMbarTimeout = 1,     // an mbarrier wait ran past its time limit
  kErrPeerTimeout = 2,     // a wait on a peer GPU's flag ran past its limit
  kErrBadShape = 3,        // device-side shape guard tripped
  kErrBadIndex = 4,        // device-side bounds guard tripped (the access was skipped)
};

// Nanoseconds a device-side wait may spin before it records a timeout.
#ifndef K8V4_WAIT_LIMIT_NS
#define K8V4_WAIT_LIMIT_NS 2000000000ull
#endif

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Device status word of this translation unit (one per device that loaded
// the library). Each .cu file exports a reader through K8V4_STATUS_API.
static __device__ int g_k8v4_status;
// Where the first recorded error happened (site id of the wait, see tc.cuh).
static __device__ int g_k8v4_site;

// Returns the status code in the low byte and the site id above it.
#define K8V4_STATUS_API(unit)                                              \
  extern "C" int k8v4_status_##unit(int clear) {                           \
    int v = 0, site = 0;                                                   \
    cudaMemcpyFromSymbol(&v, k8v4::g_k8v4_status, sizeof(int));            \
    cudaMemcpyFromSymbol(&site, k8v4::g_k8v4_site, sizeof(int));           \
    if (clear && v) {                                                      \
      int z = 0;                                                           \
      cudaMemcpyToSymbol(k8v4::g_k8v4_status, &z, sizeof(int));            \
      cudaMemcpyToSymbol(k8v4::g_k8v4_site, &z, sizeof(int));              \
    }                                                                      \
    return v ? (v | (site << 8)) : 0;                                      \
  }

// Raises Kernel's dynamic shared-memory limit to `bytes` on the current
// device. The attribute belongs to the device, so it is set once per
// (kernel, device): a process that drives several GPUs sets it on each.
template <auto Kernel>
inline cudaError_t ensure_smem_limit(int bytes) {
  static std::atomic<unsigned long long> done{0};  // bit d: set on device d
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const unsigned long long bit = dev < 64 ? 1ull << dev : 0ull;
  if (bit && (done.load(std::memory_order_acquire) & bit)) return cudaSuccess;
  e = cudaFuncSetAttribute(Kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess && bit) done.fetch_or(bit, std::memory_order_release);
  return e;
}

__device__ __forceinline__ void record_error(int code, int site = 0) {
  if (atomicCAS(&g_k8v4_status, 0, code) == 0) g_k8v4_site = site;
}

__device__ __forceinline__ float bf2f(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ __nv_bfloat16 f2bf(float v) { return __float2bfloat16_rn(v); }

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

K8V4_HOST_DEVICE inline int cdiv(int a, int b) { return (a + b - 1) / b; }

// ------------------------------------------------ programmatic dependent launch
// Kernels are launched with programmatic stream serialization (decode runs
// ~11 dependent kernels per layer inside a CUDA graph): the next kernel's
// CTAs may start once every CTA of the current one has started, set up
// barriers / TMEM and stream inputs that no earlier kernel writes (weights),
// and wait for the previous grid's completion and memory only where they
// first touch its results. Both instructions are no-ops in a kernel launched
// without the attribute.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// K8V4_PDL=0 in the environment turns the attribute off (plain stream order).
inline bool pdl_enabled() {
  static const int on = [] {
    const char* e = getenv("K8V4_PDL");
    return (e && e[0] == '0') ? 0 : 1;
  }();
  return on != 0;
}

// kern<<<grid, block, smem, st>>>(args...) with the programmatic attribute.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                           Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

}  // namespace k8v4
