// Split-K decode attention without any allocation by the library.
//
// Declared in ../k8v4_c_api.h. This entry point has no counterpart in the
// reference; it is an addition of this library.
//
// Who needs it: callers that cannot allocate device memory at the point where
// they run attention -- code running inside a host thread that must not call
// cudaMalloc (it synchronizes the device and can deadlock against work the
// caller has queued), embedders whose device memory is owned by another
// allocator, and plugin hosts that forbid allocations after start-up. They
// still pass every input and output tensor; only the split-K scratch (the
// per-split running max, row sum and partial output rows that the combine
// step merges) lives here, in a fixed array in device memory that every GPU
// which loads the library keeps until the process exits.
//
// Limits and behaviour:
//   * The scratch holds K8V4_NOALLOC_SCRATCH_FLOATS floats (4 MiB). A launch
//     needing more (see k8v4_decode_ws_floats: sequences x heads x splits x
//     padded rows x 130) is refused with return code 20 and a message on
//     stderr; use fewer splits or the allocating entry point.
//   * The first call on a device looks up the array's device address with
//     cudaGetSymbolAddress while that device is current, and caches it. Make
//     that first call before any stream capture on the device.
//   * Every call shares the one array and it keeps the last call's contents.
//     Nothing in it needs to start at zero: each split writes all of its
//     partial rows before the combine reads them. Two calls whose kernels
//     overlap on the GPU (different streams, or concurrent graph branches)
//     race on the array and corrupt each other's output; serialize them.
//   * The call allocates nothing: no cudaMalloc, cudaFree or allocating
//     library routine.
#include <atomic>
#include <cstdio>

#include "../common.cuh"
#include "../k8v4_c_api.h"

#ifndef K8V4_NOALLOC_SCRATCH_FLOATS
#define K8V4_NOALLOC_SCRATCH_FLOATS (1 << 20)
#endif

static __device__ __align__(256) float g_decode_noalloc_scratch[K8V4_NOALLOC_SCRATCH_FLOATS];

namespace {
constexpr int kMaxDevices = 64;
// Device address of the array on each device. Two host threads making their
// first call on one device at the same time both look it up and store the
// same value; the atomics make that well defined.
std::atomic<float*> g_scratch_addr[kMaxDevices];

// Device address of the scratch array on the current device (looked up once).
float* scratch_for_current_device(int* err) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    *err = 21;
    return nullptr;
  }
  float* known = g_scratch_addr[dev].load(std::memory_order_acquire);
  if (!known) {
    void* p = nullptr;
    const cudaError_t rc = cudaGetSymbolAddress(&p, g_decode_noalloc_scratch);
    if (rc != cudaSuccess || p == nullptr) {
      fprintf(stderr, "k8v4_decode_attn_noalloc: cudaGetSymbolAddress failed on device %d: %s\n", dev,
              cudaGetErrorString(rc));
      *err = 22;
      return nullptr;
    }
    known = static_cast<float*>(p);
    g_scratch_addr[dev].store(known, std::memory_order_release);
  }
  return known;
}
}  // namespace

// Capacity of the built-in scratch, in floats.
extern "C" int64_t k8v4_decode_attn_noalloc_max_floats(void) { return K8V4_NOALLOC_SCRATCH_FLOATS; }

// Same arguments and results as k8v4_decode_attn, minus the two workspace
// pointers. Returns 0 on success, 20 when the launch needs more scratch than
// the array holds, 21/22 when the device or the array's address cannot be
// obtained, and k8v4_decode_attn's codes otherwise.
extern "C" int k8v4_decode_attn_noalloc(const void* q, const int32_t* cu_q, const int32_t* seq_lens,
                                        const int32_t* q_ends, const int32_t* block_table, int bt_stride,
                                        const void* cache, int64_t num_pages, int hkv, int head_offset, int heads,
                                        int gqa, int hq_total, int nseq, int max_q_len, int nsplit, float sm_scale,
                                        void* out, cudaStream_t st) {
  float* ws_o = nullptr;
  float* ws_ml = nullptr;
  if (nsplit > 1) {
    const int64_t need = k8v4_decode_ws_floats(nseq, heads, nsplit, max_q_len, gqa);
    if (need > K8V4_NOALLOC_SCRATCH_FLOATS) {
      fprintf(stderr,
              "k8v4_decode_attn_noalloc: %lld scratch floats needed (nseq=%d heads=%d nsplit=%d q_len=%d), "
              "built-in maximum is %d; use fewer splits or k8v4_decode_attn with a workspace\n",
              (long long)need, nseq, heads, nsplit, max_q_len, K8V4_NOALLOC_SCRATCH_FLOATS);
      return 20;
    }
    int err = 0;
    float* base = scratch_for_current_device(&err);
    if (!base) return err;
    const int64_t ml = need / (128 + 2) * 2;  // (m, l) planes first, then the partial rows
    ws_ml = base;
    ws_o = base + ml;
  }
  return k8v4_decode_attn(q, cu_q, seq_lens, q_ends, block_table, bt_stride, cache, num_pages, hkv, head_offset,
                          heads, gqa, hq_total, nseq, max_q_len, nsplit, sm_scale, out, ws_o, ws_ml, st);
}
