// Cross-GPU primitives for kernels that fuse compute with a collective over
// NVLink 5 / NVSwitch: NVLS multicast reductions (multimem), system-scope
// signals, and bounded waits on them.
//
// A symmetric buffer is mapped twice in every rank's address space: a
// unicast address (this GPU's own copy) and a multicast address (every
// rank's copy at once; an access goes through the switch). The two are
// virtual aliases of the same memory, so accesses through one are ordered
// against accesses through the other with fence.proxy.alias.
#pragma once
#include "../common.cuh"

namespace k8v4 {
namespace peer {

// v is added into every rank's copy of the element (the switch fans it out).
__device__ __forceinline__ void mc_red_add_f32(float* mc_addr, float v) {
  asm volatile("multimem.red.relaxed.sys.global.add.f32 [%0], %1;" ::"l"(mc_addr), "f"(v) : "memory");
}

// Four consecutive floats added into every rank's copy (16-byte aligned).
__device__ __forceinline__ void mc_red_add_v4_f32(float* mc_addr, float4 v) {
  asm volatile("multimem.red.relaxed.sys.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc_addr), "f"(v.x),
               "f"(v.y), "f"(v.z), "f"(v.w)
               : "memory");
}

// Signal: +v on every rank's copy of a 64-bit counter, ordered after this
// thread's earlier writes (and, through a preceding bar.sync, its CTA's).
__device__ __forceinline__ void mc_signal_add_u64(unsigned long long* mc_addr, unsigned long long v) {
  asm volatile("multimem.red.release.sys.global.add.u64 [%0], %1;" ::"l"(mc_addr), "l"(v) : "memory");
}

// v is stored into every rank's copy of the element (the switch fans it out).
__device__ __forceinline__ void mc_st_f32(float* mc_addr, float v) {
  asm volatile("multimem.st.relaxed.sys.global.f32 [%0], %1;" ::"l"(mc_addr), "f"(v) : "memory");
}

// +v on a 64-bit counter (this GPU's or a peer's), ordered after this
// thread's earlier writes (and, through a preceding bar.sync and fence_sys,
// its CTA's).
__device__ __forceinline__ void red_release_add_u64(unsigned long long* addr, unsigned long long v) {
  asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(addr), "l"(v) : "memory");
}

__device__ __forceinline__ void fence_proxy_alias() { asm volatile("fence.proxy.alias;" ::: "memory"); }

__device__ __forceinline__ void fence_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Spin until *p >= target, at most K8V4_WAIT_LIMIT_NS. On timeout records
// kErrPeerTimeout with `site` and returns false (the caller proceeds; the
// host reads the status word and fails the step).
__device__ __forceinline__ bool wait_geq_u64(const unsigned long long* p, unsigned long long target, int site) {
  if (ld_acquire_sys_u64(p) >= target) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (ld_acquire_sys_u64(p) >= target) return true;
    if (globaltimer_ns() - t0 > K8V4_WAIT_LIMIT_NS) {
      record_error(kErrPeerTimeout, site);
      return false;
    }
    __nanosleep(64);
  }
}

// Completion tracking of a producer -> consumer exchange through symmetric
// memory: the producer's CTAs (on every rank) each add 1 to a counter, and
// one consumer launch waits until its copy of the counter holds one more
// call's worth of signals.
struct ReduceSync {
  const unsigned long long* flag;  // this rank's copy of the multicast counter
  unsigned long long* state;       // [0] signals consumed so far, [1] CTAs of this launch done
  unsigned long long expected;     // signals one producer call sends (world x its CTAs)
};

// Every thread of the CTA returns once the counter reached state[0] +
// expected (or the wait gave up and recorded kErrPeerTimeout at `site`).
__device__ __forceinline__ void sync_wait(const ReduceSync& s, int site) {
  if (threadIdx.x == 0) {
    const unsigned long long target = *reinterpret_cast<volatile unsigned long long*>(s.state) + s.expected;
    wait_geq_u64(s.flag, target, site);
  }
  __syncthreads();
  fence_proxy_alias();  // the data arrived through the multicast alias
}

// Every CTA of the consumer launch calls this once; the last one advances
// state[0] by `expected` (a running count: a replayed CUDA graph needs no
// reset, and calls may differ in size).
__device__ __forceinline__ void sync_done(const ReduceSync& s) {
  fence_proxy_alias();  // this CTA's reads and writes precede later multicast traffic
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned long long ctas = (unsigned long long)gridDim.x * gridDim.y * gridDim.z;
    const unsigned long long prev = atomicAdd(s.state + 1, 1ull);
    if (prev == ctas - 1) {
      s.state[1] = 0;
      s.state[0] += s.expected;
      __threadfence();
    }
  }
}

}  // namespace peer
}  // namespace k8v4
