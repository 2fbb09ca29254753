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

// Signal: +v on every rank's copy of a 64-bit counter, ordered after this
// thread's earlier writes (and, through a preceding bar.sync, its CTA's).
__device__ __forceinline__ void mc_signal_add_u64(unsigned long long* mc_addr, unsigned long long v) {
  asm volatile("multimem.red.release.sys.global.add.u64 [%0], %1;" ::"l"(mc_addr), "l"(v) : "memory");
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

}  // namespace peer
}  // namespace k8v4
