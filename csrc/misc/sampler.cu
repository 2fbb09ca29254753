// Greedy sampling: per-row argmax over (a vocab shard of) bf16 logits.
// Returns the max value and its global index (shard offset added) so a
// vocab-parallel rank can reduce (value, index) pairs across ranks instead of
// gathering full logits. Ties resolve to the lowest index, like torch.argmax.
#include "../common.cuh"

namespace k8v4 {
namespace sampler {

// Row r of the logits starts at logits + r * ld (ld >= vocab: a lm_head shard
// padded to the GEMM's 128-row tile is read only over its real columns).
__global__ void __launch_bounds__(1024) argmax_kernel(const __nv_bfloat16* __restrict__ logits, int vocab, int64_t ld,
                                                      int64_t offset, float* best_val, int64_t* best_idx) {
  pdl_trigger();
  pdl_wait();  // everything this kernel reads may come from the previous one
  __shared__ float sv[32];
  __shared__ int si[32];
  const int64_t row = blockIdx.x;
  const __nv_bfloat16* x = logits + row * ld;
  const bool vec = (ld & 7) == 0 && (reinterpret_cast<uintptr_t>(logits) & 15) == 0;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int c = threadIdx.x * 8; c < vocab; c += blockDim.x * 8) {
    if (c + 8 <= vocab && vec) {
      const uint4 raw = *reinterpret_cast<const uint4*>(x + c);
      const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float v = __bfloat162float(h[j]);
        if (v > bv) { bv = v; bi = c + j; }
      }
    } else {
      for (int j = 0; j < 8 && c + j < vocab; ++j) {
        const float v = __bfloat162float(x[c + j]);
        if (v > bv) { bv = v; bi = c + j; }
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) { sv[w] = bv; si[w] = bi; }
  __syncthreads();
  if (w == 0) {
    bv = (l < (int)(blockDim.x >> 5)) ? sv[l] : -INFINITY;
    bi = (l < (int)(blockDim.x >> 5)) ? si[l] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if (l == 0) {
      best_val[row] = bv;
      best_idx[row] = (bi == 0x7fffffff ? 0 : bi) + offset;
    }
  }
}

// The same over a cluster of kArgCluster CTAs per row, each scanning one
// contiguous slice of the row; the slices' (value, index) pairs meet through
// distributed shared memory in CTA-rank (= column) order, so ties still
// resolve to the lowest index. One CTA per row took ~14 us for a 151,936-wide
// vocabulary, bound by one SM's load rate.
constexpr int kArgCluster = 8;
constexpr int kArgThreads = 512;

__device__ __forceinline__ void argmax_cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__global__ void __launch_bounds__(kArgThreads) argmax_cluster_kernel(const __nv_bfloat16* __restrict__ logits,
                                                                     int vocab, int64_t ld, int64_t offset,
                                                                     float* best_val, int64_t* best_idx) {
  pdl_trigger();
  pdl_wait();  // the logits come from the previous kernel
  __shared__ float sv[32];
  __shared__ int si[32];
  __shared__ float cv;
  __shared__ int ci;
  const int64_t row = blockIdx.y;
  const __nv_bfloat16* x = logits + row * ld;
  const bool vec = (ld & 7) == 0 && (reinterpret_cast<uintptr_t>(logits) & 15) == 0;
  const int chunk = ((vocab + kArgCluster * 8 - 1) / (kArgCluster * 8)) * 8;  // a multiple of 8
  const int c0 = blockIdx.x * chunk;
  const int c1 = min(vocab, c0 + chunk);
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int c = c0 + threadIdx.x * 8; c < c1; c += kArgThreads * 8) {
    if (c + 8 <= c1 && vec) {
      const uint4 raw = *reinterpret_cast<const uint4*>(x + c);
      const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float v = __bfloat162float(h[j]);
        if (v > bv) { bv = v; bi = c + j; }
      }
    } else {
      for (int j = 0; j < 8 && c + j < c1; ++j) {
        const float v = __bfloat162float(x[c + j]);
        if (v > bv) { bv = v; bi = c + j; }
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) { sv[w] = bv; si[w] = bi; }
  __syncthreads();
  if (w == 0) {
    bv = (l < kArgThreads / 32) ? sv[l] : -INFINITY;
    bi = (l < kArgThreads / 32) ? si[l] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if (l == 0) { cv = bv; ci = bi; }
  }
  argmax_cluster_sync();  // every slice's best is written
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    const uint32_t av = static_cast<uint32_t>(__cvta_generic_to_shared(&cv));
    const uint32_t ai = static_cast<uint32_t>(__cvta_generic_to_shared(&ci));
    float best = -INFINITY;
    int idx = 0x7fffffff;
    for (int r = 0; r < kArgCluster; ++r) {
      uint32_t rv, ri;
      float v;
      int i;
      asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(rv) : "r"(av), "r"(r));
      asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ri) : "r"(ai), "r"(r));
      asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(rv) : "memory");
      asm volatile("ld.shared::cluster.s32 %0, [%1];" : "=r"(i) : "r"(ri) : "memory");
      if (v > best || (v == best && i < idx)) { best = v; idx = i; }
    }
    best_val[row] = best;
    best_idx[row] = (idx == 0x7fffffff ? 0 : idx) + offset;
  }
  argmax_cluster_sync();  // no CTA leaves while its slice is being read
}

}  // namespace sampler
}  // namespace k8v4

using namespace k8v4;

K8V4_STATUS_API(sampler)

// Rows of a wide vocabulary run on a cluster per row (argmax_cluster_kernel)
// unless K8V4_ARGMAX_CLUSTER=0.
static bool argmax_cluster_enabled() {
  static const bool on = [] {
    const char* v = getenv("K8V4_ARGMAX_CLUSTER");
    return !(v && (v[0] == '0' || v[0] == 'n' || v[0] == 'N' || v[0] == 'f' || v[0] == 'F'));
  }();
  return on;
}

extern "C" int k8v4_argmax(const void* logits, int rows, int vocab, int64_t ld, int64_t offset, float* best_val,
                           int64_t* best_idx, cudaStream_t st) {
  if (rows <= 0) return 0;
  if (ld < vocab) return 2;
  if (vocab >= 8192 && argmax_cluster_enabled()) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(sampler::kArgCluster, rows);
    cfg.blockDim = dim3(sampler::kArgThreads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = sampler::kArgCluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, sampler::argmax_cluster_kernel, reinterpret_cast<const __nv_bfloat16*>(logits),
                              vocab, ld, offset, best_val, best_idx) == cudaSuccess
               ? 0
               : 1;
  }
  launch_k(sampler::argmax_kernel, dim3(rows), dim3(1024), 0, st, reinterpret_cast<const __nv_bfloat16*>(logits), vocab, ld, offset,
                                                 best_val, best_idx);
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}
