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

}  // namespace sampler
}  // namespace k8v4

using namespace k8v4;

K8V4_STATUS_API(sampler)

extern "C" int k8v4_argmax(const void* logits, int rows, int vocab, int64_t ld, int64_t offset, float* best_val,
                           int64_t* best_idx, cudaStream_t st) {
  if (rows <= 0) return 0;
  if (ld < vocab) return 2;
  launch_k(sampler::argmax_kernel, dim3(rows), dim3(1024), 0, st, reinterpret_cast<const __nv_bfloat16*>(logits), vocab, ld, offset,
                                                 best_val, best_idx);
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}
