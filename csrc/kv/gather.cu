// Paged gather + dequantize of one KV head into dense K / V rows (b200
// format), the standalone counterpart of the reference's Triton gather
// (k8v4_v030/prefill_gather_triton.py:15-40; torch form dequant.py:114-157).
// The attention kernels dequantize inside their pipelines; this kernel is the
// test utility that checks them against a dense reference and the staging
// step for callers that want dense K / V rows.
//
// One warp per token: lane l handles dims [4l, 4l + 4). K = int8 x k_scale,
// V = (nibble - 8) x v_scale[dim / 32], both products exact in fp32 (an int8
// or int4 times an fp16 value), so the result is bitwise equal to the torch
// gather of the same pages.
#include "attn_common.cuh"

namespace k8v4 {
namespace attn {

template <typename OutT>
__device__ __forceinline__ void store4(OutT* dst, float a, float b, float c, float d);

template <>
__device__ __forceinline__ void store4<float>(float* dst, float a, float b, float c, float d) {
  *reinterpret_cast<float4*>(dst) = make_float4(a, b, c, d);
}

template <>
__device__ __forceinline__ void store4<__nv_bfloat16>(__nv_bfloat16* dst, float a, float b, float c, float d) {
  __nv_bfloat162 lo = __floats2bfloat162_rn(a, b), hi = __floats2bfloat162_rn(c, d);
  uint2 v;
  v.x = *reinterpret_cast<uint32_t*>(&lo);
  v.y = *reinterpret_cast<uint32_t*>(&hi);
  *reinterpret_cast<uint2*>(dst) = v;
}

template <typename OutT>
__global__ void __launch_bounds__(256) gather_dequant_kernel(const uint8_t* __restrict__ cache,
                                                             const int32_t* __restrict__ block_table, int hkv,
                                                             int head, int seq_len, int64_t num_pages,
                                                             OutT* __restrict__ k_out, OutT* __restrict__ v_out) {
  pdl_trigger();
  pdl_wait();  // everything this kernel reads may come from the previous one
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= seq_len) return;
  const int64_t page = block_table[warp / PAGE];
  const int t = warp % PAGE;
  OutT* kd = k_out + (int64_t)warp * D + lane * 4;
  OutT* vd = v_out + (int64_t)warp * D + lane * 4;
  if (page < 0 || page >= num_pages) {  // unmapped page: zeros
    store4<OutT>(kd, 0.f, 0.f, 0.f, 0.f);
    store4<OutT>(vd, 0.f, 0.f, 0.f, 0.f);
    return;
  }
  const uint8_t* run = cache + (page * hkv + head) * HEAD_BYTES;
  const uint32_t kq = *reinterpret_cast<const uint32_t*>(run + t * D + lane * 4);
  const float ks = __half2float(*reinterpret_cast<const __half*>(run + VS_OFF + KS_OFF + t * 2));
  const float k0 = (float)(int8_t)(kq & 0xff) * ks, k1 = (float)(int8_t)((kq >> 8) & 0xff) * ks;
  const float k2 = (float)(int8_t)((kq >> 16) & 0xff) * ks, k3 = (float)(int8_t)(kq >> 24) * ks;
  store4<OutT>(kd, k0, k1, k2, k3);
  const uint16_t vq = *reinterpret_cast<const uint16_t*>(run + VS_OFF + t * 64 + lane * 2);
  const float vsc = __half2float(*reinterpret_cast<const __half*>(run + VS_OFF + VSC_OFF + (t * 4 + lane / 8) * 2));
  const float v0 = (float)((int)(vq & 0xf) - 8) * vsc, v1 = (float)((int)((vq >> 4) & 0xf) - 8) * vsc;
  const float v2 = (float)((int)((vq >> 8) & 0xf) - 8) * vsc, v3 = (float)((int)(vq >> 12) - 8) * vsc;
  store4<OutT>(vd, v0, v1, v2, v3);
}

}  // namespace attn
}  // namespace k8v4

using namespace k8v4;
using namespace k8v4::attn;

K8V4_STATUS_API(gather)

// out_dtype 0: fp32, 1: bf16. k_out / v_out: [seq_len, 128].
extern "C" int k8v4_gather_dequant(const void* cache, int64_t num_pages, const int32_t* block_table, int hkv,
                                   int head, int seq_len, int out_dtype, void* k_out, void* v_out,
                                   cudaStream_t st) {
  if (seq_len <= 0) return 0;
  if (head < 0 || head >= hkv) return 1;
  const int blocks = (seq_len * 32 + 255) / 256;
  if (out_dtype == 0)
    launch_k(gather_dequant_kernel<float>, dim3(blocks), dim3(256), 0, st, reinterpret_cast<const uint8_t*>(cache), block_table, hkv,
                                                         head, seq_len, num_pages, reinterpret_cast<float*>(k_out),
                                                         reinterpret_cast<float*>(v_out));
  else
    launch_k(gather_dequant_kernel<__nv_bfloat16>, dim3(blocks), dim3(256), 0, st, 
        reinterpret_cast<const uint8_t*>(cache), block_table, hkv, head, seq_len, num_pages,
        reinterpret_cast<__nv_bfloat16*>(k_out), reinterpret_cast<__nv_bfloat16*>(v_out));
  return cudaGetLastError() == cudaSuccess ? 0 : 2;
}
