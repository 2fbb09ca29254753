// K8/V4 cache write: quantize fresh K/V rows into paged storage.
//
// One warp per (token, KV head). K: symmetric int8 with scale amax/127, V:
// symmetric int4 per 32-dim group with scale amax/7 (b200 format) or affine
// uint4 per row (ref format, the reference's K6/K7 store rules at
// k8v4_v030/native/xe2_kv_ops.cpp:536-627). Every fp32 step matches the
// torch oracle (k8v4_xpu_b200/kv/oracle.py) operation for operation, so the
// stored bytes are identical. A slot that is negative or past the cache is
// skipped (reference :549-563).
//
// The b200 variant optionally applies rotary embedding (neox halves) to K
// and to the query heads of the same fused qkv row, writing the rotated
// queries for attention, so the qkv projection output is read exactly once.
#include "../common.cuh"

namespace k8v4 {
namespace kv {

struct StoreArgs {
  const __nv_bfloat16* qkv;  // fused rows [T, (hq + 2*hkv) * D] (b200) or nullptr
  float* qkv_f;              // or the same rows as the qkv GEMM's fp32 split-K sums (read, then zeroed)
  const __nv_bfloat16* k;    // separate K rows [T, hkv, D] when qkv == nullptr
  const __nv_bfloat16* v;
  int64_t k_stride_t, v_stride_t;  // token strides (elements) of k / v
  const int64_t* slots;      // [T]
  uint8_t* cache;            // [num_pages, page_bytes]
  int64_t num_pages;
  int T, hkv, hq;
  int page_bytes;
  // rotary (b200 fused path)
  const float* cos_sin;      // [max_pos, D] as (cos[D/2], sin[D/2])
  const int64_t* positions;  // [T]
  __nv_bfloat16* q_out;      // [T, hq, D]
};

__device__ __forceinline__ float rint_f(float x) { return rintf(x); }

// ----------------------------------------------------------------- b200
// D = 128, page 16, head-major (page, head) runs of 3,232 bytes:
// [K 16x128 int8][V 16x64 u8][k_scale 16 fp16][v_scale 16x4 fp16].
template <bool ROPE>
__global__ void store_b200_kernel(StoreArgs a) {
  pdl_trigger();
  pdl_wait();  // everything this kernel reads may come from the previous one
  constexpr int D = 128, PAGE = 16, HEAD_BYTES = 3232;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int heads_per_tok = ROPE ? (a.hq + a.hkv) : a.hkv;
  if (gw >= a.T * heads_per_tok) return;
  const int t = gw / heads_per_tok;
  const int hh = gw % heads_per_tok;
  const int d0 = lane * 4;

  float x[4], y[4];
  const int row = a.hq + 2 * a.hkv;
  // 4 values of a fused qkv row: bf16, or the GEMM's fp32 split-K sums, which
  // are rounded to bf16 as the split-K finish would and zeroed for the next
  // split-K GEMM (every element of the row is read by exactly one warp)
  auto load_row4 = [&](int64_t off, float (&f)[4]) {
    if (a.qkv_f) {
      float4* p4 = reinterpret_cast<float4*>(a.qkv_f + off);
      const float4 v = *p4;
      *p4 = make_float4(0.f, 0.f, 0.f, 0.f);
      f[0] = __bfloat162float(__float2bfloat16_rn(v.x));
      f[1] = __bfloat162float(__float2bfloat16_rn(v.y));
      f[2] = __bfloat162float(__float2bfloat16_rn(v.z));
      f[3] = __bfloat162float(__float2bfloat16_rn(v.w));
    } else {
      const uint2 raw = *reinterpret_cast<const uint2*>(a.qkv + off);
      const __nv_bfloat162* p2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
      const float2 f0 = __bfloat1622float2(p2[0]), f1 = __bfloat1622float2(p2[1]);
      f[0] = f0.x; f[1] = f0.y; f[2] = f1.x; f[3] = f1.y;
    }
  };
  if (ROPE) {
    // head hh < hq: a query head; otherwise KV head hh - hq, whose V columns
    // are read here too (before any early return, so they are always consumed)
    const int col = (hh < a.hq) ? hh * D : (a.hq + (hh - a.hq)) * D;
    load_row4((int64_t)t * row * D + col + d0, x);
    if (hh >= a.hq) load_row4((int64_t)t * row * D + (a.hq + a.hkv + (hh - a.hq)) * D + d0, y);
  } else {
    const __nv_bfloat16* src = a.k + (int64_t)t * a.k_stride_t + (int64_t)hh * D;
    const uint2 raw = *reinterpret_cast<const uint2*>(src + d0);
    const __nv_bfloat162* p2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
    const float2 f0 = __bfloat1622float2(p2[0]), f1 = __bfloat1622float2(p2[1]);
    x[0] = f0.x; x[1] = f0.y; x[2] = f1.x; x[3] = f1.y;
  }
  if (ROPE) {
    // neox rotation: pair dim i (< D/2) with i + D/2. Lanes 0-15 hold the first
    // half, lanes 16-31 the second half of the same pairs.
    const int64_t pos = a.positions[t];
    const float* cs = a.cos_sin + pos * D;
    const int i0 = (lane & 15) * 4;
    float other[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) other[j] = __shfl_xor_sync(0xffffffffu, x[j], 16);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float c = cs[i0 + j], s = cs[D / 2 + i0 + j];
      // first half: x1*c - x2*s ; second half: x2*c + x1*s
      x[j] = (lane < 16) ? __fsub_rn(__fmul_rn(x[j], c), __fmul_rn(other[j], s))
                         : __fadd_rn(__fmul_rn(x[j], c), __fmul_rn(other[j], s));
    }
    if (hh < a.hq) {
      __nv_bfloat16* q = a.q_out + ((int64_t)t * a.hq + hh) * D + d0;
      __nv_bfloat162 o0 = __floats2bfloat162_rn(x[0], x[1]), o1 = __floats2bfloat162_rn(x[2], x[3]);
      uint2 w;
      w.x = *reinterpret_cast<uint32_t*>(&o0);
      w.y = *reinterpret_cast<uint32_t*>(&o1);
      *reinterpret_cast<uint2*>(q) = w;
      return;
    }
    // Round the rotated K to bf16, as a bf16 model would hold it.
#pragma unroll
    for (int j = 0; j < 4; ++j) x[j] = __bfloat162float(__float2bfloat16_rn(x[j]));
  }
  const int h = ROPE ? (hh - a.hq) : hh;
  const int64_t slot = a.slots[t];
  if (slot < 0 || slot >= a.num_pages * PAGE) return;
  const int64_t page = slot / PAGE;
  const int off = (int)(slot % PAGE);
  uint8_t* base = a.cache + page * a.page_bytes + (int64_t)h * HEAD_BYTES;

  // ---- K: int8 symmetric, fp16 scale
  float amax = fmaxf(fmaxf(fabsf(x[0]), fabsf(x[1])), fmaxf(fabsf(x[2]), fabsf(x[3])));
  amax = warp_max(amax);
  const __half ks = __float2half_rn(amax / 127.f);
  const float ksf = __half2float(ks);
  const float kinv = ksf > 0.f ? 1.f / ksf : 0.f;
  uint32_t packed = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float q = fminf(fmaxf(rint_f(__fmul_rn(x[j], kinv)), -127.f), 127.f);
    packed |= (uint32_t)((uint8_t)(int8_t)(int)q) << (8 * j);
  }
  *reinterpret_cast<uint32_t*>(base + off * D + d0) = packed;
  if (lane == 0) *reinterpret_cast<__half*>(base + 3072 + off * 2) = ks;

  // ---- V: int4 symmetric per 32-dim group (8 lanes), fp16 scale
  if (!ROPE) {
    const __nv_bfloat16* vsrc = a.v + (int64_t)t * a.v_stride_t + (int64_t)h * D;
    const uint2 raw = *reinterpret_cast<const uint2*>(vsrc + d0);
    const __nv_bfloat162* p2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
    const float2 f0 = __bfloat1622float2(p2[0]), f1 = __bfloat1622float2(p2[1]);
    y[0] = f0.x; y[1] = f0.y; y[2] = f1.x; y[3] = f1.y;
  }
  float vmax = fmaxf(fmaxf(fabsf(y[0]), fabsf(y[1])), fmaxf(fabsf(y[2]), fabsf(y[3])));
#pragma unroll
  for (int o = 1; o < 8; o <<= 1) vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, o));
  const __half vs = __float2half_rn(vmax / 7.f);
  const float vsf = __half2float(vs);
  const float vinv = vsf > 0.f ? 1.f / vsf : 0.f;
  uint32_t nib[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float q = fminf(fmaxf(rint_f(__fmul_rn(y[j], vinv)), -7.f), 7.f);
    nib[j] = (uint32_t)((int)q + 8);
  }
  const uint16_t vb = (uint16_t)(nib[0] | (nib[1] << 4) | (nib[2] << 8) | (nib[3] << 12));
  *reinterpret_cast<uint16_t*>(base + 2048 + off * 64 + lane * 2) = vb;
  if ((lane & 7) == 0) *reinterpret_cast<__half*>(base + 3104 + (off * 4 + (lane >> 3)) * 2) = vs;
}

// ------------------------------------------------------------------ ref
// D = 256, page 64, token-major regions, fp32 scales, affine V.
__global__ void store_ref_kernel(StoreArgs a) {
  pdl_trigger();
  pdl_wait();  // everything this kernel reads may come from the previous one
  constexpr int D = 256, PAGE = 64;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= a.T * a.hkv) return;
  const int t = gw / a.hkv;
  const int h = gw % a.hkv;
  const int64_t slot = a.slots[t];
  if (slot < 0 || slot >= a.num_pages * PAGE) return;
  const int64_t page = slot / PAGE;
  const int off = (int)(slot % PAGE);
  const int hkv = a.hkv;
  uint8_t* pg = a.cache + page * a.page_bytes;
  const int kbytes = PAGE * hkv * D, vbytes = PAGE * hkv * (D / 2), plane = PAGE * hkv * 4;
  const int cell = off * hkv + h;
  const int d0 = lane * 8;

  float x[8];
  const __nv_bfloat16* ks = a.k + (int64_t)t * a.k_stride_t + (int64_t)h * D + d0;
#pragma unroll
  for (int j = 0; j < 8; ++j) x[j] = __bfloat162float(ks[j]);
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(x[j]));
  amax = warp_max(amax);
  const float kscale = amax / 127.f;
  const float kinv = kscale > 0.f ? 1.f / kscale : 0.f;
  uint8_t kq[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) kq[j] = (uint8_t)(int8_t)(int)fminf(fmaxf(rint_f(__fmul_rn(x[j], kinv)), -127.f), 127.f);
  *reinterpret_cast<uint2*>(pg + (int64_t)cell * D + d0) = *reinterpret_cast<uint2*>(kq);
  if (lane == 0) *reinterpret_cast<float*>(pg + kbytes + vbytes + cell * 4) = kscale;

  float y[8];
  const __nv_bfloat16* vsrc = a.v + (int64_t)t * a.v_stride_t + (int64_t)h * D + d0;
#pragma unroll
  for (int j = 0; j < 8; ++j) y[j] = __bfloat162float(vsrc[j]);
  float lo = y[0], hi = y[0];
#pragma unroll
  for (int j = 1; j < 8; ++j) { lo = fminf(lo, y[j]); hi = fmaxf(hi, y[j]); }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
    hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, o));
  }
  const float vscale = fmaxf(__fsub_rn(hi, lo) / 15.f, 1.0e-8f);
  const float zero = fminf(fmaxf(floorf(__fadd_rn(-lo / vscale, 0.5f)), 0.f), 15.f);
  uint32_t packed = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float q = fminf(fmaxf(floorf(__fadd_rn(__fadd_rn(y[j] / vscale, zero), 0.5f)), 0.f), 15.f);
    packed |= ((uint32_t)q) << (4 * j);
  }
  *reinterpret_cast<uint32_t*>(pg + kbytes + (int64_t)cell * (D / 2) + lane * 4) = packed;
  if (lane == 0) {
    *reinterpret_cast<float*>(pg + kbytes + vbytes + plane + cell * 4) = vscale;
    *reinterpret_cast<float*>(pg + kbytes + vbytes + 2 * plane + cell * 4) = zero;
  }
}

}  // namespace kv
}  // namespace k8v4

using namespace k8v4;
using namespace k8v4::kv;

K8V4_STATUS_API(store)

// fmt 0 = ref, 1 = b200. Separate K/V rows.
extern "C" int k8v4_kv_store(int fmt, const void* k, int64_t k_stride_t, const void* v, int64_t v_stride_t,
                             const int64_t* slots, void* cache, int64_t num_pages, int page_bytes, int T, int hkv,
                             cudaStream_t st) {
  if (T <= 0) return 0;
  StoreArgs a{};
  a.k = reinterpret_cast<const __nv_bfloat16*>(k);
  a.v = reinterpret_cast<const __nv_bfloat16*>(v);
  a.k_stride_t = k_stride_t;
  a.v_stride_t = v_stride_t;
  a.slots = slots;
  a.cache = reinterpret_cast<uint8_t*>(cache);
  a.num_pages = num_pages;
  a.page_bytes = page_bytes;
  a.T = T;
  a.hkv = hkv;
  const int warps = T * hkv;
  const int blocks = cdiv(warps, 4);
  if (fmt == 0)
    launch_k(store_ref_kernel, dim3(blocks), dim3(128), 0, st, a);
  else
    launch_k(store_b200_kernel<false>, dim3(blocks), dim3(128), 0, st, a);
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}

// b200 format, fused: rotate q/k of the qkv rows, write q_out, store K/V.
// `qkv_fp32` = 1: qkv holds the qkv GEMM's fp32 split-K sums, which this
// call finishes (bf16 rounding) and leaves zeroed.
extern "C" int k8v4_rope_store(const void* qkv, int qkv_fp32, const float* cos_sin, const int64_t* positions,
                               void* q_out, const int64_t* slots, void* cache, int64_t num_pages, int page_bytes,
                               int T, int hq, int hkv, cudaStream_t st) {
  if (T <= 0) return 0;
  StoreArgs a{};
  if (qkv_fp32)
    a.qkv_f = reinterpret_cast<float*>(const_cast<void*>(qkv));
  else
    a.qkv = reinterpret_cast<const __nv_bfloat16*>(qkv);
  a.cos_sin = cos_sin;
  a.positions = positions;
  a.q_out = reinterpret_cast<__nv_bfloat16*>(q_out);
  a.slots = slots;
  a.cache = reinterpret_cast<uint8_t*>(cache);
  a.num_pages = num_pages;
  a.page_bytes = page_bytes;
  a.T = T;
  a.hkv = hkv;
  a.hq = hq;
  const int warps = T * (hq + hkv);
  launch_k(store_b200_kernel<true>, dim3(cdiv(warps, 4)), dim3(128), 0, st, a);
  return cudaGetLastError() == cudaSuccess ? 0 : 1;
}
