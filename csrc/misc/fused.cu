// Memory-bound fused elementwise kernels around the GEMMs:
//   * RMSNorm with optional residual add and optional per-token int8 output
//     (the activation quantization of the W4A8 path, reference
//     k8v4_v030/w4a8_prefill.py:192-203, fused into the norm that produces it)
//   * SiLU(gate) * up with optional per-token int8 output
//   * INT8 embedding lookup (codes x per-row fp16 scale, vocab-sharded;
//     reference k8v4_v030/embed_int8_runtime.py:53-56)
//   * split-K finish: fp32 partial sums -> bf16 (+ residual)
//   * per-token int8 quantization of bf16 rows
// One CTA per token row; 16-byte vector loads; fp32 math.
#include "../common.cuh"
#include "../comm/peer.cuh"

namespace k8v4 {
namespace misc {

constexpr int kThreads = 256;

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = (l < (int)(blockDim.x >> 5)) ? red[l] : 0.f;
  return warp_sum(t);
}
__device__ __forceinline__ float block_max(float v, float* red) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = (l < (int)(blockDim.x >> 5)) ? red[l] : 0.f;
  return warp_max(t);
}

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&f)[8]) {
  const uint4 raw = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 v = __bfloat1622float2(h[j]);
    f[2 * j] = v.x;
    f[2 * j + 1] = v.y;
  }
}
__device__ __forceinline__ void store8(__nv_bfloat16* p, const float (&f)[8]) {
  uint4 raw;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&raw);
#pragma unroll
  for (int j = 0; j < 4; ++j) h[j] = __floats2bfloat162_rn(f[2 * j], f[2 * j + 1]);
  *reinterpret_cast<uint4*>(p) = raw;
}

// Quantize the row held in registers (VPT vectors of 8 per thread) to int8
// with scale amax/127 (clamped to >= 1e-5 like the reference), write codes
// and the fp32 scale.
template <int VPT>
__device__ __forceinline__ void quant_row(const float (&v)[VPT][8], int n, int8_t* q, float* scale, float* red) {
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = (threadIdx.x + i * kThreads) * 8;
    if (c < n)
#pragma unroll
      for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(v[i][j]));
  }
  amax = block_max(amax, red);
  const float s = fmaxf(amax / 127.f, 1e-5f);
  const float inv = 1.f / s;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = (threadIdx.x + i * kThreads) * 8;
    if (c < n) {
      uint32_t w[2] = {0, 0};
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int qi = (int)fminf(fmaxf(rintf(v[i][j] * inv), -127.f), 127.f);
        w[j >> 2] |= ((uint32_t)(uint8_t)(int8_t)qi) << (8 * (j & 3));
      }
      *reinterpret_cast<uint2*>(q + c) = make_uint2(w[0], w[1]);
    }
  }
  if (threadIdx.x == 0) *scale = s;
}

// x: [T, n] bf16. If residual != nullptr: h = x + residual, residual <- h.
// y = h * rsqrt(mean(h^2) + eps) * w. Outputs bf16 y (row stride ldy, so two
// norms can write the halves of one concatenated row) and/or int8 y + scale.
template <int VPT>
// x may instead arrive as fp32 split-K partial sums `xf` (the finishing step
// of a split-K GEMM fused into this norm); xf is zeroed after it is read so
// the shared accumulator is clean for the next split-K GEMM.
//
// Tensor parallel: xf may be this rank's copy of a symmetric buffer that a
// GEMM -> all-reduce fills through its multicast address. Then `sync` is
// given: the CTAs first wait until the counter `sync.flag` reaches
// sync.state[0] + sync.expected (all ranks' GEMM CTAs have signalled), and the
// last CTA to finish advances sync.state[0] by `expected` (a running count, so
// a replayed CUDA graph needs no reset and calls may differ in size).
__global__ void __launch_bounds__(kThreads) rmsnorm_kernel(const __nv_bfloat16* __restrict__ x, float* xf,
                                                           __nv_bfloat16* residual, const __nv_bfloat16* __restrict__ w,
                                                           __nv_bfloat16* y, int8_t* yq, float* yscale, int n,
                                                           int64_t ldy, float eps, peer::ReduceSync sync) {
  pdl_trigger();
  // the norm weights come from no earlier kernel: load them before waiting
  uint4 gw[VPT];
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = (threadIdx.x + i * kThreads) * 8;
    gw[i] = c < n ? *reinterpret_cast<const uint4*>(w + c) : make_uint4(0u, 0u, 0u, 0u);
  }
  pdl_wait();  // x / xf / residual may come from the previous kernel
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  if (sync.flag) peer::sync_wait(sync, 201);
  float v[VPT][8];
  float rs[VPT][8];
  float ss = 0.f;
  // every load first: the zeroing and residual stores below would otherwise
  // order each later load behind them (the pointers may alias)
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = (threadIdx.x + i * kThreads) * 8;
    if (c < n) {
      if (xf) {
        const float4* p4 = reinterpret_cast<const float4*>(xf + row * n + c);
        const float4 a = p4[0], b = p4[1];
        v[i][0] = a.x; v[i][1] = a.y; v[i][2] = a.z; v[i][3] = a.w;
        v[i][4] = b.x; v[i][5] = b.y; v[i][6] = b.z; v[i][7] = b.w;
      } else {
        load8(x + row * n + c, v[i]);
      }
      if (residual) load8(residual + row * n + c, rs[i]);
    }
  }
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = (threadIdx.x + i * kThreads) * 8;
    if (c < n) {
      if (xf) {
        float4* p4 = reinterpret_cast<float4*>(xf + row * n + c);
        p4[0] = make_float4(0.f, 0.f, 0.f, 0.f);
        p4[1] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
      if (residual) {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] += rs[i][j];
        // the residual stream is kept in bf16
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] = __bfloat162float(__float2bfloat16_rn(v[i][j]));
        store8(residual + row * n + c, v[i]);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[i][j] * v[i][j];
    }
  }
  ss = block_sum(ss, red);
  const float inv = rsqrtf(ss / (float)n + eps);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = (threadIdx.x + i * kThreads) * 8;
    if (c < n) {
      const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&gw[i]);
      float g[8];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(g2[j]);
        g[2 * j] = f.x;
        g[2 * j + 1] = f.y;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) v[i][j] = __bfloat162float(__float2bfloat16_rn(v[i][j] * inv)) * g[j];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[i][j] = __bfloat162float(__float2bfloat16_rn(v[i][j]));
      if (y) store8(y + row * ldy + c, v[i]);
    }
  }
  if (yq) quant_row<VPT>(v, n, yq + row * n, yscale + row, red);
  if (sync.flag) peer::sync_done(sync);
}

// ------------------------------------------------------------ cluster norm
// The same norm for a few decode rows (no int8 output, no all-reduce wait):
// one thread-block cluster of kNormCluster CTAs per row, each CTA owning
// n / kNormCluster columns (one 8-wide vector per thread). The CTAs' partial
// sums of squares meet through distributed shared memory (each CTA reads the
// others' partials in CTA-rank order, so every CTA forms the same sum); a
// single CTA per row spent ~5 us on 5,120 columns, most of it latency.
constexpr int kNormCluster = 8;
constexpr int kNormThreads = 128;

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__global__ void __launch_bounds__(kNormThreads) rmsnorm_cluster_kernel(const __nv_bfloat16* __restrict__ x, float* xf,
                                                                       __nv_bfloat16* residual,
                                                                       const __nv_bfloat16* __restrict__ w,
                                                                       __nv_bfloat16* y, int n, int64_t ldy,
                                                                       float eps) {
  pdl_trigger();
  __shared__ float red[kNormThreads / 32];
  __shared__ float part;
  const int64_t row = blockIdx.y;
  const int per = n / kNormCluster;                 // columns of this CTA (a multiple of 8)
  const int c = blockIdx.x * per + threadIdx.x * 8;  // blockIdx.x is the CTA's rank in the cluster
  const bool mine = threadIdx.x * 8 < per;
  // the norm weights come from no earlier kernel: load them before waiting
  const uint4 gw = mine ? *reinterpret_cast<const uint4*>(w + c) : make_uint4(0u, 0u, 0u, 0u);
  pdl_wait();  // x / xf / residual may come from the previous kernel
  float v[8];
  float ss = 0.f;
  if (mine) {
    if (xf) {
      float4* p4 = reinterpret_cast<float4*>(xf + row * n + c);
      const float4 a = p4[0], b = p4[1];
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
      v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
      p4[0] = make_float4(0.f, 0.f, 0.f, 0.f);  // the shared split-K accumulator stays clean
      p4[1] = make_float4(0.f, 0.f, 0.f, 0.f);
    } else {
      load8(x + row * n + c, v);
    }
    if (residual) {
      float rs[8];
      load8(residual + row * n + c, rs);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = __bfloat162float(__float2bfloat16_rn(v[j] + rs[j]));
      store8(residual + row * n + c, v);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) ss += v[j] * v[j];
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < kNormThreads / 32; ++i) t += red[i];
    part = t;
  }
  cluster_sync_all();  // every CTA's partial is written
  float total = 0.f;
  {
    const uint32_t local = static_cast<uint32_t>(__cvta_generic_to_shared(&part));
#pragma unroll
    for (int r = 0; r < kNormCluster; ++r) {
      uint32_t remote;
      float pv;
      asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local), "r"(r));
      asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(pv) : "r"(remote) : "memory");
      total += pv;
    }
  }
  const float inv = rsqrtf(total / (float)n + eps);
  if (mine) {
    const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&gw);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 g = __bfloat1622float2(g2[j]);
      v[2 * j] = __bfloat162float(__float2bfloat16_rn(__bfloat162float(__float2bfloat16_rn(v[2 * j] * inv)) * g.x));
      v[2 * j + 1] =
          __bfloat162float(__float2bfloat16_rn(__bfloat162float(__float2bfloat16_rn(v[2 * j + 1] * inv)) * g.y));
    }
    store8(y + row * ldy + c, v);
  }
  cluster_sync_all();  // no CTA leaves while another still reads its partial
}

// gu: [T, 2I] = [gate | up]. out = silu(gate) * up (bf16 and/or int8 + scale).
template <int VPT>
__global__ void __launch_bounds__(kThreads) silu_mul_kernel(const __nv_bfloat16* __restrict__ gu, __nv_bfloat16* y,
                                                            int8_t* yq, float* yscale, int inter) {
  pdl_trigger();
  pdl_wait();  // everything this kernel reads may come from the previous one
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  float v[VPT][8];
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = (threadIdx.x + i * kThreads) * 8;
    if (c < inter) {
      float g[8], u[8];
      load8(gu + row * 2 * inter + c, g);
      load8(gu + row * 2 * inter + inter + c, u);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float s = g[j] / (1.f + __expf(-g[j]));
        v[i][j] = __bfloat162float(__float2bfloat16_rn(s * u[j]));
      }
      if (y) store8(y + row * inter + c, v[i]);
    }
  }
  if (yq) quant_row<VPT>(v, inter, yq + row * inter, yscale + row, red);
}

// bf16-only SiLU(gate)*up spread over the whole grid (one 8-wide vector per
// thread), for the few-token decode rows where one CTA per row is too serial.
__global__ void __launch_bounds__(256) silu_mul_wide_kernel(const __nv_bfloat16* __restrict__ gu,
                                                            __nv_bfloat16* __restrict__ y, int inter, int64_t total) {
  pdl_trigger();
  pdl_wait();  // everything this kernel reads may come from the previous one
  const int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (v >= total) return;
  const int per_row = inter / 8;
  const int64_t row = v / per_row;
  const int c = (int)(v % per_row) * 8;
  float g[8], u[8], o[8];
  load8(gu + row * 2 * inter + c, g);
  load8(gu + row * 2 * inter + inter + c, u);
#pragma unroll
  for (int j = 0; j < 8; ++j) o[j] = g[j] / (1.f + __expf(-g[j])) * u[j];
  store8(y + row * inter + c, o);
}

// The same from the gate/up projection's fp32 sums (a decode GEMV or split-K
// accumulator, [T, 2I]): each sum is rounded to bf16 first, as the GEMM's own
// bf16 output would be, and the accumulator is zeroed behind the read for
// the next GEMM.
__global__ void __launch_bounds__(256) silu_mul_f32_wide_kernel(float* __restrict__ gu, __nv_bfloat16* __restrict__ y,
                                                                int inter, int64_t total) {
  pdl_trigger();
  pdl_wait();  // the sums come from the previous kernel
  const int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (v >= total) return;
  const int per_row = inter / 8;
  const int64_t row = v / per_row;
  const int c = (int)(v % per_row) * 8;
  float4* gp = reinterpret_cast<float4*>(gu + row * 2 * inter + c);
  float4* up = reinterpret_cast<float4*>(gu + row * 2 * inter + inter + c);
  const float4 g0 = gp[0], g1 = gp[1], u0 = up[0], u1 = up[1];
  const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
  gp[0] = z;
  gp[1] = z;
  up[0] = z;
  up[1] = z;
  const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
  const float u[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
  float o[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float gb = __bfloat162float(__float2bfloat16_rn(g[j]));
    const float ub = __bfloat162float(__float2bfloat16_rn(u[j]));
    o[j] = gb / (1.f + __expf(-gb)) * ub;
  }
  store8(y + row * inter + c, o);
}

// Row-wise int8 quantization of bf16 rows.
template <int VPT>
__global__ void __launch_bounds__(kThreads) quant_rows_kernel(const __nv_bfloat16* __restrict__ x, int8_t* q, float* scale,
                                                              int n) {
  pdl_trigger();
  pdl_wait();  // everything this kernel reads may come from the previous one
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  float v[VPT][8];
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = (threadIdx.x + i * kThreads) * 8;
    if (c < n) load8(x + row * n + c, v[i]);
  }
  quant_row<VPT>(v, n, q + row * n, scale + row, red);
}

// out[t] = codes[id - start] * scale[id - start] for ids inside [start, start + rows), else 0.
__global__ void embed_int8_kernel(const int64_t* __restrict__ ids, const int8_t* __restrict__ codes,
                                  const __half* __restrict__ scales, __nv_bfloat16* out, int n, int64_t start,
                                  int64_t rows) {
  pdl_trigger();
  pdl_wait();  // everything this kernel reads may come from the previous one
  const int64_t t = blockIdx.x;
  const int64_t id = ids[t] - start;
  const bool in = id >= 0 && id < rows;
  const float s = in ? __half2float(scales[id]) : 0.f;
  for (int c = threadIdx.x * 8; c < n; c += blockDim.x * 8) {
    float f[8];
    if (in) {
      const uint2 raw = *reinterpret_cast<const uint2*>(codes + id * n + c);
      const int8_t* b = reinterpret_cast<const int8_t*>(&raw);
      // bf16 product of the two bf16-rounded factors, like F.embedding(..).to(bf16) * scale.to(bf16)
      const float sb = __bfloat162float(__float2bfloat16_rn(s));
#pragma unroll
      for (int j = 0; j < 8; ++j) f[j] = (float)b[j] * sb;
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) f[j] = 0.f;
    }
    store8(out + t * n + c, f);
  }
}

// out = bf16(ws (+ residual)); optionally zero ws for the next accumulation.
__global__ void splitk_finish_kernel(float* ws, const __nv_bfloat16* residual, __nv_bfloat16* out, int64_t total,
                                     int zero_ws) {
  pdl_trigger();
  pdl_wait();  // everything this kernel reads may come from the previous one
  const int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (i >= total) return;
  float4 a = *reinterpret_cast<float4*>(ws + i);
  if (residual) {
    const uint2 raw = *reinterpret_cast<const uint2*>(residual + i);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
    const float2 r0 = __bfloat1622float2(h[0]), r1 = __bfloat1622float2(h[1]);
    a.x += r0.x; a.y += r0.y; a.z += r1.x; a.w += r1.y;
  }
  __nv_bfloat162 o0 = __floats2bfloat162_rn(a.x, a.y), o1 = __floats2bfloat162_rn(a.z, a.w);
  uint2 w;
  w.x = *reinterpret_cast<uint32_t*>(&o0);
  w.y = *reinterpret_cast<uint32_t*>(&o1);
  *reinterpret_cast<uint2*>(out + i) = w;
  if (zero_ws) *reinterpret_cast<float4*>(ws + i) = make_float4(0.f, 0.f, 0.f, 0.f);
}

// INT8 island weights: out[n, k] = q[n, k] * scale[n] in bf16 (8 values a thread).
__global__ void __launch_bounds__(256) int8_dequant_kernel(const int8_t* __restrict__ q,
                                                          const __nv_bfloat16* __restrict__ scale,
                                                          __nv_bfloat16* __restrict__ out, int K, int64_t total8) {
  pdl_trigger();
  pdl_wait();  // the scratch it overwrites may still be read by the previous kernel
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total8) return;
  const int64_t e = i * 8;
  const float s = __bfloat162float(scale[e / K]);
  const uint2 raw = *reinterpret_cast<const uint2*>(q + e);
  const int8_t* b = reinterpret_cast<const int8_t*>(&raw);
  float f[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) f[j] = (float)b[j] * s;
  store8(out + e, f);
}

}  // namespace misc
}  // namespace k8v4

using namespace k8v4;
using namespace k8v4::misc;

K8V4_STATUS_API(misc)


// ------------------------------------------------------------ sequence parallel
// Norm of this rank's rows between a GEMM -> reduce-scatter and an
// all-gather -> GEMM (tensor-parallel prefill, see wq_gemm.cu). One CTA per
// local row r:
//   v = sum over the `world` slots of row r (bf16 partial rows that every
//       rank's reduce-scatter GEMM stored here; waited for until rs_flag >=
//       rs_target), or row r of x_local (bf16) when slots is null;
//   residual[r] <- bf16(v + residual[r]) (or bf16(v) with init_residual);
//   y = bf16(bf16(residual[r] * rsqrt(mean(residual[r]^2) + eps)) * w)
// then y (bf16) or its int8 quantization (per-row amax / 127) goes out:
// through the multicast address of the all-gather buffer at global row
// row0 + r (every rank's copy, `mc` set), followed by +1 on the multicast row
// counter ag_sig_mc; or to a local buffer at row r.
__device__ __forceinline__ void mc_st_v4(void* mc, uint4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.bf16x2 [%0], {%1,%2,%3,%4};" ::"l"(mc), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ void mc_st_b64(void* mc, uint2 v) {
  const unsigned long long b = ((unsigned long long)v.y << 32) | v.x;
  asm volatile("multimem.st.relaxed.sys.global.b64 [%0], %1;" ::"l"(mc), "l"(b) : "memory");
}

template <int VPT>
__global__ void __launch_bounds__(kThreads) rmsnorm_sp_kernel(
    const __nv_bfloat16* slots, int world, int64_t slot_stride, const __nv_bfloat16* x_local,
    __nv_bfloat16* residual, int init_residual, const __nv_bfloat16* __restrict__ w, int n, float eps,
    const unsigned long long* rs_flag, unsigned long long rs_target, __nv_bfloat16* y, int8_t* yq, float* ys,
    int64_t row0, int mc, unsigned long long* ag_sig_mc) {
  pdl_trigger();
  uint4 gw[VPT];
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = (threadIdx.x + i * kThreads) * 8;
    gw[i] = c < n ? *reinterpret_cast<const uint4*>(w + c) : make_uint4(0u, 0u, 0u, 0u);
  }
  pdl_wait();
  __shared__ float red[32];
  const int64_t r = blockIdx.x;
  if (slots && rs_flag) {
    if (threadIdx.x == 0) peer::wait_geq_u64(rs_flag, rs_target, 202);
    __syncthreads();
  }
  float v[VPT][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = (threadIdx.x + i * kThreads) * 8;
    if (c < n) {
      if (slots) {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] = 0.f;
        for (int src = 0; src < world; ++src) {
          float f[8];
          load8(slots + src * slot_stride + r * n + c, f);
#pragma unroll
          for (int j = 0; j < 8; ++j) v[i][j] += f[j];
        }
      } else {
        load8(x_local + r * n + c, v[i]);
      }
      if (!init_residual) {
        float rs[8];
        load8(residual + r * n + c, rs);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] += rs[j];
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) v[i][j] = __bfloat162float(__float2bfloat16_rn(v[i][j]));
      store8(residual + r * n + c, v[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[i][j] * v[i][j];
    }
  }
  ss = block_sum(ss, red);
  const float inv = rsqrtf(ss / (float)n + eps);
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = (threadIdx.x + i * kThreads) * 8;
    if (c < n) {
      const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&gw[i]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 g = __bfloat1622float2(g2[j]);
        v[i][2 * j] = __bfloat162float(__float2bfloat16_rn(__bfloat162float(__float2bfloat16_rn(v[i][2 * j] * inv)) * g.x));
        v[i][2 * j + 1] =
            __bfloat162float(__float2bfloat16_rn(__bfloat162float(__float2bfloat16_rn(v[i][2 * j + 1] * inv)) * g.y));
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(v[i][j]));
    }
  }
  const int64_t orow = mc ? row0 + r : r;
  if (yq) {
    amax = block_max(amax, red);
    const float sc = fmaxf(amax / 127.f, 1e-5f);
    const float qi = 1.f / sc;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int c = (threadIdx.x + i * kThreads) * 8;
      if (c < n) {
        uint32_t wq[2] = {0, 0};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int q = (int)fminf(fmaxf(rintf(v[i][j] * qi), -127.f), 127.f);
          wq[j >> 2] |= ((uint32_t)(uint8_t)(int8_t)q) << (8 * (j & 3));
        }
        int8_t* dst = yq + orow * n + c;
        if (mc) mc_st_b64(dst, make_uint2(wq[0], wq[1]));
        else *reinterpret_cast<uint2*>(dst) = make_uint2(wq[0], wq[1]);
      }
    }
    if (threadIdx.x == 0) {
      if (mc) peer::mc_st_f32(ys + orow, sc);
      else ys[orow] = sc;
    }
  } else {
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int c = (threadIdx.x + i * kThreads) * 8;
      if (c < n) {
        if (mc) {
          uint4 raw;
          __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&raw);
#pragma unroll
          for (int j = 0; j < 4; ++j) h[j] = __floats2bfloat162_rn(v[i][2 * j], v[i][2 * j + 1]);
          mc_st_v4(y + orow * n + c, raw);
        } else {
          store8(y + orow * n + c, v[i]);
        }
      }
    }
  }
  if (mc && ag_sig_mc) {
    __syncthreads();
    if (threadIdx.x == 0) {
      peer::fence_proxy_alias();
      peer::fence_sys();
      peer::mc_signal_add_u64(ag_sig_mc, 1ull);
    }
  }
}

#define K8V4_VPT_DISPATCH(n, KERNEL, ...)                                         \
  do {                                                                            \
    const int vpt_ = cdiv(cdiv((n), 8), kThreads);                                \
    if (vpt_ <= 1) launch_k(KERNEL<1>, dim3(rows), dim3(kThreads), 0, st, __VA_ARGS__);             \
    else if (vpt_ <= 2) launch_k(KERNEL<2>, dim3(rows), dim3(kThreads), 0, st, __VA_ARGS__);        \
    else if (vpt_ <= 4) launch_k(KERNEL<4>, dim3(rows), dim3(kThreads), 0, st, __VA_ARGS__);        \
    else if (vpt_ <= 9) launch_k(KERNEL<9>, dim3(rows), dim3(kThreads), 0, st, __VA_ARGS__);        \
    else return 2;                                                                \
  } while (0)

// A few decode rows without int8 output or all-reduce wait run on a cluster
// per row (rmsnorm_cluster_kernel) unless K8V4_NORM_CLUSTER=0.
static bool norm_cluster_enabled() {
  static const bool on = [] {
    const char* v = getenv("K8V4_NORM_CLUSTER");
    return !(v && (v[0] == '0' || v[0] == 'n' || v[0] == 'N' || v[0] == 'f' || v[0] == 'F'));
  }();
  return on;
}

extern "C" int k8v4_rmsnorm(const void* x, float* xf, void* residual, const void* w, void* y, int64_t ldy, void* yq,
                            float* yscale, int rows, int n, float eps, const unsigned long long* sync_flag,
                            unsigned long long* sync_state, unsigned long long sync_expected, cudaStream_t st) {
  if (rows <= 0) return 0;
  if (n % 8 || ldy < n || ldy % 8) return 1;
  if (sync_flag && (!xf || !sync_state)) return 4;
  if (rows <= 4 && !yq && y && !sync_flag && n % (8 * kNormCluster) == 0 && n / kNormCluster <= 8 * kNormThreads &&
      norm_cluster_enabled()) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kNormCluster, rows);
    cfg.blockDim = dim3(kNormThreads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kNormCluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, rmsnorm_cluster_kernel, reinterpret_cast<const __nv_bfloat16*>(x),
                                             xf, reinterpret_cast<__nv_bfloat16*>(residual),
                                             reinterpret_cast<const __nv_bfloat16*>(w),
                                             reinterpret_cast<__nv_bfloat16*>(y), n, ldy, eps);
    return e == cudaSuccess ? 0 : 3;
  }
  peer::ReduceSync sync{sync_flag, sync_state, sync_expected};
  K8V4_VPT_DISPATCH(n, rmsnorm_kernel, reinterpret_cast<const __nv_bfloat16*>(x), xf,
                    reinterpret_cast<__nv_bfloat16*>(residual), reinterpret_cast<const __nv_bfloat16*>(w),
                    reinterpret_cast<__nv_bfloat16*>(y), reinterpret_cast<int8_t*>(yq), yscale, n, ldy, eps, sync);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

// Sequence-parallel norm of `rows` local rows (see rmsnorm_sp_kernel).
extern "C" int k8v4_rmsnorm_sp(const void* slots, int world, int64_t slot_stride, const void* x_local,
                               void* residual, int init_residual, const void* w, int rows, int n, float eps,
                               const unsigned long long* rs_flag, unsigned long long rs_target, void* y, void* yq,
                               float* ys, int64_t row0, int mc, unsigned long long* ag_sig_mc, cudaStream_t st) {
  if (rows <= 0) return 0;
  if (n % 8) return 1;
  if (!slots && !x_local) return 4;
  if (!y && !yq) return 4;
  if (yq && !ys) return 4;
  if (mc && (!ag_sig_mc || (y && reinterpret_cast<uintptr_t>(y) % 16) || (yq && reinterpret_cast<uintptr_t>(yq) % 8)))
    return 4;
  K8V4_VPT_DISPATCH(n, rmsnorm_sp_kernel, reinterpret_cast<const __nv_bfloat16*>(slots), world, slot_stride,
                    reinterpret_cast<const __nv_bfloat16*>(x_local), reinterpret_cast<__nv_bfloat16*>(residual),
                    init_residual, reinterpret_cast<const __nv_bfloat16*>(w), n, eps, rs_flag, rs_target,
                    reinterpret_cast<__nv_bfloat16*>(y), reinterpret_cast<int8_t*>(yq), ys, row0, mc, ag_sig_mc);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

extern "C" int k8v4_silu_mul(const void* gu, void* y, void* yq, float* yscale, int rows, int inter,
                             cudaStream_t st) {
  if (rows <= 0) return 0;
  if (inter % 8) return 1;
  if (!yq && y && rows <= 16) {
    const int64_t total = (int64_t)rows * (inter / 8);
    launch_k(silu_mul_wide_kernel, dim3((unsigned)((total + 255) / 256)), dim3(256), 0, st,
        reinterpret_cast<const __nv_bfloat16*>(gu), reinterpret_cast<__nv_bfloat16*>(y), inter, total);
    return cudaGetLastError() == cudaSuccess ? 0 : 3;
  }
  K8V4_VPT_DISPATCH(inter, silu_mul_kernel, reinterpret_cast<const __nv_bfloat16*>(gu),
                    reinterpret_cast<__nv_bfloat16*>(y), reinterpret_cast<int8_t*>(yq), yscale, inter);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

// y = silu(gate) * up from fp32 sums [rows, 2 inter] that are zeroed after reading.
extern "C" int k8v4_silu_mul_f32(float* gu, void* y, int rows, int inter, cudaStream_t st) {
  if (rows <= 0) return 0;
  if (inter % 8) return 1;
  const int64_t total = (int64_t)rows * (inter / 8);
  launch_k(silu_mul_f32_wide_kernel, dim3((unsigned)((total + 255) / 256)), dim3(256), 0, st, gu,
           reinterpret_cast<__nv_bfloat16*>(y), inter, total);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

extern "C" int k8v4_quant_rows(const void* x, void* q, float* scale, int rows, int n, cudaStream_t st) {
  if (rows <= 0) return 0;
  if (n % 8) return 1;
  K8V4_VPT_DISPATCH(n, quant_rows_kernel, reinterpret_cast<const __nv_bfloat16*>(x), reinterpret_cast<int8_t*>(q),
                    scale, n);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

extern "C" int k8v4_embed_int8(const int64_t* ids, const void* codes, const void* scales, void* out, int T, int n,
                               int64_t start, int64_t rows, cudaStream_t st) {
  if (T <= 0) return 0;
  if (n % 8) return 1;
  launch_k(embed_int8_kernel, dim3(T), dim3(128), 0, st, ids, reinterpret_cast<const int8_t*>(codes),
                                       reinterpret_cast<const __half*>(scales), reinterpret_cast<__nv_bfloat16*>(out),
                                       n, start, rows);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

extern "C" int k8v4_splitk_finish(float* ws, const void* residual, void* out, int64_t total, int zero_ws,
                                  cudaStream_t st) {
  if (total <= 0) return 0;
  if (total % 4) return 1;
  const int64_t threads = total / 4;
  launch_k(splitk_finish_kernel, dim3((unsigned)((threads + 255) / 256)), dim3(256), 0, st,
      ws, reinterpret_cast<const __nv_bfloat16*>(residual), reinterpret_cast<__nv_bfloat16*>(out), total, zero_ws);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

// q [N, K] int8 with per-row bf16 scales -> bf16 [N, K]; K % 8 == 0.
extern "C" int k8v4_int8_dequant(const void* q, const void* scale, void* out, int N, int K, cudaStream_t st) {
  if (N <= 0 || K <= 0) return 0;
  if (K % 8) return 1;
  const int64_t total8 = (int64_t)N * K / 8;
  return launch_k(int8_dequant_kernel, dim3((unsigned)((total8 + 255) / 256)), dim3(256), 0, st,
                  reinterpret_cast<const int8_t*>(q), reinterpret_cast<const __nv_bfloat16*>(scale),
                  reinterpret_cast<__nv_bfloat16*>(out), K, total8) == cudaSuccess
             ? 0
             : 3;
}
