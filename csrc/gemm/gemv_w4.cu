// Decode GEMV for GPTQ int4 weights at 1 to 4 token rows (W4A16 numerics;
// the dispatch sends single-row calls here, see k8v4_gemv_w4_max_rows):
//   ws[t, n] += sum_k x[t, k] * scale[k / 128, n] * (q[k, n] - 8)
//
// At a handful of token rows a decode projection is a stream of int4 weights
// with about one multiply-add per weight byte and token: HBM bound. The
// tcgen05 path (wq_gemm.cu) needs every weight converted into the MMA operand
// format first, and at 1 token row its converter / MMA / accumulator pipeline
// moves ~8 KB of weights per CTA every ~0.4 us, about 0.3 of HBM. This kernel
// streams the weights once through registers instead and does the products on
// the integer pipe. (Two other forms measured slower at one row: packed fp16
// FMAs on the unpacked codes, 34.9 us for the gate/up shape, being
// instruction bound; the same fed by a 32-stage TMA ring with 12 compute
// warps, 43.0 us.)
//
//   * work unit = 128 output features x 64 k (8 packed rows of the GPTQ
//     [K/8, N] int32 layout); a lane owns 4 features and loads one 16-byte
//     vector per packed row. Units are numbered k-fastest within a feature
//     tile, and every warp of the persistent grid takes an equal contiguous
//     run of them (no wave tail; at most one unit of imbalance).
//   * the activations of the unit's 64 k are quantized by the warp itself to
//     two int8 limbs, x ~= s (128 hi + lo) with |128 hi + lo| <= 16319
//     (15 bits, s = amax / 16319 over the 64 values), so no preparation
//     kernel runs; the limbs go through 512 bytes of shared memory per warp
//     into the byte order the unpacked codes need.
//   * codes are unpacked to u8 (q + 8) with two AND and one shift per 8
//     codes; dp4a.u32.s32 multiplies 4 codes by 4 limb bytes and accumulates
//     in int32, exact. 128 D_hi + D_lo - 8 C (C = the limbs' sum over the
//     unit) is sum (q - 8) X exactly (|.| < 2^24), then fp32: times s and the
//     group scale, accumulated per lane.
//   * when a warp's run leaves a feature tile it adds its fp32 sums into ws
//     (red.global.add), the split-K accumulator protocol of wq_gemm.cu: ws is
//     zero on entry and the consumer (the fused RMSNorm, the RoPE / cache
//     store kernel or splitk_finish) reads and re-zeroes it.
//   * GEMM -> all-reduce (tensor parallel o_proj / down_proj), in two
//     phases: the warps' sums first meet in a local fp32 accumulator
//     (`ws`, L2 atomics); the CTA that finishes last (a ticket counter) then
//     reads the reduced rows once and sends them with 16-byte multimem.red
//     to the multicast address of the symmetric buffer `ws_mc` (the NVSwitch
//     sums every rank's rows into every rank's copy), re-zeroes the local
//     accumulator and the ticket, and adds 1 to the multicast counter
//     `flag_mc` with release semantics; the consuming RMSNorm waits for
//     `world` signals. Measured at TP2 (27B, 128K, c = 1): 161.9 tok/s,
//     against 172.2 for this GEMV followed by an NCCL all-reduce, so the
//     engine keeps one-row calls on NCCL unless K8V4_TP_GEMV_FUSED=1.
//     (Sending every warp's partial straight through the switch, ~60 per
//     output element, measured 110 tok/s; one send per 128-feature tile by
//     the warp that completes it, 142 tok/s.)
//
// Weights are streamed with no-allocate L1 loads; the first unit's loads go
// out before the grid waits for its predecessor (programmatic launch), the
// next unit's loads before the current unit's math.
#include "../comm/peer.cuh"

namespace k8v4 {
namespace gemv {

constexpr int kWarps = 8;           // warps per CTA
constexpr int kRows = 8;            // packed k-rows (8 codes each) per unit: 64 k
constexpr float kLimbMax = 16319.f; // |128 hi + lo| bound of the two-limb split

__device__ __forceinline__ uint4 ld_stream(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// d = c + sum_i a.u8[i] * b.s8[i]
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// CTAs per SM: two at 1-2 token rows (128 registers a thread), one above
// (the wider accumulators need more registers than half the file allows).
template <int M>
constexpr int ctas_per_sm() { return M <= 2 ? 2 : 1; }

template <int M>
__global__ void __launch_bounds__(kWarps * 32, ctas_per_sm<M>())
    gemv_w4_kernel(const uint32_t* __restrict__ qw, const __half* __restrict__ wscale,
                   const __nv_bfloat16* __restrict__ x, float* ws, int N, int K, int ldx, int ldo, int units,
                   float* ws_mc, unsigned long long* flag_mc, unsigned int* ticket) {
  pdl_trigger();
  // per warp and token row: for each packed row j of the unit the four limb
  // words {even k hi, odd k hi, even k lo, odd k lo}
  __shared__ __align__(16) uint32_t lsm[kWarps][M][kRows][4];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long nw = (long long)gridDim.x * kWarps;
  const long long gw = (long long)blockIdx.x * kWarps + warp;
  int u = (int)(gw * units / nw);
  const int uend = (int)((gw + 1) * units / nw);
  const int kunits = K / (8 * kRows);
  const size_t row_vec = (size_t)N / 4;  // uint4 vectors per packed row

  uint4 cur[kRows];
  auto load_unit = [&](int uu, uint4 (&dst)[kRows]) {
    const int tile = uu / kunits, ku = uu - tile * kunits;
    const uint4* base = reinterpret_cast<const uint4*>(qw) + (size_t)(ku * kRows) * row_vec + tile * 32 + lane;
#pragma unroll
    for (int j = 0; j < kRows; ++j) dst[j] = ld_stream(base + j * row_vec);
  };
  if (u < uend) load_unit(u, cur);
  pdl_wait();  // x comes from the previous kernel, which also re-zeroed ws

  int tile = -1;
  float facc[M][4];
  auto flush = [&]() {
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
      for (int f = 0; f < 4; ++f) {
        atomicAdd(ws + (size_t)m * ldo + tile * 128 + lane * 4 + f, facc[m][f]);
      }
  };
  uint8_t* lbytes = reinterpret_cast<uint8_t*>(&lsm[warp][0][0][0]);
  while (u < uend) {
    const int t = u / kunits, ku = u - t * kunits;
    if (t != tile) {
      if (tile >= 0) flush();
      tile = t;
#pragma unroll
      for (int m = 0; m < M; ++m)
#pragma unroll
        for (int f = 0; f < 4; ++f) facc[m][f] = 0.f;
    }
    uint4 nxt[kRows];
    const bool more = u + 1 < uend;
    if (more) load_unit(u + 1, nxt);
    const int k0 = ku * 8 * kRows;
    // ---- the warp's own limbs of the unit's 64 activations per token row.
    // Lane l holds k0 + 2l and k0 + 2l + 1: packed row j = l / 4, byte l % 4
    // of the even-k word (codes 0, 2, 4, 6 after the unpack) and of the odd one.
    float s[M];
    int csum[M];
#pragma unroll
    for (int m = 0; m < M; ++m) {
      const __nv_bfloat162 xv = *reinterpret_cast<const __nv_bfloat162*>(x + (size_t)m * ldx + k0 + 2 * lane);
      const float2 xf = __bfloat1622float2(xv);
      const float am = warp_max(fmaxf(fabsf(xf.x), fabsf(xf.y)));
      const float sc = am > 0.f ? am / kLimbMax : 1.f;
      const float inv = 1.f / sc;
      const int X0 = (int)fminf(fmaxf(rintf(xf.x * inv), -kLimbMax), kLimbMax);
      const int X1 = (int)fminf(fmaxf(rintf(xf.y * inv), -kLimbMax), kLimbMax);
      const int h0 = (X0 + 64) >> 7, h1 = (X1 + 64) >> 7;  // floor: hi in [-127, 127], lo in [-64, 63]
      uint8_t* rb = lbytes + ((m * kRows + (lane >> 2)) * 16) + (lane & 3);
      rb[0] = (uint8_t)(int8_t)h0;
      rb[4] = (uint8_t)(int8_t)h1;
      rb[8] = (uint8_t)(int8_t)(X0 - 128 * h0);
      rb[12] = (uint8_t)(int8_t)(X1 - 128 * h1);
      csum[m] = warp_sum_i(X0 + X1);
      s[m] = sc;
    }
    __syncwarp();
    int ah[M][4], al[M][4];
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
      for (int f = 0; f < 4; ++f) ah[m][f] = al[m][f] = 0;
#pragma unroll
    for (int j = 0; j < kRows; ++j) {
      uint4 lw[M];
#pragma unroll
      for (int m = 0; m < M; ++m) lw[m] = *reinterpret_cast<const uint4*>(&lsm[warp][m][j][0]);
      const uint32_t wv[4] = {cur[j].x, cur[j].y, cur[j].z, cur[j].w};
#pragma unroll
      for (int f = 0; f < 4; ++f) {
        const uint32_t ev = wv[f] & 0x0F0F0F0Fu;         // codes of k 0, 2, 4, 6 (+8)
        const uint32_t od = (wv[f] >> 4) & 0x0F0F0F0Fu;  // codes of k 1, 3, 5, 7 (+8)
#pragma unroll
        for (int m = 0; m < M; ++m) {
          ah[m][f] = dp4a_us(ev, lw[m].x, ah[m][f]);
          ah[m][f] = dp4a_us(od, lw[m].y, ah[m][f]);
          al[m][f] = dp4a_us(ev, lw[m].z, al[m][f]);
          al[m][f] = dp4a_us(od, lw[m].w, al[m][f]);
        }
      }
    }
    // group scales of the unit's 4 features (fp16)
    const uint2 sraw = *reinterpret_cast<const uint2*>(wscale + (size_t)(k0 >> 7) * N + tile * 128 + lane * 4);
    const __half2* sh = reinterpret_cast<const __half2*>(&sraw);
    const float2 g01 = __half22float2(sh[0]), g23 = __half22float2(sh[1]);
    const float gsc[4] = {g01.x, g01.y, g23.x, g23.y};
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
      for (int f = 0; f < 4; ++f) {
        const int v = ah[m][f] * 128 + al[m][f] - 8 * csum[m];  // sum (q - 8) X, exact
        facc[m][f] = fmaf((float)v * s[m], gsc[f], facc[m][f]);
      }
    __syncwarp();  // every lane read the limbs before the next unit rewrites them
    if (more) {
#pragma unroll
      for (int j = 0; j < kRows; ++j) cur[j] = nxt[j];
    }
    ++u;
  }
  if (tile >= 0) flush();
  if (flag_mc) {
    // second phase: the last CTA to finish sends the reduced rows to every rank
    __shared__ int last;
    __threadfence();  // this thread's atomics are visible before the ticket
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(ticket, 1u) == gridDim.x - 1;
    __syncthreads();
    if (last) {
      __threadfence();  // every other CTA's atomics (ordered by their tickets)
      for (int r = 0; r < M; ++r) {
        float4* src = reinterpret_cast<float4*>(ws + (size_t)r * ldo);
        for (int i = threadIdx.x; i < N / 4; i += blockDim.x) {
          const float4 v = __ldcg(src + i);
          src[i] = make_float4(0.f, 0.f, 0.f, 0.f);  // clean for the next call
          peer::mc_red_add_v4_f32(ws_mc + (size_t)r * ldo + 4 * i, v);
        }
      }
      peer::fence_proxy_alias();
      __syncthreads();
      if (threadIdx.x == 0) {
        *ticket = 0u;
        peer::mc_signal_add_u64(flag_mc, 1ull);
      }
    }
  }
}

// SM count of the current device, cached per device (host threads may race
// to fill an entry; they store the same value, and the atomics keep that
// well defined). The grid size, and so the all-reduce signal count, follows it.
static int sm_count() {
  static std::atomic<int> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev < 0 || dev >= 64) return 148;
  int n = cache[dev].load(std::memory_order_relaxed);
  if (n <= 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

// CTAs of one launch (persistent: at most ctas_per_sm per SM).
static int grid_ctas(int M, int N, int K) {
  const int units = (N / 128) * (K / (8 * kRows));
  const int ctas = (M <= 2 ? ctas_per_sm<1>() : ctas_per_sm<4>()) * sm_count();
  const int need = cdiv(units, kWarps);
  return ctas < need ? ctas : need;
}

template <int M>
static int launch(const void* w, const void* wscale, const void* x, float* ws, int N, int K, int ldx, int ldo,
                  float* ws_mc, unsigned long long* flag_mc, unsigned int* ticket, cudaStream_t st) {
  const int units = (N / 128) * (K / (8 * kRows));
  return launch_k(gemv_w4_kernel<M>, dim3(grid_ctas(M, N, K)), dim3(kWarps * 32), 0, st,
                  reinterpret_cast<const uint32_t*>(w), reinterpret_cast<const __half*>(wscale),
                  reinterpret_cast<const __nv_bfloat16*>(x), ws, N, K, ldx, ldo, units, ws_mc, flag_mc,
                  ticket) == cudaSuccess
             ? 0
             : 300;
}

static int dispatch(const void* w, const void* wscale, const void* x, float* ws, int M, int N, int K, int ldx,
                    int ldo, float* ws_mc, unsigned long long* flag_mc, unsigned int* ticket, cudaStream_t st) {
  if (M < 1 || M > 4 || N % 128 || K % 128 || ldx % 2 || ldo < N || !w || !wscale || !x || !ws) return 1;
  if (flag_mc && (!ws_mc || !ticket || ldo % 4 || (reinterpret_cast<uintptr_t>(ws) & 15) ||
                  (reinterpret_cast<uintptr_t>(ws_mc) & 15)))
    return 1;
  switch (M) {
    case 1: return launch<1>(w, wscale, x, ws, N, K, ldx, ldo, ws_mc, flag_mc, ticket, st);
    case 2: return launch<2>(w, wscale, x, ws, N, K, ldx, ldo, ws_mc, flag_mc, ticket, st);
    case 3: return launch<3>(w, wscale, x, ws, N, K, ldx, ldo, ws_mc, flag_mc, ticket, st);
    default: return launch<4>(w, wscale, x, ws, N, K, ldx, ldo, ws_mc, flag_mc, ticket, st);
  }
}

}  // namespace gemv
}  // namespace k8v4

// Rows up to which the decode GEMV serves a W4A16 call. Measured (graph-timed,
// L2 flushed, 27B shapes): at one row the GEMV beats the tcgen05 path
// (gate/up 28.7 vs 43.0 us, down 20.5 vs 32.6 us); at four rows the integer
// dot-product pipe (~16-21 dp4a per clock per SM here) makes it slower
// (gate/up 71.6 vs 45.1 us), so wider calls stay on the tensor cores. The
// kernel itself takes up to 4 rows.
extern "C" int k8v4_gemv_w4_max_rows() { return 1; }

// ws[t, n] (row stride ldo, fp32, zero on entry) += x[t, :] (bf16, row stride
// ldx) times the GPTQ int4 weights [K/8, N] with fp16 group scales [K/128, N].
// Returns 0, 1 for an unsupported shape, 300 for a launch error.
extern "C" int k8v4_gemv_w4(const void* w, const void* wscale, const void* x, float* ws, int M, int N, int K,
                            int ldx, int ldo, cudaStream_t st) {
  return k8v4::gemv::dispatch(w, wscale, x, ws, M, N, K, ldx, ldo, nullptr, nullptr, nullptr, st);
}

// GEMM -> all-reduce: the sums meet in `local` (this rank's fp32 [M, ldo]
// accumulator, zero on entry and left zero), then the last CTA adds them into
// every rank's copy of a symmetric fp32 buffer through its multicast address
// ws_mc and adds 1 to the multicast counter flag_mc; `ticket` (one unsigned
// int, zero on entry and left zero) picks that CTA. The consumer expects
// `world` signals for one call. Calls that overlap on the GPU must not share
// `local` or `ticket`.
extern "C" int k8v4_gemv_w4_allreduce(const void* w, const void* wscale, const void* x, float* local, float* ws_mc,
                                      unsigned long long* flag_mc, unsigned int* ticket, int M, int N, int K,
                                      int ldx, int ldo, cudaStream_t st) {
  if (!local || !ws_mc || !flag_mc || !ticket) return 4;
  return k8v4::gemv::dispatch(w, wscale, x, local, M, N, K, ldx, ldo, ws_mc, flag_mc, ticket, st);
}

// CTAs one call launches (0 for an unsupported shape).
extern "C" int k8v4_gemv_w4_ctas(int M, int N, int K) {
  if (M < 1 || M > 4 || N % 128 || K % 128) return 0;
  return k8v4::gemv::grid_ctas(M, N, K);
}
