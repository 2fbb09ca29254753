// tcgen05.mma issue cost at decode sizes (M = 128, N = 16, K = 16, A from
// TMEM): (a) one issuing thread, (b) two issuing threads in different warps
// with separate accumulators, (c) one issuer while four other warps stream
// tcgen05.st into other TMEM columns. Every loop is bounded.
//
//   nvcc -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 -Icsrc \
//        -o mma_issue_probe bench/mma_issue_probe.cu && ./mma_issue_probe
//
// Measured on one B200: (a) 52.1 cycles per MMA, (b) 56.1 per issuer = 28.0
// aggregate, (c) 60.1; the decode GEMM splits its MMA issue over warps.
#include <cstdio>
#include "../csrc/tc.cuh"
using namespace k8v4; using namespace k8v4::tc;
template <int MODE>
__global__ void probe(long long* out, int iters) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = align_smem_1024(smem_raw);
  __shared__ uint64_t bar[2];
  __shared__ uint32_t holder;
  __shared__ int abortf;
  __shared__ volatile int stop;
  for (int i = threadIdx.x; i < 32768 / 4; i += blockDim.x) ((uint32_t*)sm)[i] = 0;
  if (threadIdx.x == 0) { mbar_init(&bar[0], 1); mbar_init(&bar[1], 1); abortf = 0; stop = 0; fence_mbar_init(); }
  if (threadIdx.x < 32) { tmem_alloc(&holder, 512); tmem_relinquish(); }
  fence_async_smem(); tc_fence_before(); __syncthreads(); tc_fence_after();
  uint32_t tmem = holder;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t idesc = idesc_bf16(128, 16);
  const uint32_t b = smem_u32(sm);
  const bool issuer = (lane == 0) && (warp == 0 || (MODE == 1 && warp == 1));
  if (issuer) {
    const uint32_t d = tmem + warp * 32;           // accumulators cols 0 / 32
    const uint32_t a = tmem + 128 + warp * 64;     // A cols 128.. / 192..
    long long t0 = clock64();
    for (int i = 0; i < iters; ++i) {
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) mma_f16_ts(d, a + kk * 8, sdesc_sw128(b + (kk >> 2) * 2048 + (kk & 3) * 32, 16, 1024), idesc, 1);
      mma_commit(&bar[warp]);
    }
    long long t1 = clock64();
    out[warp] = t1 - t0;
    if (warp == 0) stop = 1;
  } else if (MODE == 2 && warp >= 4 && warp < 8) {
    // stream tcgen05.st into cols 256..511 of this warp's lane quadrant until the issuer is done
    uint32_t v[32];
    for (int i = 0; i < 32; ++i) v[i] = i;
    const uint32_t base = tmem + 256 + ((uint32_t)((warp & 3) * 32) << 16);
    for (int it = 0; it < 1000000 && !stop; ++it) {
      tmem_st32(base + (it & 7) * 32, v);
      tmem_st_wait();
    }
  }
  tc_fence_before(); __syncthreads();
  if (threadIdx.x < 32) { tc_fence_after(); tmem_dealloc(tmem, 512); }
}
template <int MODE> void run(const char* name, long long* d) {
  int iters = 2000;
  cudaFuncSetAttribute(probe<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, 40000);
  cudaMemset(d, 0, 16);
  probe<MODE><<<1, 256, 40000>>>(d, iters);
  long long h[2]; cudaMemcpy(h, d, 16, cudaMemcpyDeviceToHost);
  cudaError_t e = cudaGetLastError();
  int n = iters * 8;
  if (MODE == 1) printf("%-28s issuer0 %.1f cyc/mma issuer1 %.1f cyc/mma -> aggregate %.1f cyc/mma (%s)\n", name, (double)h[0] / n, (double)h[1] / n, (double)(h[0] > h[1] ? h[0] : h[1]) / (2 * n), cudaGetErrorString(e));
  else printf("%-28s %.1f cyc/mma (%s)\n", name, (double)h[0] / n, cudaGetErrorString(e));
}
int main() {
  long long* d; cudaMalloc(&d, 16);
  run<0>("one issuer", d);
  run<1>("two issuers", d);
  run<2>("one issuer + tcgen05.st load", d);
  return 0;
}
