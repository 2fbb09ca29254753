// Pieces shared by the paged K8/V4 attention kernels (b200 format).
//
// Page format: each (page, head) is one 3,232-byte run
//   [K 16 x 128 int8][V 16 x 64 u8][k_scale 16 fp16][v_scale 16 x 4 fp16].
// A 128-key tile = 8 pages. K rows reach shared memory through a 3D TMA
// tensor map (128-byte swizzle, the tcgen05 K-major layout); the V + scale
// tail of each run (1,184 bytes) through one plain bulk copy.
#pragma once
#include "../tc.cuh"

namespace k8v4 {
namespace attn {

constexpr int D = 128;
constexpr int PAGE = 16;
constexpr int HEAD_BYTES = 3232;
constexpr int K_BYTES = PAGE * D;      // 2048
constexpr int VS_OFF = K_BYTES;        // V + scales start inside a head run
constexpr int VS_BYTES = 1184;         // V (1024) + k_scale (32) + v_scale (128)
constexpr int KS_OFF = 1024;           // k_scale inside the VS block
constexpr int VSC_OFF = 1056;          // v_scale inside the VS block
constexpr int TILE = 128;              // keys per tile
constexpr int TILE_PAGES = TILE / PAGE;
constexpr int K_TILE_BYTES = TILE * D; // 16 KB
constexpr int VS_TILE_BYTES = TILE_PAGES * VS_BYTES;
constexpr int VT_BYTES = TILE * D * 2; // fp16 V tile, 32 KB
constexpr int VT_LBO = 16 * 1024;      // MN-major: next 64 dims
constexpr float LOG2E = 1.4426950408889634f;

// TMA maps of one KV cache: `page` moves one (page, head) K block (2 KB);
// `k8` moves the K blocks of 8 consecutive pages of one head (16 KB, the
// whole tile) and `vs8` their V + scale blocks (9,472 B). A tile whose pages
// are consecutive (the usual case: the block manager hands out pages in
// order) then costs 2 copy requests instead of 16; the TMA's per-request
// issue cost, not bandwidth, set the tile rate with one request per page.
struct KVTileMaps {
  CUtensorMap page;
  CUtensorMap k8;
  CUtensorMap vs8;
};
// Lazy rescale threshold (log2 units): the running max used for exp2 only
// moves when a new score exceeds it by more than this, so p <= 2^8.
constexpr float RESCALE_TAU = 8.0f;

// Instruction descriptor, fp16 inputs, fp32 accumulate.
K8V4_HOST_DEVICE constexpr uint32_t idesc_f16(int M, int N, bool a_mn, bool b_mn) {
  return (1u << 4) | (0u << 7) | (0u << 10) | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// Convert one 8-dim chunk (4 bytes of packed V, low nibble = even dim) of one
// key into 8 fp16 values (q-8)*scale, stored at the MN-major 128B-swizzled
// position of a [128 dims] x [128 keys] tile (dims contiguous).
__device__ __forceinline__ void v_chunk_to_f16(uint32_t w, __half scale, uint8_t* vt, int key, int chunk) {
  const uint32_t w4 = w >> 4;
  const __half2 bias = __halves2half2(__float2half(1032.f), __float2half(1032.f));
  const __half2 s2 = __halves2half2(scale, scale);
  uint32_t o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t dup = __byte_perm(w, w4, 0x0400 + j * 0x0101);
    const uint32_t m = (dup & 0x000F000Fu) | 0x64006400u;  // fp16 (1024 + c0, 1024 + c1)
    __half2 v = *reinterpret_cast<const __half2*>(&m);
    v = __hmul2(__hsub2(v, bias), s2);
    o[j] = *reinterpret_cast<uint32_t*>(&v);
  }
  const int atom_m = chunk >> 3, c = chunk & 7, g = key >> 3, r = key & 7;
  *reinterpret_cast<uint4*>(vt + atom_m * VT_LBO + g * 1024 + r * 128 + ((c ^ r) << 4)) =
      make_uint4(o[0], o[1], o[2], o[3]);
}

__device__ __forceinline__ void v_chunk_zero(uint8_t* vt, int key, int chunk) {
  const int atom_m = chunk >> 3, c = chunk & 7, g = key >> 3, r = key & 7;
  *reinterpret_cast<uint4*>(vt + atom_m * VT_LBO + g * 1024 + r * 128 + ((c ^ r) << 4)) = make_uint4(0, 0, 0, 0);
}

// 2^x with the SFU's ex2.approx (flush-to-zero). Softmax arguments are <= 0
// after max subtraction (<= tau with the lazy rescale), and -inf gives +0.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Exact int32 -> fp32 for |v| < 2^22 (QK dot products are below 2^21).
__device__ __forceinline__ float i2f_small(uint32_t v) {
  return __int_as_float(static_cast<int>(v) + 0x4B400000) - 12582912.0f;
}

}  // namespace attn
}  // namespace k8v4
