// Paged causal prefill attention directly on int8-K / int4-V pages.
//
// Replaces the reference's per-KV-head gather + oneDNN SDPA pipeline
// (k8v4_v030/onednn_prefill.py:188-241, native/k8v4_sdpa.cpp:83-228 and the
// Triton gather prefill_gather_triton.py:15-66): K stays int8 (read by TMA
// straight from the pages), only V is dequantized, once per tile and KV head
// into a staging buffer in the MMA's own layout (prefill_stage_kernel);
// nothing is compiled per shape and there are no host waits.
//
// One CTA per (query tile, KV head, sequence). A query tile is TQ = 128/gqa
// consecutive tokens x the gqa query heads of this KV head = up to 128 rows,
// so every K/V tile read serves all grouped heads. Causality is bottom-right:
// the chunk's tokens are the last q_len tokens of the sequence.
//
//   S[row, key]  = Q8(int8, per-row scale) x K_tile^T      tcgen05 kind::i8
//   softmax      : two threads per row (64 keys each), lazy rescale (tau 8, log2 units)
//   O[row, dim] += P(fp16, TMEM) x V_tile(fp16, MN-major)   tcgen05 kind::f16, A from TMEM
//
// Warp roles: 0 = producer (K pages by TMA, staged V and k-scales by bulk
// copies), 1 = TMEM owner + MMA issuer, 2-9 = softmax / epilogue (lane
// quadrant = warp & 3, key and O-column half = (warp - 2) >> 2). S and P are
// double-buffered in TMEM, so the softmax of tile j overlaps QK(j + 1) and
// PV(j - 1).
#include "attn_common.cuh"

namespace k8v4 {
namespace attn {

using namespace tc;

constexpr int MAX_SRC = 8;  // KV page sources: this GPU plus context-parallel peers

// Context parallelism: a block-table entry is (source << 24) | page, source
// 0 .. nsrc-1 indexing `caches` (this GPU's cache or a peer's, mapped into
// this process) and the matching TMA map. With one source the entry is the
// page number itself.
struct KVMaps {
  KVTileMaps m[MAX_SRC];
};

struct PrefillParams {
  const __nv_bfloat16* q;      // [T, hq_total, D]
  const int32_t* cu_q;         // [nseq + 1]
  const int32_t* seq_lens;     // [nseq]
  const int32_t* block_table;  // [nseq, bt_stride]
  const int32_t* q_pos;        // optional [T] global position of each query token (CP: strided tokens)
  const uint8_t* caches[MAX_SRC];
  int nsrc;
  int64_t num_pages;           // pages of every source cache
  __nv_bfloat16* out;          // [T, hq_total, D]
  uint8_t* vstage;             // staged tiles [nseq][stage_tiles][heads] x STAGE_TILE_BYTES
  int stage_tiles;             // tiles per sequence in the staging buffer
  int bt_stride;
  int hkv, gqa, hq_total, head_offset;
  int n_qtiles;
  float sm_scale_log2;
};

// Every query tile of a KV head reads the same V pages, so V is dequantized
// once per (sequence, 128-key tile, KV head) by prefill_stage_kernel instead
// of in each of the ~128 / TQ-times-more attention CTAs. A staged tile is the
// fp16 MN-major SW128 image the PV MMA reads (32 KB) followed by the tile's
// 128 k-scales as fp32 (512 B); keys past the sequence are zero. The
// attention kernel moves it with two plain bulk copies.
constexpr int STAGE_V_BYTES = VT_BYTES;
constexpr int STAGE_KS_BYTES = TILE * 4;
constexpr int STAGE_TILE_BYTES = STAGE_V_BYTES + STAGE_KS_BYTES;

__device__ __forceinline__ uint8_t* stage_tile(const PrefillParams& p, int seq, int j, int hl, int heads) {
  return p.vstage + (((size_t)seq * p.stage_tiles + j) * heads + hl) * STAGE_TILE_BYTES;
}

__global__ void __launch_bounds__(256) prefill_stage_kernel(const PrefillParams p) {
  pdl_trigger();
  pdl_wait();  // everything this kernel reads may come from the previous one
  __shared__ __align__(1024) uint8_t sV[VT_BYTES];
  const int j = blockIdx.x, hl = blockIdx.y, h = hl + p.head_offset, seq = blockIdx.z;
  const int seq_len = p.seq_lens[seq];
  const int key0 = j * TILE;
  if (key0 >= seq_len) return;  // uniform for the CTA
  const int nvalid = min(TILE, seq_len - key0);
  const int32_t* bt = p.block_table + (int64_t)seq * p.bt_stride + j * TILE_PAGES;
  uint8_t* dst = stage_tile(p, seq, j, hl, gridDim.y);
  float* ks_out = reinterpret_cast<float*>(dst + STAGE_V_BYTES);
  // one item = 32 dims (one scale group) of one key: a 16-byte load of packed
  // V and one scale feed four 16-byte stores of the fp16 tile
  for (int item = threadIdx.x; item < TILE * 4; item += 256) {
    const int key = item >> 2, grp = item & 3;
    const uint32_t e = key < nvalid ? (uint32_t)bt[key >> 4] : 0u;
    const bool in_pool = (int64_t)(e & 0xFFFFFFu) < p.num_pages;
    if (key < nvalid && !in_pool && grp == 0 && (key & 15) == 0) record_error(kErrBadIndex, 301);
    if (key < nvalid && in_pool) {  // a page outside the pool reads as zeros (and is reported)
      const int src = (int)(e >> 24) < p.nsrc ? (int)(e >> 24) : 0;  // a bad source reads source 0
      const uint8_t* run = p.caches[src] + ((int64_t)(e & 0xFFFFFFu) * p.hkv + h) * HEAD_BYTES + VS_OFF;
      const int kk = key & 15;
      const uint4 w = *reinterpret_cast<const uint4*>(run + kk * 64 + grp * 16);
      const __half sc = *reinterpret_cast<const __half*>(run + VSC_OFF + (kk * 4 + grp) * 2);
      v_chunk_to_f16(w.x, sc, sV, key, grp * 4);
      v_chunk_to_f16(w.y, sc, sV, key, grp * 4 + 1);
      v_chunk_to_f16(w.z, sc, sV, key, grp * 4 + 2);
      v_chunk_to_f16(w.w, sc, sV, key, grp * 4 + 3);
      if (grp == 0) ks_out[key] = __half2float(*reinterpret_cast<const __half*>(run + KS_OFF + kk * 2));
    } else {
#pragma unroll
      for (int q = 0; q < 4; ++q) v_chunk_zero(sV, key, grp * 4 + q);
      if (grp == 0) ks_out[key] = 0.f;
    }
  }
  __syncthreads();
  const uint4* s4 = reinterpret_cast<const uint4*>(sV);
  uint4* d4 = reinterpret_cast<uint4*>(dst);
  for (int i = threadIdx.x; i < VT_BYTES / 16; i += 256) d4[i] = s4[i];
}

struct PCfg {
  static constexpr int STAGES = 4;
  static constexpr int NWARPS = 10;
  static constexpr int NTHREADS = NWARPS * 32;
  static constexpr int NSOFT = 8;   // warps 2-9: quadrant = warp & 3, key half = (warp - 2) >> 2
  static constexpr int TMEM_COLS = 512;
  static constexpr uint32_t COL_S = 0, COL_P = 256, COL_O = 384;  // S [2 x 128], P fp16 pairs [2 x 64], O [128]
  static constexpr int OFF_K = 0;                                  // [STAGES] int8 K tiles (TMA, SW128)
  static constexpr int OFF_V = OFF_K + STAGES * K_TILE_BYTES;      // [STAGES] staged fp16 V tiles
  static constexpr int OFF_KS = OFF_V + STAGES * STAGE_V_BYTES;    // [STAGES] k-scales (fp32)
  static constexpr int OFF_Q = OFF_KS + STAGES * STAGE_KS_BYTES;
  static constexpr int OFF_MISC = OFF_Q + 128 * 128;
  static constexpr int MISC_BYTES = 5120;
  static constexpr int SMEM_BYTES = 1024 + OFF_MISC + MISC_BYTES;
};
static_assert(PCfg::SMEM_BYTES <= 232448, "prefill shared memory");
static_assert(PCfg::OFF_V % 1024 == 0 && PCfg::OFF_Q % 1024 == 0, "SW128 operands on 1 KB boundaries");

__global__ void __launch_bounds__(PCfg::NTHREADS, 1)
    prefill_attn_kernel(const __grid_constant__ KVMaps maps, const PrefillParams p) {
  pdl_trigger();
  pdl_wait();  // Q, the KV pages and the block table may come from the previous kernels
  using C = PCfg;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = align_smem_1024(smem_raw);
  uint8_t* sK = sm + C::OFF_K;
  uint8_t* sV = sm + C::OFF_V;
  const float* sKS = reinterpret_cast<const float*>(sm + C::OFF_KS);
  uint8_t* sQ = sm + C::OFF_Q;
  uint8_t* misc = sm + C::OFF_MISC;
  uint64_t* kv_full = reinterpret_cast<uint64_t*>(misc);
  uint64_t* kv_empty = kv_full + C::STAGES;  // PV of the stage's tile done (K, V and k-scales all read)
  uint64_t* s_full = kv_empty + C::STAGES;   // [2] QK of the tile in S[b] done
  uint64_t* s_empty = s_full + 2;            // [2] every softmax warp loaded S[b]
  uint64_t* p_full = s_empty + 2;            // [2] P[b] written (and O rescaled)
  uint64_t* pv_empty = p_full + 2;           // [2] PV that read P[b] done
  uint64_t* mx_full = pv_empty + 2;          // [2][4] both key halves of quadrant q published their max
  uint64_t* l_full = mx_full + 8;            // [4] both halves published their row sum
  uint64_t* done_bar = l_full + 4;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(done_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  float* q_scale = reinterpret_cast<float*>(misc + 512);   // [128]
  int* row_end = reinterpret_cast<int*>(misc + 1024);       // [128]
  float* mx_buf = reinterpret_cast<float*>(misc + 1536);    // [2 buffers][2 halves][128 rows]
  float* l_buf = reinterpret_cast<float*>(misc + 3584);     // [2 halves][128 rows]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = p.n_qtiles - 1 - blockIdx.x;  // longest tiles first
  const int hl = blockIdx.y, h = hl + p.head_offset, seq = blockIdx.z;
  const int qb = p.cu_q[seq], q_len = p.cu_q[seq + 1] - qb;
  const int TQ = 128 / p.gqa;
  const int t0 = qt * TQ;
  if (t0 >= q_len) return;  // uniform for the CTA: nothing allocated yet
  const int tq = min(TQ, q_len - t0);
  const int R = tq * p.gqa;
  const int seq_len = p.seq_lens[seq];
  const int ctx = seq_len - q_len;
  // without positions the chunk is the sequence's last q_len tokens (bottom-right causal)
  const int32_t* qpos = p.q_pos ? p.q_pos + qb : nullptr;
  const int n_keys = qpos ? qpos[t0 + tq - 1] + 1 : ctx + t0 + tq;  // keys the last token of the tile sees
  const int nt = (n_keys + TILE - 1) / TILE;
  const int32_t* bt = p.block_table + (int64_t)seq * p.bt_stride;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&s_empty[b], C::NSOFT);
      mbar_init(&p_full[b], C::NSOFT);
      mbar_init(&pv_empty[b], 1);
    }
    for (int i = 0; i < 8; ++i) mbar_init(&mx_full[i], 2);
    for (int i = 0; i < 4; ++i) mbar_init(&l_full[i], 2);
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, C::TMEM_COLS);
    tmem_relinquish();
  }
  // ---- prologue: quantized query rows (A operand, K-major SW128)
  for (int r = warp; r < 128; r += C::NWARPS) {
    float x[4] = {0.f, 0.f, 0.f, 0.f};
    int end = 0;
    if (r < R) {
      const int t = t0 + r / p.gqa, g = r % p.gqa;
      const __nv_bfloat16* src = p.q + ((int64_t)(qb + t) * p.hq_total + (int64_t)h * p.gqa + g) * D + lane * 4;
      const uint2 raw = *reinterpret_cast<const uint2*>(src);
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
      const float2 a = __bfloat1622float2(h2[0]), b = __bfloat1622float2(h2[1]);
      x[0] = a.x; x[1] = a.y; x[2] = b.x; x[3] = b.y;
      end = qpos ? qpos[t] + 1 : ctx + t + 1;
    }
    float amax = fmaxf(fmaxf(fabsf(x[0]), fabsf(x[1])), fmaxf(fabsf(x[2]), fabsf(x[3])));
    amax = warp_max(amax);
    const float s = amax / 127.f;
    const float inv = s > 0.f ? 1.f / s : 0.f;
    uint32_t w = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int qi = (int)fminf(fmaxf(rintf(x[j] * inv), -127.f), 127.f);
      w |= ((uint32_t)(uint8_t)(int8_t)qi) << (8 * j);
    }
    *reinterpret_cast<uint32_t*>(sQ + sw128_offset(r, lane >> 2) + (lane & 3) * 4) = w;
    if (lane == 0) {
      q_scale[r] = s * p.sm_scale_log2;
      row_end[r] = end;
    }
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const int n_pages = (n_keys + PAGE - 1) / PAGE;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // per tile: the K pages by TMA (one 3D map per source; lane i issues
    // page i, its block-table entry read STAGES tiles ahead in a register
    // ring), the staged V image and k-scales by two bulk copies (lane 0)
    if (lane == 0)
      for (int i = 0; i < p.nsrc; ++i) {
        prefetch_tmap(&maps.m[i].page);
        prefetch_tmap(&maps.m[i].k8);
      }
    auto entry_of = [&](int jt) -> uint32_t {
      const int pg = jt * TILE_PAGES + lane;
      return (jt < nt && lane < TILE_PAGES && pg < n_pages) ? (uint32_t)bt[pg] : 0u;
    };
    static_assert(C::STAGES == 4, "page-id ring depth");
    uint32_t eq0 = entry_of(0), eq1 = entry_of(1), eq2 = entry_of(2), eq3 = entry_of(3);
    int issued = 0;
    for (int j = 0; j < nt; ++j) {
      const int s = j % C::STAGES;
      const uint32_t e = eq0;
      eq0 = eq1;
      eq1 = eq2;
      eq2 = eq3;
      eq3 = entry_of(j + 4);
      if (j >= C::STAGES && !mbar_wait_all(&kv_empty[s], ((j / C::STAGES) - 1) & 1, abort_flag, 301)) break;
      const int npg = min(TILE_PAGES, n_pages - j * TILE_PAGES);
      const uint32_t e0 = __shfl_sync(0xffffffffu, e, 0);
      if (__all_sync(0xffffffffu, lane >= npg || e == e0 + (uint32_t)lane)) {
        // 8 consecutive pages of one source: one box for the tile's K
        if (lane == 0) {
          const int src = (int)(e0 >> 24) < p.nsrc ? (int)(e0 >> 24) : 0;  // a bad source reads source 0
          mbar_arrive_expect_tx(&kv_full[s], TILE_PAGES * K_BYTES + STAGE_TILE_BYTES);
          tma_load_4d(sK + s * K_TILE_BYTES, &maps.m[src].k8, &kv_full[s], 0, 0, h, (int)(e0 & 0xFFFFFFu));
        }
      } else {
        if (lane == 0) mbar_arrive_expect_tx(&kv_full[s], npg * K_BYTES + STAGE_TILE_BYTES);
        __syncwarp();
        if (lane < npg) {
          const int src = (int)(e >> 24) < p.nsrc ? (int)(e >> 24) : 0;  // a bad source reads source 0
          const int64_t run = (int64_t)(e & 0xFFFFFFu) * p.hkv + h;
          tma_load_3d(sK + s * K_TILE_BYTES + lane * K_BYTES, &maps.m[src].page, &kv_full[s], 0, 0, (int)run);
        }
      }
      if (lane == 0) {
        const uint8_t* st = stage_tile(p, seq, j, hl, gridDim.y);
        bulk_load(sV + s * STAGE_V_BYTES, st, STAGE_V_BYTES, &kv_full[s]);
        bulk_load(sm + C::OFF_KS + s * STAGE_KS_BYTES, st + STAGE_V_BYTES, STAGE_KS_BYTES, &kv_full[s]);
      }
      ++issued;
    }
    if (lane == 0 && *abort_flag)
      for (int j = issued - 1; j >= 0 && j >= issued - C::STAGES; --j)
        mbar_wait_drain(&kv_full[j % C::STAGES], (j / C::STAGES) & 1);
  } else if (warp == 1) {
    // ----------------------------------------------------------------- MMA
    // QK(j) into S[j & 1] once the softmax loaded S of tile j - 2; PV(j - 1)
    // with P[(j - 1) & 1] read from TMEM (TS form) once the softmax wrote it.
    if (lane == 0) {
      const uint32_t id_qk = idesc_s8(128, 128);
      const uint32_t id_pv = idesc_f16(128, 128, false, true);
      const uint32_t q_base = smem_u32(sQ);
      bool ok = true;
      for (int j = 0; j <= nt && ok; ++j) {
        if (j < nt) {
          const int s = j % C::STAGES, b = j & 1;
          if (!mbar_wait(&kv_full[s], (j / C::STAGES) & 1, abort_flag, 302) ||
              (j >= 2 && !mbar_wait(&s_empty[b], ((j >> 1) - 1) & 1, abort_flag, 311)))
            break;
          tc_fence_after();
          const uint32_t k_base = smem_u32(sK + s * K_TILE_BYTES);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_i8(tmem + C::COL_S + b * 128, sdesc_sw128(q_base + kk * 32, 16, 1024),
                   sdesc_sw128(k_base + kk * 32, 16, 1024), id_qk, kk > 0 ? 1u : 0u);
          mma_commit(&s_full[b]);
        }
        if (j >= 1) {
          const int jj = j - 1, b = jj & 1, s = jj % C::STAGES;
          if (!mbar_wait(&p_full[b], (jj >> 1) & 1, abort_flag, 303)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t v_base = smem_u32(sV + s * STAGE_V_BYTES);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            mma_f16_ts(tmem + C::COL_O, tmem + C::COL_P + b * 64 + kk * 8,
                       sdesc_sw128(v_base + kk * 2048, VT_LBO, 1024), id_pv, (jj > 0 || kk > 0) ? 1u : 0u);
          mma_commit(&pv_empty[b]);
          mma_commit(&kv_empty[s]);  // the stage's K, V and k-scales are all consumed
        }
      }
      mma_commit(done_bar);
      mbar_wait_drain(done_bar, 0);
    }
  } else {
    // ------------------------------------------------------------- softmax
    // Two warps per TMEM lane quadrant: each owns 32 rows x 64 keys of every
    // tile (scores held in registers, one pass) and 64 columns of O. The two
    // halves of a row agree on the running max through shared memory.
    const int quad = warp & 3, hf = (warp - 2) >> 2;
    const int row = quad * 32 + lane;
    const bool live = row < R;
    // a zero query row (scale 0) keeps finite scores: scores x qs stay 0 and masked keys -inf
    const float qs = fmaxf(q_scale[row], 1e-30f);
    const int end = row_end[row];
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t tS = tmem + C::COL_S + lane_off + hf * 64;
    const uint32_t tP = tmem + C::COL_P + lane_off + hf * 32;
    const uint32_t tO = tmem + C::COL_O + lane_off + hf * 64;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    // Every softmax warp runs every iteration (the halves exchange maxima each
    // tile); a failed wait only turns the work off.
    for (int j = 0; j < nt; ++j) {
      const int s = j % C::STAGES, b = j & 1;
      if (ok && !mbar_wait_all(&s_full[b], (j >> 1) & 1, abort_flag, 307)) ok = false;
      float sc[64];
      if (ok) {
        tc_fence_after();
        uint32_t v[32];
        tmem_ld32(tS + b * 128, v);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) sc[i] = i2f_small(v[i]);
        tmem_ld32(tS + b * 128 + 32, v);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) sc[32 + i] = i2f_small(v[i]);
        tc_fence_before();
      }
      __syncwarp();
      if (ok && lane == 0) mbar_arrive(&s_empty[b]);
      // the stage's k-scales (landed with its K tile; QK completing implies it)
      if (ok && !mbar_wait_all(&kv_full[s], (j / C::STAGES) & 1, abort_flag, 308)) ok = false;
      const int key0 = j * TILE + hf * 64;
      float tmax = -INFINITY;
      if (ok) {
        const float4* ks4 = reinterpret_cast<const float4*>(sKS + s * TILE + hf * 64);
#pragma unroll
        for (int k = 0; k < 64; k += 4) {
          const float4 kq = ks4[k >> 2];
          sc[k] *= kq.x;
          sc[k + 1] *= kq.y;
          sc[k + 2] *= kq.z;
          sc[k + 3] *= kq.w;
        }
        const bool full = __all_sync(0xffffffffu, end >= key0 + 64 || !live);
        if (!full) {
#pragma unroll
          for (int k = 0; k < 64; ++k) sc[k] = (key0 + k < end) ? sc[k] : -INFINITY;
        }
        float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int k = 0; k < 64; k += 4) {
          mx[0] = fmaxf(mx[0], sc[k]);
          mx[1] = fmaxf(mx[1], sc[k + 1]);
          mx[2] = fmaxf(mx[2], sc[k + 2]);
          mx[3] = fmaxf(mx[3], sc[k + 3]);
        }
        tmax = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])) * qs;
      }
      // publish this half's max, combine with the other half of the same rows
      mx_buf[(b * 2 + hf) * 128 + row] = tmax;
      __syncwarp();
      if (lane == 0) mbar_arrive(&mx_full[b * 4 + quad]);
      if (ok && !mbar_wait_all(&mx_full[b * 4 + quad], (j >> 1) & 1, abort_flag, 309)) ok = false;
      if (ok) {
        tmax = fmaxf(tmax, mx_buf[(b * 2 + (hf ^ 1)) * 128 + row]);
        float alpha = 1.f;
        if (tmax > m + RESCALE_TAU || (m == -INFINITY && tmax > -INFINITY)) {
          alpha = (m == -INFINITY) ? 0.f : ex2_approx(m - tmax);
          m = tmax;
        }
        l *= alpha;
        // O holds PV(0..j-1) after PV(j-1): rescale this half's columns when any row of the warp moved its max
        if (j >= 1 && __any_sync(0xffffffffu, alpha != 1.f)) {
          if (!mbar_wait_all(&pv_empty[(j - 1) & 1], ((j - 1) >> 1) & 1, abort_flag, 310)) {
            ok = false;
          } else {
            tc_fence_after();
            // 16 columns at a time: the 64 scores stay live in registers meanwhile
#pragma unroll
            for (int c = 0; c < 64; c += 16) {
              uint32_t v[16];
              tmem_ld16(tO + c, v);
              tmem_ld_wait();
#pragma unroll
              for (int i = 0; i < 16; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * alpha);
              tmem_st16(tO + c, v);
            }
          }
        }
        // P[b] is free once the PV of tile j-2 finished
        if (ok && j >= 2 && !mbar_wait_all(&pv_empty[b], ((j >> 1) - 1) & 1, abort_flag, 312)) ok = false;
        if (ok) {
          tc_fence_after();
          // rows with no visible key keep m = -inf: exponentiate against 0 (all p = 0)
          const float nm = (m == -INFINITY) ? 0.f : -m;
          float ls[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int hh = 0; hh < 64; hh += 32) {
            uint32_t pk[16];
#pragma unroll
            for (int k = 0; k < 32; k += 2) {
              const float p0 = ex2_approx(fmaf(sc[hh + k], qs, nm));
              const float p1 = ex2_approx(fmaf(sc[hh + k + 1], qs, nm));
              ls[(k >> 1) & 3] += p0 + p1;
              const __half2 hp = __floats2half2_rn(p0, p1);
              pk[k >> 1] = *reinterpret_cast<const uint32_t*>(&hp);
            }
            tmem_st16(tP + b * 64 + (hh >> 1), pk);
          }
          l += (ls[0] + ls[1]) + (ls[2] + ls[3]);
          tmem_st_wait();
          tc_fence_before();
        }
      }
      __syncwarp();
      if (ok && lane == 0) mbar_arrive(&p_full[b]);
    }
    // ------------------------------------------------------------ epilogue
    // each warp writes its 64 columns of its 32 rows; the row sum is the sum of both halves
    l_buf[hf * 128 + row] = l;
    __syncwarp();
    if (lane == 0) mbar_arrive(&l_full[quad]);
    if (ok && nt > 0 && !mbar_wait_all(&pv_empty[(nt - 1) & 1], ((nt - 1) >> 1) & 1, abort_flag, 313)) ok = false;
    if (ok && !mbar_wait_all(&l_full[quad], 0, abort_flag, 314)) ok = false;
    if (ok && nt > 0) {  // warp-uniform (voted waits): every lane joins the TMEM loads
      tc_fence_after();
      const float lt = l + l_buf[(hf ^ 1) * 128 + row];
      const int t = t0 + (live ? row : 0) / p.gqa, g = (live ? row : 0) % p.gqa;
      __nv_bfloat16* dst = p.out + ((int64_t)(qb + t) * p.hq_total + (int64_t)h * p.gqa + g) * D + hf * 64;
      const float inv_l = lt > 0.f ? 1.f / lt : 0.f;
#pragma unroll
      for (int c = 0; c < 64; c += 32) {
        uint32_t r32[32];
        tmem_ld32(tO + c, r32);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          uint4 o;
          __nv_bfloat162 b0 = __floats2bfloat162_rn(__uint_as_float(r32[i]) * inv_l, __uint_as_float(r32[i + 1]) * inv_l);
          __nv_bfloat162 b1 = __floats2bfloat162_rn(__uint_as_float(r32[i + 2]) * inv_l, __uint_as_float(r32[i + 3]) * inv_l);
          __nv_bfloat162 b2 = __floats2bfloat162_rn(__uint_as_float(r32[i + 4]) * inv_l, __uint_as_float(r32[i + 5]) * inv_l);
          __nv_bfloat162 b3 = __floats2bfloat162_rn(__uint_as_float(r32[i + 6]) * inv_l, __uint_as_float(r32[i + 7]) * inv_l);
          o.x = *reinterpret_cast<uint32_t*>(&b0);
          o.y = *reinterpret_cast<uint32_t*>(&b1);
          o.z = *reinterpret_cast<uint32_t*>(&b2);
          o.w = *reinterpret_cast<uint32_t*>(&b3);
          if (live) *reinterpret_cast<uint4*>(dst + c + i) = o;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

}  // namespace attn
}  // namespace k8v4

using namespace k8v4;
using namespace k8v4::attn;

extern "C" int k8v4_make_kv_maps(void* maps_out, const void* cache, int64_t num_pages, int hkv);

K8V4_STATUS_API(prefill)

// Bytes of the V staging buffer for `nseq` sequences whose block-table rows
// hold `bt_width` pages, over `heads` KV heads.
extern "C" int64_t k8v4_prefill_stage_bytes(int nseq, int bt_width, int heads) {
  return (int64_t)nseq * cdiv(bt_width, TILE_PAGES) * heads * STAGE_TILE_BYTES;
}

// Paged causal prefill over `heads` KV heads starting at head_offset. With
// `nsrc` > 1 the pages come from several caches (context parallelism: this
// GPU's and its peers', block-table entries (source << 24) | page), and
// `q_pos` gives each query token's global position (the tokens of a rank are
// then not contiguous). All caches share num_pages and the head layout.
// `stage` holds k8v4_prefill_stage_bytes(nseq, bt_width, heads) bytes of
// scratch for the dequantized V tiles.
extern "C" int k8v4_prefill_attn_multi(const void* q, const int32_t* cu_q, const int32_t* seq_lens,
                                       const int32_t* block_table, int bt_stride, int bt_width,
                                       const void* const* caches, int nsrc, int64_t num_pages,
                                       const int32_t* q_pos, int hkv, int head_offset, int heads, int gqa,
                                       int hq_total, int nseq, int max_q_len, float sm_scale, void* stage,
                                       void* out, cudaStream_t st) {
  if (nseq <= 0 || max_q_len <= 0) return 0;
  if (gqa < 1 || 128 / gqa < 1) return 1;
  if (nsrc < 1 || nsrc > MAX_SRC) return 2;
  if (!stage || bt_width < 1) return 4;
  KVMaps maps;
  PrefillParams p;
  for (int i = 0; i < nsrc; ++i) {
    if (k8v4_make_kv_maps(&maps.m[i], caches[i], num_pages, hkv)) return 3;
    p.caches[i] = reinterpret_cast<const uint8_t*>(caches[i]);
  }
  for (int i = nsrc; i < MAX_SRC; ++i) {
    maps.m[i] = maps.m[0];
    p.caches[i] = p.caches[0];
  }
  p.nsrc = nsrc;
  p.num_pages = num_pages;
  p.q = reinterpret_cast<const __nv_bfloat16*>(q);
  p.cu_q = cu_q;
  p.seq_lens = seq_lens;
  p.block_table = block_table;
  p.q_pos = q_pos;
  p.out = reinterpret_cast<__nv_bfloat16*>(out);
  p.vstage = reinterpret_cast<uint8_t*>(stage);
  p.stage_tiles = cdiv(bt_width, TILE_PAGES);
  p.bt_stride = bt_stride;
  p.hkv = hkv;
  p.gqa = gqa;
  p.hq_total = hq_total;
  p.head_offset = head_offset;
  p.n_qtiles = cdiv(max_q_len, 128 / gqa);
  p.sm_scale_log2 = sm_scale * LOG2E;
  if (ensure_smem_limit<prefill_attn_kernel>(PCfg::SMEM_BYTES) != cudaSuccess) return 10;
  if (launch_k(prefill_stage_kernel, dim3(p.stage_tiles, heads, nseq), dim3(256), 0, st, p) != cudaSuccess) return 10;
  dim3 grid(p.n_qtiles, heads, nseq);
  return launch_k(prefill_attn_kernel, grid, dim3(PCfg::NTHREADS), PCfg::SMEM_BYTES, st, maps, p) == cudaSuccess ? 0
                                                                                                              : 10;
}

extern "C" int k8v4_prefill_attn(const void* q, const int32_t* cu_q, const int32_t* seq_lens,
                                 const int32_t* block_table, int bt_stride, int bt_width, const void* cache,
                                 int64_t num_pages, int hkv, int head_offset, int heads, int gqa, int hq_total,
                                 int nseq, int max_q_len, float sm_scale, void* stage, void* out, cudaStream_t st) {
  const void* caches[1] = {cache};
  return k8v4_prefill_attn_multi(q, cu_q, seq_lens, block_table, bt_stride, bt_width, caches, 1, num_pages, nullptr,
                                 hkv, head_offset, heads, gqa, hq_total, nseq, max_q_len, sm_scale, stage, out, st);
}
