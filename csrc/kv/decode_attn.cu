// Split-K paged decode / MTP-verify attention over int8-K / int4-V pages.
//
// One CTA per (split, KV head, sequence). Query rows are the (token, q-head)
// pairs of the sequence that share this KV head (q_len * gqa <= 64); they are
// quantized to int8 per row in the prologue (the reference's Q-once
// quantization, k8v4_v030/native/xe2_kv_ops.cpp:205-257). Rows run on the
// TMEM lanes, keys / dims on the columns:
//
//   S[row, key]  = Q8 (A, smem) x K_tile^T (B, TMA)       tcgen05 kind::i8 -> TMEM
//   softmax      : the rows are replicated down the 128 lanes; each lane
//                  quadrant's warp takes its slice of every tile's keys
//                  (tcgen05.ld), slice maxima meet through shared memory,
//                  lazy rescale (tau = 8 in log2 units), P -> TMEM (tcgen05.st)
//   O[row, dim] += P (A, TMEM) x V_tile (B, fp16 smem)     tcgen05 kind::f16 -> TMEM
//
// V int4 is dequantized by converter warps into the MN-major fp16 tile the
// PV MMA reads. Each split writes its (m, l, O) partial; k8v4_decode_combine
// merges the splits (the reference's stage-2 merge, :847-1246). With one
// split the CTA writes the normalized output directly.
//
// Warp roles: 0 = producer (a tile of 8 consecutive pages in two TMA boxes,
// else per-page copies), 1 = TMEM owner + MMA issuer (polls its QK and PV
// queues), 4-7 = softmax / epilogue (one per TMEM lane quadrant), 2, 3, 8..
// = V converters.
#include "attn_common.cuh"
#include "../comm/peer.cuh"
#include "../k8v4_c_api.h"

namespace k8v4 {
namespace attn {

using namespace tc;

struct DecodeParams {
  const __nv_bfloat16* q;     // [T, hq_total, D] rotated queries
  const int32_t* cu_q;        // [nseq + 1] token offsets
  const int32_t* seq_lens;    // [nseq] context length incl. the new tokens
  const int32_t* q_ends;      // optional [T] per-token visible end
  const int32_t* block_table; // [nseq, bt_stride]
  const uint8_t* cache;       // [pages, hkv * 3232]
  __nv_bfloat16* out;         // [T, hq_total, D]
  float* ws_o;                // [nseq, hkv, nsplit, NPAD, D]
  float* ws_ml;               // [nseq, hkv, nsplit, 2, NPAD]
  int bt_stride;
  int hkv, gqa, hq_total;     // hq_total: query heads in q / out rows
  int head_offset;            // first KV head of this launch (for replicated layouts)
  int nsplit;
  float sm_scale_log2;        // softmax scale * log2(e)
  // context parallelism, fused exchange: ws_o / ws_ml are multicast addresses
  // (this rank's slot in every rank's copy of a symmetric gather buffer), the
  // partials go out with multimem stores even when nsplit == 1, and each CTA
  // then adds 1 to the multicast counter flag_mc
  int push;
  unsigned long long* flag_mc;
};

#ifdef K8V4_TRACE
// Timeline of CTA (0,0,0) (trace builds only): rows = 0 producer issued,
// 1 converters done, 2 QK issued, 3 softmax done (p_full), 4 PV issued;
// keys-on-lanes kernel only: 5 softmax read S, 6 softmax past the maxima
// barrier, 7 softmax past the P^T buffer wait.
__device__ uint64_t g_attn_trace[8 * 256];
#define K8V4_ATRACE(row, idx)                                                             \
  do {                                                                                    \
    if (blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && (idx) < 256)             \
      g_attn_trace[(row) * 256 + (idx)] = globaltimer_ns();                               \
  } while (0)
#else
#define K8V4_ATRACE(row, idx) do { } while (0)
#endif

template <int NPAD>
struct DCfg {
  static constexpr int STAGES = 4;
  static constexpr int NVT = 3;             // fp16 V tiles (conversion runs ahead of the PV MMAs)
  // 0 TMA, 1 MMA, 4-7 softmax (one per TMEM lane quadrant), 2, 3, 8.. V converters
#ifndef K8V4_DECODE_NCONV
#define K8V4_DECODE_NCONV 6
#endif
  static constexpr int NCONV = K8V4_DECODE_NCONV;
  static constexpr int NWARPS = 8 + (NCONV - 2);
  static constexpr int NTHREADS = 32 * NWARPS;
  static constexpr int Q_BYTES = 128 * 128; // Q8 tile: 128 lanes (replicated rows) x 128 dims
  // TMEM columns: S[2] (int32, 128 keys each), P[2] (fp16 pairs, 64 each), O (fp32, 128 dims)
  static constexpr uint32_t COL_S = 0, COL_P = 256, COL_O = 384;
  static constexpr int TMEM_COLS = 512;
  static constexpr int OFF_K = 0;
  static constexpr int OFF_VT = OFF_K + STAGES * K_TILE_BYTES;
  static constexpr int OFF_Q = OFF_VT + NVT * VT_BYTES;
  static constexpr int OFF_VS = OFF_Q + Q_BYTES;
  // k scales of a tile (fp32, one per key), copied out of the stage by the
  // converters so the stage is released as soon as QK and conversion are done
  static constexpr int OFF_KS = OFF_VS + STAGES * VS_TILE_BYTES;
  static constexpr int OFF_MISC = OFF_KS + NVT * TILE * 4;
  static constexpr int SMEM_BYTES = 1024 + OFF_MISC + 512 + 2 * 64 * 4 + 2 * 128 * 4 + 128 * 4;
  // epilogue scratch (the K stages, idle by then): 128 lanes x 132 floats
  static constexpr int EPI_STRIDE = 132;
  static_assert(128 * EPI_STRIDE * 4 <= STAGES * K_TILE_BYTES + NVT * VT_BYTES, "epilogue scratch");
};

// Rows on TMEM lanes: the QK MMA puts query rows in lanes (A = Q8, M = 128)
// and the tile's 128 keys in columns (B = K page tile, N = 128). The real
// rows (R <= 64) are replicated NREP = 128 / LPR times down the lanes
// (LPR = 32 lanes per replica for R <= 32, else 64), which costs the tensor
// core nothing: replica e's threads own keys [e*KPR, (e+1)*KPR) of every
// tile (KPR = 128 / NREP). The four softmax warps (one per lane quadrant,
// so one per SM sub-partition) load only their key slice of S with
// tcgen05.ld, exchange the slice maxima through an mbarrier, and write their
// slice of P (fp16 pairs) into TMEM; a lane's P row is zero outside its
// slice, so the PV MMA (A = P from TMEM, B = V fp16 MN-major) produces one
// partial O row per replica, summed in the epilogue. O stays in TMEM across
// tiles; each thread rescales its own row when the shared running max moves
// (lazy, tau = 8 in log2 units).
template <int NPAD>
__global__ void __launch_bounds__(DCfg<NPAD>::NTHREADS, 1)
    decode_attn_kernel(const __grid_constant__ KVTileMaps tm, const DecodeParams p) {
  pdl_trigger();
  pdl_wait();  // Q, the KV pages and the block table may come from the previous kernels
  using C = DCfg<NPAD>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = align_smem_1024(smem_raw);
  uint8_t* sK = sm + C::OFF_K;
  uint8_t* sVT = sm + C::OFF_VT;
  uint8_t* sQ = sm + C::OFF_Q;
  uint8_t* sVS = sm + C::OFF_VS;
  float* sKS = reinterpret_cast<float*>(sm + C::OFF_KS);
  uint8_t* misc = sm + C::OFF_MISC;
  uint64_t* kv_full = reinterpret_cast<uint64_t*>(misc);
  uint64_t* kv_empty = kv_full + C::STAGES;  // QK commit + converter warps
  uint64_t* s_full = kv_empty + C::STAGES;   // [2] QK done
  uint64_t* s_empty = s_full + 2;            // [2] softmax read S
  uint64_t* p_full = s_empty + 2;            // [2] softmax wrote P (and rescaled O)
  uint64_t* pv_empty = p_full + 2;           // [2] PV that read P[b] done (O current)
  uint64_t* v_full = pv_empty + 2;           // [NVT] V tile converted
  uint64_t* vt_empty = v_full + C::NVT;      // [NVT] PV that read the V tile done
  uint64_t* ks_full = vt_empty + C::NVT;     // [NVT] k scales copied out
  uint64_t* mx_full = ks_full + C::NVT;      // [2] slice maxima of a tile published
  uint64_t* done_bar = mx_full + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(done_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  float* q_scale = reinterpret_cast<float*>(misc + 512);  // [64] q scale * softmax scale (log2)
  int* row_end = reinterpret_cast<int*>(q_scale + 64);     // [64] visible keys per row
  float* mx_buf = reinterpret_cast<float*>(row_end + 64);  // [2][128] slice max per lane
  float* l_buf = mx_buf + 2 * 128;                         // [128] partial row sums per lane

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int split = blockIdx.x, h = blockIdx.y + p.head_offset, seq = blockIdx.z;
  const int hl = blockIdx.y;  // head index within this launch's workspace
  const int qb = p.cu_q[seq], q_len = p.cu_q[seq + 1] - qb;
  const int R = q_len * p.gqa;  // real rows (<= 64)
  constexpr int LPR = NPAD > 32 ? 64 : 32;  // lanes per replica (rows R <= NPAD)
  constexpr int NREP = 128 / LPR;
  constexpr int KPR = TILE / NREP;          // keys per replica slice
  const int seq_len = p.seq_lens[seq];
  const int n_pages = (seq_len + PAGE - 1) / PAGE;
  const int n_tiles_all = (n_pages + TILE_PAGES - 1) / TILE_PAGES;
  const int tile_beg = (int)(((int64_t)n_tiles_all * split) / p.nsplit);
  const int tile_end = (int)(((int64_t)n_tiles_all * (split + 1)) / p.nsplit);
  const int nt = tile_end - tile_beg;
  const int32_t* bt = p.block_table + (int64_t)seq * p.bt_stride;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1 + C::NCONV);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&s_empty[b], 4);
      mbar_init(&p_full[b], 4);
      mbar_init(&pv_empty[b], 1);
      mbar_init(&mx_full[b], 4);
    }
    for (int v = 0; v < C::NVT; ++v) {
      mbar_init(&v_full[v], C::NCONV);
      mbar_init(&vt_empty[v], 1);
      mbar_init(&ks_full[v], 4);
    }
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, C::TMEM_COLS);
    tmem_relinquish();
  }
  // ---- prologue: zero the Q8 tile, then quantize the real rows into every replica (K-major SW128)
  for (int i = threadIdx.x; i < C::Q_BYTES / 16; i += C::NTHREADS)
    reinterpret_cast<uint4*>(sQ)[i] = make_uint4(0, 0, 0, 0);
  if (threadIdx.x < 64) {
    q_scale[threadIdx.x] = 0.f;
    row_end[threadIdx.x] = 0;
  }
  __syncthreads();
  for (int r = warp; r < R; r += C::NWARPS) {
    const int t = r / p.gqa, g = r % p.gqa;
    const __nv_bfloat16* src = p.q + ((int64_t)(qb + t) * p.hq_total + (int64_t)h * p.gqa + g) * D + lane * 4;
    const uint2 raw = *reinterpret_cast<const uint2*>(src);
    const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
    const float2 a = __bfloat1622float2(h2[0]), b2 = __bfloat1622float2(h2[1]);
    const float x[4] = {a.x, a.y, b2.x, b2.y};
    float amax = fmaxf(fmaxf(fabsf(x[0]), fabsf(x[1])), fmaxf(fabsf(x[2]), fabsf(x[3])));
    amax = warp_max(amax);
    const float sc = amax / 127.f;
    const float inv = sc > 0.f ? 1.f / sc : 0.f;
    uint32_t w = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int qi = (int)fminf(fmaxf(rintf(x[j] * inv), -127.f), 127.f);
      w |= ((uint32_t)(uint8_t)(int8_t)qi) << (8 * j);
    }
    for (int e = 0; e < NREP; ++e)
      *reinterpret_cast<uint32_t*>(sQ + sw128_offset(e * LPR + r, lane >> 2) + (lane & 3) * 4) = w;
    if (lane == 0) {
      q_scale[r] = sc * p.sm_scale_log2;
      row_end[r] = p.q_ends ? p.q_ends[qb + t] : (seq_len - q_len + t + 1);
    }
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // Lane i holds page i of a tile (8 pages), its id read one tile ahead.
    // Consecutive pages: lane 0 moves the tile with two TMA boxes; otherwise
    // each lane issues its page's K TMA and V + scales bulk copy.
    if (lane == 0) {
      prefetch_tmap(&tm.page);
      prefetch_tmap(&tm.k8);
      prefetch_tmap(&tm.vs8);
    }
    auto page_of = [&](int jt) -> int64_t {
      const int pg = (tile_beg + jt) * TILE_PAGES + lane;
      return (jt < nt && lane < TILE_PAGES && pg < n_pages) ? (int64_t)bt[pg] : 0;
    };
    int64_t next_page = page_of(0);
    int issued = 0;
    for (int j = 0; j < nt; ++j) {
      const int s = j % C::STAGES;
      const int64_t page = next_page;
      next_page = page_of(j + 1);
      if (j >= C::STAGES && !mbar_wait_all(&kv_empty[s], ((j / C::STAGES) - 1) & 1, abort_flag, 201)) break;
      const int pg0 = (tile_beg + j) * TILE_PAGES;
      const int npg = min(TILE_PAGES, n_pages - pg0);
      const int64_t page0 = __shfl_sync(0xffffffffu, page, 0);
      if (__all_sync(0xffffffffu, lane >= npg || page == page0 + lane)) {
        // 8-page boxes (pages past the cache arrive zero-filled; pages past
        // the sequence are masked like any key beyond its end)
        if (lane == 0) {
          mbar_arrive_expect_tx(&kv_full[s], TILE_PAGES * (K_BYTES + VS_BYTES));
          tma_load_4d(sK + s * K_TILE_BYTES, &tm.k8, &kv_full[s], 0, 0, h, (int)page0);
          tma_load_3d(sVS + s * VS_TILE_BYTES, &tm.vs8, &kv_full[s], 0, h, (int)page0);
        }
      } else {
        if (lane == 0) mbar_arrive_expect_tx(&kv_full[s], npg * (K_BYTES + VS_BYTES));
        __syncwarp();
        if (lane < npg) {
          const int64_t run = page * p.hkv + h;
          tma_load_3d(sK + s * K_TILE_BYTES + lane * K_BYTES, &tm.page, &kv_full[s], 0, 0, (int)run);
          bulk_load(sVS + s * VS_TILE_BYTES + lane * VS_BYTES, p.cache + run * HEAD_BYTES + VS_OFF, VS_BYTES,
                    &kv_full[s]);
        }
      }
      if (lane == 0) K8V4_ATRACE(0, j);
      ++issued;
    }
    if (lane == 0 && *abort_flag)
      for (int j = issued - 1; j >= 0 && j >= issued - C::STAGES; --j)
        mbar_wait_drain(&kv_full[j % C::STAGES], (j / C::STAGES) & 1);
  } else if (warp == 1) {
    // ----------------------------------------------------------------- MMA
    if (lane == 0 && nt > 0) {
      const uint32_t id_qk = idesc_s8(128, 128);
      const uint32_t id_pv = idesc_f16(128, 128, false, true);
      const uint32_t q_base = smem_u32(sQ);
      // One thread feeds the in-order tensor pipe from two queues: QK(jq)
      // as soon as its K stage landed and the softmax has loaded S of tile
      // jq - 2, PV(jp) as soon as P and V of tile jp are ready. QK thus runs
      // up to two tiles ahead instead of queueing behind PV(jq - 2), which
      // waits for the softmax. The polls are bounded like every wait.
      int jq = 0, jp = 0, idle = 0;
      uint64_t t_idle = globaltimer_ns();
      while (jp < nt) {
        bool progressed = false;
        if (jq < nt) {
          const int s = jq % C::STAGES, b = jq & 1;
          if (mbar_test_wait(&kv_full[s], (jq / C::STAGES) & 1) &&
              (jq < 2 || mbar_test_wait(&s_empty[b], ((jq >> 1) - 1) & 1))) {
            tc_fence_after();
            const uint32_t k_base = smem_u32(sK + s * K_TILE_BYTES);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              mma_i8(tmem + C::COL_S + b * 128, sdesc_sw128(q_base + kk * 32, 16, 1024),
                     sdesc_sw128(k_base + kk * 32, 16, 1024), id_qk, kk > 0 ? 1u : 0u);
            mma_commit(&s_full[b]);
            mma_commit(&kv_empty[s]);
            K8V4_ATRACE(2, jq);
            ++jq;
            progressed = true;
          }
        }
        if (jp < jq) {
          const int b = jp & 1, vb = jp % C::NVT;
          if (mbar_test_wait(&p_full[b], (jp >> 1) & 1) && mbar_test_wait(&v_full[vb], (jp / C::NVT) & 1)) {
            tc_fence_after();
            const uint32_t vt_base = smem_u32(sVT + vb * VT_BYTES);
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
              mma_f16_ts(tmem + C::COL_O, tmem + C::COL_P + b * 64 + kk * 8,
                         sdesc_sw128(vt_base + kk * 2048, VT_LBO, 1024), id_pv, (jp > 0 || kk > 0) ? 1u : 0u);
            mma_commit(&pv_empty[b]);
            mma_commit(&vt_empty[vb]);
            K8V4_ATRACE(4, jp);
            ++jp;
            progressed = true;
          }
        }
        if (progressed) {
          idle = 0;
        } else {
          // idle: yield the issue slots to this sub-partition's other warps,
          // look at the clock and the abort flag every 64 polls
          __nanosleep(20);
          if (++idle == 1) t_idle = globaltimer_ns();
          if ((idle & 63) == 0) {
            if (*abort_flag) break;
            if (globaltimer_ns() - t_idle > K8V4_WAIT_LIMIT_NS) {
              *abort_flag = 1;
              record_error(kErrMbarTimeout, 203);
              break;
            }
          }
        }
      }
      mma_commit(done_bar);
      mbar_wait_drain(done_bar, 0);
    }
  } else if (warp >= 4 && warp < 8) {
    // ---------------------------------------- softmax (lane = replica x row)
    const int quad = warp - 4;
    const int lane_id = quad * 32 + lane;  // TMEM lane
    const int rep = lane_id / LPR, r = lane_id % LPR;
    const bool real = r < R;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t tS = tmem + C::COL_S + lane_off, tP = tmem + C::COL_P + lane_off, tO = tmem + C::COL_O + lane_off;
    const float qs = real ? q_scale[r] : 0.f;
    const int end = real ? row_end[r] : 0;
    const int kofs = rep * KPR;  // this lane's key slice within a tile
    // P rows are zero outside the lane's slice: clear both P buffers once
    {
      uint32_t z[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) z[i] = 0u;
#pragma unroll
      for (int c = 0; c < 128; c += 32) tmem_st32(tP + c, z);
      tmem_st_wait();
    }
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    // Every softmax warp runs every iteration (the slice maxima are exchanged
    // each tile); a failed wait only turns the work off.
    for (int j = 0; j < nt; ++j) {
      const int b = j & 1, vb = j % C::NVT;
      if (ok && !mbar_wait_all(&s_full[b], (j >> 1) & 1, abort_flag, 207)) ok = false;
      float sc[KPR];
      if (ok) {
        tc_fence_after();
        uint32_t v[32];
        tmem_ld32(tS + b * 128 + kofs, v);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) sc[i] = i2f_small(v[i]);
        if constexpr (KPR > 32) {
          tmem_ld32(tS + b * 128 + kofs + 32, v);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) sc[32 + i] = i2f_small(v[i]);
        }
        tc_fence_before();
      }
      __syncwarp();
      if (ok && lane == 0) mbar_arrive(&s_empty[b]);
      if (ok && !mbar_wait_all(&ks_full[vb], (j / C::NVT) & 1, abort_flag, 208)) ok = false;
      const int key0 = (tile_beg + j) * TILE + kofs;
      float tmax = -INFINITY;
      if (ok) {
        const float4* ks4 = reinterpret_cast<const float4*>(sKS + vb * TILE + kofs);
        const bool full = __all_sync(0xffffffffu, end >= key0 + KPR || !real);
        float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int k = 0; k < KPR; k += 4) {
          {
            const float4 kq = ks4[k >> 2];
            float v0 = sc[k] * (qs * kq.x), v1 = sc[k + 1] * (qs * kq.y);
            float v2 = sc[k + 2] * (qs * kq.z), v3 = sc[k + 3] * (qs * kq.w);
            if (!full) {
              v0 = (key0 + k < end) ? v0 : -INFINITY;
              v1 = (key0 + k + 1 < end) ? v1 : -INFINITY;
              v2 = (key0 + k + 2 < end) ? v2 : -INFINITY;
              v3 = (key0 + k + 3 < end) ? v3 : -INFINITY;
            }
            sc[k] = v0; sc[k + 1] = v1; sc[k + 2] = v2; sc[k + 3] = v3;
            mx[0] = fmaxf(mx[0], v0); mx[1] = fmaxf(mx[1], v1);
            mx[2] = fmaxf(mx[2], v2); mx[3] = fmaxf(mx[3], v3);
          }
        }
        tmax = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
      }
      // publish the slice max, combine the row's slices (all replicas of row r)
      mx_buf[b * 128 + lane_id] = tmax;
      __syncwarp();
      if (lane == 0) mbar_arrive(&mx_full[b]);
      if (ok && !mbar_wait_all(&mx_full[b], (j >> 1) & 1, abort_flag, 213)) ok = false;
      if (ok) {
        for (int e = 0; e < NREP; ++e) tmax = fmaxf(tmax, mx_buf[b * 128 + e * LPR + r]);
        float alpha = 1.f;
        if (tmax > m + RESCALE_TAU || (m == -INFINITY && tmax > -INFINITY)) {
          alpha = (m == -INFINITY) ? 0.f : ex2_approx(m - tmax);
          m = tmax;
        }
        l *= alpha;
        // O holds PV(0..j-1) after PV(j-1): rescale it when any row of the warp moved its max
        if (j >= 1 && __any_sync(0xffffffffu, alpha != 1.f)) {
          if (!mbar_wait_all(&pv_empty[(j - 1) & 1], ((j - 1) >> 1) & 1, abort_flag, 211)) {
            ok = false;
          } else {
            tc_fence_after();
#pragma unroll
            for (int c = 0; c < D; c += 32) {
              uint32_t v[32];
              tmem_ld32(tO + c, v);
              tmem_ld_wait();
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * alpha);
              tmem_st32(tO + c, v);
            }
          }
        }
        // P[b] is free once the PV of tile j-2 finished
        if (ok && j >= 2 && !mbar_wait_all(&pv_empty[b], ((j >> 1) - 1) & 1, abort_flag, 210)) ok = false;
        if (ok) {
          tc_fence_after();
          // rows with no visible key keep m = -inf: exponentiate against 0 (all p = 0)
          const float mref = (m == -INFINITY) ? 0.f : m;
          float ls[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int hlf = 0; hlf < KPR; hlf += 32) {
            uint32_t pk[16];
#pragma unroll
            for (int k = 0; k < 32; k += 2) {
              const float p0 = ex2_approx(sc[hlf + k] - mref);
              const float p1 = ex2_approx(sc[hlf + k + 1] - mref);
              ls[(k >> 1) & 3] += p0 + p1;
              const __half2 hp = __floats2half2_rn(p0, p1);
              pk[k >> 1] = *reinterpret_cast<const uint32_t*>(&hp);
            }
            tmem_st16(tP + b * 64 + ((kofs + hlf) >> 1), pk);
          }
          l += (ls[0] + ls[1]) + (ls[2] + ls[3]);
          tmem_st_wait();
          tc_fence_before();
        }
      }
      __syncwarp();
      if (ok && lane == 0) {
        mbar_arrive(&p_full[b]);
        if (quad == 0) K8V4_ATRACE(3, j);
      }
    }
    // ------------------------------------------------------------ epilogue
    // sum the replicas' partial O rows and row sums through shared memory
    // (the K / V stage buffers are idle once the last PV finished)
    if (ok && nt > 0 && !mbar_wait_all(&pv_empty[(nt - 1) & 1], ((nt - 1) >> 1) & 1, abort_flag, 212)) ok = false;
    tc_fence_after();
    float* epi = reinterpret_cast<float*>(sm);
#pragma unroll
    for (int c = 0; c < D; c += 32) {
      uint32_t v[32];
      if (ok && nt > 0) {
        tmem_ld32(tO + c, v);
        tmem_ld_wait();
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = 0u;
      }
      float* row = epi + lane_id * C::EPI_STRIDE + c;
#pragma unroll
      for (int i = 0; i < 32; i += 4)
        *reinterpret_cast<float4*>(row + i) = make_float4(__uint_as_float(v[i]), __uint_as_float(v[i + 1]),
                                                          __uint_as_float(v[i + 2]), __uint_as_float(v[i + 3]));
    }
    l_buf[lane_id] = (ok && nt > 0) ? l : 0.f;
    if (lane_id < 64) mx_buf[lane_id] = (ok && nt > 0) ? m : -INFINITY;  // replica 0 rows (lanes < LPR)
    asm volatile("bar.sync 1, 128;" ::: "memory");
    // thread d of the 128 softmax threads writes dim d of every real row
    const int d = lane_id;
    const int64_t wsi = (((int64_t)seq * gridDim.y + hl) * p.nsplit + split);
    for (int rr = 0; rr < R; ++rr) {
      float o = 0.f, lt = 0.f;
      for (int e = 0; e < NREP; ++e) {
        o += epi[(e * LPR + rr) * C::EPI_STRIDE + d];
        lt += l_buf[e * LPR + rr];
      }
      if (p.push) {
        peer::mc_st_f32(p.ws_o + (wsi * NPAD + rr) * D + d, o);
        if (d == 0) {
          peer::mc_st_f32(p.ws_ml + (wsi * 2) * NPAD + rr, mx_buf[rr]);
          peer::mc_st_f32(p.ws_ml + (wsi * 2 + 1) * NPAD + rr, lt);
        }
      } else if (p.nsplit == 1) {
        const int t = rr / p.gqa, g = rr % p.gqa;
        p.out[((int64_t)(qb + t) * p.hq_total + (int64_t)h * p.gqa + g) * D + d] =
            __float2bfloat16_rn(lt > 0.f ? o / lt : 0.f);
      } else {
        p.ws_o[(wsi * NPAD + rr) * D + d] = o;
        if (d == 0) {
          p.ws_ml[(wsi * 2) * NPAD + rr] = mx_buf[rr];
          p.ws_ml[(wsi * 2 + 1) * NPAD + rr] = lt;
        }
      }
    }
  } else {
    // ---------------------------------------------------------- converters
    // One item = 32 dims (one scale group) of one key: a 16-byte load of
    // packed V and one scale feed four 16-byte stores of the fp16 tile.
    const int cw = (warp < 4) ? warp - 2 : warp - 6;  // warps 2, 3, 8, 9, ... -> 0 .. NCONV-1
    const int ct = cw * 32 + lane;
    constexpr int CT = C::NCONV * 32;
    for (int j = 0; j < nt; ++j) {
      const int s = j % C::STAGES;
      if (!mbar_wait_all(&kv_full[s], (j / C::STAGES) & 1, abort_flag, 205)) break;
      const int vb = j % C::NVT;
      if (j >= C::NVT && !mbar_wait_all(&vt_empty[vb], ((j / C::NVT) - 1) & 1, abort_flag, 206)) break;
      const int key0 = (tile_beg + j) * TILE;
      const int nvalid = min(TILE, seq_len - key0);
      const uint8_t* vs = sVS + s * VS_TILE_BYTES;
      uint8_t* vt = sVT + vb * VT_BYTES;
      // k scales first: the softmax of this tile needs only these
      if (cw < 4) {
        sKS[vb * TILE + ct] = (ct < nvalid) ? __half2float(*reinterpret_cast<const __half*>(
                                                  vs + (ct >> 4) * VS_BYTES + KS_OFF + (ct & 15) * 2))
                                            : 0.f;
        __syncwarp();
        if (lane == 0) mbar_arrive(&ks_full[vb]);
      }
#pragma unroll
      for (int item = ct; item < TILE * 4; item += CT) {
        const int key = item >> 2, grp = item & 3;
        if (key < nvalid) {
          const uint8_t* run = vs + (key >> 4) * VS_BYTES;
          const int kk = key & 15;
          const uint4 w = *reinterpret_cast<const uint4*>(run + kk * 64 + grp * 16);
          const __half sc = *reinterpret_cast<const __half*>(run + VSC_OFF + (kk * 4 + grp) * 2);
          v_chunk_to_f16(w.x, sc, vt, key, grp * 4);
          v_chunk_to_f16(w.y, sc, vt, key, grp * 4 + 1);
          v_chunk_to_f16(w.z, sc, vt, key, grp * 4 + 2);
          v_chunk_to_f16(w.w, sc, vt, key, grp * 4 + 3);
        } else {
#pragma unroll
          for (int q = 0; q < 4; ++q) v_chunk_zero(vt, key, grp * 4 + q);
        }
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&v_full[vb]);
        mbar_arrive(&kv_empty[s]);
        if (ct < 32) K8V4_ATRACE(1, j);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
  if (p.push && threadIdx.x == 0) {
    // the CTA's multicast stores (ordered before this point by the barrier)
    // are out: publish them to every rank
    peer::fence_proxy_alias();
    peer::mc_signal_add_u64(p.flag_mc, 1ull);
  }
}

// ---------------------------------------------------------------------------
// Keys on TMEM lanes, query rows as the MMA N dimension (rows <= 16).
//
// With a handful of query rows per KV head (one decode token x GQA 6 at
// c = 1), an MMA with the rows as M wastes most of its 128 lanes: QK and PV
// of one 128-key tile then cost the tensor pipe ~800 cycles. Here the keys
// (QK) and the head dims (PV) are M and the rows are N = 16:
//
//   S^T[key, row] = K_tile (A, smem, K-major) x Q8^T (B, smem)  kind::i8, N = 16
//   softmax       : thread = key (4 warps = 128 TMEM lanes) holding its 16
//                   row scores; per-row tile maxima through redux.sync on an
//                   order-preserving integer image of the floats, then shared
//                   memory across the 4 warps; lazy rescale (tau = 8, log2)
//   P^T           : each thread writes its key's fp16 probabilities into the
//                   K-major B operand [16 rows x 128 keys] in shared memory
//   O^T[dim, row] += V^T (A, the converted fp16 tile, MN-major) x P^T (B)
//                   kind::f16, N = 16; O^T stays in TMEM (16 columns)
//
// so a tile costs the tensor pipe ~100 cycles. The row sums stay per thread
// until the epilogue. The producer, the V converters and the (m, l, O)
// partial layout are the rows-on-lanes kernel's (decode_attn_kernel), so
// decode_combine merges either kernel's splits.
template <int NPAD>
struct TCfg {
  static constexpr int STAGES = 4;
  static constexpr int NVT = 3;
  static constexpr int NCONV = K8V4_DECODE_NCONV;
  static constexpr int NWARPS = 8 + (NCONV - 2);
  static constexpr int NTHREADS = 32 * NWARPS;
  static constexpr int Q_BYTES = NPAD * 128;         // Q8 rows, K-major SW128 (NPAD % 8 == 0)
  static constexpr int P_ATOM = NPAD * 128;          // 64 keys of every row (fp16), K-major SW128
  static constexpr int P_BYTES = 2 * P_ATOM;         // one P^T buffer: 128 keys
  static constexpr uint32_t COL_S = 0, COL_O = 2 * NPAD;
  static constexpr int TMEM_COLS = (3 * NPAD <= 32) ? 32 : (3 * NPAD <= 64 ? 64 : 128);
  static constexpr int OFF_K = 0;
  static constexpr int OFF_VT = OFF_K + STAGES * K_TILE_BYTES;
  static constexpr int OFF_Q = OFF_VT + NVT * VT_BYTES;
  static constexpr int OFF_P = OFF_Q + ((Q_BYTES + 1023) / 1024) * 1024;
  static constexpr int OFF_VS = OFF_P + 2 * P_BYTES;
  static constexpr int OFF_KS = OFF_VS + STAGES * VS_TILE_BYTES;
  static constexpr int OFF_MISC = OFF_KS + NVT * TILE * 4;
  // misc: barriers (512 B), q_scale / row_end [NPAD], tile maxima [2][4][NPAD], row sums [4][NPAD]
  static constexpr int SMEM_BYTES = 1024 + OFF_MISC + 512 + 2 * NPAD * 4 + 2 * 4 * NPAD * 4 + 4 * NPAD * 4;
  static_assert(NPAD % 16 == 0 && NPAD <= 32, "rows as MMA N");
  static_assert(SMEM_BYTES <= 232448, "shared memory per CTA");
};

// Order-preserving map float -> int32 (and back): redux.sync works on integers.
__device__ __forceinline__ int f2ord(float f) {
  const int i = __float_as_int(f);
  return i >= 0 ? i : (i ^ 0x7FFFFFFF);
}
__device__ __forceinline__ float ord2f(int i) { return __int_as_float(i >= 0 ? i : (i ^ 0x7FFFFFFF)); }
__device__ __forceinline__ int redux_max(int v) {
  int r;
  asm volatile("redux.sync.max.s32 %0, %1, 0xffffffff;" : "=r"(r) : "r"(v));
  return r;
}

template <int NPAD>
__global__ void __launch_bounds__(TCfg<NPAD>::NTHREADS, 1)
    decode_attn_t_kernel(const __grid_constant__ KVTileMaps tm, const DecodeParams p) {
  pdl_trigger();
  pdl_wait();  // Q, the KV pages and the block table may come from the previous kernels
  using C = TCfg<NPAD>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = align_smem_1024(smem_raw);
  uint8_t* sK = sm + C::OFF_K;
  uint8_t* sVT = sm + C::OFF_VT;
  uint8_t* sQ = sm + C::OFF_Q;
  uint8_t* sP = sm + C::OFF_P;
  uint8_t* sVS = sm + C::OFF_VS;
  float* sKS = reinterpret_cast<float*>(sm + C::OFF_KS);
  uint8_t* misc = sm + C::OFF_MISC;
  uint64_t* kv_full = reinterpret_cast<uint64_t*>(misc);
  uint64_t* kv_empty = kv_full + C::STAGES;  // QK commit + converter warps
  uint64_t* s_full = kv_empty + C::STAGES;   // [2] QK done
  uint64_t* s_empty = s_full + 2;            // [2] softmax read S
  uint64_t* p_full = s_empty + 2;            // [2] softmax wrote P^T (and rescaled O)
  uint64_t* pv_done = p_full + 2;            // [2] PV that read P^T[b] done (O current)
  uint64_t* v_full = pv_done + 2;            // [NVT] V tile converted
  uint64_t* vt_empty = v_full + C::NVT;      // [NVT] PV that read the V tile done
  uint64_t* ks_full = vt_empty + C::NVT;     // [NVT] k scales copied out
  uint64_t* done_bar = ks_full + C::NVT;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(done_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  float* q_scale = reinterpret_cast<float*>(misc + 512);  // [NPAD] q scale * softmax scale (log2)
  int* row_end = reinterpret_cast<int*>(q_scale + NPAD);  // [NPAD] visible keys per row
  float* mx_w = reinterpret_cast<float*>(row_end + NPAD); // [2][4][NPAD] per-warp tile maxima
  float* l_w = mx_w + 2 * 4 * NPAD;                        // [4][NPAD] per-warp row sums

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int split = blockIdx.x, h = blockIdx.y + p.head_offset, seq = blockIdx.z;
  const int hl = blockIdx.y;
  const int qb = p.cu_q[seq], q_len = p.cu_q[seq + 1] - qb;
  const int R = q_len * p.gqa;  // real rows (<= NPAD)
  const int seq_len = p.seq_lens[seq];
  const int n_pages = (seq_len + PAGE - 1) / PAGE;
  const int n_tiles_all = (n_pages + TILE_PAGES - 1) / TILE_PAGES;
  const int tile_beg = (int)(((int64_t)n_tiles_all * split) / p.nsplit);
  const int tile_end = (int)(((int64_t)n_tiles_all * (split + 1)) / p.nsplit);
  const int nt = tile_end - tile_beg;
  const int32_t* bt = p.block_table + (int64_t)seq * p.bt_stride;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1 + C::NCONV);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&s_empty[b], 4);
      mbar_init(&p_full[b], 4);
      mbar_init(&pv_done[b], 1);
    }
    for (int v = 0; v < C::NVT; ++v) {
      mbar_init(&v_full[v], C::NCONV);
      mbar_init(&vt_empty[v], 1);
      mbar_init(&ks_full[v], 4);
    }
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, C::TMEM_COLS);
    tmem_relinquish();
  }
  // ---- prologue: zero the Q8 tile, then quantize the real rows (K-major SW128)
  for (int i = threadIdx.x; i < C::Q_BYTES / 16; i += C::NTHREADS)
    reinterpret_cast<uint4*>(sQ)[i] = make_uint4(0, 0, 0, 0);
  if (threadIdx.x < NPAD) {
    q_scale[threadIdx.x] = 0.f;
    row_end[threadIdx.x] = 0;
  }
  __syncthreads();
  for (int r = warp; r < R; r += C::NWARPS) {
    const int t = r / p.gqa, g = r % p.gqa;
    const __nv_bfloat16* src = p.q + ((int64_t)(qb + t) * p.hq_total + (int64_t)h * p.gqa + g) * D + lane * 4;
    const uint2 raw = *reinterpret_cast<const uint2*>(src);
    const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
    const float2 a = __bfloat1622float2(h2[0]), b2 = __bfloat1622float2(h2[1]);
    const float x[4] = {a.x, a.y, b2.x, b2.y};
    float amax = fmaxf(fmaxf(fabsf(x[0]), fabsf(x[1])), fmaxf(fabsf(x[2]), fabsf(x[3])));
    amax = warp_max(amax);
    const float sc = amax / 127.f;
    const float inv = sc > 0.f ? 1.f / sc : 0.f;
    uint32_t w = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int qi = (int)fminf(fmaxf(rintf(x[j] * inv), -127.f), 127.f);
      w |= ((uint32_t)(uint8_t)(int8_t)qi) << (8 * j);
    }
    *reinterpret_cast<uint32_t*>(sQ + sw128_offset(r, lane >> 2) + (lane & 3) * 4) = w;
    if (lane == 0) {
      q_scale[r] = sc * p.sm_scale_log2;
      row_end[r] = p.q_ends ? p.q_ends[qb + t] : (seq_len - q_len + t + 1);
    }
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // (as in decode_attn_kernel) lane i holds page i of a tile, read one tile
    // ahead; consecutive pages move in two TMA boxes, others page by page
    if (lane == 0) {
      prefetch_tmap(&tm.page);
      prefetch_tmap(&tm.k8);
      prefetch_tmap(&tm.vs8);
    }
    auto page_of = [&](int jt) -> int64_t {
      const int pg = (tile_beg + jt) * TILE_PAGES + lane;
      return (jt < nt && lane < TILE_PAGES && pg < n_pages) ? (int64_t)bt[pg] : 0;
    };
    int64_t next_page = page_of(0);
    int issued = 0;
    for (int j = 0; j < nt; ++j) {
      const int s = j % C::STAGES;
      const int64_t page = next_page;
      next_page = page_of(j + 1);
      if (j >= C::STAGES && !mbar_wait_all_backoff(&kv_empty[s], ((j / C::STAGES) - 1) & 1, abort_flag, 221, 64))
        break;
      const int pg0 = (tile_beg + j) * TILE_PAGES;
      const int npg = min(TILE_PAGES, n_pages - pg0);
      const int64_t page0 = __shfl_sync(0xffffffffu, page, 0);
      if (__all_sync(0xffffffffu, lane >= npg || page == page0 + lane)) {
        if (lane == 0) {
          mbar_arrive_expect_tx(&kv_full[s], TILE_PAGES * (K_BYTES + VS_BYTES));
          tma_load_4d(sK + s * K_TILE_BYTES, &tm.k8, &kv_full[s], 0, 0, h, (int)page0);
          tma_load_3d(sVS + s * VS_TILE_BYTES, &tm.vs8, &kv_full[s], 0, h, (int)page0);
        }
      } else {
        if (lane == 0) mbar_arrive_expect_tx(&kv_full[s], npg * (K_BYTES + VS_BYTES));
        __syncwarp();
        if (lane < npg) {
          const int64_t run = page * p.hkv + h;
          tma_load_3d(sK + s * K_TILE_BYTES + lane * K_BYTES, &tm.page, &kv_full[s], 0, 0, (int)run);
          bulk_load(sVS + s * VS_TILE_BYTES + lane * VS_BYTES, p.cache + run * HEAD_BYTES + VS_OFF, VS_BYTES,
                    &kv_full[s]);
        }
      }
      if (lane == 0) K8V4_ATRACE(0, j);
      ++issued;
    }
    if (lane == 0 && *abort_flag)
      for (int j = issued - 1; j >= 0 && j >= issued - C::STAGES; --j)
        mbar_wait_drain(&kv_full[j % C::STAGES], (j / C::STAGES) & 1);
  } else if (warp == 1) {
    // ----------------------------------------------------------------- MMA
    if (lane == 0 && nt > 0) {
      const uint32_t id_qk = idesc_s8(128, NPAD);                 // M = keys, N = rows
      const uint32_t id_pv = idesc_f16(128, NPAD, true, false);   // M = dims (MN-major V), N = rows
      const uint32_t q_base = smem_u32(sQ);
      const uint32_t p_base = smem_u32(sP);
      int jq = 0, jp = 0, idle = 0;
      uint64_t t_idle = globaltimer_ns();
      while (jp < nt) {
        bool progressed = false;
        if (jq < nt) {
          const int s = jq % C::STAGES, b = jq & 1;
          if (mbar_test_wait(&kv_full[s], (jq / C::STAGES) & 1) &&
              (jq < 2 || mbar_test_wait(&s_empty[b], ((jq >> 1) - 1) & 1))) {
            tc_fence_after();
            const uint32_t k_base = smem_u32(sK + s * K_TILE_BYTES);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              mma_i8(tmem + C::COL_S + b * NPAD, sdesc_sw128(k_base + kk * 32, 16, 1024),
                     sdesc_sw128(q_base + kk * 32, 16, 1024), id_qk, kk > 0 ? 1u : 0u);
            mma_commit(&s_full[b]);
            mma_commit(&kv_empty[s]);
            K8V4_ATRACE(2, jq);
            ++jq;
            progressed = true;
          }
        }
        if (jp < jq) {
          const int b = jp & 1, vb = jp % C::NVT;
          if (mbar_test_wait(&p_full[b], (jp >> 1) & 1) && mbar_test_wait(&v_full[vb], (jp / C::NVT) & 1)) {
            tc_fence_after();
            const uint32_t vt_base = smem_u32(sVT + vb * VT_BYTES);
            const uint32_t pb = p_base + b * C::P_BYTES;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
              mma_f16(tmem + C::COL_O, sdesc_sw128(vt_base + kk * 2048, VT_LBO, 1024),
                      sdesc_sw128(pb + (kk >> 2) * C::P_ATOM + (kk & 3) * 32, 16, 1024), id_pv,
                      (jp > 0 || kk > 0) ? 1u : 0u);
            mma_commit(&pv_done[b]);
            mma_commit(&vt_empty[vb]);
            K8V4_ATRACE(4, jp);
            ++jp;
            progressed = true;
          }
        }
        if (progressed) {
          idle = 0;
        } else {
          __nanosleep(20);
          if (++idle == 1) t_idle = globaltimer_ns();
          if ((idle & 63) == 0) {
            if (*abort_flag) break;
            if (globaltimer_ns() - t_idle > K8V4_WAIT_LIMIT_NS) {
              *abort_flag = 1;
              record_error(kErrMbarTimeout, 223);
              break;
            }
          }
        }
      }
      mma_commit(done_bar);
      mbar_wait_drain(done_bar, 0);
    }
  } else if (warp >= 4 && warp < 8) {
    // ------------------------------------------------- softmax (lane = key)
    const int quad = warp - 4;
    const int key = quad * 32 + lane;  // TMEM lane: key of the tile (S^T), head dim (O^T)
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t tS = tmem + C::COL_S + lane_off, tO = tmem + C::COL_O + lane_off;
    float qs[NPAD], m[NPAD], l[NPAD];
    int rend[NPAD];
#pragma unroll
    for (int r = 0; r < NPAD; ++r) {
      qs[r] = q_scale[r];
      rend[r] = row_end[r];  // 0 past the real rows: no key visible
      m[r] = -INFINITY;
      l[r] = 0.f;
    }
    // this thread's key inside a P^T buffer (K-major SW128, 64-key atoms)
    const int patom = (key >> 6) * C::P_ATOM, pchunk = (key & 63) >> 3, pbyte = (key & 7) * 2;
    bool ok = true;
    // Every softmax warp runs every iteration (the tile maxima meet at a
    // named barrier); a failed wait only turns the work off.
    for (int j = 0; j < nt; ++j) {
      const int b = j & 1, vb = j % C::NVT;
      if (ok && !mbar_wait_all(&s_full[b], (j >> 1) & 1, abort_flag, 224)) ok = false;
      uint32_t sv[NPAD];
      if (ok) {
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < NPAD; c += 16) tmem_ld16(tS + b * NPAD + c, *reinterpret_cast<uint32_t(*)[16]>(&sv[c]));
        tmem_ld_wait();
        tc_fence_before();
      }
      __syncwarp();
      if (ok && lane == 0) mbar_arrive(&s_empty[b]);
      if (quad == 0 && lane == 0) K8V4_ATRACE(5, j);
      if (ok && !mbar_wait_all(&ks_full[vb], (j / C::NVT) & 1, abort_flag, 225)) ok = false;
      const int keyg = (tile_beg + j) * TILE + key;
      const float ks = ok ? sKS[vb * TILE + key] : 0.f;
      float s[NPAD];
#pragma unroll
      for (int r = 0; r < NPAD; ++r)
        if (r < R) s[r] = (ok && keyg < rend[r]) ? i2f_small(sv[r]) * (qs[r] * ks) : -INFINITY;
      float* mxb = mx_w + b * 4 * NPAD;
#pragma unroll
      for (int r = 0; r < NPAD; ++r)
        if (r < R) {
          const int wm = redux_max(f2ord(s[r]));
          if (lane == r) mxb[quad * NPAD + r] = ord2f(wm);
        }
      asm volatile("bar.sync 1, 128;" ::: "memory");  // the four warps' maxima of tile j
      if (quad == 0 && lane == 0) K8V4_ATRACE(6, j);
      float alpha[NPAD];
      bool moved = false;
#pragma unroll
      for (int r = 0; r < NPAD; ++r) {
        alpha[r] = 1.f;
        if (r < R) {
          const float tmax = fmaxf(fmaxf(mxb[r], mxb[NPAD + r]), fmaxf(mxb[2 * NPAD + r], mxb[3 * NPAD + r]));
          if (tmax > m[r] + RESCALE_TAU || (m[r] == -INFINITY && tmax > -INFINITY)) {
            alpha[r] = (m[r] == -INFINITY) ? 0.f : ex2_approx(m[r] - tmax);
            m[r] = tmax;
            moved = true;
          }
          l[r] *= alpha[r];
        }
      }
      // O^T holds PV(0..j-1) after PV(j-1): rescale its row columns when a max moved
      // (`moved` is the same in every thread: all read the same maxima)
      if (ok && j >= 1 && moved) {
        if (!mbar_wait_all(&pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1, abort_flag, 226)) {
          ok = false;
        } else {
          tc_fence_after();
          uint32_t ov[NPAD];
#pragma unroll
          for (int c = 0; c < NPAD; c += 16) tmem_ld16(tO + c, *reinterpret_cast<uint32_t(*)[16]>(&ov[c]));
          tmem_ld_wait();
#pragma unroll
          for (int r = 0; r < NPAD; ++r) ov[r] = __float_as_uint(__uint_as_float(ov[r]) * alpha[r]);
#pragma unroll
          for (int c = 0; c < NPAD; c += 16) tmem_st16(tO + c, *reinterpret_cast<uint32_t(*)[16]>(&ov[c]));
          tmem_st_wait();
        }
      }
      // P^T[b] is free once the PV of tile j-2 finished
      if (ok && j >= 2 && !mbar_wait_all(&pv_done[b], ((j >> 1) - 1) & 1, abort_flag, 227)) ok = false;
      if (quad == 0 && lane == 0) K8V4_ATRACE(7, j);
      if (ok) {
        // rows past R are never read back (their O^T columns are ignored)
        uint8_t* pt = sP + b * C::P_BYTES + patom;
#pragma unroll
        for (int r = 0; r < NPAD; ++r)
          if (r < R) {
            // rows with no visible key keep m = -inf: exponentiate against 0 (p = 0)
            const float pr = ex2_approx(s[r] - (m[r] == -INFINITY ? 0.f : m[r]));
            l[r] += pr;
            *reinterpret_cast<__half*>(pt + sw128_offset(r, pchunk) + pbyte) = __float2half_rn(pr);
          }
        fence_async_smem();  // the tensor core reads P^T through the async proxy
        tc_fence_before();
      }
      __syncwarp();
      if (ok && lane == 0) {
        mbar_arrive(&p_full[b]);
        if (quad == 0) K8V4_ATRACE(3, j);
      }
    }
    // ------------------------------------------------------------ epilogue
    if (ok && nt > 0 && !mbar_wait_all(&pv_done[(nt - 1) & 1], ((nt - 1) >> 1) & 1, abort_flag, 228)) ok = false;
#pragma unroll
    for (int r = 0; r < NPAD; ++r)
      if (r < R) {
        const float ls = warp_sum(l[r]);
        if (lane == 0) l_w[quad * NPAD + r] = ls;
      }
    asm volatile("bar.sync 1, 128;" ::: "memory");
    tc_fence_after();
    uint32_t ov[NPAD];
    const bool have = ok && nt > 0;
    if (have) {
#pragma unroll
      for (int c = 0; c < NPAD; c += 16) tmem_ld16(tO + c, *reinterpret_cast<uint32_t(*)[16]>(&ov[c]));
      tmem_ld_wait();
    } else {
#pragma unroll
      for (int r = 0; r < NPAD; ++r) ov[r] = 0u;
    }
    // thread d of the 128 softmax threads writes dim d of every real row
    const int d = key;
    const int64_t wsi = (((int64_t)seq * gridDim.y + hl) * p.nsplit + split);
#pragma unroll
    for (int rr = 0; rr < NPAD; ++rr) {
      if (rr >= R) break;
      const float o = __uint_as_float(ov[rr]);
      const float lt = have ? (l_w[rr] + l_w[NPAD + rr]) + (l_w[2 * NPAD + rr] + l_w[3 * NPAD + rr]) : 0.f;
      const float mr = have ? m[rr] : -INFINITY;
      if (p.push) {
        peer::mc_st_f32(p.ws_o + (wsi * NPAD + rr) * D + d, o);
        if (d == 0) {
          peer::mc_st_f32(p.ws_ml + (wsi * 2) * NPAD + rr, mr);
          peer::mc_st_f32(p.ws_ml + (wsi * 2 + 1) * NPAD + rr, lt);
        }
      } else if (p.nsplit == 1) {
        const int t = rr / p.gqa, g = rr % p.gqa;
        p.out[((int64_t)(qb + t) * p.hq_total + (int64_t)h * p.gqa + g) * D + d] =
            __float2bfloat16_rn(lt > 0.f ? o / lt : 0.f);
      } else {
        p.ws_o[(wsi * NPAD + rr) * D + d] = o;
        if (d == 0) {
          p.ws_ml[(wsi * 2) * NPAD + rr] = mr;
          p.ws_ml[(wsi * 2 + 1) * NPAD + rr] = lt;
        }
      }
    }
  } else {
    // ---------------------------------------------------------- converters
    // (as in decode_attn_kernel) one item = 32 dims (one scale group) of one key
    const int cw = (warp < 4) ? warp - 2 : warp - 6;  // warps 2, 3, 8, 9, ... -> 0 .. NCONV-1
    const int ct = cw * 32 + lane;
    constexpr int CT = C::NCONV * 32;
    for (int j = 0; j < nt; ++j) {
      const int s = j % C::STAGES;
      if (!mbar_wait_all_backoff(&kv_full[s], (j / C::STAGES) & 1, abort_flag, 229, 64)) break;
      const int vb = j % C::NVT;
      if (j >= C::NVT && !mbar_wait_all_backoff(&vt_empty[vb], ((j / C::NVT) - 1) & 1, abort_flag, 230, 64)) break;
      const int key0 = (tile_beg + j) * TILE;
      const int nvalid = min(TILE, seq_len - key0);
      const uint8_t* vs = sVS + s * VS_TILE_BYTES;
      uint8_t* vt = sVT + vb * VT_BYTES;
      if (cw < 4) {
        sKS[vb * TILE + ct] = (ct < nvalid) ? __half2float(*reinterpret_cast<const __half*>(
                                                  vs + (ct >> 4) * VS_BYTES + KS_OFF + (ct & 15) * 2))
                                            : 0.f;
        __syncwarp();
        if (lane == 0) mbar_arrive(&ks_full[vb]);
      }
#pragma unroll
      for (int item = ct; item < TILE * 4; item += CT) {
        const int key = item >> 2, grp = item & 3;
        if (key < nvalid) {
          const uint8_t* run = vs + (key >> 4) * VS_BYTES;
          const int kk = key & 15;
          const uint4 w = *reinterpret_cast<const uint4*>(run + kk * 64 + grp * 16);
          const __half sc = *reinterpret_cast<const __half*>(run + VSC_OFF + (kk * 4 + grp) * 2);
          v_chunk_to_f16(w.x, sc, vt, key, grp * 4);
          v_chunk_to_f16(w.y, sc, vt, key, grp * 4 + 1);
          v_chunk_to_f16(w.z, sc, vt, key, grp * 4 + 2);
          v_chunk_to_f16(w.w, sc, vt, key, grp * 4 + 3);
        } else {
#pragma unroll
          for (int q = 0; q < 4; ++q) v_chunk_zero(vt, key, grp * 4 + q);
        }
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&v_full[vb]);
        mbar_arrive(&kv_empty[s]);
        if (ct < 32) K8V4_ATRACE(1, j);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
  if (p.push && threadIdx.x == 0) {
    peer::fence_proxy_alias();
    peer::mc_signal_add_u64(p.flag_mc, 1ull);
  }
}

// Merge split partials: grid (rows, heads, seqs), 128 threads (dims). The
// per-split weights are computed once by the block; the O loads of all splits
// are independent, so their latencies overlap. Context parallelism adds a
// rank dimension: split index s of the merged set is (rank s / nsplit, split
// s % nsplit), each rank's partials `rank_stride_*` floats apart (the
// all-gathered workspaces of every rank).
// Merge the split partials of one query row: threads (group g, dim d), group
// g takes splits g, g + 4, ... so every O load of the row is in flight at
// once; the groups' sums meet in shared memory.
constexpr int COMBINE_GROUPS = 4;
// NC: the partials were written before this launch (read-only data path);
// otherwise they arrived from peers during it (plain coherent loads).
template <bool NC>
__device__ __forceinline__ float ld_part(const float* p) {
  if constexpr (NC) return __ldg(p);
  else return *p;
}

template <bool NC>
__device__ __forceinline__ void combine_row(const float* ws_o, const float* ws_ml, __nv_bfloat16* out, int r, int hl,
                                            int seq, int qb, int nsplit, int npad, int gqa, int hq_total,
                                            int head_offset, int nrank, int64_t rank_stride_o,
                                            int64_t rank_stride_ml) {
  __shared__ float wsh[128];
  __shared__ float red[8];
  __shared__ float part[COMBINE_GROUPS - 1][D];
  const int d = threadIdx.x & (D - 1), grp = threadIdx.x / D;
  const int64_t base = ((int64_t)seq * gridDim.y + hl) * nsplit;
  const int ntot = nsplit * nrank;  // <= 128
  // (m, l) of every split: threads of group 0, one split each
  float m = -INFINITY, l = 0.f;
  if (grp == 0 && d < ntot) {
    const int rk = d / nsplit, sp = d % nsplit;
    const float* ml = ws_ml + rk * rank_stride_ml;
    m = ld_part<NC>(ml + ((base + sp) * 2) * npad + r);
    l = ld_part<NC>(ml + ((base + sp) * 2 + 1) * npad + r);
  }
  if (grp == 0) {
    const float M0 = warp_max(m);
    if ((d & 31) == 0) red[d >> 5] = M0;
  }
  __syncthreads();
  const float M = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  float L = 0.f;
  if (grp == 0) {
    const float w = (m == -INFINITY || M == -INFINITY) ? 0.f : exp2f(m - M);
    if (d < ntot) wsh[d] = w;
    const float Lw = warp_sum(w * l);
    if ((d & 31) == 0) red[4 + (d >> 5)] = Lw;
  }
  __syncthreads();
  L = red[4] + red[5] + red[6] + red[7];
  const int64_t stride = (int64_t)npad * D;
  float acc = 0.f;
  for (int rk = 0; rk < nrank; ++rk) {
    const float* o = ws_o + rk * rank_stride_o + (base * npad + r) * D + d;
    const float* wr = wsh + rk * nsplit;
    int s = grp;
    for (; s + 7 * COMBINE_GROUPS < nsplit; s += 8 * COMBINE_GROUPS) {
      float v[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = ld_part<NC>(o + (s + i * COMBINE_GROUPS) * stride);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float wi = wr[s + i * COMBINE_GROUPS];
        acc += wi > 0.f ? wi * v[i] : 0.f;
      }
    }
    for (; s < nsplit; s += COMBINE_GROUPS) acc += wr[s] > 0.f ? wr[s] * ld_part<NC>(o + s * stride) : 0.f;
  }
  if (grp > 0) part[grp - 1][d] = acc;
  __syncthreads();
  if (grp == 0) {
#pragma unroll
    for (int g = 0; g < COMBINE_GROUPS - 1; ++g) acc += part[g][d];
    const int t = r / gqa, g = r % gqa, h = hl + head_offset;
    out[((int64_t)(qb + t) * hq_total + (int64_t)h * gqa + g) * D + d] = __float2bfloat16_rn(L > 0.f ? acc / L : 0.f);
  }
}

__global__ void __launch_bounds__(128 * COMBINE_GROUPS) decode_combine_kernel(
    const float* __restrict__ ws_o, const float* __restrict__ ws_ml, const int32_t* cu_q, __nv_bfloat16* out,
    int nsplit, int npad, int gqa, int hq_total, int head_offset, int nrank, int64_t rank_stride_o,
    int64_t rank_stride_ml) {
  pdl_trigger();
  pdl_wait();  // everything this kernel reads may come from the previous one
  const int r = blockIdx.x, hl = blockIdx.y, seq = blockIdx.z;
  const int qb = cu_q[seq], q_len = cu_q[seq + 1] - qb;
  if (r >= q_len * gqa) return;  // uniform for the CTA
  combine_row<true>(ws_o, ws_ml, out, r, hl, seq, qb, nsplit, npad, gqa, hq_total, head_offset, nrank,
                    rank_stride_o, rank_stride_ml);
}

// The same merge over every rank's slot of a symmetric gather buffer that
// the ranks' decode kernels fill with multicast stores (`ws_all` is this
// rank's copy). Every CTA, rows past a sequence's end included, waits until
// all ranks' CTAs have signalled; the last CTA advances the running count.
__global__ void __launch_bounds__(128 * COMBINE_GROUPS) decode_combine_sync_kernel(
    const float* ws_o, const float* ws_ml, const int32_t* cu_q, __nv_bfloat16* out, int nsplit, int npad, int gqa,
    int hq_total, int head_offset, int nrank, int64_t rank_stride, peer::ReduceSync sync) {
  pdl_trigger();
  pdl_wait();
  const int r = blockIdx.x, hl = blockIdx.y, seq = blockIdx.z;
  const int qb = cu_q[seq], q_len = cu_q[seq + 1] - qb;
  peer::sync_wait(sync, 213);
  if (r < q_len * gqa)  // uniform for the CTA
    combine_row<false>(ws_o, ws_ml, out, r, hl, seq, qb, nsplit, npad, gqa, hq_total, head_offset, nrank,
                       rank_stride, rank_stride);
  peer::sync_done(sync);
}

}  // namespace attn
}  // namespace k8v4

using namespace k8v4;
using namespace k8v4::attn;

namespace {
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}
}  // namespace

// 3D map over the cache's K rows: (128 bytes, 16 tokens, page*hkv + head), 128B swizzle.
extern "C" int k8v4_make_kv_tmap(void* map_out, const void* cache, int64_t num_pages, int hkv) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return -1;
  cuuint64_t dims[3] = {128, 16, (cuuint64_t)(num_pages * hkv)};
  cuuint64_t strides[2] = {128, HEAD_BYTES};
  cuuint32_t box[3] = {128, 16, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(reinterpret_cast<CUtensorMap*>(map_out), CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(cache),
                   dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -2;
}

// All three maps of a cache (KVTileMaps).
extern "C" int k8v4_make_kv_maps(void* maps_out, const void* cache, int64_t num_pages, int hkv) {
  KVTileMaps* m = reinterpret_cast<KVTileMaps*>(maps_out);
  if (k8v4_make_kv_tmap(&m->page, cache, num_pages, hkv)) return -3;
  EncodeTiledFn enc = encode_fn();
  if (!enc) return -1;
  {
    // K: (128 bytes, 16 rows, hkv heads, pages), box = one head's rows of 8 pages
    cuuint64_t dims[4] = {128, 16, (cuuint64_t)hkv, (cuuint64_t)num_pages};
    cuuint64_t strides[3] = {128, HEAD_BYTES, (cuuint64_t)hkv * HEAD_BYTES};
    cuuint32_t box[4] = {128, 16, 1, TILE_PAGES};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = enc(&m->k8, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<void*>(cache), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return -4;
  }
  {
    // V + scales: (148 x 8 bytes, hkv heads, pages) from VS_OFF, box = 8 pages of one head
    cuuint64_t dims[3] = {VS_BYTES / 8, (cuuint64_t)hkv, (cuuint64_t)num_pages};
    cuuint64_t strides[2] = {HEAD_BYTES, (cuuint64_t)hkv * HEAD_BYTES};
    cuuint32_t box[3] = {VS_BYTES / 8, 1, TILE_PAGES};
    cuuint32_t estr[3] = {1, 1, 1};
    void* base = const_cast<uint8_t*>(reinterpret_cast<const uint8_t*>(cache)) + VS_OFF;
    CUresult r = enc(&m->vs8, CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, base, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return -5;
  }
  return 0;
}

K8V4_STATUS_API(decode)

#ifdef K8V4_TRACE
extern "C" int k8v4_attn_trace(uint64_t* host) {
  return cudaMemcpyFromSymbol(host, g_attn_trace, sizeof(uint64_t) * 8 * 256);
}
#endif

template <int NPAD>
static int launch_decode(const KVTileMaps& tm, const DecodeParams& p, int heads, int nseq, cudaStream_t st) {
  using C = DCfg<NPAD>;
  if (ensure_smem_limit<decode_attn_kernel<NPAD>>(C::SMEM_BYTES) != cudaSuccess) return 10;
  dim3 grid(p.nsplit, heads, nseq);
  return launch_k(decode_attn_kernel<NPAD>, grid, dim3(C::NTHREADS), C::SMEM_BYTES, st, tm, p) == cudaSuccess ? 0 : 10;
}

template <int NPAD>
static int launch_decode_t(const KVTileMaps& tm, const DecodeParams& p, int heads, int nseq, cudaStream_t st) {
  using C = TCfg<NPAD>;
  if (ensure_smem_limit<decode_attn_t_kernel<NPAD>>(C::SMEM_BYTES) != cudaSuccess) return 10;
  dim3 grid(p.nsplit, heads, nseq);
  return launch_k(decode_attn_t_kernel<NPAD>, grid, dim3(C::NTHREADS), C::SMEM_BYTES, st, tm, p) == cudaSuccess ? 0
                                                                                                            : 10;
}

// Launches of at most 16 query rows per KV head run keys-on-lanes
// (decode_attn_t_kernel) with K8V4_DECODE_ATTN_T=1; rows on lanes otherwise.
// (Read at every launch, so a process can switch between the two.)
static bool keys_on_lanes() {
  const char* v = getenv("K8V4_DECODE_ATTN_T");
  return v && (v[0] == '1' || v[0] == 'y' || v[0] == 'Y' || v[0] == 't' || v[0] == 'T');
}

namespace {
// Builds the parameters and launches the decode kernel; the npad the launch
// used comes back in *npad_out.
int decode_core(const void* q, const int32_t* cu_q, const int32_t* seq_lens, const int32_t* q_ends,
                const int32_t* block_table, int bt_stride, const void* cache, int64_t num_pages, int hkv,
                int head_offset, int heads, int gqa, int hq_total, int nseq, int max_q_len, int nsplit,
                float sm_scale, void* out, float* ws_o, float* ws_ml, unsigned long long* flag_mc, int* npad_out,
                cudaStream_t st) {
  const int rows = max_q_len * gqa;
  KVTileMaps tm;
  if (k8v4_make_kv_maps(&tm, cache, num_pages, hkv)) return 3;
  DecodeParams p;
  p.q = reinterpret_cast<const __nv_bfloat16*>(q);
  p.cu_q = cu_q;
  p.seq_lens = seq_lens;
  p.q_ends = q_ends;
  p.block_table = block_table;
  p.cache = reinterpret_cast<const uint8_t*>(cache);
  p.out = reinterpret_cast<__nv_bfloat16*>(out);
  p.ws_o = ws_o;
  p.ws_ml = ws_ml;
  p.bt_stride = bt_stride;
  p.hkv = hkv;
  p.gqa = gqa;
  p.hq_total = hq_total;
  p.head_offset = head_offset;
  p.nsplit = nsplit;
  p.sm_scale_log2 = sm_scale * LOG2E;
  p.push = flag_mc != nullptr;
  p.flag_mc = flag_mc;
  int npad, rc;
  if (rows <= 16 && keys_on_lanes()) { npad = 16; rc = launch_decode_t<16>(tm, p, heads, nseq, st); }
  else if (rows <= 16) { npad = 16; rc = launch_decode<16>(tm, p, heads, nseq, st); }
  else if (rows <= 32) { npad = 32; rc = launch_decode<32>(tm, p, heads, nseq, st); }
  else if (rows <= 48) { npad = 48; rc = launch_decode<48>(tm, p, heads, nseq, st); }
  else { npad = 64; rc = launch_decode<64>(tm, p, heads, nseq, st); }
  *npad_out = npad;
  return rc;
}

int npad_of(int rows) { return rows <= 16 ? 16 : rows <= 32 ? 32 : rows <= 48 ? 48 : 64; }
}  // namespace

// Paged decode attention (b200 format). `heads` KV heads starting at
// `head_offset` are processed; q/out rows hold hq_total query heads.
// ws_o / ws_ml must hold nseq*heads*nsplit*npad*(D+2) floats when nsplit > 1.
extern "C" int k8v4_decode_attn(const void* q, const int32_t* cu_q, const int32_t* seq_lens, const int32_t* q_ends,
                                const int32_t* block_table, int bt_stride, const void* cache, int64_t num_pages,
                                int hkv, int head_offset, int heads, int gqa, int hq_total, int nseq, int max_q_len,
                                int nsplit, float sm_scale, void* out, float* ws_o, float* ws_ml, cudaStream_t st) {
  const int rows = max_q_len * gqa;
  if (rows <= 0 || nseq <= 0) return 0;
  if (rows > 64) return 1;  // longer query runs use the prefill kernel
  if (nsplit > 128) return 4;
  if (nsplit < 1) nsplit = 1;
  if (nsplit > 1 && (!ws_o || !ws_ml)) return 2;
  int npad = 0;
  const int rc = decode_core(q, cu_q, seq_lens, q_ends, block_table, bt_stride, cache, num_pages, hkv, head_offset,
                             heads, gqa, hq_total, nseq, max_q_len, nsplit, sm_scale, out, ws_o, ws_ml, nullptr,
                             &npad, st);
  if (rc || nsplit == 1) return rc;
  return launch_k(decode_combine_kernel, dim3(rows, heads, nseq), dim3(D * COMBINE_GROUPS), 0, st, (const float*)ws_o,
                  (const float*)ws_ml, cu_q, reinterpret_cast<__nv_bfloat16*>(out), nsplit, npad, gqa, hq_total,
                  head_offset, 1, (int64_t)0, (int64_t)0) == cudaSuccess
             ? 0
             : 11;
}

// Context parallelism, exchange fused into the decode kernel: each CTA stores
// its (m, l, O) partial through `slot_mc`, the multicast address of this
// rank's slot in a symmetric gather buffer (the slot lands in every rank's
// copy; (m, l) first, then O, k8v4_decode_ws_floats floats), then adds 1 to
// the multicast counter `flag_mc`. k8v4_decode_combine_ranks_sync merges the
// slots. Every rank must launch the same shape (nseq, heads, nsplit, rows).
extern "C" int k8v4_decode_attn_push(const void* q, const int32_t* cu_q, const int32_t* seq_lens,
                                     const int32_t* q_ends, const int32_t* block_table, int bt_stride,
                                     const void* cache, int64_t num_pages, int hkv, int head_offset, int heads,
                                     int gqa, int hq_total, int nseq, int max_q_len, int nsplit, float sm_scale,
                                     float* slot_mc, unsigned long long* flag_mc, cudaStream_t st) {
  const int rows = max_q_len * gqa;
  if (rows <= 0 || nseq <= 0) return 0;
  if (rows > 64) return 1;
  if (nsplit < 1 || nsplit > 128) return 4;
  if (!slot_mc || !flag_mc) return 2;
  const int64_t ml_floats = (int64_t)nseq * heads * nsplit * 2 * npad_of(rows);
  int npad = 0;
  return decode_core(q, cu_q, seq_lens, q_ends, block_table, bt_stride, cache, num_pages, hkv, head_offset, heads,
                     gqa, hq_total, nseq, max_q_len, nsplit, sm_scale, nullptr, slot_mc + ml_floats, slot_mc, flag_mc,
                     &npad, st);
}

// CTAs one k8v4_decode_attn_push launch signals with (per rank).
extern "C" int64_t k8v4_decode_push_ctas(int nseq, int heads, int nsplit) {
  return (int64_t)nseq * heads * nsplit;
}

// Merge the split partials of `nrank` ranks (context parallelism): `ws_all`
// holds every rank's decode workspace back to back, `rank_floats` apart (one
// launch shape's partials: (m, l) first, then O, as k8v4_decode_attn lays
// them out).
extern "C" int k8v4_decode_combine_ranks(const float* ws_all, int64_t rank_floats, const int32_t* cu_q, void* out,
                                         int nrank, int nsplit, int nseq, int heads, int head_offset, int gqa,
                                         int hq_total, int max_q_len, cudaStream_t st) {
  const int rows = max_q_len * gqa;
  if (rows <= 0 || nseq <= 0) return 0;
  if (rows > 64 || nrank < 1 || nsplit < 1 || nrank * nsplit > 128) return 1;
  const int npad = rows <= 16 ? 16 : rows <= 32 ? 32 : rows <= 48 ? 48 : 64;
  const int64_t ml_floats = (int64_t)nseq * heads * nsplit * 2 * npad;
  return launch_k(decode_combine_kernel, dim3(rows, heads, nseq), dim3(D * COMBINE_GROUPS), 0, st, ws_all + ml_floats, ws_all, cu_q,
                  reinterpret_cast<__nv_bfloat16*>(out), nsplit, npad, gqa, hq_total, head_offset, nrank,
                  rank_floats, rank_floats) == cudaSuccess
             ? 0
             : 11;
}

// Merge every rank's slot of the gather buffer that k8v4_decode_attn_push
// fills (`ws_all`: this rank's copy, slots `rank_floats` apart). The kernel
// waits until the counter `sync_flag` (this rank's copy) reaches
// sync_state[0] + sync_expected, then the last CTA adds sync_expected to
// sync_state[0]; sync_expected = ranks x k8v4_decode_push_ctas.
extern "C" int k8v4_decode_combine_ranks_sync(const float* ws_all, int64_t rank_floats, const int32_t* cu_q,
                                              void* out, int nrank, int nsplit, int nseq, int heads, int head_offset,
                                              int gqa, int hq_total, int max_q_len,
                                              const unsigned long long* sync_flag, unsigned long long* sync_state,
                                              unsigned long long sync_expected, cudaStream_t st) {
  const int rows = max_q_len * gqa;
  if (rows <= 0 || nseq <= 0) return 0;
  if (rows > 64 || nrank < 1 || nsplit < 1 || nrank * nsplit > 128) return 1;
  if (!sync_flag || !sync_state) return 2;
  const int npad = npad_of(rows);
  const int64_t ml_floats = (int64_t)nseq * heads * nsplit * 2 * npad;
  peer::ReduceSync sync{sync_flag, sync_state, sync_expected};
  return launch_k(decode_combine_sync_kernel, dim3(rows, heads, nseq), dim3(D * COMBINE_GROUPS), 0, st,
                  (const float*)(ws_all + ml_floats), ws_all, cu_q, reinterpret_cast<__nv_bfloat16*>(out), nsplit,
                  npad, gqa, hq_total, head_offset, nrank, rank_floats, sync) == cudaSuccess
             ? 0
             : 11;
}

// Workspace floats needed for a given launch shape.
extern "C" int64_t k8v4_decode_ws_floats(int nseq, int heads, int nsplit, int max_q_len, int gqa) {
  const int rows = max_q_len * gqa;
  const int npad = rows <= 16 ? 16 : rows <= 32 ? 32 : rows <= 48 ? 48 : 64;
  return (int64_t)nseq * heads * nsplit * npad * (D + 2);
}
