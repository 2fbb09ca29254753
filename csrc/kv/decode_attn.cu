// Split-K paged decode / MTP-verify attention over int8-K / int4-V pages.
//
// One CTA per (split, KV head, sequence). Query rows are the (token, q-head)
// pairs of the sequence that share this KV head (q_len * gqa <= NPAD); they
// are quantized to int8 per row in the prologue (the reference's Q-once
// quantization, k8v4_v030/native/xe2_kv_ops.cpp:205-257) and held as the
// MMA B operand. Keys run on the MMA M dimension (TMEM lanes):
//
//   S^T[key, row]  = K_tile(int8, TMA) x Q8^T          tcgen05 kind::i8 -> TMEM
//   softmax        : one thread per key, per-row max over the 128 keys via
//                    warp shuffles, lazy rescale (tau = 8 in log2 units)
//   O^T[dim, row] += V^T_tile(fp16) x P^T(fp16)       tcgen05 kind::f16 -> TMEM
//
// V int4 is dequantized by converter warps into the MN-major fp16 tile the
// PV MMA reads. Each split writes its (m, l, O) partial; k8v4_decode_combine
// merges the splits (the reference's stage-2 merge, :847-1246). With one
// split the CTA writes the normalized output directly.
//
// Warp roles: 0 = TMA producer, 1 = TMEM owner + MMA issuer, 2-5 = V
// converters, 6-9 = softmax / epilogue.
#include "attn_common.cuh"

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
};

#ifdef K8V4_TRACE
// Timeline of CTA (0,0,0) (trace builds only): rows = 0 producer issued,
// 1 converters done, 2 QK issued, 3 softmax done (p_full), 4 PV issued.
__device__ uint64_t g_attn_trace[5 * 256];
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
  static constexpr int NGRP = 2;  // softmax warpgroups, ping-pong over tiles
  static constexpr int NWARPS = 2 + 4 + 4 * NGRP;
  static constexpr int NTHREADS = 32 * NWARPS;
  static constexpr int Q_BYTES = NPAD * 128;
  static constexpr int PT_BYTES = 2 * NPAD * 128;   // P^T fp16: 2 K-atoms of NPAD rows
  static constexpr int TMEM_NEED = 4 * NPAD;        // S^T[2] + O^T[2]
  static constexpr int TMEM_COLS = TMEM_NEED <= 32 ? 32 : TMEM_NEED <= 64 ? 64 : TMEM_NEED <= 128 ? 128
                                   : TMEM_NEED <= 256 ? 256 : 512;
  // layout (offsets from the 1024-aligned base)
  static constexpr int OFF_K = 0;
  // fp16 V^T tiles: three when shared memory allows, so conversion of tile
  // j+1 never waits for the PV MMA of tile j-2
  static constexpr int NVT = (NPAD <= 32) ? 3 : 2;
  static constexpr int OFF_VT = OFF_K + STAGES * K_TILE_BYTES;
  static constexpr int OFF_PT = OFF_VT + NVT * VT_BYTES;
  static constexpr int OFF_Q = OFF_PT + 2 * PT_BYTES;
  static constexpr int OFF_VS = OFF_Q + ((Q_BYTES + 1023) / 1024) * 1024;
  static constexpr int OFF_MISC = OFF_VS + STAGES * VS_TILE_BYTES;
  static constexpr int SMEM_BYTES = 1024 + OFF_MISC + 256 + 32 * NPAD * 4 + 64;
};

// Two softmax warpgroups take alternate tiles (group g owns tiles j = g mod 2)
// with their own S^T / P^T / O^T buffers and their own running max and sums,
// so one group's softmax overlaps the other's MMAs and handoffs. Their
// (m, l, O) are merged in the epilogue like two splits.
template <int NPAD>
__global__ void __launch_bounds__(DCfg<NPAD>::NTHREADS, 1)
    decode_attn_kernel(const __grid_constant__ CUtensorMap tm_k, const DecodeParams p) {
  using C = DCfg<NPAD>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = sm + C::OFF_K;
  uint8_t* sVT = sm + C::OFF_VT;
  uint8_t* sPT = sm + C::OFF_PT;
  uint8_t* sQ = sm + C::OFF_Q;
  uint8_t* sVS = sm + C::OFF_VS;
  uint8_t* misc = sm + C::OFF_MISC;
  uint64_t* kv_full = reinterpret_cast<uint64_t*>(misc);
  uint64_t* kv_empty = kv_full + C::STAGES;
  uint64_t* s_full = kv_empty + C::STAGES;  // [2] (buffer = owning group)
  uint64_t* p_full = s_full + 2;            // [2]
  uint64_t* v_full = p_full + 2;            // [NVT] V^T tile converted
  uint64_t* pv_empty = v_full + 3;          // [2] PV of the group's last tile done (P^T / O^T reusable)
  uint64_t* vt_empty = pv_empty + 2;        // [NVT] PV that read the V^T tile done
  uint64_t* done_bar = vt_empty + 3;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(done_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  int* grp_ok = const_cast<int*>(abort_flag) + 1;            // [2]
  float* q_scale = reinterpret_cast<float*>(misc + 256);     // [NPAD] q scale * softmax scale
  int* row_end = reinterpret_cast<int*>(q_scale + NPAD);     // [NPAD] visible keys per row
  float* m_ref = reinterpret_cast<float*>(row_end + NPAD);   // [2][4][NPAD] running max per warp (log2)
  float* alpha = m_ref + 8 * NPAD;                           // [2][4][NPAD] this tile's rescale per warp
  float* red = alpha + 8 * NPAD;                             // [2][4][NPAD] cross-warp partials
  float* fin = red + 8 * NPAD;                               // [2][2][NPAD] final (m, l) per group

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int split = blockIdx.x, h = blockIdx.y + p.head_offset, seq = blockIdx.z;
  const int hl = blockIdx.y;  // head index within this launch's workspace
  const int qb = p.cu_q[seq], q_len = p.cu_q[seq + 1] - qb;
  const int R = q_len * p.gqa;  // real rows
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
      mbar_init(&kv_empty[s], 1 + 4 + 4);  // MMA commit + converter warps + owning group's warps
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&p_full[b], 4);
      mbar_init(&pv_empty[b], 1);
    }
    for (int v = 0; v < C::NVT; ++v) {
      mbar_init(&v_full[v], 4);
      mbar_init(&vt_empty[v], 1);
    }
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    grp_ok[0] = grp_ok[1] = 1;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, C::TMEM_COLS);
    tmem_relinquish();
  }
  // ---- prologue: quantize the query rows into the Q8 tile (K-major SW128)
  for (int r = warp; r < NPAD; r += C::NWARPS) {
    float x[4] = {0.f, 0.f, 0.f, 0.f};
    int end = 0;
    if (r < R) {
      const int t = r / p.gqa, g = r % p.gqa;
      const __nv_bfloat16* src = p.q + ((int64_t)(qb + t) * p.hq_total + (int64_t)h * p.gqa + g) * D + lane * 4;
      const uint2 raw = *reinterpret_cast<const uint2*>(src);
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
      const float2 a = __bfloat1622float2(h2[0]), b = __bfloat1622float2(h2[1]);
      x[0] = a.x; x[1] = a.y; x[2] = b.x; x[3] = b.y;
      end = p.q_ends ? p.q_ends[qb + t] : (seq_len - q_len + t + 1);
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
    // lane covers bytes [4*lane, 4*lane+4) of the 128-byte row: chunk lane/4
    *reinterpret_cast<uint32_t*>(sQ + sw128_offset(r, lane >> 2) + (lane & 3) * 4) = w;
    if (lane == 0) {
      q_scale[r] = s * p.sm_scale_log2;
      row_end[r] = end;
      for (int c = 0; c < 8; ++c) m_ref[c * NPAD + r] = -INFINITY;
    }
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const uint32_t tm_s = tmem;                 // S^T buffers: cols [0, 2*NPAD)
  const uint32_t tm_o = tmem + 2 * NPAD;      // O^T buffers: cols [2*NPAD, 4*NPAD)

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tmap(&tm_k);
      int issued = 0;
      for (int j = 0; j < nt; ++j) {
        const int s = j % C::STAGES;
        if (j >= C::STAGES && !mbar_wait(&kv_empty[s], ((j / C::STAGES) - 1) & 1, abort_flag, 201)) break;
        const int pg0 = (tile_beg + j) * TILE_PAGES;
        const int npg = min(TILE_PAGES, n_pages - pg0);
        mbar_arrive_expect_tx(&kv_full[s], npg * (K_BYTES + VS_BYTES));
        for (int i = 0; i < npg; ++i) {
          const int64_t page = bt[pg0 + i];
          const int64_t run = page * p.hkv + h;
          tma_load_3d(sK + s * K_TILE_BYTES + i * K_BYTES, &tm_k, &kv_full[s], 0, 0, (int)run);
          bulk_load(sVS + s * VS_TILE_BYTES + i * VS_BYTES, p.cache + run * HEAD_BYTES + VS_OFF, VS_BYTES,
                    &kv_full[s]);
        }
        K8V4_ATRACE(0, j);
        ++issued;
      }
      if (*abort_flag)
        for (int j = issued - 1; j >= 0 && j >= issued - C::STAGES; --j)
          mbar_wait_drain(&kv_full[j % C::STAGES], (j / C::STAGES) & 1);
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------------- MMA
    if (lane == 0 && nt > 0) {
      const uint32_t id_qk = idesc_s8(128, NPAD);
      const uint32_t id_pv = idesc_f16(128, NPAD, true, false);
      const uint32_t q_base = smem_u32(sQ);
      bool ok = true;
      for (int j = 0; j <= nt && ok; ++j) {
        if (j < nt) {
          const int s = j % C::STAGES, b = j & 1;
          if (!mbar_wait(&kv_full[s], (j / C::STAGES) & 1, abort_flag, 202)) break;
          tc_fence_after();
          const uint32_t k_base = smem_u32(sK + s * K_TILE_BYTES);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_i8(tm_s + b * NPAD, sdesc_sw128(k_base + kk * 32, 16, 1024), sdesc_sw128(q_base + kk * 32, 16, 1024),
                   id_qk, kk > 0 ? 1u : 0u);
          mma_commit(&s_full[b]);
          mma_commit(&kv_empty[s]);
          K8V4_ATRACE(2, j);
        }
        if (j >= 1) {
          const int jj = j - 1, b = jj & 1;
          const int vb = jj % C::NVT;
          if (!mbar_wait(&p_full[b], (jj >> 1) & 1, abort_flag, 203) ||
              !mbar_wait(&v_full[vb], (jj / C::NVT) & 1, abort_flag, 204)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t vt_base = smem_u32(sVT + vb * VT_BYTES);
          const uint32_t pt_base = smem_u32(sPT + b * C::PT_BYTES);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint64_t ad = sdesc_sw128(vt_base + kk * 2048, VT_LBO, 1024);
            const uint64_t bd = sdesc_sw128(pt_base + (kk >> 2) * (NPAD * 128) + (kk & 3) * 32, 16, 1024);
            mma_f16(tm_o + b * NPAD, ad, bd, id_pv, (jj >= 2 || kk > 0) ? 1u : 0u);
          }
          mma_commit(&pv_empty[b]);
          mma_commit(&vt_empty[vb]);
          K8V4_ATRACE(4, jj);
        }
      }
      mma_commit(done_bar);
      mbar_wait_drain(done_bar, 0);
    }
  } else if (warp < 6) {
    // ---------------------------------------------------------- converters
    const int ct = threadIdx.x - 64;  // 0..127
    for (int j = 0; j < nt; ++j) {
      const int s = j % C::STAGES, b = j & 1;
      if (!mbar_wait_all(&kv_full[s], (j / C::STAGES) & 1, abort_flag, 205)) break;
      const int vb = j % C::NVT;
      if (j >= C::NVT && !mbar_wait_all(&vt_empty[vb], ((j / C::NVT) - 1) & 1, abort_flag, 206)) break;
      const int key0 = (tile_beg + j) * TILE;
      const int nvalid = min(TILE, seq_len - key0);
      const uint8_t* vs = sVS + s * VS_TILE_BYTES;
      uint8_t* vt = sVT + vb * VT_BYTES;
#pragma unroll 4
      for (int item = ct; item < TILE * 16; item += 128) {
        const int key = item >> 4, chunk = item & 15;
        if (key < nvalid) {
          const uint8_t* run = vs + (key >> 4) * VS_BYTES;
          const int kk = key & 15;
          const uint32_t w = *reinterpret_cast<const uint32_t*>(run + kk * 64 + chunk * 4);
          const __half sc = *reinterpret_cast<const __half*>(run + VSC_OFF + (kk * 4 + (chunk >> 2)) * 2);
          v_chunk_to_f16(w, sc, vt, key, chunk);
        } else {
          v_chunk_zero(vt, key, chunk);
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
  } else {
    // ------------------------------------------------------------- softmax
    const int grp = (warp - 6) >> 2;           // warpgroup: owns tiles j = grp mod 2
    const int sw = (warp - 6) & 3;             // warp within the group
    const int quad = warp & 3;                 // TMEM lane quadrant
    const int key_local = quad * 32 + lane;    // this thread's key (S^T lane) and dim (O^T lane)
    const int bar_id = 1 + grp;
    float* mw = m_ref + (grp * 4 + sw) * NPAD;
    float* aw = alpha + (grp * 4 + sw) * NPAD;
    float* rd = red + grp * 4 * NPAD;
    const uint32_t tm_og = tm_o + grp * NPAD;
    float l_acc[NPAD];
#pragma unroll
    for (int r = 0; r < NPAD; ++r) l_acc[r] = 0.f;
    // Every warp of a group runs every iteration and every named barrier,
    // even after a failed (timed-out) wait: a failure only turns the work
    // off, so the four warps always meet at the same bar.sync.
    bool ok = true;
    for (int j = grp; j < nt; j += 2) {
      const int s = j % C::STAGES, b = grp;
      if (ok && (!mbar_wait_all(&s_full[b], (j >> 1) & 1, abort_flag, 207) ||
                 !mbar_wait_all(&kv_full[s], (j / C::STAGES) & 1, abort_flag, 208)))
        ok = false;
      const int key = (tile_beg + j) * TILE + key_local;
      float sc[NPAD];
#pragma unroll
      for (int r = 0; r < NPAD; ++r) sc[r] = -INFINITY;
      if (ok) {
        tc_fence_after();
        const uint8_t* vs = sVS + s * VS_TILE_BYTES;
        const float ks = (key < seq_len)
                             ? __half2float(*reinterpret_cast<const __half*>(vs + (key_local >> 4) * VS_BYTES + KS_OFF +
                                                                             (key_local & 15) * 2))
                             : 0.f;
        const uint32_t ta = tm_s + b * NPAD + ((uint32_t)(quad * 32) << 16);
#pragma unroll
        for (int c = 0; c < NPAD; c += 16) {
          uint32_t r16[16];
          tmem_ld16(ta + c, r16);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 16; ++i) sc[c + i] = i2f_small(r16[i]);
        }
        // scores (log2 domain), masked, and this warp's per-row max
#pragma unroll
        for (int r = 0; r < NPAD; ++r) {
          if (r < R) {
            const float v = sc[r] * (q_scale[r] * ks);
            sc[r] = (key < row_end[r]) ? v : -INFINITY;
            const float wm = warp_max(sc[r]);
            if (lane == 0) rd[sw * NPAD + r] = wm;
          }
        }
      }
      asm volatile("bar.sync %0, 128;" ::"r"(bar_id) : "memory");
      int any_rescale = 0;
      if (ok) {
#pragma unroll
        for (int r = 0; r < NPAD; ++r) {
          if (r < R) {
            const float tmax = fmaxf(fmaxf(rd[r], rd[NPAD + r]), fmaxf(rd[2 * NPAD + r], rd[3 * NPAD + r]));
            const float mo = mw[r];
            float a = 1.f, mn = mo;
            if (tmax > mo + RESCALE_TAU || (mo == -INFINITY && tmax > -INFINITY)) {
              mn = tmax;
              a = (mo == -INFINITY) ? 0.f : exp2f(mo - mn);
              any_rescale = 1;
            }
            l_acc[r] *= a;
            sc[r] = (sc[r] == -INFINITY || mn == -INFINITY) ? 0.f : exp2f(sc[r] - mn);
            l_acc[r] += sc[r];
            __syncwarp();
            if (lane == 0) {
              mw[r] = mn;
              aw[r] = a;
            }
          }
        }
        __syncwarp();
      }
      // this group's previous PV (tile j-2) read P^T[b] and wrote O^T[b]
      if (ok && j >= 2 && !mbar_wait_all(&pv_empty[b], ((j >> 1) - 1) & 1, abort_flag, 210)) ok = false;
      if (ok && any_rescale && j >= 2) {
        tc_fence_after();
        const uint32_t ta = tm_og + ((uint32_t)(quad * 32) << 16);
#pragma unroll
        for (int c = 0; c < NPAD; c += 8) {
          uint32_t r8[8];
          tmem_ld8(ta + c, r8);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 8; ++i)
            r8[i] = __float_as_uint(__uint_as_float(r8[i]) * (c + i < R ? aw[c + i] : 1.f));
          tmem_st8(ta + c, r8);
        }
        tmem_st_wait();
      }
      if (ok) {
        uint8_t* pt = sPT + b * C::PT_BYTES + (key_local >> 6) * (NPAD * 128) + (key_local & 7) * 2;
        const int kc = (key_local & 63) >> 3;
#pragma unroll
        for (int r = 0; r < NPAD; ++r) {
          const __half hv = __float2half_rn(r < R ? sc[r] : 0.f);
          *reinterpret_cast<__half*>(pt + r * 128 + ((kc ^ (r & 7)) << 4)) = hv;
        }
        fence_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&p_full[b]);
          mbar_arrive(&kv_empty[s]);
          if (sw == 0) K8V4_ATRACE(3, j);
        }
      }
      asm volatile("bar.sync %0, 128;" ::"r"(bar_id) : "memory");  // rd / m reads done before the next tile
    }
    // ------------------------------------------------------------ epilogue
    const bool has = nt > grp;  // this group processed at least one tile
    if (ok && has) {
      const int jl = grp + 2 * ((nt - 1 - grp) / 2);  // this group's last tile
      if (!mbar_wait_all(&pv_empty[grp], (jl >> 1) & 1, abort_flag, 211)) ok = false;
    }
#pragma unroll
    for (int r = 0; r < NPAD; ++r) {
      if (r < R) {
        const float ws = warp_sum(l_acc[r]);
        if (lane == 0) rd[sw * NPAD + r] = ws;
      }
    }
    asm volatile("bar.sync %0, 128;" ::"r"(bar_id) : "memory");
    if (sw == 0) {
      for (int r = lane; r < NPAD; r += 32) {
        fin[(grp * 2) * NPAD + r] = has ? mw[r] : -INFINITY;
        fin[(grp * 2 + 1) * NPAD + r] = rd[r] + rd[NPAD + r] + rd[2 * NPAD + r] + rd[3 * NPAD + r];
      }
      if (lane == 0 && !ok) grp_ok[grp] = 0;
    }
    asm volatile("bar.sync 3, 256;" ::: "memory");  // both groups' (m, l) published
    if (grp == 0 && grp_ok[0] && grp_ok[1]) {
      tc_fence_after();
      float o0[NPAD], o1[NPAD];
#pragma unroll
      for (int r = 0; r < NPAD; ++r) o0[r] = o1[r] = 0.f;
      const uint32_t lo = (uint32_t)(quad * 32) << 16;
      if (nt > 0) {
#pragma unroll
        for (int c = 0; c < NPAD; c += 16) {
          uint32_t r16[16];
          tmem_ld16(tm_o + lo + c, r16);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 16; ++i) o0[c + i] = __uint_as_float(r16[i]);
        }
      }
      if (nt > 1) {
#pragma unroll
        for (int c = 0; c < NPAD; c += 16) {
          uint32_t r16[16];
          tmem_ld16(tm_o + NPAD + lo + c, r16);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 16; ++i) o1[c + i] = __uint_as_float(r16[i]);
        }
      }
      const int d = key_local;
      const int64_t wsi = (((int64_t)seq * gridDim.y + hl) * p.nsplit + split);
#pragma unroll
      for (int r = 0; r < NPAD; ++r) {
        if (r < R) {
          const float m0 = fin[r], l0 = fin[NPAD + r], m1 = fin[2 * NPAD + r], l1 = fin[3 * NPAD + r];
          const float M = fmaxf(m0, m1);
          const float w0 = (m0 == -INFINITY) ? 0.f : exp2f(m0 - M);
          const float w1 = (m1 == -INFINITY) ? 0.f : exp2f(m1 - M);
          const float o = (w0 > 0.f ? w0 * o0[r] : 0.f) + (w1 > 0.f ? w1 * o1[r] : 0.f);
          const float l = w0 * l0 + w1 * l1;
          if (p.nsplit == 1) {
            const int t = r / p.gqa, g = r % p.gqa;
            const float v = l > 0.f ? o / l : 0.f;
            p.out[((int64_t)(qb + t) * p.hq_total + (int64_t)h * p.gqa + g) * D + d] = __float2bfloat16_rn(v);
          } else {
            p.ws_o[(wsi * NPAD + r) * D + d] = o;
            if (d == 0) {
              p.ws_ml[(wsi * 2) * NPAD + r] = M;
              p.ws_ml[(wsi * 2 + 1) * NPAD + r] = l;
            }
          }
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

// Merge split partials: grid (rows, heads, seqs), 128 threads (dims). The
// per-split weights are computed once by the block; the O loads of all splits
// are independent, so their latencies overlap.
__global__ void __launch_bounds__(128) decode_combine_kernel(const float* __restrict__ ws_o,
                                                             const float* __restrict__ ws_ml, const int32_t* cu_q,
                                                             __nv_bfloat16* out, int nsplit, int npad, int gqa,
                                                             int hq_total, int head_offset) {
  __shared__ float wsh[128];
  __shared__ float red[8];
  const int r = blockIdx.x, hl = blockIdx.y, seq = blockIdx.z, d = threadIdx.x;
  const int qb = cu_q[seq], q_len = cu_q[seq + 1] - qb;
  if (r >= q_len * gqa) return;
  const int64_t base = ((int64_t)seq * gridDim.y + hl) * nsplit;
  float m = -INFINITY, l = 0.f;
  if (d < nsplit) {
    m = ws_ml[((base + d) * 2) * npad + r];
    l = ws_ml[((base + d) * 2 + 1) * npad + r];
  }
  float M = warp_max(m);
  if ((d & 31) == 0) red[d >> 5] = M;
  __syncthreads();
  M = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  const float w = (m == -INFINITY || M == -INFINITY) ? 0.f : exp2f(m - M);
  if (d < nsplit) wsh[d] = w;
  float L = warp_sum(w * l);
  __syncthreads();
  if ((d & 31) == 0) red[4 + (d >> 5)] = L;
  __syncthreads();
  L = red[4] + red[5] + red[6] + red[7];
  const float* o = ws_o + (base * npad + r) * D + d;
  const int64_t stride = (int64_t)npad * D;
  float acc = 0.f;
  int s = 0;
  for (; s + 8 <= nsplit; s += 8) {
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = o[(s + i) * stride];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc += wsh[s + i] > 0.f ? wsh[s + i] * v[i] : 0.f;
  }
  for (; s < nsplit; ++s) acc += wsh[s] > 0.f ? wsh[s] * o[s * stride] : 0.f;
  const int t = r / gqa, g = r % gqa, h = hl + head_offset;
  out[((int64_t)(qb + t) * hq_total + (int64_t)h * gqa + g) * D + d] = __float2bfloat16_rn(L > 0.f ? acc / L : 0.f);
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

K8V4_STATUS_API(decode)

#ifdef K8V4_TRACE
extern "C" int k8v4_attn_trace(uint64_t* host) {
  return cudaMemcpyFromSymbol(host, g_attn_trace, sizeof(uint64_t) * 5 * 256);
}
#endif

template <int NPAD>
static int launch_decode(const CUtensorMap& tm, const DecodeParams& p, int heads, int nseq, cudaStream_t st) {
  using C = DCfg<NPAD>;
  static bool set = false;
  if (!set) {
    cudaFuncSetAttribute(decode_attn_kernel<NPAD>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
    set = true;
  }
  dim3 grid(p.nsplit, heads, nseq);
  decode_attn_kernel<NPAD><<<grid, C::NTHREADS, C::SMEM_BYTES, st>>>(tm, p);
  return cudaGetLastError() == cudaSuccess ? 0 : 10;
}

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
  CUtensorMap tm;
  if (k8v4_make_kv_tmap(&tm, cache, num_pages, hkv)) return 3;
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
  int npad, rc;
  if (rows <= 16) { npad = 16; rc = launch_decode<16>(tm, p, heads, nseq, st); }
  else if (rows <= 32) { npad = 32; rc = launch_decode<32>(tm, p, heads, nseq, st); }
  else if (rows <= 48) { npad = 48; rc = launch_decode<48>(tm, p, heads, nseq, st); }
  else { npad = 64; rc = launch_decode<64>(tm, p, heads, nseq, st); }
  if (rc || nsplit == 1) return rc;
  decode_combine_kernel<<<dim3(rows, heads, nseq), D, 0, st>>>(ws_o, ws_ml, cu_q, reinterpret_cast<__nv_bfloat16*>(out),
                                                               nsplit, npad, gqa, hq_total, head_offset);
  return cudaGetLastError() == cudaSuccess ? 0 : 11;
}

// Workspace floats needed for a given launch shape.
extern "C" int64_t k8v4_decode_ws_floats(int nseq, int heads, int nsplit, int max_q_len, int gqa) {
  const int rows = max_q_len * gqa;
  const int npad = rows <= 16 ? 16 : rows <= 32 ? 32 : rows <= 48 ? 48 : 64;
  return (int64_t)nseq * heads * nsplit * npad * (D + 2);
}
