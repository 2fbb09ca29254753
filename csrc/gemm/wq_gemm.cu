// Quantized-weight GEMM on tcgen05: Y[t, n] = sum_k X[t, k] * W[n, k].
//
// Weights are the MMA "A" operand (128 output features per CTA = the TMEM
// lanes) and tokens are the MMA "N" dimension (BT = 16..128 per CTA), so one
// kernel serves decode (a handful of tokens) and prefill (thousands).
//
//   mode W4A16 : GPTQ int4 (group 128, symmetric, codes q+8) x bf16 tokens.
//                Converter warps turn each int4 code into the exact bf16
//                integer (q-8); tcgen05.mma.kind::f16 accumulates one K group
//                into a TMEM partial; accumulator warps fold the fp32 group
//                scale in: acc += partial * scale[g][n].
//   mode W4A8  : same weights x int8 tokens (per-token scale). Converters
//                emit int8 (q-8); tcgen05.mma.kind::i8 gives an int32 group
//                partial; accumulator warps rescale in fp32 and apply the
//                token scale at the end. (reference: int4_gemm_w4a8 called at
//                k8v4_v030/w4a8_prefill.py:146-157)
//   mode W8A8  : int8 per-row weights (lm_head) x int8 tokens; the weight
//                tile goes straight from TMA into the MMA, one group = all K.
//   mode W4L   : W4A16 at decode sizes (at most 32 tokens) through 8-bit
//                integer MMAs. Each token row x is written as two int8 limbs
//                x ~= s (128 hi + lo) with |128 hi + lo| <= 16319 (15 bits,
//                finer than bf16 for the row's large entries); the limbs_kernel
//                makes them, with the row scale s and the integer sum C of
//                each 128-k group. Converters only unpack int4 codes to u8
//                (q + 8, five instructions per 8 codes, no subtraction); one
//                kind::i8 MMA of N = 2 BT takes the hi and the lo rows
//                together (an MMA of N <= 64 costs the tensor pipe the same
//                ~45 cycles as one of N = 16) with K = 32 per instruction, so
//                a 128-k block is 4 MMAs instead of 8. The accumulators form
//                128 D_hi + D_lo - 8 C = sum q X exactly in int32, scale it by
//                the group scale, and apply s at the end.
//
// Roles: warp 0 issues TMA, warp 1 owns TMEM and issues MMAs (one elected
// thread; at decode sizes two more warps issue too, each taking every third
// K group into its own accumulator buffers), the next NCONV warps convert
// raw weights, the NACC accumulator warps fold TMEM partials into fp32 and
// write the output. NBUF TMEM partial buffers let group g+1's MMAs overlap
// group g's rescale.
//
// Split-K: gridDim.z slices K; with more than one slice the CTA adds fp32
// partial sums into `ws` with red.global.add, and a consumer finishes them
// (the splitk_finish kernel, the fused RMSNorm, or the RoPE / cache-store
// kernel for the qkv projection), zeroing `ws` for the next GEMM.
//
// Sequence-parallel prefill (tensor parallel, 128-row token tiles owned by
// ranks in contiguous runs, sp_tile0[o] .. sp_tile0[o + 1] for rank o):
//   all-gather -> GEMM (qkv, gate/up): the token rows are this rank's copy of
//     a symmetric buffer that every rank's norm fills through its multicast
//     address. The CTAs of tile j start at this rank's own tiles, and the
//     producer waits (bounded) until ag_flag[owner(j)] reaches
//     ag_target[owner(j)] before the first TMA load of the tile, so tiles of
//     ranks that are still normalizing come last.
//   GEMM -> reduce-scatter (o_proj, down): each CTA stores its bf16 partial
//     rows straight into the owner's slot for this rank (rs_dst[owner], peer
//     memory over NVLink, row stride ldo) and then adds 1 to the owner's
//     counter rs_sig[owner] with release semantics; the owner's norm sums the
//     slots once every rank's CTAs have signalled. The transfer of early
//     tiles overlaps the math of later ones.
//
// GEMM -> all-reduce (tensor parallel row-parallel projections): with
// `ws_mc` set, the partial sums go to the multicast address of a symmetric
// fp32 buffer instead (multimem.red: the NVSwitch adds them into every
// rank's copy), and each CTA then adds 1 to the multicast counter `flag_mc`
// with release semantics. The consumer (the fused RMSNorm) waits until its
// local copy of the counter shows every rank's CTAs, then reads the reduced
// sums from its own copy: the reduction and its broadcast happen inside the
// GEMM's epilogue, overlapped with the other tiles' MMAs.
#include "../tc.cuh"
#include "../comm/peer.cuh"

namespace k8v4 {
namespace gemm {

using namespace tc;

enum Mode : int { W4A16 = 0, W4A8 = 1, W8A8 = 2, W4L = 3 };

struct Params {
  const int32_t* qweight;      // W4: [K/8, N] int32 (GPTQ, low nibble first)
  const __half* wscale;        // W4: [K/128, N]; W8: [N]
  const float* xscale;         // A8: [M] per-token scale
  const __nv_bfloat16* residual;  // optional [M, ldo]
  __nv_bfloat16* out;          // [M, ldo] (split == 1)
  float* ws;                   // [M, ldo] fp32 accumulation (split > 1)
  float* ws_mc;                // multicast alias of a symmetric [M, ldo] fp32 buffer (GEMM -> all-reduce)
  unsigned long long* flag_mc; // multicast alias of the counter each CTA signals when its sums are out
  const int32_t* csum;         // W4L: [M, K/128] integer sum of each token's limb values per 128-k group
  // sequence-parallel prefill (sp_world > 1; token tiles of 128 rows)
  int sp_world, sp_rank;
  int sp_tile0[9];                   // rank o owns token tiles [sp_tile0[o], sp_tile0[o + 1])
  const unsigned long long* ag_flag; // all-gather -> GEMM: this rank's copy of the per-owner row counters
  unsigned long long ag_target[8];   //   rows of owner o are all here once ag_flag[o] >= ag_target[o]
  __nv_bfloat16* rs_dst[8];          // GEMM -> reduce-scatter: owner o's slot for this rank (peer memory)
  unsigned long long* rs_sig[8];     //   owner o's completion counter (peer memory)
  int M, N, K, ldo;
  int k_per_split;             // multiple of 128
};

template <int MODE, int BT, int NCONV, int NACC, int STAGES, int RSTAGES, int BSTAGES>
struct Cfg {
  // Decode-sized tiles keep the converted weights in TMEM (the MMA reads A
  // from TMEM): no shared-memory round trip for A, and 128-k stages so each
  // wait / commit of the MMA thread covers eight MMAs.
  static constexpr bool LIMB = (MODE == W4L);
  static constexpr bool TA = ((MODE == W4A16) && (BT <= 64)) || LIMB;
  static constexpr int BK = (MODE == W4A16 && !TA) ? 64 : 128;  // k per stage
  static constexpr int KB_PER_GROUP = (BK == 64) ? 2 : 1;  // stages per K group (W8: all)
  static constexpr int A_BYTES = 128 * 128;                // 128 rows x 128 B
  static constexpr int BROWS = LIMB ? 2 * BT : BT;         // B operand rows: tokens, or hi then lo limbs
  static constexpr int B_ATOMS = (MODE == W4A16) ? BK / 64 : 1;  // 128-byte k atoms per token row
  static constexpr int B_BYTES = BROWS * 128 * B_ATOMS;
  static constexpr int RAW_BYTES = (MODE == W8A8) ? 0 : (BK / 8) * 128 * 4;
  // Two MMA-issuing warps on the TMEM-A path (even / odd K groups, separate
  // accumulator buffers): at N <= 64 one tcgen05.mma costs its issuing thread
  // ~50 cycles regardless of N, and a second issuer overlaps that cost
  // (measured 28 cycles per MMA aggregate with two issuers, 52 with one).
#ifndef K8V4_GEMM_NMMA
#define K8V4_GEMM_NMMA 3
#endif
  static constexpr int NMMA = TA ? K8V4_GEMM_NMMA : 1;
  static constexpr int NWARPS = 2 + NCONV + NACC + (NMMA - 1);
  static constexpr int NTHREADS = NWARPS * 32;
  static constexpr int NBUF = 4;                           // TMEM group partials in flight
  static constexpr int D_COLS = NBUF * BROWS;
  static constexpr int A_COLS = LIMB ? BK / 4 : BK / 2;    // TMEM columns of one A stage (u8: 4 k per column)
  static constexpr int TSTAGES = TA ? ((512 - D_COLS) / A_COLS > 12 ? 12 : (512 - D_COLS) / A_COLS) : 0;
  static constexpr int TMEM_NEED = D_COLS + TSTAGES * A_COLS;
  static constexpr int TMEM_COLS = TMEM_NEED <= 32 ? 32 : TMEM_NEED <= 64 ? 64 : TMEM_NEED <= 128 ? 128
                                   : TMEM_NEED <= 256 ? 256 : 512;
  static constexpr int ASMEM = TA ? 0 : STAGES;            // A stages in shared memory
  static constexpr int AR = TA ? TSTAGES : STAGES;         // A ring depth (either place)
  // With A in TMEM the token ring shares the A ring's slots and its empty
  // barrier (one commit per k-block); otherwise it has its own depth.
  static constexpr int BR = TA ? TSTAGES : BSTAGES;
  static constexpr int BAR_BYTES = 2048;
  static constexpr int MAXG = 144;                         // K groups whose scales fit the smem table
  static constexpr int ACC_SPLIT = NACC / 4;               // column slices per lane quadrant
  static constexpr int COLS = BT / ACC_SPLIT;              // columns per accumulator thread
  static constexpr int UMMA_K = (MODE == W4A16) ? 16 : 32;
  static constexpr int CSUM_BYTES = LIMB ? MAXG * BT * 4 : 0;  // W4L: group sums of the CTA's tokens
  static constexpr int SMEM_BYTES =
      1024 + ASMEM * A_BYTES + BR * B_BYTES + RSTAGES * RAW_BYTES + BAR_BYTES + MAXG * 128 * 2 + CSUM_BYTES;
  static_assert(TMEM_NEED <= 512, "TMEM budget");
  static_assert(!TA || NCONV % 4 == 0, "TMEM converters work in teams of 4 warps (one per lane quadrant)");
  static_assert(NACC == 4 || NACC == 8, "accumulator warps cover the 4 lane quadrants");
  static_assert(COLS % 8 == 0, "columns per accumulator thread");
  static_assert(BT % 16 == 0 && BT >= 16 && BT <= 256, "MMA N");
  static_assert(!LIMB || BT <= 32, "limb GEMMs serve at most 32 tokens (MMA N = 2 BT <= 64)");
  static_assert(SMEM_BYTES <= 232448, "shared memory per CTA");
};

// int4 x 8 (GPTQ low nibble first) -> 8 exact bf16 values (q-8) as 4 words.
__device__ __forceinline__ void int4x8_to_bf16(uint32_t w, uint32_t (&o)[4]) {
  // Byte j of w holds codes (2j, 2j+1); byte j of w>>4 holds code 2j+1 in its
  // low nibble. One byte_perm puts code 2j in bits 0-3 and code 2j+1 in bits
  // 16-19; OR-ing exponent 2^7 (bf16 ulp 1) makes the pair (128+c0, 128+c1)
  // and one bf16x2 subtraction of 136 leaves (c0-8, c1-8) exactly.
  const uint32_t w4 = w >> 4;
  const __nv_bfloat162 bias = __halves2bfloat162(__float2bfloat16(136.0f), __float2bfloat16(136.0f));
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t dup = __byte_perm(w, w4, 0x0400 + j * 0x0101);
    const uint32_t m = (dup & 0x000F000Fu) | 0x43004300u;
    __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(&m);
    v = __hsub2(v, bias);
    o[j] = *reinterpret_cast<uint32_t*>(&v);
  }
}

// int4 x 8 -> 8 int8 values (q-8) as 2 words (bytes in k order).
__device__ __forceinline__ void int4x8_to_s8(uint32_t w, uint32_t& o0, uint32_t& o1) {
  const uint32_t lo = (w & 0x0F0F0F0Fu) | 0x80808080u;         // codes 0,2,4,6
  const uint32_t hi = ((w >> 4) & 0x0F0F0F0Fu) | 0x80808080u;  // codes 1,3,5,7
  uint32_t a = __byte_perm(lo, hi, 0x5140);                     // 0,1,2,3
  uint32_t b = __byte_perm(lo, hi, 0x7362);                     // 4,5,6,7
  // per-byte (c | 0x80) - 8 never borrows across bytes; xor restores sign.
  o0 = (a - 0x08080808u) ^ 0x80808080u;
  o1 = (b - 0x08080808u) ^ 0x80808080u;
}

// Exact int32 -> fp32 for |v| < 2^22 with full-rate integer/float ops.
__device__ __forceinline__ float i2f_small(uint32_t v) {
  return __int_as_float(static_cast<int>(v) + 0x4B400000) - 12582912.0f;
}

#ifdef K8V4_TRACE
// Timeline of CTA (0,0,0) for pipeline studies (trace builds only):
// row 0 producer issue, 1 converter done, 2 MMA issued, 3 accumulate done,
// 4 MMA wait for the converted stage (ns), 5 converter past its waits,
// 6 MMA wait for a free accumulator buffer (ns), 7 converter stores issued.
__device__ uint64_t g_gemm_trace[8 * 256];
#define K8V4_TRACE_EVENT(row, idx)                                                        \
  do {                                                                                    \
    if (blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && (idx) < 256)             \
      g_gemm_trace[(row) * 256 + (idx)] = globaltimer_ns();                               \
  } while (0)
#else
#define K8V4_TRACE_EVENT(row, idx) do { } while (0)
#endif

template <int MODE, int BT, int NCONV, int NACC, int STAGES, int RSTAGES, int BSTAGES>
__global__ void __launch_bounds__(Cfg<MODE, BT, NCONV, NACC, STAGES, RSTAGES, BSTAGES>::NTHREADS, 1)
    wq_gemm_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                   const __grid_constant__ CUtensorMap tm_s, const Params p) {
  using C = Cfg<MODE, BT, NCONV, NACC, STAGES, RSTAGES, BSTAGES>;
  pdl_trigger();
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = align_smem_1024(smem_raw);
  uint8_t* sA = smem;
  uint8_t* sB = sA + C::ASMEM * C::A_BYTES;
  uint8_t* sR = sB + C::BR * C::B_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sR + RSTAGES * C::RAW_BYTES);
  // Three rings with their own depths: converted weights A (STAGES), token
  // tiles B (BSTAGES) and raw int4 weights (RSTAGES). The producer only
  // blocks on the raw and B rings, so weight bytes run RSTAGES k-blocks ahead
  // of the tensor cores.
  uint64_t* a_full = bars;                 // converters (or TMA for W8) -> MMA
  uint64_t* a_empty = a_full + C::AR;      // MMA -> converters (TMA for W8)
  uint64_t* b_full = a_empty + C::AR;      // TMA -> MMA (TMEM-A path: -> converters)
  uint64_t* b_empty_own = b_full + C::BR;  // MMA -> TMA (own ring)
  uint64_t* b_empty = C::TA ? a_empty : b_empty_own;
  uint64_t* r_full = b_empty_own + C::BR;  // TMA -> converters
  uint64_t* r_empty = r_full + RSTAGES;    // converters -> TMA
  uint64_t* acc_full = r_empty + RSTAGES;  // MMA -> accumulators (NBUF)
  uint64_t* acc_empty = acc_full + C::NBUF;  // accumulators -> MMA (NBUF)
  uint64_t* done_bar = acc_empty + C::NBUF;  // MMA drain on exit
  uint64_t* scale_bar = done_bar + 1;        // group-scale table loaded
  uint64_t* done_more = scale_bar + 1;       // [NMMA-1] drains of the other MMA issuers
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(done_more + C::NMMA);
  __half* sScale = reinterpret_cast<__half*>(reinterpret_cast<uint8_t*>(bars) + C::BAR_BYTES);  // [MAXG][128]
  int32_t* sCsum = reinterpret_cast<int32_t*>(sScale + C::MAXG * 128);  // W4L: [MAXG][BT]
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * 128;
  // token tile: under sequence parallelism the CTAs start at this rank's own tiles
  const int tile = p.sp_world > 1 ? (int)((blockIdx.y + p.sp_tile0[p.sp_rank]) % gridDim.y) : (int)blockIdx.y;
  int owner = 0;
  if (p.sp_world > 1)
    while (owner + 1 < p.sp_world && tile >= p.sp_tile0[owner + 1]) ++owner;
  const int t0 = tile * BT;
  const int kbeg = blockIdx.z * p.k_per_split;
  const int kend = min(p.K, kbeg + p.k_per_split);
  const int nkb = (kend - kbeg) / C::BK;
  const int kb_per_group = (MODE == W8A8) ? nkb : C::KB_PER_GROUP;
  const int ngroups = (MODE == W8A8) ? 1 : nkb / kb_per_group;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::AR; ++s) {
      mbar_init(&a_full[s], (MODE == W8A8) ? 1 : (C::TA ? 4 : NCONV));
      mbar_init(&a_empty[s], 1);
    }
    for (int s = 0; s < C::BR; ++s) {
      mbar_init(&b_full[s], 1);
      mbar_init(&b_empty_own[s], 1);
    }
    mbar_init(scale_bar, 1);
    for (int s = 0; s < RSTAGES; ++s) {
      mbar_init(&r_full[s], 1);
      mbar_init(&r_empty[s], C::TA ? 4 : NCONV);
    }
    for (int s = 0; s < C::NBUF; ++s) {
      mbar_init(&acc_full[s], 1);
      mbar_init(&acc_empty[s], NACC);
    }
    mbar_init(done_bar, 1);
    for (int i = 0; i < C::NMMA - 1; ++i) mbar_init(&done_more[i], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && nkb > 0) {
      prefetch_tmap(&tm_w);
      prefetch_tmap(&tm_x);
      if (MODE != W8A8) prefetch_tmap(&tm_s);
      const bool scale_copy = MODE != W8A8 && p.k_per_split / 128 <= C::MAXG;
      if (scale_copy) {
        // the CTA's scale block in one copy: the box always moves k_per_split/128
        // rows (rows past K arrive zero-filled and are never read)
        mbar_arrive_expect_tx(scale_bar, (p.k_per_split / 128) * 256);
        tma_load_2d(sScale, &tm_s, scale_bar, n0, kbeg / 128);
      }
      int issued = 0, raw_issued = 0;
      // The weights (and their scales) come from no earlier kernel: a few raw
      // stages go out before this grid waits for the previous one
      // (programmatic dependent launch), so the first weight bytes overlap its
      // tail. Only a few: the token tiles issued after the wait queue behind
      // them in the TMA unit.
      const int pre = (MODE != W8A8) ? min(min(RSTAGES, 4), nkb) : 0;
      for (int kb = 0; kb < pre; ++kb) {
        mbar_arrive_expect_tx(&r_full[kb], C::RAW_BYTES);
        tma_load_2d(sR + kb * C::RAW_BYTES, &tm_w, &r_full[kb], n0, (kbeg + kb * C::BK) / 8);
        ++raw_issued;
      }
      pdl_wait();
      if (p.ag_flag) {
        // all-gather -> GEMM: the tile's rows arrived from their owner
        if (!peer::wait_geq_u64(p.ag_flag + owner, p.ag_target[owner], 114)) *abort_flag = 1;
        peer::fence_proxy_alias();                                 // written through the multicast alias
        asm volatile("fence.proxy.async.global;" ::: "memory");    // read by TMA (the async proxy)
      }
      for (int kb = 0; kb < nkb && !*abort_flag; ++kb) {
        const int k0 = kbeg + kb * C::BK;
        if (MODE != W8A8) {
          if (kb >= pre) {
            const int rs = kb % RSTAGES;
            if (kb >= RSTAGES && !mbar_wait(&r_empty[rs], ((kb / RSTAGES) & 1) ^ 1, abort_flag, 101)) break;
            mbar_arrive_expect_tx(&r_full[rs], C::RAW_BYTES);
            tma_load_2d(sR + rs * C::RAW_BYTES, &tm_w, &r_full[rs], n0, k0 / 8);
            ++raw_issued;
          }
        } else {
          const int s = kb % STAGES;
          if (kb >= STAGES && !mbar_wait(&a_empty[s], ((kb / STAGES) & 1) ^ 1, abort_flag, 102)) break;
          mbar_arrive_expect_tx(&a_full[s], C::A_BYTES);
          tma_load_2d(sA + s * C::A_BYTES, &tm_w, &a_full[s], k0, n0);
        }
        const int bs = kb % C::BR;
        if (kb >= C::BR && !mbar_wait(&b_empty[bs], ((kb / C::BR) & 1) ^ 1, abort_flag, 109)) break;
        mbar_arrive_expect_tx(&b_full[bs], C::B_BYTES);
#pragma unroll
        for (int at = 0; at < C::B_ATOMS; ++at)
          tma_load_2d(sB + bs * C::B_BYTES + at * (BT * 128), &tm_x, &b_full[bs], k0 + at * 64,
                      C::LIMB ? blockIdx.y * C::BROWS : t0);
        K8V4_TRACE_EVENT(0, kb);
        ++issued;
      }
      if (*abort_flag) {
        // Wait (bounded) for this CTA's own copies still in flight.
        if (scale_copy) mbar_wait_drain(scale_bar, 0);
        for (int kb = issued - 1; kb >= 0 && kb >= issued - C::BR; --kb)
          mbar_wait_drain(&b_full[kb % C::BR], (kb / C::BR) & 1);
        if (MODE == W8A8)
          for (int kb = issued - 1; kb >= 0 && kb >= issued - STAGES; --kb)
            mbar_wait_drain(&a_full[kb % STAGES], (kb / STAGES) & 1);
        if (MODE != W8A8)
          for (int kb = raw_issued - 1; kb >= 0 && kb >= raw_issued - RSTAGES; --kb)
            mbar_wait_drain(&r_full[kb % RSTAGES], (kb / RSTAGES) & 1);
      }
    }
  } else if (warp == 1 || warp >= 2 + NCONV + NACC) {
    // ----------------------------------------------------------------- MMA
    // issuer i (warp 1, then the last NMMA-1 warps) takes K groups g with
    // g % NMMA == i; group g accumulates into buffer g % NBUF, whose reuse
    // waits on the accumulators whichever issuer filled it last.
    if (lane == 0 && nkb > 0) {
      const int issuer = (warp == 1) ? 0 : warp - (2 + NCONV + NACC) + 1;
      const uint32_t idesc = (MODE == W4A16) ? idesc_bf16(128, BT)
                             : C::LIMB     ? idesc_i8(128, C::BROWS, false, true)  // u8 codes x s8 limbs
                                           : idesc_s8(128, BT);
      bool ok = true;
      for (int g = issuer; g < ngroups && ok; g += C::NMMA) {
        const int buf = g % C::NBUF;
#ifdef K8V4_TRACE
        const uint64_t te0 = globaltimer_ns();
#endif
        if (g >= C::NBUF && !mbar_wait(&acc_empty[buf], ((g / C::NBUF) - 1) & 1, abort_flag, 103)) break;
#ifdef K8V4_TRACE
        if (blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && g < 256)
          g_gemm_trace[6 * 256 + g] = globaltimer_ns() - te0;
#endif
        tc_fence_after();
        const uint32_t dtm = tmem + buf * C::BROWS;
        for (int j = 0; j < kb_per_group; ++j) {
          const int kb = g * kb_per_group + j;
          const int s = kb % C::AR, bs = kb % C::BR;
          // TMEM-A path: the converters already waited for this stage's token tile
#ifdef K8V4_TRACE
          const uint64_t tw0 = globaltimer_ns();
#endif
          if (!mbar_wait(&a_full[s], (kb / C::AR) & 1, abort_flag, 104) ||
              (!C::TA && !mbar_wait(&b_full[bs], (kb / C::BR) & 1, abort_flag, 105))) {
            ok = false;
            break;
          }
#ifdef K8V4_TRACE
          if (blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && kb < 256)
            g_gemm_trace[4 * 256 + kb] = globaltimer_ns() - tw0;
#endif
          tc_fence_after();
          const uint32_t b_base = smem_u32(sB + bs * C::B_BYTES);
          if (C::LIMB) {
            const uint32_t a_tm = tmem + C::D_COLS + s * C::A_COLS;
#pragma unroll
            for (int kk = 0; kk < C::BK / C::UMMA_K; ++kk)  // 4 MMAs of K = 32 (8 TMEM columns of A each)
              mma_i8_ts(dtm, a_tm + kk * 8, sdesc_sw128(b_base + kk * 32, 16, 1024), idesc, kk > 0 ? 1u : 0u);
            mma_commit(&a_empty[s]);  // frees the TMEM A stage and the limb stage
          } else if (C::TA) {
            const uint32_t a_tm = tmem + C::D_COLS + s * C::A_COLS;
#pragma unroll
            for (int kk = 0; kk < C::BK / C::UMMA_K; ++kk)
              mma_f16_ts(dtm, a_tm + kk * 8,
                         sdesc_sw128(b_base + (kk >> 2) * (BT * 128) + (kk & 3) * 32, 16, 1024), idesc,
                         (j > 0 || kk > 0) ? 1u : 0u);
            mma_commit(&a_empty[s]);  // frees the TMEM A stage and the token stage
          } else {
            const uint32_t a_base = smem_u32(sA + s * C::A_BYTES);
#pragma unroll
            for (int kk = 0; kk < C::BK / C::UMMA_K; ++kk) {
              const uint64_t ad = sdesc_sw128(a_base + kk * 32, 16, 1024);
              const uint64_t bd = sdesc_sw128(b_base + kk * 32, 16, 1024);
              if (MODE == W4A16)
                mma_f16(dtm, ad, bd, idesc, (j > 0 || kk > 0) ? 1u : 0u);
              else
                mma_i8(dtm, ad, bd, idesc, (j > 0 || kk > 0) ? 1u : 0u);
            }
            mma_commit(&a_empty[s]);
            mma_commit(&b_empty[bs]);
          }
          K8V4_TRACE_EVENT(2, kb);
        }
        if (ok) mma_commit(&acc_full[buf]);
      }
      // Every MMA this thread issued must finish before TMEM is released.
      uint64_t* dbar = issuer == 0 ? done_bar : &done_more[issuer - 1];
      mma_commit(dbar);
      mbar_wait_drain(dbar, 0);
    }
  } else if (warp < 2 + NCONV) {
    // ---------------------------------------------------------- converters
    if (C::TA) {
      // Teams of 4 warps (one per TMEM lane quadrant) take alternate
      // k-blocks; each thread converts one weight row (feature) of the block
      // into 32 columns of bf16 pairs and stores them with one tcgen05.st.
      const int cw = warp - 2;
      const int team = cw >> 2, nteams = NCONV / 4;
      const int quad = warp & 3;
      const int f = quad * 32 + lane;
      const uint32_t lane_base = tmem + C::D_COLS + ((uint32_t)(quad * 32) << 16);
      for (int kb = team; kb < nkb; kb += nteams) {
        const int rs = kb % RSTAGES, ts = kb % C::AR;
        if (!mbar_wait_all(&r_full[rs], (kb / RSTAGES) & 1, abort_flag, 110)) break;
        if (kb >= C::AR && !mbar_wait_all(&a_empty[ts], ((kb / C::AR) - 1) & 1, abort_flag, 111)) break;
        if (quad == 0 && lane == 0) K8V4_TRACE_EVENT(5, kb);
        const uint32_t* raw = reinterpret_cast<const uint32_t*>(sR + rs * C::RAW_BYTES);
        const uint32_t dst = lane_base + ts * C::A_COLS;
        if (C::LIMB) {
          // 16 words of 8 codes -> 32 columns of 4 u8 codes (q + 8) in k order
          uint32_t v[32];
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            const uint32_t w = raw[c * 128 + f];
            const uint32_t lo = w & 0x0F0F0F0Fu;          // codes k0 k2 k4 k6
            const uint32_t hi = (w >> 4) & 0x0F0F0F0Fu;   // codes k1 k3 k5 k7
            v[2 * c] = __byte_perm(lo, hi, 0x5140);       // k0 k1 k2 k3
            v[2 * c + 1] = __byte_perm(lo, hi, 0x7362);   // k4 k5 k6 k7
          }
          tc_fence_after();  // the MMA that read this TMEM stage has completed
          tmem_st32(dst, v);
        } else {
#pragma unroll
          for (int half = 0; half < C::BK / 64; ++half) {
            uint32_t v[32];
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              uint32_t o[4];
              int4x8_to_bf16(raw[(half * 8 + c) * 128 + f], o);
              v[4 * c] = o[0];
              v[4 * c + 1] = o[1];
              v[4 * c + 2] = o[2];
              v[4 * c + 3] = o[3];
            }
            if (half == 0) tc_fence_after();  // the MMA that read this TMEM stage has completed
            tmem_st32(dst + half * 32, v);
          }
        }
        if (quad == 0 && lane == 0) K8V4_TRACE_EVENT(7, kb);
        tmem_st_wait();
        tc_fence_before();
        // the MMA waits only on a_full: hand over once the token tile landed too
        if (!mbar_wait_all(&b_full[ts], (kb / C::AR) & 1, abort_flag, 112)) break;
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&r_empty[rs]);
          mbar_arrive(&a_full[ts]);
          if (quad == 0) K8V4_TRACE_EVENT(1, kb);
        }
      }
    } else if (MODE != W8A8) {
      const int ct = threadIdx.x - 64;  // 0 .. NCONV*32-1
      int rs = 0, rphase = 0;
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % STAGES;
        const uint32_t ph = (kb / STAGES) & 1;
        if (!mbar_wait_all(&r_full[rs], rphase, abort_flag, 106)) break;
        if (kb >= STAGES && !mbar_wait_all(&a_empty[s], ph ^ 1, abort_flag, 107)) break;
        const uint32_t* raw = reinterpret_cast<const uint32_t*>(sR + rs * C::RAW_BYTES);
        uint8_t* dst = sA + s * C::A_BYTES;
#pragma unroll 4
        for (int item = ct; item < 1024; item += NCONV * 32) {
          const int f = item & 127;
          const int c = item >> 7;
          uint4 v;
          if (MODE == W4A16) {
            uint32_t o[4];
            int4x8_to_bf16(raw[c * 128 + f], o);
            v = make_uint4(o[0], o[1], o[2], o[3]);
          } else {
            uint32_t o0, o1, o2, o3;
            int4x8_to_s8(raw[(2 * c) * 128 + f], o0, o1);
            int4x8_to_s8(raw[(2 * c + 1) * 128 + f], o2, o3);
            v = make_uint4(o0, o1, o2, o3);
          }
          *reinterpret_cast<uint4*>(dst + sw128_offset(f, c)) = v;
        }
        fence_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&r_empty[rs]);
          mbar_arrive(&a_full[s]);
        }
        if (++rs == RSTAGES) { rs = 0; rphase ^= 1; }
      }
    }
  } else {
    // --------------------------------------------------------- accumulators
    const int aw = warp - 2 - NCONV;  // 0 .. NACC-1
    const int quad = warp & 3;        // TMEM lane quadrant this warp may access
    const int slice = aw / 4;         // column slice
    const int row = quad * 32 + lane; // feature within the tile
    const int n = n0 + row;
    const int c0 = slice * C::COLS;
    float acc[C::COLS];
#pragma unroll
    for (int i = 0; i < C::COLS; ++i) acc[i] = 0.f;
    // Group scales of this CTA's K range: one TMA copy into shared memory
    // (issued by the producer at start), so no global load sits between an
    // MMA's completion and the release of its TMEM buffer.
    const bool staged = (MODE != W8A8) && p.k_per_split / 128 <= C::MAXG && nkb > 0;
    bool scales_ok = true;
    if (C::LIMB) {
      // the group sums of this CTA's tokens (made by the previous kernel)
      pdl_wait();
      const int kg0 = kbeg / 128, kgs = p.K / 128;
      for (int i = threadIdx.x - 32 * (2 + NCONV); i < ngroups * BT; i += 32 * NACC) {
        const int g = i / BT, c = i % BT, t = t0 + c;
        sCsum[g * BT + c] = (t < p.M && g < C::MAXG) ? p.csum[(size_t)t * kgs + kg0 + g] : 0;
      }
      asm volatile("bar.sync 1, %0;" ::"n"(32 * NACC) : "memory");  // the accumulator warps only
    }
    if (staged) scales_ok = mbar_wait_all(scale_bar, 0, abort_flag, 113);
    bool ok = nkb > 0 && scales_ok;
    for (int g = 0; g < ngroups && ok; ++g) {
      const int buf = g % C::NBUF;
      if (!mbar_wait_all(&acc_full[buf], (g / C::NBUF) & 1, abort_flag, 108)) { ok = false; break; }
      tc_fence_after();
      float gs = 1.f;
      if (MODE != W8A8)
        gs = staged ? __half2float(sScale[g * 128 + row])
                    : (n < p.N ? __half2float(p.wscale[(size_t)((kbeg / 128) + g) * p.N + n]) : 0.f);
      const uint32_t taddr = tmem + ((uint32_t)(quad * 32) << 16) + buf * C::BROWS + c0;
      if (C::LIMB) {
#pragma unroll
        for (int cc = 0; cc < C::COLS; cc += 8) {
          uint32_t h[8], l[8];
          tmem_ld8(taddr + cc, h);
          tmem_ld8(taddr + BT + cc, l);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            // 128 D_hi + D_lo - 8 C = sum over the group of q * X, exactly
            const int v = (int)h[i] * 128 + (int)l[i] - 8 * sCsum[g * BT + c0 + cc + i];
            acc[cc + i] = fmaf((float)v, gs, acc[cc + i]);
          }
        }
      } else {
#pragma unroll
        for (int cc = 0; cc < C::COLS; cc += 16) {
          uint32_t r[16];
          tmem_ld8(taddr + cc, *reinterpret_cast<uint32_t(*)[8]>(&r[0]));
          if (cc + 8 < C::COLS) tmem_ld8(taddr + cc + 8, *reinterpret_cast<uint32_t(*)[8]>(&r[8]));
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            if (cc + i < C::COLS) {
              const float v = (MODE == W4A16) ? __uint_as_float(r[i])
                                              : ((MODE == W4A8) ? i2f_small(r[i]) : (float)(int)r[i]);
              acc[cc + i] = fmaf(v, gs, acc[cc + i]);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
      if (lane == 0 && aw == 0) K8V4_TRACE_EVENT(3, g);
    }
    if (ok && n < p.N) {
      const float rs = (MODE == W8A8) ? __half2float(p.wscale[n]) : 1.f;
#pragma unroll
      for (int i = 0; i < C::COLS; ++i) {
        const int t = t0 + c0 + i;
        if (t < p.M) {
          float v = acc[i] * rs;
          if (MODE != W4A16) v *= p.xscale[t];
          const size_t o = (size_t)t * p.ldo + n;
          if (p.ws_mc) {
            peer::mc_red_add_f32(p.ws_mc + o, v);
          } else if (p.rs_dst[0]) {
            // reduce-scatter: this rank's partial row goes to the owner's slot
            p.rs_dst[owner][(size_t)(t - p.sp_tile0[owner] * BT) * p.ldo + n] = __float2bfloat16_rn(v);
          } else if (gridDim.z > 1) {
            atomicAdd(p.ws + o, v);
          } else {
            if (p.residual) v += __bfloat162float(p.residual[o]);
            p.out[o] = __float2bfloat16_rn(v);
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
  if (p.rs_dst[0] && threadIdx.x == 0) {
    // the CTA's partial rows (ordered before this point by the barrier) are
    // in the owner's slot: signal it
    peer::fence_sys();
    peer::red_release_add_u64(p.rs_sig[owner], 1ull);
  }
  if (p.flag_mc && threadIdx.x == 0) {
    // the CTA's multicast adds (ordered before this point by the barrier) are
    // out: publish them to every rank
    peer::fence_proxy_alias();
#ifdef K8V4_AR_FENCE_SYS
    peer::fence_sys();
#endif
    peer::mc_signal_add_u64(p.flag_mc, 1ull);
  }
}

// ------------------------------------------------------------ limb preparation
// One CTA per token row of x [M, K] (bf16): s = amax / 16319, X = rint(x / s)
// (|X| <= 16319), hi = floor((X + 64) / 128) in [-127, 127], lo = X - 128 hi
// in [-64, 63]. Rows go to the limb operand of tile t / bt: hi at row
// t % bt, lo at row bt + t % bt. Also the per-row scale and the integer sum
// of X over every 128-k group (the correction of the unsigned weight codes).
constexpr float kLimbMax = 16319.f;

__global__ void __launch_bounds__(256) limbs_kernel(const __nv_bfloat16* __restrict__ x, int K, int bt,
                                                    int8_t* __restrict__ limbs, float* __restrict__ scale,
                                                    int32_t* __restrict__ gsum) {
  pdl_trigger();
  pdl_wait();  // x comes from the previous kernel
  __shared__ float red[8];
  const int t = blockIdx.x;
  const __nv_bfloat16* row = x + (size_t)t * K;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float am = 0.f;
  for (int k = threadIdx.x * 8; k < K; k += 256 * 8) {
    const uint4 raw = *reinterpret_cast<const uint4*>(row + k);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 v = __bfloat1622float2(h[j]);
      am = fmaxf(am, fmaxf(fabsf(v.x), fabsf(v.y)));
    }
  }
  am = warp_max(am);
  if (lane == 0) red[warp] = am;
  __syncthreads();
  am = lane < 8 ? red[lane] : 0.f;
  am = warp_max(am);
  const float s = am > 0.f ? am / kLimbMax : 1.f;
  const float inv = 1.f / s;
  int8_t* hi_row = limbs + ((size_t)(t / bt) * 2 * bt + (t % bt)) * K;
  int8_t* lo_row = hi_row + (size_t)bt * K;
  const int groups = K / 128;
  for (int g = warp; g < groups; g += 8) {
    const int k = g * 128 + lane * 4;
    const uint2 raw = *reinterpret_cast<const uint2*>(row + k);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
    uint32_t hw = 0, lw = 0;
    int sum = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float v = __bfloat162float(j & 1 ? h[j >> 1].y : h[j >> 1].x);
      const int X = (int)fminf(fmaxf(rintf(v * inv), -kLimbMax), kLimbMax);
      const int hv = (X + 64) >> 7;  // arithmetic shift: floor
      const int lv = X - 128 * hv;
      hw |= ((uint32_t)(uint8_t)(int8_t)hv) << (8 * j);
      lw |= ((uint32_t)(uint8_t)(int8_t)lv) << (8 * j);
      sum += X;
    }
    *reinterpret_cast<uint32_t*>(hi_row + k) = hw;
    *reinterpret_cast<uint32_t*>(lo_row + k) = lw;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) gsum[(size_t)t * groups + g] = sum;
  }
  if (threadIdx.x == 0) scale[t] = s;
}

// -------------------------------------------------------------------- host
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode() {
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

// 2D row-major tensor map: inner dim `cols` (elements), `rows` rows, row stride in bytes.
int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem_bytes, uint64_t cols,
                 uint64_t rows, uint64_t row_stride_bytes, uint32_t box_cols, uint32_t box_rows, bool swizzle128) {
  EncodeTiledFn enc = get_encode();
  if (!enc) return -1;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  (void)elem_bytes;
  CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -2;
}

// Sequence-parallel arguments of one GEMM call (see the kernel's notes).
struct SpArgs {
  int world, rank;
  int tile0[9];
  const unsigned long long* ag_flag;  // null: no all-gather wait
  unsigned long long ag_target[8];
  __nv_bfloat16* rs_dst[8];           // rs_dst[0] null: no reduce-scatter
  unsigned long long* rs_sig[8];
};

struct LimbBufs {
  int8_t* limbs;   // [tiles x 2 bt, K]
  float* scale;    // [M]
  int32_t* gsum;   // [M, K / 128]
};

template <int MODE, int BT, int NCONV, int NACC, int STAGES, int RSTAGES, int BSTAGES>
static int launch_cfg(const void* w, const void* x, const Params& p, int split, cudaStream_t st) {
  const void* wscale_ptr = p.wscale;
  using C = Cfg<MODE, BT, NCONV, NACC, STAGES, RSTAGES, BSTAGES>;
  CUtensorMap tw, tx;
  int rc;
  if (MODE == W8A8)
    rc = make_tmap_2d(&tw, w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, p.K, p.N, p.K, 128, 128, true);
  else
    rc = make_tmap_2d(&tw, w, CU_TENSOR_MAP_DATA_TYPE_INT32, 4, p.N, p.K / 8, (uint64_t)p.N * 4, 128, C::BK / 8,
                      false);
  if (rc) return 100 + rc;
  if (MODE == W4A16)
    rc = make_tmap_2d(&tx, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, p.K, p.M, (uint64_t)p.K * 2, 64, BT, true);
  else if (MODE == W4L)  // the limb operand: [tiles x (hi rows, lo rows), K] int8
    rc = make_tmap_2d(&tx, x, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, p.K, (uint64_t)cdiv(p.M, BT) * 2 * BT, p.K, 128,
                      2 * BT, true);
  else
    rc = make_tmap_2d(&tx, x, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, p.K, p.M, p.K, 128, BT, true);
  if (rc) return 200 + rc;
  CUtensorMap ts;
  if (MODE != W8A8) {
    // group scales [K/128, N] fp16: one box of (128 features x groups of one split)
    const int groups = p.k_per_split / 128;
    rc = make_tmap_2d(&ts, wscale_ptr, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p.N, p.K / 128, (uint64_t)p.N * 2, 128,
                      groups <= C::MAXG ? groups : 1, false);
    if (rc) return 400 + rc;
  } else {
    ts = tx;  // unused
  }
  auto kern = wq_gemm_kernel<MODE, BT, NCONV, NACC, STAGES, RSTAGES, BSTAGES>;
  if (ensure_smem_limit<wq_gemm_kernel<MODE, BT, NCONV, NACC, STAGES, RSTAGES, BSTAGES>>(C::SMEM_BYTES) != cudaSuccess)
    return 300;
  dim3 grid(cdiv(p.N, 128), cdiv(p.M, BT), split);
  return launch_k(kern, grid, dim3(C::NTHREADS), C::SMEM_BYTES, st, tw, tx, ts, p) == cudaSuccess ? 0 : 300;
}

}  // namespace gemm
}  // namespace k8v4

using namespace k8v4;
using namespace k8v4::gemm;

K8V4_STATUS_API(gemm)

#ifdef K8V4_TRACE
extern "C" int k8v4_gemm_trace(uint64_t* host, int clear) {
  int rc = cudaMemcpyFromSymbol(host, g_gemm_trace, sizeof(uint64_t) * 8 * 256);
  if (clear) {
    static uint64_t zeros[8 * 256] = {0};
    cudaMemcpyToSymbol(g_gemm_trace, zeros, sizeof(zeros));
  }
  return rc;
}
#endif

// Tokens per CTA for a given M: small M streams weights (decode), large M
// reuses each converted weight tile over 128 tokens (prefill).
// converter warps of the decode (TMEM-A) configurations: teams of 4
#ifndef K8V4_GEMM_NCONV
#define K8V4_GEMM_NCONV 12
#endif

static int pick_bt(int mode, int M) {
  if (mode == W4A16) return M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : 128;
  return M <= 32 ? 32 : 128;
}

static int k_per_split_for(int K, int split) {
  const int kgroups = K / 128;
  if (split < 1) split = 1;
  if (split > kgroups) split = kgroups;
  return cdiv(kgroups, split) * 128;
}

// Token rows up to which a W4A16 call runs as W4L (when the caller gave limb buffers).
constexpr int kLimbMaxRows = 32;

static int limb_bt(int M) { return M <= 16 ? 16 : 32; }

static int gemm_impl(int mode, const void* w, const void* wscale, const void* x, const float* xscale,
                     const void* residual, void* out, float* ws, float* ws_mc, unsigned long long* flag_mc, int M,
                     int N, int K, int ldo, int split, cudaStream_t st, const LimbBufs* lb = nullptr,
                     const SpArgs* sp = nullptr) {
  if (N % 128 || K % 128 || M <= 0) return 1;
  Params p;
  p.qweight = reinterpret_cast<const int32_t*>(w);
  p.wscale = reinterpret_cast<const __half*>(wscale);
  p.xscale = xscale;
  p.residual = reinterpret_cast<const __nv_bfloat16*>(residual);
  p.out = reinterpret_cast<__nv_bfloat16*>(out);
  p.ws = ws;
  p.ws_mc = ws_mc;
  p.flag_mc = flag_mc;
  p.csum = nullptr;
  p.sp_world = 0;
  p.sp_rank = 0;
  p.ag_flag = nullptr;
  for (int i = 0; i < 9; ++i) p.sp_tile0[i] = 0;
  for (int i = 0; i < 8; ++i) {
    p.ag_target[i] = 0;
    p.rs_dst[i] = nullptr;
    p.rs_sig[i] = nullptr;
  }
  if (sp) {
    // sequence parallelism works on whole 128-row token tiles
    if (sp->world < 2 || sp->world > 8 || sp->rank < 0 || sp->rank >= sp->world || pick_bt(mode, M) != 128 ||
        split != 1 || ws_mc || (!sp->ag_flag && !sp->rs_dst[0]))
      return 6;
    p.sp_world = sp->world;
    p.sp_rank = sp->rank;
    for (int i = 0; i <= sp->world; ++i) p.sp_tile0[i] = sp->tile0[i];
    if (p.sp_tile0[0] != 0 || p.sp_tile0[sp->world] != cdiv(M, 128)) return 6;
    p.ag_flag = sp->ag_flag;
    for (int i = 0; i < sp->world; ++i) {
      p.ag_target[i] = sp->ag_target[i];
      p.rs_dst[i] = sp->rs_dst[i];
      p.rs_sig[i] = sp->rs_sig[i];
    }
  }
  p.M = M;
  p.N = N;
  p.K = K;
  p.ldo = ldo;
  p.k_per_split = k_per_split_for(K, split);
  split = cdiv(K, p.k_per_split);
  if (split > 1 && !ws && !ws_mc) return 2;
  const int bt = pick_bt(mode, M);
  if (mode == W4A16 && lb && lb->limbs && M <= kLimbMaxRows && K / 128 <= 144) {
    const int lbt = limb_bt(M);
    if (launch_k(limbs_kernel, dim3(M), dim3(256), 0, st, reinterpret_cast<const __nv_bfloat16*>(x), K, lbt,
                 lb->limbs, lb->scale, lb->gsum) != cudaSuccess)
      return 5;
    p.xscale = lb->scale;
    p.csum = lb->gsum;
    if (lbt == 16) return launch_cfg<W4L, 16, K8V4_GEMM_NCONV, 4, 4, 12, 16>(w, lb->limbs, p, split, st);
    return launch_cfg<W4L, 32, K8V4_GEMM_NCONV, 4, 4, 12, 16>(w, lb->limbs, p, split, st);
  }
  if (mode == W4A16) {
    if (bt == 16) return launch_cfg<W4A16, 16, K8V4_GEMM_NCONV, 4, 4, 16, 16>(w, x, p, split, st);
    if (bt == 32) return launch_cfg<W4A16, 32, K8V4_GEMM_NCONV, 4, 4, 12, 16>(w, x, p, split, st);
    if (bt == 64) return launch_cfg<W4A16, 64, K8V4_GEMM_NCONV, 4, 4, 8, 8>(w, x, p, split, st);
    return launch_cfg<W4A16, 128, 4, 8, 4, 8, 4>(w, x, p, split, st);
  }
  if (mode == W4A8) {
    if (bt == 32) return launch_cfg<W4A8, 32, 8, 4, 4, 8, 12>(w, x, p, split, st);
    return launch_cfg<W4A8, 128, 4, 8, 4, 4, 4>(w, x, p, split, st);
  }
  if (mode == W8A8) {
    if (bt == 32) return launch_cfg<W8A8, 32, 4, 4, 6, 1, 6>(w, x, p, split, st);
    return launch_cfg<W8A8, 128, 4, 8, 4, 1, 4>(w, x, p, split, st);
  }
  return 3;
}

extern "C" int k8v4_wq_gemm(int mode, const void* w, const void* wscale, const void* x, const float* xscale,
                            const void* residual, void* out, float* ws, int M, int N, int K, int ldo, int split,
                            cudaStream_t st) {
  return gemm_impl(mode, w, wscale, x, xscale, residual, out, ws, nullptr, nullptr, M, N, K, ldo, split, st);
}

// Bytes of the limb buffers a W4A16 call of M rows and K columns needs (0
// when the call does not take the limb path): limb operand, row scales, group
// sums, each part 256-byte aligned.
extern "C" int64_t k8v4_wq_gemm_limb_bytes(int M, int K) {
  if (M <= 0 || M > kLimbMaxRows || K % 128 || K / 128 > 144) return 0;
  const int bt = limb_bt(M);
  auto up = [](int64_t b) { return (b + 255) / 256 * 256; };
  return up((int64_t)cdiv(M, bt) * 2 * bt * K) + up((int64_t)M * 4) + up((int64_t)M * (K / 128) * 4);
}

static LimbBufs carve_limbs(void* buf, int M, int K) {
  LimbBufs lb{nullptr, nullptr, nullptr};
  if (!buf) return lb;
  const int bt = limb_bt(M);
  auto up = [](int64_t b) { return (b + 255) / 256 * 256; };
  uint8_t* b = static_cast<uint8_t*>(buf);
  lb.limbs = reinterpret_cast<int8_t*>(b);
  b += up((int64_t)cdiv(M, bt) * 2 * bt * K);
  lb.scale = reinterpret_cast<float*>(b);
  b += up((int64_t)M * 4);
  lb.gsum = reinterpret_cast<int32_t*>(b);
  return lb;
}

// W4A16 with the limb buffers of k8v4_wq_gemm_limb_bytes(M, K) bytes: calls of
// at most 32 rows run as W4L (limbs_kernel, then the int8 GEMM); others as
// k8v4_wq_gemm.
extern "C" int k8v4_wq_gemm_limbs(const void* w, const void* wscale, const void* x, const void* residual, void* out,
                                  float* ws, void* limb_buf, int M, int N, int K, int ldo, int split,
                                  cudaStream_t st) {
  const LimbBufs lb = carve_limbs(limb_buf, M, K);
  return gemm_impl(W4A16, w, wscale, x, nullptr, residual, out, ws, nullptr, nullptr, M, N, K, ldo, split, st, &lb);
}

// GEMM -> all-reduce: fp32 sums into every rank's copy of a symmetric buffer
// through its multicast address `ws_mc`, then one signal per CTA on the
// multicast counter `flag_mc`. The consumer expects world x
// k8v4_wq_gemm_ctas(...) signals for one call.
extern "C" int k8v4_wq_gemm_allreduce(int mode, const void* w, const void* wscale, const void* x, const float* xscale,
                                      float* ws_mc, unsigned long long* flag_mc, int M, int N, int K, int ldo,
                                      int split, cudaStream_t st, void* limb_buf) {
  if (!ws_mc || !flag_mc) return 4;
  const LimbBufs lb = carve_limbs(mode == W4A16 ? limb_buf : nullptr, M, K);
  return gemm_impl(mode, w, wscale, x, xscale, nullptr, nullptr, nullptr, ws_mc, flag_mc, M, N, K, ldo, split, st,
                   &lb);
}

// Sequence-parallel prefill GEMM (tensor parallel, token tiles of 128 rows
// owned by ranks in runs tile0[o] .. tile0[o + 1]). With ag_flag set, x is
// this rank's copy of the all-gathered rows and each CTA first waits until
// ag_flag[owner] >= ag_target[owner]. With rs_dst set, the output goes as bf16
// partial rows into rs_dst[owner] (row stride ldo) and each CTA then adds 1 to
// rs_sig[owner]; `out` is not written. Returns 6 for an unsupported call.
extern "C" int k8v4_wq_gemm_sp(int mode, const void* w, const void* wscale, const void* x, const float* xscale,
                               void* out, int M, int N, int K, int ldo, int world, int rank, const int* tile0,
                               const unsigned long long* ag_flag, const unsigned long long* ag_target,
                               void* const* rs_dst, unsigned long long* const* rs_sig, cudaStream_t st) {
  SpArgs sp;
  sp.world = world;
  sp.rank = rank;
  if (world < 2 || world > 8) return 6;
  for (int i = 0; i <= world; ++i) sp.tile0[i] = tile0[i];
  sp.ag_flag = ag_flag;
  for (int i = 0; i < 8; ++i) {
    sp.ag_target[i] = (ag_target && i < world) ? ag_target[i] : 0;
    sp.rs_dst[i] = (rs_dst && i < world) ? reinterpret_cast<__nv_bfloat16*>(rs_dst[i]) : nullptr;
    sp.rs_sig[i] = (rs_sig && i < world) ? rs_sig[i] : nullptr;
  }
  if (rs_dst && (!sp.rs_dst[0] || !sp.rs_sig[0])) return 6;
  return gemm_impl(mode, w, wscale, x, xscale, nullptr, out, nullptr, nullptr, nullptr, M, N, K, ldo, 1, st, nullptr,
                   &sp);
}

// CTAs one call launches (the number of signals it sends per rank).
extern "C" int k8v4_wq_gemm_ctas(int mode, int M, int N, int K, int split) {
  if (N % 128 || K % 128 || M <= 0) return 0;
  const int kps = k_per_split_for(K, split);
  return (N / 128) * cdiv(M, pick_bt(mode, M)) * cdiv(K, kps);
}
