// Torch op registry for the k8v4 sm_100a kernel library: torch.ops.k8v4.*.
//
// Each op validates dtypes, devices, shapes and strides on the host, then
// calls the raw-pointer launcher of its .cu file on the current stream. The
// op set mirrors the reference's xe2_kv registry (k8v4_v030/native/
// xe2_kv_ops.cpp:1779-1837) where the semantics carry over (paged store,
// batched decode over every request in one launch) and adds the GEMM, norm,
// activation, embedding and prefill-attention ops the reference took from
// libraries.
#include <string>
#include <vector>
#include <torch/library.h>
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_runtime.h>

extern "C" {
int k8v4_kv_store(int fmt, const void* k, int64_t k_stride_t, const void* v, int64_t v_stride_t, const int64_t* slots,
                  void* cache, int64_t num_pages, int page_bytes, int T, int hkv, cudaStream_t st);
int k8v4_rope_store(const void* qkv, int qkv_fp32, const float* cos_sin, const int64_t* positions, void* q_out,
                    const int64_t* slots, void* cache, int64_t num_pages, int page_bytes, int T, int hq, int hkv,
                    cudaStream_t st);
int k8v4_decode_attn(const void* q, const int32_t* cu_q, const int32_t* seq_lens, const int32_t* q_ends,
                     const int32_t* block_table, int bt_stride, const void* cache, int64_t num_pages, int hkv,
                     int head_offset, int heads, int gqa, int hq_total, int nseq, int max_q_len, int nsplit,
                     float sm_scale, void* out, float* ws_o, float* ws_ml, cudaStream_t st);
int64_t k8v4_decode_ws_floats(int nseq, int heads, int nsplit, int max_q_len, int gqa);
int k8v4_decode_attn_push(const void* q, const int32_t* cu_q, const int32_t* seq_lens, const int32_t* q_ends,
                          const int32_t* block_table, int bt_stride, const void* cache, int64_t num_pages, int hkv,
                          int head_offset, int heads, int gqa, int hq_total, int nseq, int max_q_len, int nsplit,
                          float sm_scale, float* slot_mc, unsigned long long* flag_mc, cudaStream_t st);
int k8v4_decode_combine_ranks_sync(const float* ws_all, int64_t rank_floats, const int32_t* cu_q, void* out,
                                   int nrank, int nsplit, int nseq, int heads, int head_offset, int gqa, int hq_total,
                                   int max_q_len, const unsigned long long* sync_flag, unsigned long long* sync_state,
                                   unsigned long long sync_expected, cudaStream_t st);
int k8v4_prefill_attn(const void* q, const int32_t* cu_q, const int32_t* seq_lens, const int32_t* block_table,
                      int bt_stride, int bt_width, const void* cache, int64_t num_pages, int hkv, int head_offset,
                      int heads, int gqa, int hq_total, int nseq, int max_q_len, float sm_scale, void* stage,
                      void* out, cudaStream_t st);
int64_t k8v4_prefill_stage_bytes(int nseq, int bt_width, int heads);
int k8v4_wq_gemm(int mode, const void* w, const void* wscale, const void* x, const float* xscale,
                 const void* residual, void* out, float* ws, int M, int N, int K, int ldo, int split,
                 cudaStream_t st);
int k8v4_rmsnorm(const void* x, float* xf, void* residual, const void* w, void* y, int64_t ldy, void* yq,
                 float* yscale, int rows, int n, float eps, const unsigned long long* sync_flag,
                 unsigned long long* sync_state, unsigned long long sync_expected, cudaStream_t st);
int k8v4_wq_gemm_allreduce(int mode, const void* w, const void* wscale, const void* x, const float* xscale,
                           float* ws_mc, unsigned long long* flag_mc, int M, int N, int K, int ldo, int split,
                           cudaStream_t st, void* limb_buf);
int64_t k8v4_wq_gemm_limb_bytes(int M, int K);
int k8v4_wq_gemm_sp(int mode, const void* w, const void* wscale, const void* x, const float* xscale, void* out, int M,
                    int N, int K, int ldo, int world, int rank, const int* tile0, const unsigned long long* ag_flag,
                    const unsigned long long* ag_target, void* const* rs_dst, unsigned long long* const* rs_sig,
                    cudaStream_t st);
int k8v4_rmsnorm_sp(const void* slots, int world, int64_t slot_stride, const void* x_local, void* residual,
                    int init_residual, const void* w, int rows, int n, float eps, const unsigned long long* rs_flag,
                    unsigned long long rs_target, void* y, void* yq, float* ys, int64_t row0, int mc,
                    unsigned long long* ag_sig_mc, cudaStream_t st);
int k8v4_wq_gemm_limbs(const void* w, const void* wscale, const void* x, const void* residual, void* out, float* ws,
                       void* limb_buf, int M, int N, int K, int ldo, int split, cudaStream_t st);
int k8v4_wq_gemm_ctas(int mode, int M, int N, int K, int split);
int k8v4_silu_mul(const void* gu, void* y, void* yq, float* yscale, int rows, int inter, cudaStream_t st);
int k8v4_silu_mul_f32(float* gu, void* y, int rows, int inter, cudaStream_t st);
int k8v4_quant_rows(const void* x, void* q, float* scale, int rows, int n, cudaStream_t st);
int k8v4_embed_int8(const int64_t* ids, const void* codes, const void* scales, void* out, int T, int n,
                    int64_t start, int64_t rows, cudaStream_t st);
int k8v4_splitk_finish(float* ws, const void* residual, void* out, int64_t total, int zero_ws, cudaStream_t st);
int k8v4_gemv_w4_max_rows();
int k8v4_gemv_w4_allreduce(const void* w, const void* wscale, const void* x, float* local, float* ws_mc,
                           unsigned long long* flag_mc, unsigned int* ticket, int M, int N, int K, int ldx, int ldo,
                           cudaStream_t st);
int k8v4_gemv_w4_ctas(int M, int N, int K);
int k8v4_gemv_w4(const void* w, const void* wscale, const void* x, float* ws, int M, int N, int K, int ldx, int ldo,
                 cudaStream_t st);
int k8v4_int8_dequant(const void* q, const void* scale, void* out, int N, int K, cudaStream_t st);
int k8v4_argmax(const void* logits, int rows, int vocab, int64_t ld, int64_t offset, float* best_val,
                int64_t* best_idx, cudaStream_t st);
int k8v4_status_gemm(int clear);
int k8v4_status_store(int clear);
int k8v4_status_misc(int clear);
int k8v4_status_decode(int clear);
int k8v4_status_prefill(int clear);
int k8v4_status_sampler(int clear);
int k8v4_status_gather(int clear);
int k8v4_prefill_attn_multi(const void* q, const int32_t* cu_q, const int32_t* seq_lens, const int32_t* block_table,
                            int bt_stride, int bt_width, const void* const* caches, int nsrc, int64_t num_pages,
                            const int32_t* q_pos, int hkv, int head_offset, int heads, int gqa, int hq_total, int nseq,
                            int max_q_len, float sm_scale, void* stage, void* out, cudaStream_t st);
int k8v4_decode_combine_ranks(const float* ws_all, int64_t rank_floats, const int32_t* cu_q, void* out, int nrank,
                              int nsplit, int nseq, int heads, int head_offset, int gqa, int hq_total, int max_q_len,
                              cudaStream_t st);
int k8v4_gather_dequant(const void* cache, int64_t num_pages, const int32_t* block_table, int hkv, int head,
                        int seq_len, int out_dtype, void* k_out, void* v_out, cudaStream_t st);
}

namespace {

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

void check_cuda(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
}
void check_contig(const at::Tensor& t, const char* name) {
  check_cuda(t, name);
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
}
void check_rc(int rc, const char* what) { TORCH_CHECK(rc == 0, "k8v4 ", what, " launch failed (code ", rc, ")"); }

// ------------------------------------------------------------------ KV store
void kv_store(int64_t fmt, const at::Tensor& k, const at::Tensor& v, const at::Tensor& slots, at::Tensor& cache,
              int64_t hkv) {
  check_cuda(k, "k");
  check_cuda(v, "v");
  check_contig(slots, "slot_mapping");
  check_contig(cache, "cache");
  TORCH_CHECK(k.scalar_type() == at::kBFloat16 && v.scalar_type() == at::kBFloat16, "k/v must be bf16");
  TORCH_CHECK(slots.scalar_type() == at::kLong, "slot_mapping must be int64");
  TORCH_CHECK(cache.scalar_type() == at::kByte && cache.dim() == 2, "cache must be uint8 [pages, page_bytes]");
  TORCH_CHECK(k.dim() == 3 && v.dim() == 3 && k.size(1) == hkv && v.size(1) == hkv, "k/v must be [T, hkv, D]");
  TORCH_CHECK(k.stride(2) == 1 && v.stride(2) == 1 && k.stride(1) == k.size(2) && v.stride(1) == v.size(2),
              "k/v heads must be dense");
  const int D = fmt == 0 ? 256 : 128;
  TORCH_CHECK(k.size(2) == D && v.size(2) == D, "head_dim must be ", D);
  TORCH_CHECK(slots.numel() == k.size(0) && v.size(0) == k.size(0), "token count mismatch");
  const int page = fmt == 0 ? 64 : 16;
  const int64_t per_head = fmt == 0 ? 396 : 202;
  TORCH_CHECK(cache.size(1) == page * hkv * per_head, "cache page_bytes mismatch");
  c10::cuda::CUDAGuard g(cache.device());
  check_rc(k8v4_kv_store((int)fmt, k.data_ptr(), k.stride(0), v.data_ptr(), v.stride(0), slots.data_ptr<int64_t>(),
                         cache.data_ptr(), cache.size(0), (int)cache.size(1), (int)k.size(0), (int)hkv, cur_stream()),
           "kv_store");
}

void rope_store(const at::Tensor& qkv, const at::Tensor& cos_sin, const at::Tensor& positions, at::Tensor& q_out,
                const at::Tensor& slots, at::Tensor& cache, int64_t hq, int64_t hkv) {
  check_contig(qkv, "qkv");
  check_contig(cos_sin, "cos_sin");
  check_contig(positions, "positions");
  check_contig(q_out, "q_out");
  check_contig(slots, "slot_mapping");
  check_contig(cache, "cache");
  // qkv: bf16 rows, or the qkv GEMM's fp32 split-K sums (finished and zeroed here)
  TORCH_CHECK((qkv.scalar_type() == at::kBFloat16 || qkv.scalar_type() == at::kFloat) &&
                  q_out.scalar_type() == at::kBFloat16,
              "qkv bf16 or fp32 split-K sums, q_out bf16");
  TORCH_CHECK(cos_sin.scalar_type() == at::kFloat && cos_sin.size(-1) == 128, "cos_sin fp32 [pos, 128]");
  TORCH_CHECK(positions.scalar_type() == at::kLong && slots.scalar_type() == at::kLong, "positions/slots int64");
  const int64_t T = qkv.size(0);
  TORCH_CHECK(qkv.numel() == T * (hq + 2 * hkv) * 128, "qkv must be [T, (hq + 2 hkv) * 128]");
  TORCH_CHECK(q_out.numel() == T * hq * 128, "q_out must be [T, hq, 128]");
  TORCH_CHECK(positions.numel() == T && slots.numel() == T, "positions/slots length");
  TORCH_CHECK(cache.scalar_type() == at::kByte && cache.size(1) == 16 * hkv * 202, "b200 cache layout");
  c10::cuda::CUDAGuard g(cache.device());
  check_rc(k8v4_rope_store(qkv.data_ptr(), qkv.scalar_type() == at::kFloat ? 1 : 0, cos_sin.data_ptr<float>(),
                           positions.data_ptr<int64_t>(), q_out.data_ptr(),
                           slots.data_ptr<int64_t>(), cache.data_ptr(), cache.size(0), (int)cache.size(1), (int)T,
                           (int)hq, (int)hkv, cur_stream()),
           "rope_store");
}

// ----------------------------------------------------------------- attention
void check_attn_common(const at::Tensor& q, const at::Tensor& cu_q, const at::Tensor& seq_lens,
                       const at::Tensor& block_table, const at::Tensor& cache, const at::Tensor& out, int64_t hkv) {
  check_contig(q, "q");
  check_contig(cu_q, "cu_q");
  check_contig(seq_lens, "seq_lens");
  check_contig(block_table, "block_table");
  check_contig(cache, "cache");
  check_contig(out, "out");
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && out.scalar_type() == at::kBFloat16, "q/out bf16");
  TORCH_CHECK(q.dim() == 3 && q.size(2) == 128 && out.sizes() == q.sizes(), "q/out must be [T, hq, 128]");
  TORCH_CHECK(cu_q.scalar_type() == at::kInt && seq_lens.scalar_type() == at::kInt &&
                  block_table.scalar_type() == at::kInt,
              "cu_q / seq_lens / block_table must be int32");
  TORCH_CHECK(block_table.dim() == 2 && block_table.size(0) == seq_lens.numel() &&
                  cu_q.numel() == seq_lens.numel() + 1,
              "batch metadata shapes");
  TORCH_CHECK(cache.scalar_type() == at::kByte && cache.dim() == 2 && cache.size(1) == 16 * hkv * 202,
              "cache must be b200 [pages, 16*hkv*202]");
}

void decode_attn(const at::Tensor& q, const at::Tensor& cu_q, const at::Tensor& seq_lens,
                 const c10::optional<at::Tensor>& q_ends, const at::Tensor& block_table, const at::Tensor& cache,
                 int64_t hkv, int64_t head_offset, int64_t heads, int64_t gqa, int64_t max_q_len, int64_t nsplit,
                 double sm_scale, at::Tensor& out, const c10::optional<at::Tensor>& ws) {
  check_attn_common(q, cu_q, seq_lens, block_table, cache, out, hkv);
  TORCH_CHECK(max_q_len * gqa <= 64, "decode tile holds at most 64 query rows per KV head");
  TORCH_CHECK(head_offset >= 0 && heads >= 1 && head_offset + heads <= hkv, "head range");
  TORCH_CHECK(q.size(1) == hkv * gqa || q.size(1) == heads * gqa, "q heads vs layout");
  const int32_t* qe = nullptr;
  if (q_ends.has_value()) {
    check_contig(*q_ends, "q_ends");
    TORCH_CHECK(q_ends->scalar_type() == at::kInt && q_ends->numel() == q.size(0), "q_ends int32 [T]");
    qe = q_ends->data_ptr<int32_t>();
  }
  const int nseq = (int)seq_lens.numel();
  float* ws_o = nullptr;
  float* ws_ml = nullptr;
  if (nsplit > 1) {
    TORCH_CHECK(ws.has_value(), "nsplit > 1 needs a workspace");
    check_contig(*ws, "ws");
    TORCH_CHECK(ws->scalar_type() == at::kFloat, "ws fp32");
    const int64_t need = k8v4_decode_ws_floats(nseq, (int)heads, (int)nsplit, (int)max_q_len, (int)gqa);
    TORCH_CHECK(ws->numel() >= need, "decode workspace too small: need ", need, " floats");
    const int64_t ml = need / (128 + 2) * 2;
    ws_ml = ws->data_ptr<float>();
    ws_o = ws_ml + ml;
  }
  c10::cuda::CUDAGuard g(cache.device());
  check_rc(k8v4_decode_attn(q.data_ptr(), cu_q.data_ptr<int32_t>(), seq_lens.data_ptr<int32_t>(), qe,
                            block_table.data_ptr<int32_t>(), (int)block_table.stride(0), cache.data_ptr(),
                            cache.size(0), (int)hkv, (int)head_offset, (int)heads, (int)gqa, (int)q.size(1), nseq,
                            (int)max_q_len, (int)nsplit, (float)sm_scale, out.data_ptr(), ws_o, ws_ml, cur_stream()),
           "decode_attn");
}

int64_t decode_ws_floats(int64_t nseq, int64_t heads, int64_t nsplit, int64_t max_q_len, int64_t gqa) {
  return k8v4_decode_ws_floats((int)nseq, (int)heads, (int)nsplit, (int)max_q_len, (int)gqa);
}

// Context parallelism: decode attention whose partials go straight into
// every rank's copy of this rank's gather slot (multicast address `slot_mc`),
// then one signal per CTA on the multicast counter `flag_mc`.
void decode_attn_push(const at::Tensor& q, const at::Tensor& cu_q, const at::Tensor& seq_lens,
                      const c10::optional<at::Tensor>& q_ends, const at::Tensor& block_table, const at::Tensor& cache,
                      int64_t hkv, int64_t head_offset, int64_t heads, int64_t gqa, int64_t max_q_len, int64_t nsplit,
                      double sm_scale, int64_t slot_mc, int64_t flag_mc) {
  check_attn_common(q, cu_q, seq_lens, block_table, cache, q, hkv);
  TORCH_CHECK(max_q_len * gqa <= 64, "decode tile holds at most 64 query rows per KV head");
  TORCH_CHECK(head_offset >= 0 && heads >= 1 && head_offset + heads <= hkv, "head range");
  TORCH_CHECK(q.size(1) == hkv * gqa || q.size(1) == heads * gqa, "q heads vs layout");
  TORCH_CHECK(slot_mc != 0 && flag_mc != 0 && slot_mc % 16 == 0 && flag_mc % 8 == 0, "multicast addresses");
  const int32_t* qe = nullptr;
  if (q_ends.has_value()) {
    check_contig(*q_ends, "q_ends");
    TORCH_CHECK(q_ends->scalar_type() == at::kInt && q_ends->numel() == q.size(0), "q_ends int32 [T]");
    qe = q_ends->data_ptr<int32_t>();
  }
  c10::cuda::CUDAGuard g(cache.device());
  check_rc(k8v4_decode_attn_push(q.data_ptr(), cu_q.data_ptr<int32_t>(), seq_lens.data_ptr<int32_t>(), qe,
                                 block_table.data_ptr<int32_t>(), (int)block_table.stride(0), cache.data_ptr(),
                                 cache.size(0), (int)hkv, (int)head_offset, (int)heads, (int)gqa, (int)q.size(1),
                                 (int)seq_lens.numel(), (int)max_q_len, (int)nsplit, (float)sm_scale,
                                 reinterpret_cast<float*>(slot_mc), reinterpret_cast<unsigned long long*>(flag_mc),
                                 cur_stream()),
           "decode_attn_push");
}

void prefill_attn(const at::Tensor& q, const at::Tensor& cu_q, const at::Tensor& seq_lens,
                  const at::Tensor& block_table, const at::Tensor& cache, int64_t hkv, int64_t head_offset,
                  int64_t heads, int64_t gqa, int64_t max_q_len, double sm_scale, at::Tensor& out) {
  check_attn_common(q, cu_q, seq_lens, block_table, cache, out, hkv);
  TORCH_CHECK(head_offset >= 0 && heads >= 1 && head_offset + heads <= hkv, "head range");
  c10::cuda::CUDAGuard g(cache.device());
  const int nseq = (int)seq_lens.numel(), width = (int)block_table.size(1);
  // scratch for the once-dequantized V tiles (stream-ordered caching allocator)
  at::Tensor stage = at::empty({k8v4_prefill_stage_bytes(nseq, width, (int)heads)}, cache.options());
  check_rc(k8v4_prefill_attn(q.data_ptr(), cu_q.data_ptr<int32_t>(), seq_lens.data_ptr<int32_t>(),
                             block_table.data_ptr<int32_t>(), (int)block_table.stride(0), width, cache.data_ptr(),
                             cache.size(0), (int)hkv, (int)head_offset, (int)heads, (int)gqa, (int)q.size(1), nseq,
                             (int)max_q_len, (float)sm_scale, stage.data_ptr(), out.data_ptr(), cur_stream()),
           "prefill_attn");
}

// --------------------------------------------------------------------- GEMM
// Decode-sized W4A16 calls (at most 32 rows) can run on 8-bit MMAs over two
// int8 limbs of each token row (see wq_gemm.cu, mode W4L), at the cost of one
// small preparation kernel. K8V4_DECODE_LIMBS: "auto" (default) takes that
// path for wide outputs (N >= 16384, the gate/up projection up to TP2, where
// it measured 17% faster; the narrower decode GEMMs measured 2 us slower with
// the extra kernel), "1" for every decode-sized call, "0" never.
static int limbs_policy() {  // 0 never, 1 always, 2 auto
  static const int pol = [] {
    const char* v = std::getenv("K8V4_DECODE_LIMBS");
    if (!v || !*v || v[0] == 'a' || v[0] == 'A') return 2;
    return (v[0] == '0' || v[0] == 'n' || v[0] == 'N' || v[0] == 'f' || v[0] == 'F') ? 0 : 1;
  }();
  return pol;
}

// The limb buffers of one W4A16 call (an empty tensor when the call does not take that path).
static at::Tensor limb_buffer(const at::Tensor& x, int64_t M, int64_t N, int64_t K) {
  const int pol = limbs_policy();
  const bool use = pol == 1 || (pol == 2 && N >= 16384);
  const int64_t bytes = use ? k8v4_wq_gemm_limb_bytes((int)M, (int)K) : 0;
  return at::empty({bytes}, x.options().dtype(at::kByte));
}

// W4A16 calls of at most k8v4_gemv_w4_max_rows() rows that come with an fp32
// workspace run as the decode GEMV (gemv_w4.cu: weights streamed once through
// registers, dp4a over two int8 limbs of each activation), whose sums land in
// the workspace like a split-K GEMM's. K8V4_DECODE_GEMV=0 keeps them on the
// tcgen05 path.
static bool gemv_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("K8V4_DECODE_GEMV");
    return !(v && (v[0] == '0' || v[0] == 'n' || v[0] == 'N' || v[0] == 'f' || v[0] == 'F'));
  }();
  return on;
}

// mode 0: W4A16 (x bf16), 1: W4A8 (x int8 + xscale), 2: W8A8 (w int8 [N,K] + per-row scale).
void wq_gemm(int64_t mode, const at::Tensor& w, const at::Tensor& wscale, const at::Tensor& x,
             const c10::optional<at::Tensor>& xscale, const c10::optional<at::Tensor>& residual, at::Tensor& out,
             const c10::optional<at::Tensor>& ws, int64_t split, bool finish) {
  check_contig(w, "weight");
  check_contig(wscale, "weight scale");
  check_contig(x, "x");
  check_contig(out, "out");
  TORCH_CHECK(x.dim() == 2, "x must be 2D");
  const int64_t M = x.size(0), K = x.size(1);
  int64_t N;
  if (mode == 2) {
    TORCH_CHECK(w.scalar_type() == at::kChar && w.dim() == 2 && w.size(1) == K, "W8 weight int8 [N, K]");
    N = w.size(0);
    TORCH_CHECK(wscale.numel() == N && wscale.scalar_type() == at::kHalf, "W8 scale fp16 [N]");
  } else {
    TORCH_CHECK(w.scalar_type() == at::kInt && w.dim() == 2 && w.size(0) * 8 == K, "W4 qweight int32 [K/8, N]");
    N = w.size(1);
    TORCH_CHECK(wscale.scalar_type() == at::kHalf && wscale.dim() == 2 && wscale.size(0) * 128 == K &&
                    wscale.size(1) == N,
                "W4 scales fp16 [K/128, N]");
  }
  TORCH_CHECK(N % 128 == 0 && K % 128 == 0, "N and K must be multiples of 128");
  if (mode == 0) {
    TORCH_CHECK(x.scalar_type() == at::kBFloat16, "W4A16 takes bf16 activations");
  } else {
    TORCH_CHECK(x.scalar_type() == at::kChar, "A8 modes take int8 activations");
    TORCH_CHECK(xscale.has_value() && xscale->is_cuda() && xscale->scalar_type() == at::kFloat &&
                    xscale->numel() == M,
                "A8 modes need fp32 per-token scales");
  }
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.dim() == 2 && out.size(0) == M && out.size(1) == N,
              "out must be bf16 [M, N]");
  const void* res = nullptr;
  if (residual.has_value()) {
    check_contig(*residual, "residual");
    TORCH_CHECK(residual->sizes() == out.sizes() && residual->scalar_type() == at::kBFloat16, "residual shape");
    res = residual->data_ptr();
  }
  float* wsp = nullptr;
  if (split > 1) {
    TORCH_CHECK(ws.has_value(), "split-K needs an fp32 workspace");
    check_contig(*ws, "ws");
    TORCH_CHECK(ws->scalar_type() == at::kFloat && ws->numel() >= M * N, "workspace [M, N] fp32");
    wsp = ws->data_ptr<float>();
  }
  c10::cuda::CUDAGuard g(x.device());
  if (mode == 0 && M <= k8v4_gemv_w4_max_rows() && gemv_enabled() && ws.has_value() && ws->is_cuda() &&
      ws->scalar_type() == at::kFloat && ws->is_contiguous() && ws->numel() >= M * N) {
    float* wsg = ws->data_ptr<float>();
    check_rc(k8v4_gemv_w4(w.data_ptr(), wscale.data_ptr(), x.data_ptr(), wsg, (int)M, (int)N, (int)K, (int)K,
                          (int)N, cur_stream()),
             "gemv_w4");
    if (finish)  // else the sums stay in ws for a consumer that finishes them
      check_rc(k8v4_splitk_finish(wsg, res, out.data_ptr(), M * N, 1, cur_stream()), "splitk_finish");
    return;
  }
  const float* xs = (mode == 0) ? nullptr : xscale->data_ptr<float>();
  at::Tensor limbs = mode == 0 ? limb_buffer(x, M, N, K) : at::Tensor();
  if (limbs.defined() && limbs.numel() > 0) {
    check_rc(k8v4_wq_gemm_limbs(w.data_ptr(), wscale.data_ptr(), x.data_ptr(), res, out.data_ptr(), wsp,
                                limbs.data_ptr(), (int)M, (int)N, (int)K, (int)N, (int)split, cur_stream()),
             "wq_gemm (limbs)");
  } else {
    check_rc(k8v4_wq_gemm((int)mode, w.data_ptr(), wscale.data_ptr(), x.data_ptr(), xs, res, out.data_ptr(), wsp,
                          (int)M, (int)N, (int)K, (int)N, (int)split, cur_stream()),
             "wq_gemm");
  }
  if (split > 1 && finish) {
    check_rc(k8v4_splitk_finish(wsp, res, out.data_ptr(), M * N, 1, cur_stream()), "splitk_finish");
  }
}

// -------------------------------------------------------------- fused misc
void rmsnorm(at::Tensor& x, const c10::optional<at::Tensor>& residual, const at::Tensor& w,
             const c10::optional<at::Tensor>& y, const c10::optional<at::Tensor>& yq,
             const c10::optional<at::Tensor>& yscale, double eps, const c10::optional<at::Tensor>& sync_flag,
             const c10::optional<at::Tensor>& sync_state, int64_t sync_expected) {
  check_contig(x, "x");
  check_contig(w, "weight");
  TORCH_CHECK((x.scalar_type() == at::kBFloat16 || x.scalar_type() == at::kFloat) && w.scalar_type() == at::kBFloat16,
              "x bf16 (or fp32 split-K partials, zeroed after reading) and bf16 weight");
  const bool f32 = x.scalar_type() == at::kFloat;
  const int64_t n = x.size(-1), rows = x.numel() / n;
  TORCH_CHECK(w.numel() == n, "weight size");
  void* r = nullptr;
  if (residual.has_value()) {
    check_contig(*residual, "residual");
    TORCH_CHECK(residual->numel() == x.numel(), "residual size");
    r = residual->data_ptr();
  }
  void* yp = nullptr;
  int64_t ldy = n;
  if (y.has_value()) {
    // y may be a row-strided view (e.g. one half of a concatenated [rows, 2n] buffer)
    check_cuda(*y, "y");
    TORCH_CHECK(y->scalar_type() == at::kBFloat16 && y->numel() == x.numel() && y->size(-1) == n &&
                    y->stride(-1) == 1 && (y->dim() == 1 || y->dim() == 2),
                "y: bf16 [rows, n] with unit inner stride");
    if (y->dim() == 2) ldy = y->stride(0);
    TORCH_CHECK(ldy >= n && ldy % 8 == 0 && reinterpret_cast<uintptr_t>(y->data_ptr()) % 16 == 0,
                "y rows must be 16-byte aligned");
    yp = y->data_ptr();
  }
  void* qp = nullptr;
  float* sp = nullptr;
  if (yq.has_value()) {
    check_contig(*yq, "yq");
    TORCH_CHECK(yq->numel() == x.numel() && yq->scalar_type() == at::kChar, "yq int8");
    TORCH_CHECK(yscale.has_value() && yscale->numel() == rows && yscale->scalar_type() == at::kFloat, "yscale");
    qp = yq->data_ptr();
    sp = yscale->data_ptr<float>();
  }
  c10::cuda::CUDAGuard g(x.device());
  const unsigned long long* sf = nullptr;
  unsigned long long* ss = nullptr;
  if (sync_flag.has_value()) {
    // x is this rank's copy of a GEMM -> all-reduce buffer: wait for every rank's signals
    TORCH_CHECK(f32, "an all-reduce consumer reads fp32 sums");
    TORCH_CHECK(sync_state.has_value() && sync_state->scalar_type() == at::kLong && sync_state->numel() >= 2 &&
                    sync_state->is_contiguous(),
                "sync_state: int64 [2]");
    TORCH_CHECK(sync_flag->scalar_type() == at::kLong && sync_flag->numel() >= 1, "sync_flag: int64 counter");
    sf = reinterpret_cast<const unsigned long long*>(sync_flag->data_ptr());
    ss = reinterpret_cast<unsigned long long*>(sync_state->data_ptr());
  }
  check_rc(k8v4_rmsnorm(f32 ? nullptr : x.data_ptr(), f32 ? x.data_ptr<float>() : nullptr, r, w.data_ptr(), yp, ldy,
                        qp, sp, (int)rows, (int)n, (float)eps, sf, ss, (unsigned long long)sync_expected,
                        cur_stream()),
           "rmsnorm");
}

void silu_mul(const at::Tensor& gu, const c10::optional<at::Tensor>& y, const c10::optional<at::Tensor>& yq,
              const c10::optional<at::Tensor>& yscale) {
  check_contig(gu, "gate_up");
  TORCH_CHECK(gu.scalar_type() == at::kBFloat16 && gu.dim() == 2 && gu.size(1) % 2 == 0, "gate_up bf16 [T, 2I]");
  const int64_t rows = gu.size(0), inter = gu.size(1) / 2;
  void* yp = nullptr;
  if (y.has_value()) {
    check_contig(*y, "y");
    TORCH_CHECK(y->numel() == rows * inter && y->scalar_type() == at::kBFloat16, "y");
    yp = y->data_ptr();
  }
  void* qp = nullptr;
  float* sp = nullptr;
  if (yq.has_value()) {
    check_contig(*yq, "yq");
    TORCH_CHECK(yq->numel() == rows * inter && yq->scalar_type() == at::kChar, "yq");
    TORCH_CHECK(yscale.has_value() && yscale->numel() == rows && yscale->scalar_type() == at::kFloat, "yscale");
    qp = yq->data_ptr();
    sp = yscale->data_ptr<float>();
  }
  c10::cuda::CUDAGuard g(gu.device());
  check_rc(k8v4_silu_mul(gu.data_ptr(), yp, qp, sp, (int)rows, (int)inter, cur_stream()), "silu_mul");
}

// y = silu(gate) * up from the gate/up projection's fp32 sums, which are zeroed.
void silu_mul_f32(at::Tensor& sums, at::Tensor& y) {
  check_contig(sums, "sums");
  check_contig(y, "y");
  TORCH_CHECK(sums.scalar_type() == at::kFloat && sums.dim() == 2 && sums.size(1) % 2 == 0, "sums fp32 [T, 2I]");
  const int64_t rows = sums.size(0), inter = sums.size(1) / 2;
  TORCH_CHECK(y.numel() == rows * inter && y.scalar_type() == at::kBFloat16, "y bf16 [T, I]");
  c10::cuda::CUDAGuard g(sums.device());
  check_rc(k8v4_silu_mul_f32(sums.data_ptr<float>(), y.data_ptr(), (int)rows, (int)inter, cur_stream()),
           "silu_mul_f32");
}

void quant_rows(const at::Tensor& x, at::Tensor& q, at::Tensor& scale) {
  check_contig(x, "x");
  check_contig(q, "q");
  check_contig(scale, "scale");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && q.scalar_type() == at::kChar && scale.scalar_type() == at::kFloat,
              "dtypes");
  const int64_t n = x.size(-1), rows = x.numel() / n;
  TORCH_CHECK(q.numel() == x.numel() && scale.numel() == rows, "shapes");
  c10::cuda::CUDAGuard g(x.device());
  check_rc(k8v4_quant_rows(x.data_ptr(), q.data_ptr(), scale.data_ptr<float>(), (int)rows, (int)n, cur_stream()),
           "quant_rows");
}

// INT8 island weights -> bf16 (per-row scales).
void int8_dequant(const at::Tensor& q, const at::Tensor& scale, at::Tensor& out) {
  check_contig(q, "q");
  check_contig(scale, "scale");
  check_contig(out, "out");
  TORCH_CHECK(q.scalar_type() == at::kChar && q.dim() == 2, "q int8 [N, K]");
  TORCH_CHECK(scale.scalar_type() == at::kBFloat16 && scale.numel() == q.size(0), "scale bf16 [N]");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.numel() >= q.numel(), "out bf16, at least N * K");
  TORCH_CHECK(q.size(1) % 8 == 0, "K must be a multiple of 8");
  c10::cuda::CUDAGuard g(q.device());
  check_rc(k8v4_int8_dequant(q.data_ptr(), scale.data_ptr(), out.data_ptr(), (int)q.size(0), (int)q.size(1),
                             cur_stream()),
           "int8_dequant");
}

void embed_int8(const at::Tensor& ids, const at::Tensor& codes, const at::Tensor& scales, at::Tensor& out,
                int64_t start) {
  check_contig(ids, "ids");
  check_contig(codes, "codes");
  check_contig(scales, "scales");
  check_contig(out, "out");
  TORCH_CHECK(ids.scalar_type() == at::kLong && codes.scalar_type() == at::kChar && scales.scalar_type() == at::kHalf &&
                  out.scalar_type() == at::kBFloat16,
              "dtypes");
  TORCH_CHECK(codes.dim() == 2 && scales.numel() == codes.size(0) && out.numel() == ids.numel() * codes.size(1),
              "shapes");
  c10::cuda::CUDAGuard g(out.device());
  check_rc(k8v4_embed_int8(ids.data_ptr<int64_t>(), codes.data_ptr(), scales.data_ptr(), out.data_ptr(),
                           (int)ids.numel(), (int)codes.size(1), start, codes.size(0), cur_stream()),
           "embed_int8");
}

void argmax(const at::Tensor& logits, int64_t offset, at::Tensor& best_val, at::Tensor& best_idx) {
  check_cuda(logits, "logits");
  check_contig(best_val, "best_val");
  check_contig(best_idx, "best_idx");
  TORCH_CHECK(logits.scalar_type() == at::kBFloat16 && logits.dim() == 2, "logits bf16 [rows, vocab]");
  TORCH_CHECK(logits.stride(1) == 1 && logits.stride(0) >= logits.size(1), "logits rows must be unit-stride");
  TORCH_CHECK(best_val.scalar_type() == at::kFloat && best_idx.scalar_type() == at::kLong &&
                  best_val.numel() == logits.size(0) && best_idx.numel() == logits.size(0),
              "outputs");
  c10::cuda::CUDAGuard g(logits.device());
  check_rc(k8v4_argmax(logits.data_ptr(), (int)logits.size(0), (int)logits.size(1), logits.stride(0), offset,
                       best_val.data_ptr<float>(), best_idx.data_ptr<int64_t>(), cur_stream()),
           "argmax");
}

// GEMM -> all-reduce: `ws` is this rank's copy of a symmetric fp32 [M, N]
// buffer, `ws_mc` / `flag_mc` the multicast addresses of that buffer and of
// the completion counter (from the symmetric-memory rendezvous).
void wq_gemm_allreduce(int64_t mode, const at::Tensor& w, const at::Tensor& wscale, const at::Tensor& x,
                       const c10::optional<at::Tensor>& xscale, at::Tensor& ws, int64_t ws_mc, int64_t flag_mc,
                       int64_t split, const c10::optional<at::Tensor>& gemv_local,
                       const c10::optional<at::Tensor>& gemv_ticket) {
  check_contig(w, "weight");
  check_contig(wscale, "weight scale");
  check_contig(x, "x");
  check_contig(ws, "ws");
  TORCH_CHECK(mode == 0 || mode == 1, "all-reduce GEMMs are W4A16 or W4A8");
  TORCH_CHECK(x.dim() == 2 && w.scalar_type() == at::kInt && w.size(0) * 8 == x.size(1), "W4 qweight [K/8, N]");
  const int64_t M = x.size(0), K = x.size(1), N = w.size(1);
  TORCH_CHECK(ws.scalar_type() == at::kFloat && ws.dim() == 2 && ws.size(0) == M && ws.size(1) == N, "ws fp32 [M, N]");
  TORCH_CHECK(ws_mc != 0 && flag_mc != 0 && ws_mc % 16 == 0 && flag_mc % 8 == 0, "multicast addresses");
  if (mode == 0) {
    TORCH_CHECK(x.scalar_type() == at::kBFloat16, "W4A16 takes bf16 activations");
  } else {
    TORCH_CHECK(x.scalar_type() == at::kChar && xscale.has_value() && xscale->numel() == M &&
                    xscale->scalar_type() == at::kFloat,
                "W4A8 takes int8 activations + fp32 scales");
  }
  c10::cuda::CUDAGuard g(x.device());
  if (mode == 0 && M <= k8v4_gemv_w4_max_rows() && gemv_enabled()) {
    // the decode GEMV: partial sums meet in a local accumulator, then one
    // CTA adds the rows into every rank's copy (one signal per rank)
    TORCH_CHECK(gemv_local.has_value() && gemv_ticket.has_value(), "the GEMV all-reduce needs its local buffers");
    check_contig(*gemv_local, "gemv_local");
    TORCH_CHECK(gemv_local->scalar_type() == at::kFloat && gemv_local->numel() >= M * N, "gemv_local fp32 [M, N]");
    TORCH_CHECK(gemv_ticket->scalar_type() == at::kInt && gemv_ticket->numel() >= 1, "gemv_ticket int32");
    check_rc(k8v4_gemv_w4_allreduce(w.data_ptr(), wscale.data_ptr(), x.data_ptr(), gemv_local->data_ptr<float>(),
                                    reinterpret_cast<float*>(ws_mc), reinterpret_cast<unsigned long long*>(flag_mc),
                                    reinterpret_cast<unsigned int*>(gemv_ticket->data_ptr<int>()), (int)M, (int)N,
                                    (int)K, (int)K, (int)N, cur_stream()),
             "gemv_w4_allreduce");
    return;
  }
  at::Tensor limbs = mode == 0 ? limb_buffer(x, M, N, K) : at::Tensor();
  check_rc(k8v4_wq_gemm_allreduce((int)mode, w.data_ptr(), wscale.data_ptr(), x.data_ptr(),
                                  mode == 0 ? nullptr : xscale->data_ptr<float>(), reinterpret_cast<float*>(ws_mc),
                                  reinterpret_cast<unsigned long long*>(flag_mc), (int)M, (int)N, (int)K, (int)N,
                                  (int)split, cur_stream(),
                                  limbs.defined() && limbs.numel() > 0 ? limbs.data_ptr() : nullptr),
           "wq_gemm_allreduce");
}

// Sequence-parallel prefill GEMM (see k8v4_wq_gemm_sp). Addresses that may
// belong to peers (rs_dst, rs_sig) or to this rank's symmetric buffers
// (ag_flag) come as integers; x is this rank's view of the input rows.
void wq_gemm_sp(int64_t mode, const at::Tensor& w, const at::Tensor& wscale, const at::Tensor& x,
                const c10::optional<at::Tensor>& xscale, const c10::optional<at::Tensor>& out, int64_t world,
                int64_t rank, at::IntArrayRef tile0, int64_t ag_flag, at::IntArrayRef ag_target,
                at::IntArrayRef rs_dst, at::IntArrayRef rs_sig) {
  check_contig(w, "weight");
  check_contig(wscale, "weight scale");
  check_contig(x, "x");
  TORCH_CHECK(mode == 0 || mode == 1, "sequence-parallel GEMMs are W4A16 or W4A8");
  TORCH_CHECK(x.dim() == 2 && w.scalar_type() == at::kInt && w.size(0) * 8 == x.size(1), "W4 qweight [K/8, N]");
  TORCH_CHECK(world >= 2 && world <= 8 && (int64_t)tile0.size() == world + 1, "tile0 has world + 1 entries");
  const int64_t M = x.size(0), K = x.size(1), N = w.size(1);
  if (mode == 0) {
    TORCH_CHECK(x.scalar_type() == at::kBFloat16, "W4A16 takes bf16 activations");
  } else {
    TORCH_CHECK(x.scalar_type() == at::kChar && xscale.has_value() && xscale->numel() >= M &&
                    xscale->scalar_type() == at::kFloat,
                "W4A8 takes int8 activations + fp32 scales");
  }
  const bool rs = !rs_dst.empty();
  TORCH_CHECK(!rs || ((int64_t)rs_dst.size() == world && (int64_t)rs_sig.size() == world), "rs_dst / rs_sig per rank");
  TORCH_CHECK(ag_flag == 0 || (int64_t)ag_target.size() == world, "ag_target per rank");
  TORCH_CHECK(rs || ag_flag != 0, "neither a gather wait nor a scatter");
  void* outp = nullptr;
  if (!rs) {
    TORCH_CHECK(out.has_value() && out->scalar_type() == at::kBFloat16 && out->size(0) == M && out->size(1) == N &&
                    out->is_contiguous(),
                "out bf16 [M, N]");
    outp = out->data_ptr();
  }
  int t0[9];
  for (int i = 0; i <= world; ++i) t0[i] = (int)tile0[i];
  unsigned long long tg[8] = {0};
  void* dst[8] = {nullptr};
  unsigned long long* sig[8] = {nullptr};
  for (int i = 0; i < world; ++i) {
    if (ag_flag) tg[i] = (unsigned long long)ag_target[i];
    if (rs) {
      TORCH_CHECK(rs_dst[i] % 16 == 0 && rs_sig[i] % 8 == 0 && rs_dst[i] && rs_sig[i], "peer addresses");
      dst[i] = reinterpret_cast<void*>(rs_dst[i]);
      sig[i] = reinterpret_cast<unsigned long long*>(rs_sig[i]);
    }
  }
  c10::cuda::CUDAGuard g(x.device());
  check_rc(k8v4_wq_gemm_sp((int)mode, w.data_ptr(), wscale.data_ptr(), x.data_ptr(),
                           mode == 0 ? nullptr : xscale->data_ptr<float>(), outp, (int)M, (int)N, (int)K, (int)N,
                           (int)world, (int)rank, t0, reinterpret_cast<const unsigned long long*>(ag_flag),
                           ag_flag ? tg : nullptr, rs ? dst : nullptr, rs ? sig : nullptr, cur_stream()),
           "wq_gemm_sp");
}

// Sequence-parallel norm of this rank's rows (see k8v4_rmsnorm_sp). y / yq /
// ys are addresses: multicast addresses of the all-gather buffers (mc) or
// local buffers.
void rmsnorm_sp(const c10::optional<at::Tensor>& slots, int64_t world, int64_t slot_stride,
                const c10::optional<at::Tensor>& x_local, at::Tensor& residual, bool init_residual, const at::Tensor& w,
                int64_t rows, double eps, int64_t rs_flag, int64_t rs_target, int64_t y, int64_t yq, int64_t ys,
                int64_t row0, bool mc, int64_t ag_sig) {
  check_contig(residual, "residual");
  check_contig(w, "w");
  TORCH_CHECK(residual.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16, "bf16 residual / w");
  const int64_t n = w.numel();
  TORCH_CHECK(residual.numel() >= rows * n, "residual holds the rows");
  const void* sp = nullptr;
  if (slots.has_value()) {
    check_contig(*slots, "slots");
    TORCH_CHECK(slots->scalar_type() == at::kBFloat16 && slots->numel() >= world * slot_stride &&
                    slot_stride >= rows * n,
                "slots bf16 [world][rows >= %d][n]");
    sp = slots->data_ptr();
  }
  const void* xl = nullptr;
  if (x_local.has_value()) {
    check_contig(*x_local, "x_local");
    TORCH_CHECK(x_local->scalar_type() == at::kBFloat16 && x_local->numel() >= rows * n, "x_local bf16 [rows, n]");
    xl = x_local->data_ptr();
  }
  c10::cuda::CUDAGuard g(residual.device());
  check_rc(k8v4_rmsnorm_sp(sp, (int)world, slot_stride, xl, residual.data_ptr(), init_residual ? 1 : 0, w.data_ptr(),
                           (int)rows, (int)n, (float)eps, reinterpret_cast<const unsigned long long*>(rs_flag),
                           (unsigned long long)rs_target, reinterpret_cast<void*>(y), reinterpret_cast<void*>(yq),
                           reinterpret_cast<float*>(ys), row0, mc ? 1 : 0,
                           reinterpret_cast<unsigned long long*>(ag_sig), cur_stream()),
           "rmsnorm_sp");
}

// CTAs (= signals per rank) of one wq_gemm_allreduce call.
int64_t wq_gemm_ctas(int64_t mode, int64_t M, int64_t N, int64_t K, int64_t split) {
  if (mode == 0 && M <= k8v4_gemv_w4_max_rows() && gemv_enabled()) return 1;  // the GEMV's last CTA signals
  return k8v4_wq_gemm_ctas((int)mode, (int)M, (int)N, (int)K, (int)split);
}

// Gather + dequantize one KV head of a sequence's pages into dense [seq_len, 128] K and V.
void gather_dequant(const at::Tensor& cache, const at::Tensor& block_table, int64_t hkv, int64_t head,
                    int64_t seq_len, at::Tensor& k_out, at::Tensor& v_out) {
  check_contig(cache, "cache");
  check_contig(block_table, "block_table");
  check_contig(k_out, "k_out");
  check_contig(v_out, "v_out");
  TORCH_CHECK(cache.scalar_type() == at::kByte && cache.dim() == 2 && cache.size(1) == hkv * 3232,
              "cache: uint8 [pages, hkv * 3232] (b200 format)");
  TORCH_CHECK(block_table.scalar_type() == at::kInt && block_table.numel() * 16 >= seq_len, "block_table int32");
  TORCH_CHECK(k_out.scalar_type() == v_out.scalar_type() &&
                  (k_out.scalar_type() == at::kFloat || k_out.scalar_type() == at::kBFloat16),
              "outputs fp32 or bf16");
  TORCH_CHECK(k_out.numel() >= seq_len * 128 && v_out.numel() >= seq_len * 128, "outputs [seq_len, 128]");
  c10::cuda::CUDAGuard g(cache.device());
  check_rc(k8v4_gather_dequant(cache.data_ptr(), cache.size(0), block_table.data_ptr<int32_t>(), (int)hkv, (int)head,
                               (int)seq_len, k_out.scalar_type() == at::kFloat ? 0 : 1, k_out.data_ptr(),
                               v_out.data_ptr(), cur_stream()),
           "gather_dequant");
}

// Context-parallel prefill: pages from several caches (this GPU's and peers'
// mapped into this process), block-table entries (source << 24) | page, and
// optional per-token global positions.
void prefill_attn_cp(const at::Tensor& q, const at::Tensor& cu_q, const at::Tensor& seq_lens,
                     const at::Tensor& block_table, at::TensorList caches, const c10::optional<at::Tensor>& q_pos,
                     int64_t hkv, int64_t head_offset, int64_t heads, int64_t gqa, int64_t max_q_len, double sm_scale,
                     at::Tensor& out) {
  check_contig(q, "q");
  check_contig(block_table, "block_table");
  check_contig(out, "out");
  TORCH_CHECK(!caches.empty() && caches.size() <= 8, "1 to 8 KV sources");
  std::vector<const void*> ptrs;
  const int64_t pages = caches[0].size(0);
  for (const auto& c : caches) {
    TORCH_CHECK(c.scalar_type() == at::kByte && c.dim() == 2 && c.size(1) == hkv * 3232 && c.is_contiguous(),
                "caches: uint8 [pages, hkv * 3232]");
    TORCH_CHECK(c.size(0) == pages, "every KV source has the same page count");
    ptrs.push_back(c.data_ptr());
  }
  const int32_t* qp = nullptr;
  if (q_pos.has_value()) {
    check_contig(*q_pos, "q_pos");
    TORCH_CHECK(q_pos->scalar_type() == at::kInt && q_pos->numel() == q.size(0), "q_pos int32 [T]");
    qp = q_pos->data_ptr<int32_t>();
  }
  c10::cuda::CUDAGuard g(q.device());
  const int nseq = (int)seq_lens.numel(), width = (int)block_table.size(1);
  at::Tensor stage = at::empty({k8v4_prefill_stage_bytes(nseq, width, (int)heads)}, q.options().dtype(at::kByte));
  check_rc(k8v4_prefill_attn_multi(q.data_ptr(), cu_q.data_ptr<int32_t>(), seq_lens.data_ptr<int32_t>(),
                                   block_table.data_ptr<int32_t>(), (int)block_table.stride(0), width, ptrs.data(),
                                   (int)ptrs.size(), pages, qp, (int)hkv, (int)head_offset, (int)heads, (int)gqa,
                                   (int)q.size(1), nseq, (int)max_q_len, (float)sm_scale, stage.data_ptr(),
                                   out.data_ptr(), cur_stream()),
           "prefill_attn_cp");
}

// Merge every rank's split-K decode partials (all-gathered workspaces).
// With sync_flag: ws_all is this rank's copy of the gather buffer that
// decode_attn_push fills; the merge first waits for every rank's signals.
void decode_combine_ranks(const at::Tensor& ws_all, int64_t rank_floats, const at::Tensor& cu_q, int64_t nrank,
                          int64_t nsplit, int64_t heads, int64_t head_offset, int64_t gqa, int64_t max_q_len,
                          at::Tensor& out, const c10::optional<at::Tensor>& sync_flag,
                          const c10::optional<at::Tensor>& sync_state, int64_t sync_expected) {
  check_contig(ws_all, "ws_all");
  check_contig(out, "out");
  TORCH_CHECK(ws_all.scalar_type() == at::kFloat && ws_all.numel() >= nrank * rank_floats, "ws_all fp32");
  c10::cuda::CUDAGuard g(out.device());
  if (sync_flag.has_value()) {
    TORCH_CHECK(sync_state.has_value() && sync_state->scalar_type() == at::kLong && sync_state->numel() >= 2 &&
                    sync_state->is_contiguous(),
                "sync_state: int64 [2]");
    TORCH_CHECK(sync_flag->scalar_type() == at::kLong && sync_flag->numel() >= 1, "sync_flag: int64 counter");
    TORCH_CHECK(sync_expected > 0, "sync_expected: signals of one exchange");
    check_rc(k8v4_decode_combine_ranks_sync(
                 ws_all.data_ptr<float>(), rank_floats, cu_q.data_ptr<int32_t>(), out.data_ptr(), (int)nrank,
                 (int)nsplit, (int)(cu_q.numel() - 1), (int)heads, (int)head_offset, (int)gqa, (int)out.size(1),
                 (int)max_q_len, reinterpret_cast<const unsigned long long*>(sync_flag->data_ptr()),
                 reinterpret_cast<unsigned long long*>(sync_state->data_ptr()), (unsigned long long)sync_expected,
                 cur_stream()),
             "decode_combine_ranks");
    return;
  }
  check_rc(k8v4_decode_combine_ranks(ws_all.data_ptr<float>(), rank_floats, cu_q.data_ptr<int32_t>(), out.data_ptr(),
                                     (int)nrank, (int)nsplit, (int)(cu_q.numel() - 1), (int)heads, (int)head_offset,
                                     (int)gqa, (int)out.size(1), (int)max_q_len, cur_stream()),
           "decode_combine_ranks");
}

#ifndef K8V4_SOURCE_HASH
#define K8V4_SOURCE_HASH "unknown"
#endif
// Hash of the csrc/ tree this library was built from (setup.py passes it).
std::string source_hash() { return K8V4_SOURCE_HASH; }

// Let kernels on the current device read and write `peer`'s memory (context
// parallelism maps peer KV pools through CUDA IPC; the mapping alone does not
// grant this device access). Returns false when the pair cannot peer.
bool enable_peer_access(int64_t peer) {
  int here = -1;
  C10_CUDA_CHECK(cudaGetDevice(&here));
  if (peer == here) return true;
  int can = 0;
  C10_CUDA_CHECK(cudaDeviceCanAccessPeer(&can, here, (int)peer));
  if (!can) return false;
  const cudaError_t e = cudaDeviceEnablePeerAccess((int)peer, 0);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    (void)cudaGetLastError();
    return true;
  }
  C10_CUDA_CHECK(e);
  return true;
}

// Read (and optionally clear) the device status words of every kernel unit.
int64_t status(bool clear) {
  int v = 0;
  const int c = clear ? 1 : 0;
  int s[7] = {k8v4_status_gemm(c), k8v4_status_store(c), k8v4_status_misc(c), k8v4_status_decode(c),
              k8v4_status_prefill(c), k8v4_status_sampler(c), k8v4_status_gather(c)};
  for (int i = 0; i < 7; ++i)
    if (s[i]) v = s[i];
  return v;
}

}  // namespace

TORCH_LIBRARY(k8v4, m) {
  m.def("kv_store(int fmt, Tensor k, Tensor v, Tensor slot_mapping, Tensor(a!) cache, int hkv) -> ()");
  m.def(
      "rope_store(Tensor qkv, Tensor cos_sin, Tensor positions, Tensor(a!) q_out, Tensor slot_mapping, "
      "Tensor(b!) cache, int hq, int hkv) -> ()");
  m.def(
      "decode_attn(Tensor q, Tensor cu_q, Tensor seq_lens, Tensor? q_ends, Tensor block_table, Tensor cache, "
      "int hkv, int head_offset, int heads, int gqa, int max_q_len, int nsplit, float sm_scale, Tensor(a!) out, "
      "Tensor(b!)? ws) -> ()");
  m.def("decode_ws_floats(int nseq, int heads, int nsplit, int max_q_len, int gqa) -> int");
  m.def(
      "prefill_attn(Tensor q, Tensor cu_q, Tensor seq_lens, Tensor block_table, Tensor cache, int hkv, "
      "int head_offset, int heads, int gqa, int max_q_len, float sm_scale, Tensor(a!) out) -> ()");
  m.def(
      "wq_gemm(int mode, Tensor w, Tensor wscale, Tensor x, Tensor? xscale, Tensor? residual, Tensor(a!) out, "
      "Tensor(b!)? ws, int split, bool finish=True) -> ()");
  m.def(
      "rmsnorm(Tensor(e!) x, Tensor(a!)? residual, Tensor w, Tensor(b!)? y, Tensor(c!)? yq, Tensor(d!)? yscale, "
      "float eps, Tensor? sync_flag=None, Tensor(f!)? sync_state=None, int sync_expected=0) -> ()");
  m.def(
      "wq_gemm_allreduce(int mode, Tensor w, Tensor wscale, Tensor x, Tensor? xscale, Tensor(a!) ws, int ws_mc, "
      "int flag_mc, int split, Tensor(b!)? gemv_local=None, Tensor(c!)? gemv_ticket=None) -> ()");
  m.def("wq_gemm_ctas(int mode, int M, int N, int K, int split) -> int");
  m.def(
      "wq_gemm_sp(int mode, Tensor w, Tensor wscale, Tensor x, Tensor? xscale, Tensor(a!)? out, int world, int rank, "
      "int[] tile0, int ag_flag, int[] ag_target, int[] rs_dst, int[] rs_sig) -> ()");
  m.def(
      "rmsnorm_sp(Tensor? slots, int world, int slot_stride, Tensor? x_local, Tensor(a!) residual, bool init_residual, "
      "Tensor w, int rows, float eps, int rs_flag, int rs_target, int y, int yq, int ys, int row0, bool mc, "
      "int ag_sig) -> ()");
  m.def("silu_mul(Tensor gate_up, Tensor(a!)? y, Tensor(b!)? yq, Tensor(c!)? yscale) -> ()");
  m.def("silu_mul_f32(Tensor(a!) sums, Tensor(b!) y) -> ()");
  m.def("quant_rows(Tensor x, Tensor(a!) q, Tensor(b!) scale) -> ()");
  m.def("int8_dequant(Tensor q, Tensor scale, Tensor(a!) out) -> ()");
  m.def("embed_int8(Tensor ids, Tensor codes, Tensor scales, Tensor(a!) out, int start) -> ()");
  m.def("argmax(Tensor logits, int offset, Tensor(a!) best_val, Tensor(b!) best_idx) -> ()");
  m.def("status(bool clear) -> int");
  m.def("source_hash() -> str");
  m.def("enable_peer_access(int peer) -> bool");
  m.def(
      "prefill_attn_cp(Tensor q, Tensor cu_q, Tensor seq_lens, Tensor block_table, Tensor[] caches, Tensor? q_pos, "
      "int hkv, int head_offset, int heads, int gqa, int max_q_len, float sm_scale, Tensor(a!) out) -> ()");
  m.def(
      "decode_combine_ranks(Tensor ws_all, int rank_floats, Tensor cu_q, int nrank, int nsplit, int heads, "
      "int head_offset, int gqa, int max_q_len, Tensor(a!) out, Tensor? sync_flag=None, "
      "Tensor(b!)? sync_state=None, int sync_expected=0) -> ()");
  m.def(
      "decode_attn_push(Tensor q, Tensor cu_q, Tensor seq_lens, Tensor? q_ends, Tensor block_table, Tensor cache, "
      "int hkv, int head_offset, int heads, int gqa, int max_q_len, int nsplit, float sm_scale, int slot_mc, "
      "int flag_mc) -> ()");
  m.def(
      "gather_dequant(Tensor cache, Tensor block_table, int hkv, int head, int seq_len, Tensor(a!) k_out, "
      "Tensor(b!) v_out) -> ()");
}

TORCH_LIBRARY_IMPL(k8v4, CUDA, m) {
  m.impl("wq_gemm_sp", &wq_gemm_sp);
  m.impl("rmsnorm_sp", &rmsnorm_sp);
  m.impl("kv_store", &kv_store);
  m.impl("rope_store", &rope_store);
  m.impl("decode_attn", &decode_attn);
  m.impl("prefill_attn", &prefill_attn);
  m.impl("wq_gemm", &wq_gemm);
  m.impl("wq_gemm_allreduce", &wq_gemm_allreduce);
  m.impl("rmsnorm", &rmsnorm);
  m.impl("silu_mul", &silu_mul);
  m.impl("silu_mul_f32", &silu_mul_f32);
  m.impl("quant_rows", &quant_rows);
  m.impl("int8_dequant", &int8_dequant);
  m.impl("embed_int8", &embed_int8);
  m.impl("argmax", &argmax);
  m.impl("gather_dequant", &gather_dequant);
  m.impl("prefill_attn_cp", &prefill_attn_cp);
  m.impl("decode_combine_ranks", &decode_combine_ranks);
  m.impl("decode_attn_push", &decode_attn_push);
}

TORCH_LIBRARY_IMPL(k8v4, CompositeExplicitAutograd, m) {
  m.impl("decode_ws_floats", &decode_ws_floats);
  m.impl("wq_gemm_ctas", &wq_gemm_ctas);
  m.impl("status", &status);
  m.impl("source_hash", &source_hash);
  m.impl("enable_peer_access", &enable_peer_access);
}
