// C entry points of the k8v4 kernel library, for callers outside PyTorch.
//
// Every function takes device pointers and a CUDA stream, launches its
// kernels on that stream and returns 0 on success or a nonzero code (the
// codes are listed beside each function). None of them synchronizes.
#pragma once
#include <stdint.h>
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

// Split-K decode attention over K8/V4 pages (b200 format). ws_o / ws_ml are
// the caller's workspace of k8v4_decode_ws_floats(...) floats (unused when
// nsplit == 1). Returns 1 when q_len x GQA exceeds 64 rows (use prefill
// attention), 10 when the launch fails.
int k8v4_decode_attn(const void* q, const int32_t* cu_q, const int32_t* seq_lens, const int32_t* q_ends,
                     const int32_t* block_table, int bt_stride, const void* cache, int64_t num_pages, int hkv,
                     int head_offset, int heads, int gqa, int hq_total, int nseq, int max_q_len, int nsplit,
                     float sm_scale, void* out, float* ws_o, float* ws_ml, cudaStream_t st);

// Floats of split-K workspace one k8v4_decode_attn launch needs.
int64_t k8v4_decode_ws_floats(int nseq, int heads, int nsplit, int max_q_len, int gqa);

// ---------------------------------------------------------------------------
// Allocation-free decode attention. This entry point has no counterpart in
// the reference (k8v4-xpu); it is an addition of this library.
//
// For callers that cannot allocate device memory at the moment they run
// attention: a host thread that must not call cudaMalloc (the call can
// synchronize the device and deadlock against work the caller has queued),
// an embedder whose device memory belongs to another allocator, or a plugin
// host that forbids allocations after start-up. The split-K scratch lives in
// a fixed array inside the library; inputs and outputs are still the
// caller's.
//
//  * Capacity: k8v4_decode_attn_noalloc_max_floats() floats (4 MiB), held on
//    every GPU that loads the library until the process exits. A launch that
//    needs more is refused with code 20 and a message on stderr.
//  * The first call on a device looks up the array's device address with
//    that device current; make that first call before any stream capture.
//  * All calls share the array, which keeps the last call's contents. Calls
//    whose kernels overlap on the GPU race on it: serialize them.
//  * Codes: 0 ok, 20 too large, 21 no current device, 22 the array's address
//    could not be obtained, else k8v4_decode_attn's codes.
int64_t k8v4_decode_attn_noalloc_max_floats(void);
int k8v4_decode_attn_noalloc(const void* q, const int32_t* cu_q, const int32_t* seq_lens, const int32_t* q_ends,
                             const int32_t* block_table, int bt_stride, const void* cache, int64_t num_pages,
                             int hkv, int head_offset, int heads, int gqa, int hq_total, int nseq, int max_q_len,
                             int nsplit, float sm_scale, void* out, cudaStream_t st);

#ifdef __cplusplus
}  // extern "C"
#endif
