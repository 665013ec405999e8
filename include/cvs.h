/*
 * cvs.h - C ABI of the B200 exact top-k search library (libcvs_b200.so).
 *
 * Plain C: raw device pointers, sizes, a cudaStream_t passed as void*, and a
 * status code per call. Nothing here allocates device memory, synchronises the
 * stream or keeps state between calls, except where a function says so. Every
 * kernel is enqueued on the given stream; results are stream ordered.
 *
 * Data layout shared by all calls: row-major fp16 matrices whose width d_pad is
 * a multiple of 64 halves (zero padded), 16-byte aligned base addresses.
 *
 * Each entry point names the reference interface it replaces (paths inside
 * the sonhoang/cuda-vector-search project).
 */
#ifndef CVS_H_
#define CVS_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CVS_ABI_VERSION 1
#define CVS_PAD 64           /* width granularity (reference: index.py:14 PAD) */
#define CVS_MAX_FUSED_K 1024 /* reference limit is 256 (index.py:15 MAX_FUSED_K) */

typedef enum cvs_status {
  CVS_OK = 0,
  CVS_ERR_INVALID_ARGUMENT = 1, /* a size, pointer or alignment contract is violated */
  CVS_ERR_UNSUPPORTED = 2,      /* the current device is not an sm_100 GPU */
  CVS_ERR_WORKSPACE = 3,        /* workspace missing or smaller than required */
  CVS_ERR_CUDA = 4,             /* a CUDA runtime / driver call failed */
  CVS_ERR_DEVICE_TIMEOUT = 5    /* a kernel gave up on a pipeline wait (see cvs_poll_device_error) */
} cvs_status;

typedef enum cvs_dtype { CVS_F32 = 0, CVS_F16 = 1, CVS_BF16 = 2, CVS_F64 = 3 } cvs_dtype;

/* Message for the last non-OK status returned on this host thread. */
const char* cvs_last_error(void);

/* CVS_ABI_VERSION of the loaded library. */
int cvs_abi_version(void);

/* ceil(d / 64) * 64. Reference: cuda_vector_search/index.py:27-32 (_pad_width). */
int cvs_pad_width(int d);

/*
 * Ingest: dst[n][d_pad] (fp16) = pad(normalise?(fp16(src[n][d]))).
 * src rows are src_row_stride elements apart and may live on the device or in
 * host memory the device can address (pinned / managed). With cosine != 0 each
 * row is divided by max(||row||_2, 1e-12) in fp32 after rounding to fp16, then
 * rounded to fp16 again. src == dst is allowed for fp16 input with d == d_pad.
 * Replaces: cuda_vector_search/index.py:69-77 (to fp16, _normalize_ at
 * index.py:35-41, _pad_width at index.py:27-32) and the query preparation of
 * index.py:89-98 (_prep_queries).
 */
cvs_status cvs_ingest(const void* src, int src_dtype, int64_t n, int d, int64_t src_row_stride,
                      int d_pad, int cosine, void* dst_f16, void* stream);

/*
 * Bytes of device workspace cvs_fused_topk needs for this problem and plan
 * (plan_bq / plan_chunks as for cvs_fused_topk). Uses the current device's SM
 * count. Replaces the part_v / part_i allocation of
 * cuda_vector_search/csrc/kernels.cu:538-546.
 */
cvs_status cvs_fused_topk_workspace_size(int64_t b, int64_t n, int d_pad, int k, int plan_bq,
                                         int plan_chunks, size_t* bytes);

/*
 * Exact top-k inner-product search, scores fp32-accumulated from fp16 inputs.
 *   q[b][d_pad], x[n][d_pad]: fp16, device memory.
 *   out_scores[b][k] (fp32), out_ids[b][k] (int64): best first (score
 *   descending, then smaller id); ids are row indices of x plus id_offset.
 *   workspace: at least cvs_fused_topk_workspace_size() bytes, 256-byte aligned.
 *   plan_bq: query-tile hint, echoed in plan_out[0]: 0 = auto (CUDA-core GEMV,
 *   echoing b, for k <= 32 and d_pad <= 1024 when b = 1, or for b <= 8 on a
 *   small corpus: at most two 256-row tiles per SM, d_pad <= 640 and
 *   n x max(d_pad, 256) x (2, 4 or 8) <= 3e7 at k <= 16, 1.2e8 at k <= 32;
 *   tcgen05 tiles otherwise), 16..128 = tcgen05, one
 *   CTA per 128-query tile, 256 = CTA pairs (256-query tiles) when b > 128;
 *   plan_chunks: corpus segments per query tile (0 = auto, one CTA per SM).
 *   plan_out (host, may be NULL): {bq, segments actually used}.
 * Requires 1 <= k <= min(n, CVS_MAX_FUSED_K), n < 2^31.
 * Replaces: fused_topk (cuda_vector_search/csrc/kernels.cu:501-582, bound at
 * :590-591; kernels fused_topk_kernel :313-371 and merge_topk_kernel :373-445).
 */
cvs_status cvs_fused_topk(const void* q_f16, int64_t b, const void* x_f16, int64_t n, int d_pad,
                          int k, int64_t id_offset, float* out_scores, int64_t* out_ids,
                          void* workspace, size_t workspace_bytes, int plan_bq, int plan_chunks,
                          int64_t* plan_out, void* stream);

/*
 * Bytes of device workspace cvs_search needs (automatic plan): the candidate
 * lists and bounds of cvs_fused_topk plus the prepared queries, padded to
 * whole query tiles.
 */
cvs_status cvs_search_workspace_size(int64_t b, int64_t n, int d_pad, int k, size_t* bytes);

/*
 * Exact top-k search straight from raw queries, as Index.search does it: the
 * queries' preparation (cvs_ingest's arithmetic: to fp16, L2 normalisation when
 * cosine != 0, zero padding to d_pad) runs in the same launch that clears the
 * workspace, and writes the prepared queries into the workspace, so a search
 * is three launches (prepare, search, merge) and the caller keeps no
 * prepared-query buffer. Results as for cvs_fused_topk with the automatic plan.
 *   q_src: [b][d] rows src_row_stride elements apart, dtype src_dtype, in
 *   device memory or host memory the device can address; d <= d_pad.
 *   workspace: at least cvs_search_workspace_size() bytes, 256-byte aligned.
 * Replaces: Index._prep_queries + fused_topk as called by Index.search
 * (cuda_vector_search/index.py:89-98, 118-125).
 */
cvs_status cvs_search(const void* q_src, int src_dtype, int64_t b, int d, int64_t src_row_stride, int cosine,
                      const void* x_f16, int64_t n, int d_pad, int k, int64_t id_offset, float* out_scores,
                      int64_t* out_ids, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Full score matrix out[b][n] = q . x^T, fp32 (out_fp32 != 0) or fp16.
 * Replaces: scores (cuda_vector_search/csrc/kernels.cu:472-497, bound at
 * :588-589; kernel score_kernel :285-311).
 */
cvs_status cvs_scores(const void* q_f16, int64_t b, const void* x_f16, int64_t n, int d_pad,
                      void* out, int out_fp32, void* stream);

/*
 * Merge `lists` result lists of shape [lists][b][len] (fp32 scores, int64 ids
 * in [0, 2^31), id < 0 = empty slot) into the best k per query, best first.
 * Used after gathering per-shard results of a row-sharded corpus. Replaces the
 * running chunk merge of cuda_vector_search/reference.py:22-33 (the reference
 * has no multi-GPU path).
 */
cvs_status cvs_merge_lists(const float* scores, const int64_t* ids, int64_t lists, int64_t b,
                           int64_t len, int k, float* out_scores, int64_t* out_ids, void* stream);

/*
 * cvs_merge_lists with the lists anywhere in memory: list l's [b][len] scores
 * start at scores + l * scores_list_stride (floats) and its ids at
 * ids + l * ids_list_stride (int64); strides of at least b * len. Lets a caller
 * gather each rank's scores and ids in ONE block per rank (one collective) and
 * merge straight out of the gathered buffer. No counterpart in the reference.
 */
cvs_status cvs_merge_lists_strided(const float* scores, int64_t scores_list_stride, const int64_t* ids,
                                   int64_t ids_list_stride, int64_t lists, int64_t b, int64_t len, int k,
                                   float* out_scores, int64_t* out_ids, void* stream);

/*
 * Same search as cvs_fused_topk, for callers that cannot allocate device
 * memory (a host application that owns the device-memory budget and forbids
 * plugins from calling cudaMalloc, a serving loop that cannot afford
 * cudaMalloc's synchronisation, a language binding without a device
 * allocator). The candidate lists live in a 16 MiB array built into the
 * library (reserved on every GPU that loads it until the process exits). With
 * plan_chunks = 0 a plan that needs more (b * segments * list slots * 8 bytes,
 * as reported by cvs_fused_topk_workspace_size) is replaced by one with fewer
 * corpus segments; a problem that does not fit even with one segment, or an
 * explicit plan_chunks that does not fit, is rejected with CVS_ERR_WORKSPACE. The first
 * call on a device looks up the array's address (make it before any stream
 * capture). All calls share the array: calls that overlap on the GPU race, so
 * issue them on one stream. Allocates nothing. No counterpart in the reference.
 */
cvs_status cvs_fused_topk_noalloc(const void* q_f16, int64_t b, const void* x_f16, int64_t n,
                                  int d_pad, int k, int64_t id_offset, float* out_scores,
                                  int64_t* out_ids, int plan_chunks, void* stream);

/*
 * Reads and clears the device error word of `device` (synchronous). *code is 0
 * when no kernel reported an error since the last poll; otherwise the status is
 * CVS_ERR_DEVICE_TIMEOUT and *code says which wait gave up. No reference
 * counterpart (the reference has no device-side error reporting).
 */
cvs_status cvs_poll_device_error(int device, int* code);

/*
 * Test hook for the failure path (no reference counterpart). Arms the next
 * cvs_fused_topk call made on this host thread, and only that one. If its plan
 * is the one-CTA tcgen05 kernel (2..128 queries, or 1 query with k > 32), that
 * kernel's producer claims and loads no corpus tile and its pipeline waits give
 * up after wait_cycles SM clocks instead of ~1 s, so every wait runs out: the
 * kernel records kErrTimeout | site (0x100 | site) in the device error word,
 * releases its tensor memory and returns; cvs_poll_device_error then reports
 * CVS_ERR_DEVICE_TIMEOUT with that code, and the GPU stays usable. The armed
 * call's results are undefined. Any other plan disarms the hook and returns
 * CVS_ERR_INVALID_ARGUMENT. wait_cycles: 1000 .. 2^40.
 */
cvs_status cvs_debug_stall_next_search(int64_t wait_cycles);

/*
 * Profiling hook: when both are non-NULL (cudaEvent_t handles), every
 * cvs_fused_topk call records start_event just before its main search kernel
 * and stop_event right after it, on the call's stream. NULL disables. Process
 * wide, not thread safe. No reference counterpart.
 */
cvs_status cvs_set_profile_events(void* start_event, void* stop_event);

#ifdef __cplusplus
}
#endif

#endif /* CVS_H_ */
