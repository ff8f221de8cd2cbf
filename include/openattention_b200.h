/* OpenAttention decode path on B200 (sm_100a): C ABI.
 *
 * Every entry point takes raw device pointers, 64-bit sizes/strides (in ELEMENTS, not bytes) and a
 * cudaStream_t (passed as void*), launches on that stream without synchronising, and returns an int
 * status: 0 = OK, 1 = invalid argument (shape, stride, alignment, size limit), 2 = unsupported
 * configuration, 3 = CUDA launch error.  On a nonzero status, oa_last_error_string() (thread-local)
 * describes the failure.  No entry point allocates device memory unless its comment says so;
 * scratch space is passed in by the caller.
 *
 * Fixed model geometry (Llama-3.1-8B attention): head_dim D = 128, 32 query heads, 8 KV heads
 * (G = 4 query heads per KV head), QGS rank 32, QGC rank 16.  A "row" is one (request, query head)
 * pair r = b*32 + h; its KV row is b*8 + h/4.
 *
 * Dtype codes: OA_BF16 = 0, OA_F32 = 1.
 */
#ifndef OPENATTENTION_B200_H
#define OPENATTENTION_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define OA_BF16 0
#define OA_F32 1

/* Library identification and the message of the last failing call on this host thread. */
const char* oa_version(void);
const char* oa_last_error_string(void);

/* ------------------------------------------------------------------------------------------------
 * OpenAttention.flash, proxies per KV head.
 * Replaces decode_expand_attention / _decode_expand_kernel (triton_expand_decode.py:31-165).
 *
 * One online softmax per query row over three streams: sel_idx tokens (P1), exp_idx tokens (P2)
 * and NB cluster proxies (P3).  Token logit z = q.k * sm_scale; proxy logit z = q.kbar * sm_scale
 * + log_n (natural log).  Index -1 (or any index outside [0, K)) is a pad and is skipped;
 * log_n = -inf skips a proxy.  A row with nothing to attend returns zeros.
 *   q      (BQ, D)  bf16, row stride q_stride
 *   k, v   (BH, K, D) bf16, strides kv_stride_h, kv_stride_t (last dim contiguous)
 *   sel    (BQ, n_sel) int32 contiguous;   exp (BQ, n_exp) int32 contiguous
 *   kbar, vbar (BH, NB, D) bf16, strides kbar_stride_h, kbar_stride_b
 *   log_n  (BQ, NB) fp32, row stride log_n_stride
 *   out    (BQ, D) bf16 or fp32 (out_dtype), row stride out_stride
 *   G = BQ / BH.  nsplit: 0 = automatic, 1 = one CTA per row, >1 = split the concatenated list
 *   [sel | exp | proxies] into nsplit chunks merged by a log-sum-exp combine; splitting needs
 *   `workspace` of oa_flash_workspace_bytes(BQ, nsplit) bytes, zero-filled before its first use
 *   (the kernel leaves it reusable).  Calls that share one workspace must not overlap on the GPU.
 * ----------------------------------------------------------------------------------------------*/
int oa_flash_kvhead_proxies(const void* q, int64_t q_stride, const void* k, const void* v,
                            int64_t kv_stride_h, int64_t kv_stride_t, const int32_t* sel, int64_t n_sel,
                            const int32_t* exp_idx, int64_t n_exp, const void* kbar, const void* vbar,
                            int64_t kbar_stride_h, int64_t kbar_stride_b, const float* log_n,
                            int64_t log_n_stride, void* out, int64_t out_stride, int out_dtype, int64_t BQ,
                            int64_t BH, int64_t K, int64_t NB, float sm_scale, int nsplit, void* workspace,
                            size_t workspace_bytes, void* stream);

/* OpenAttention.flash, proxies per QUERY head (kbar, vbar: (BQ, NB, D)).
 * Replaces ours_flash / _ours_flash_kernel (inference/methods_eager.py:91-172) and, with nsplit>1,
 * the split-K pair _k_ours_flash_split + _k_dense_combine (inference/ours_graph.py:214-262,
 * inference/graph_runner.py:299-312).  Arguments as oa_flash_kvhead_proxies; NB = 0 disables P3. */
int oa_flash_qhead_proxies(const void* q, int64_t q_stride, const void* k, const void* v,
                           int64_t kv_stride_h, int64_t kv_stride_t, const int32_t* sel, int64_t n_sel,
                           const int32_t* exp_idx, int64_t n_exp, const void* kbar, const void* vbar,
                           int64_t kbar_stride_h, int64_t kbar_stride_b, const float* log_n,
                           int64_t log_n_stride, void* out, int64_t out_stride, int out_dtype, int64_t BQ,
                           int64_t BH, int64_t K, int64_t NB, float sm_scale, int nsplit, void* workspace,
                           size_t workspace_bytes, void* stream);

/* Bytes of workspace the flash entry points need for `nsplit` chunks per row (0 when nsplit <= 1;
 * nsplit = 0 is resolved the same way the entry points resolve it). */
size_t oa_flash_workspace_bytes(int64_t BQ, int64_t n_sel, int64_t n_exp, int64_t NB, int nsplit);

#ifdef __cplusplus
}
#endif

#endif /* OPENATTENTION_B200_H */
