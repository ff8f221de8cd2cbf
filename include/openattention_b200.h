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
 * pair; its KV row is row / 4.  Entry points that take `hkv` (1..8) work on arrays that hold hkv of
 * each request's 8 KV heads and the 4*hkv query heads that read them (a KV-head shard of the
 * requests; hkv = 8 is whole requests): row r = b*4*hkv + h, KV row b*hkv + h/4, and every shape
 * below written with 8 / 32 heads has hkv / 4*hkv there.
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
 *   `workspace` of oa_flash_workspace_bytes(...) bytes whose first BQ*4 bytes (one ticket counter
 *   per row) are zero before its first use; every call leaves them zero again, so a workspace can
 *   be reused by later calls with the same BQ (any nsplit).  Calls that share one workspace must
 *   not overlap on the GPU.
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

/* oa_flash_qhead_proxies for callers that cannot allocate device memory.  This entry point has no
 * counterpart in the reference.
 *
 * Who needs it: a plugin that is handed only raw device pointers across a foreign-function
 * boundary and has no allocator of its own; a serving host that has already given all device
 * memory to its own pool, so cudaMalloc would fail; a decode loop that cannot let an allocation
 * stall the device.  Such callers pass inputs and outputs only.  The split-K scratch (ticket
 * counters and partial softmax states) lives in one fixed 4 MiB (4194304-byte) array inside the
 * library, held by every GPU that loads the library until the process exits.
 *
 * Arguments and results are those of oa_flash_qhead_proxies without workspace/workspace_bytes.
 * A call whose split needs more than 4 MiB (oa_flash_workspace_bytes(...) > 4194304) is rejected
 * with status 1 and a message; pass a smaller nsplit, or use oa_flash_qhead_proxies.  The entry
 * point calls no cudaMalloc, cudaFree or other allocating routine.
 *
 * Set-up: the first call on a device (with that device current) looks up the array's device
 * address and keeps it; make that first call before any stream capture.  The kept address belongs to
 * the device's primary context: after cudaDeviceReset (or anything else that destroys that context)
 * it is stale, so do not call this entry point again in that process.  Every call that passes its
 * argument checks clears the ticket counters on `stream` before its kernel (a rejected call touches
 * nothing).  All calls on one device share the one array, which
 * keeps the last call's contents: calls that overlap on the GPU (other streams, other host threads)
 * race on it and give wrong results, so order them (one stream, or events). */
int oa_flash_qhead_proxies_noalloc(const void* q, int64_t q_stride, const void* k, const void* v,
                                   int64_t kv_stride_h, int64_t kv_stride_t, const int32_t* sel, int64_t n_sel,
                                   const int32_t* exp_idx, int64_t n_exp, const void* kbar, const void* vbar,
                                   int64_t kbar_stride_h, int64_t kbar_stride_b, const float* log_n,
                                   int64_t log_n_stride, void* out, int64_t out_stride, int out_dtype,
                                   int64_t BQ, int64_t BH, int64_t K, int64_t NB, float sm_scale, int nsplit,
                                   void* stream);

/* ------------------------------------------------------------------------------------------------
 * Decode-step selection.  State layouts (all contiguous; B requests, C clusters, Lmax positions):
 *   K, V     (B, 8, Lmax, 128) bf16 caches, new token already written at position n-1
 *   codes    (B, 8, Lmax, 32) int8       U (B, 8, 128, 32) fp32      scale (B, 8, 32) fp32
 *   W        (B, 32, 128, 16) bf16       colmean (B, 32, 16) fp32    cent (B, 32, C, 16) fp32
 *   asg      (B, 32, Lmax) int32         nb (B, 32, C) fp32          Sk, Sk2, Sv (B, 32, C, 128) fp32
 *   mem      (B, 32, Lmax) int32 CSR member lists, cstart / clen (B, 32, C) int32
 *   reclist  (B, 32, C, rmax) int32 generated tokens per cluster, reccnt (B, 32, C) int32
 * n_dev / n0_dev are device int32 scalars (current length incl. the new token; prefix length at
 * build), so a captured CUDA graph replays correctly as n grows.
 * ----------------------------------------------------------------------------------------------*/

/* Index update of the new token at position n-1 plus the QGS query projection.
 * Replaces _k_index_update_d2 (inference/ours_graph.py:43-90) and the zq matmul
 * (inference/ours_graph.py:298, methods_eager.py:603).  Per KV head: code = clamp(rint(k.U/scale),
 * +-127); per query head: nearest centroid of bf16(k.W) - colmean (ties -> lower id), asg, nb += 1,
 * Sk += k, Sk2 += k*k, Sv += v, generated-token list append (reclist may be NULL).  If q is not
 * NULL, zq (B*32, 32) bf16 = bf16((q.U) * scale) for q (B*32, 128) bf16 with row stride q_stride. */
int oa_index_update(const void* K, const void* V, int64_t B, int64_t hkv, int64_t Lmax, int64_t C, int8_t* codes,
                    const float* U, const float* scale, const void* W, const float* colmean, const float* cent,
                    int32_t* asg, float* nb, float* Sk, float* Sk2, float* Sv, int32_t* reclist, int32_t* reccnt,
                    int rmax, const void* q, int64_t q_stride, void* zq, const int32_t* n_dev, void* stream);

/* oa_index_update with the new token's K/V write fused in (the "fused KV-write + index update" step
 * that precedes the path on every layer; the reference writes the cache in its attention hook,
 * graph_runner.py:479-480, then runs _k_index_update_d2, ours_graph.py:43-90): k_new, v_new (B, 8, 128)
 * bf16 contiguous are the new token's rows; they are written into K, V at position n_dev[0] - 1 and
 * the index is updated from them, in one launch.  Other arguments as oa_index_update. */
int oa_index_update_append(void* K, void* V, int64_t B, int64_t hkv, int64_t Lmax, int64_t C, const void* k_new,
                           const void* v_new,
                           int8_t* codes, const float* U, const float* scale, const void* W, const float* colmean,
                           const float* cent, int32_t* asg, float* nb, float* Sk, float* Sk2, float* Sv,
                           int32_t* reclist, int32_t* reccnt, int rmax, const void* q, int64_t q_stride, void* zq,
                           const int32_t* n_dev, void* stream);

/* Runner helper with no counterpart in the reference (its decode loop does this with two index
 * copies and two counter increments): appends one token per request to the K/V caches in one
 * launch.  k_new, v_new (B, 8, 128) bf16 contiguous are written at position p = n_dev[0] + offset
 * of K, V (B, 8, Lmax, 128) (nothing is written when p is outside [0, Lmax)); then, if advance,
 * n_dev[0] becomes n_dev[0] + 1 and, if kv_idx is not NULL, kv_idx[0] (int64) the old n_dev[0].
 * A decode step that appends before the index update uses offset 0 and advance 1; a layer loop
 * that advanced the counters already uses offset -1 and advance 0. */
int oa_append_kv(void* K, void* V, int64_t B, int64_t hkv, int64_t Lmax, const void* k_new, const void* v_new,
                 int32_t* n_dev, int offset, int advance, int64_t* kv_idx, void* stream);

/* QGS scan: scores (B*32, score_stride) bf16 = exact int8 dot products of codes and zq, rounded to
 * fp32 then bf16, -inf for t < ns and t >= n - nl; tile_max (B*32, tile_max_stride) fp32 = maximum
 * of each 32-token tile (tile_max_stride >= ceil(Lmax / 32)).  Replaces _k_qgs_scan_tm (inference/graph_runner.py:100-120).
 * status (may be NULL): device int32 set to 1 if a bulk copy of the codes did not complete within
 * the kernel's bounded wait (the affected tiles are then not computed). */
int oa_qgs_scan(const int8_t* codes, const void* zq, int64_t B, int64_t hkv, int64_t Lmax, const int32_t* n_dev,
                int ns, int nl, void* scores, int64_t score_stride, float* tile_max, int64_t tile_max_stride,
                int32_t* status, void* stream);

/* Row top-k among the 2k 32-token tiles with the largest maxima (exact), ties -> lower position;
 * sel (R, ns+nl+k_top) int32 = [0..ns-1, n-nl..n-1, top-k by rank]; the selected scores are set to
 * -inf in `scores`.  Replaces _k_select (inference/graph_runner.py:123-159).  k_top <= 64. */
int oa_qgs_select(void* scores, int64_t score_stride, const float* tile_max, int64_t tile_max_stride, int64_t R,
                  int64_t Lmax, const int32_t* n_dev, int ns, int nl, int k_top, int32_t* sel, void* stream);

/* ErrorGate (wl1) + hierarchical water-filling per row: tail statistics (pooled sums minus the
 * selected tokens), score = zbar + ln n + s2/2 + ln erf(sqrt(s2/2)), quotas q_b = min(n_b,
 * floor(lambda w_b)) plus leftover whole tokens to the best-scoring clusters with room.
 * Outputs score, nt (tail counts) and quota, each (B*32, C) fp32; zdot (may be NULL): the unscaled
 * dot q . kbar_b of each cluster's tail mean (the value zbar is formed from), which
 * oa_residual_flash can use instead of re-reading Sk.  Replaces _k_errorgate + _k_waterfill
 * (inference/ours_fused.py:122-216).  C <= 256, n_sel <= 512.  Sk and Sk2 16-byte aligned.
 * status (may be NULL): device int32, unused by this entry (kept for a uniform stage signature). */
int oa_errorgate_waterfill(const void* q, int64_t q_stride, const void* K, int64_t B, int64_t hkv, int64_t Lmax,
                           int64_t C,
                           const int32_t* asg, const int32_t* sel, int64_t n_sel, const float* Sk, const float* Sk2,
                           const float* nb, float E, float* score, float* nt, float* quota, float* zdot,
                           int32_t* status, void* stream);

/* Within-cluster top-q: for each cluster with quota q > 0, its q best members by QGS score (the
 * selected tokens are already -inf), ties -> lower position, written to exp_idx (R, E) int32 at the
 * cluster's offset sum_{c'<c} q_c' in ascending position; -1 pads.  Candidates are the cluster's CSR
 * members (positions < n0) and its generated tokens: reclist (may be NULL) while it holds them all
 * (reccnt <= rmax), else positions in [n0, n) with asg == c.  C <= 256.  status (may be NULL): set to
 * 4 if a bulk copy of the score row did not complete in the bounded wait.  Quotas are whole numbers
 * (as oa_errorgate_waterfill writes them); a value outside [0, E] is clamped to it.  E < 2^23.
 * workspace (may be NULL): oa_topq_workspace_bytes(R, Lmax, E) bytes, 16-byte aligned, used for rows
 * too long for the shared-memory kernel (their member keys are permuted into it); without it such
 * rows read their keys from global memory, which is much slower.
 * Replaces _k_topq_d2 (inference/ours_graph.py:93-166). */
int oa_topq(const void* scores, int64_t score_stride, int64_t R, int64_t Lmax, int64_t C, const int32_t* mem,
            const int32_t* cstart, const int32_t* clen, const int32_t* asg, const int32_t* reclist,
            const int32_t* reccnt, int rmax, const float* quota, int64_t E, const int32_t* n_dev,
            const int32_t* n0_dev, int32_t* exp_idx, int32_t* status, void* workspace, size_t workspace_bytes,
            void* stream);

/* Bytes of workspace oa_topq uses for these sizes (0 when its rows fit the shared-memory kernel). */
size_t oa_topq_workspace_bytes(int64_t R, int64_t Lmax, int64_t E);

/* Which oa_topq kernel rows of Lmax positions take: 0 the pipelined one (two key buffers in shared
 * memory, the next row keyed while the current one is selected; up to about 35K positions at C = 64,
 * E = 216), 1 the one-buffer one (up to about 47K), 2 the long-row kernels (workspace, or keys read
 * from global memory). */
int oa_topq_variant(int64_t Lmax, int64_t E, int64_t C);

/* Residual proxies: per (row, cluster) the pooled sums minus every token read (sel in order, then
 * the cluster's exp segment), n' = nt - quota, kbar' / vbar' = bf16(sums / max(n', 1)) (R, C, 128),
 * log_n = ln max(n', 1) if n' > 0.5 else -inf (R, C) fp32.  Replaces _k_resid_scatter +
 * _k_resid_norm (inference/ours_fused.py:367-407), without atomics.  Quotas outside [0, E] are clamped
 * to it when the segments are placed.  status: as oa_errorgate_waterfill (value 3). */
int oa_residual(const void* K, const void* V, int64_t B, int64_t hkv, int64_t Lmax, int64_t C, const int32_t* asg,
                const int32_t* sel, int64_t n_sel, const int32_t* exp_idx, int64_t E, const float* Sk,
                const float* Sv, const float* nt, const float* quota, void* kbar, void* vbar, float* log_n,
                int32_t* status, void* stream);

/* Residual proxies and OpenAttention.flash in one kernel (per-query-head proxies: the deployed
 * combination of oa_residual + oa_flash_qhead_proxies).  Inputs as oa_residual; out (B*32, 128)
 * bf16 or fp32 (out_dtype) with row stride out_stride.
 *  - kbar, vbar and log_n all NULL (the deployed step): the proxies are folded into the flash pass.
 *    For a live cluster, q . kbar'_b = (q . Sk_b - sum of its read tokens' q . k) / n'_b needs only
 *    scalar sums of the token dots, and the value side is sum_t (p_t - w_b(t)) v_t + sum_b w_b Sv_b
 *    with w_b = p_b / n'_b.  The proxies are the fp32 estimator's (un-rounded).  zdot (may be NULL):
 *    oa_errorgate_waterfill's zdot for this step; then q . Sk_b is taken from it and Sk is not read.
 *  - kbar / vbar (and optionally log_n) given: the bf16 proxies are formed exactly as oa_residual
 *    forms them (bit-identical), written, and attended; zdot is ignored.
 * Quotas outside [0, E] are clamped to it when the segments are placed; a selected token whose
 * assignment is outside [0, C) counts as in no cluster.
 * status (may be NULL): device int32, unused by this entry. */
int oa_residual_flash(const void* q, int64_t q_stride, const void* K, const void* V, int64_t B, int64_t hkv,
                      int64_t Lmax, int64_t C,
                      const int32_t* asg, const int32_t* sel, int64_t n_sel, const int32_t* exp_idx, int64_t E,
                      const float* Sk, const float* Sv, const float* nt, const float* quota, const float* zdot,
                      void* kbar, void* vbar, float* log_n, void* out, int64_t out_stride, int out_dtype,
                      float sm_scale, int32_t* status, void* stream);

/* ------------------------------------------------------------------------------------------------
 * Per-request build (prefill).  Each call works on ONE request: K, V (hkv, Lmax, 128) bf16 with the
 * first T positions valid; state pointers address that request's slice ((hkv, ...) for QGS arrays,
 * (4*hkv, ...) for QGC arrays; hkv = 8 is the whole request).  Replaces methods_eager.Ours.build (inference/methods_eager.py:519-555)
 * and the fast build (inference/ours_fastbuild.py:253-304); the eigen-decomposition and the k-means
 * seeds stay on the host (torch), as in the reference.
 * ----------------------------------------------------------------------------------------------*/

/* QGS codes: z = k.U (8, T, 32), scale = max(amax_t |z| / 127, 1e-12) (8, 32), codes (8, Lmax, 32)
 * = clamp(rint(z / scale), +-127).  amax_ws: 256 uint32 of scratch. */
int oa_build_codes(const void* K, int64_t hkv, int64_t Lmax, int64_t T, const float* U, float* scale, int8_t* codes,
                   uint32_t* amax_ws, void* stream);

/* QGC projection: zP (32, T, 16) fp32 = bf16(k . W[h]) - colmean, colmean (32, 16) = column means
 * (double accumulation per 256-token tile, then over tiles).  W (32, 128, 16) bf16. */
size_t oa_build_project_workspace_bytes(int64_t T);
int oa_build_project(const void* K, int64_t hkv, int64_t Lmax, int64_t T, const void* W, float* zP, float* colmean,
                     void* workspace, size_t workspace_bytes, void* stream);

/* One Lloyd assignment for the 32 query heads: asg[h, t] = argmax_c bf16(bf16(bf16(zP).bf16(cent_c))
 * - bf16(|cent_c|^2 / 2)), ties -> lower c (inference/ours_fastbuild.py:52-82). */
int oa_kmeans_assign(const float* zP, int64_t hkv, int64_t T, int64_t C, const float* cent, int32_t* asg,
                     int64_t asg_stride, void* stream);

/* Stable CSR member lists of an assignment: mem[h, cstart[h,c] + i] = i-th position (ascending) with
 * asg == c; clen = counts (inference/ours_fused.py:436-445).  mem (32, mem_stride) int32. */
size_t oa_csr_workspace_bytes(int64_t T, int64_t C);
int oa_csr_build(const int32_t* asg, int64_t asg_stride, int64_t hkv, int64_t T, int64_t C, int32_t* mem,
                 int64_t mem_stride, int32_t* cstart, int32_t* clen, void* workspace, size_t workspace_bytes,
                 void* stream);

/* Lloyd update: cent_c = (sum of member zP, in position order, fp32) / count, an empty cluster takes
 * zP[init_c]; nb = counts (inference/methods_eager.py:543-545). init: (C,) int64 seed positions. */
int oa_kmeans_update(const float* zP, int64_t hkv, int64_t T, int64_t C, const int32_t* mem, int64_t mem_stride,
                     const int32_t* cstart, const int32_t* clen, const int64_t* init, float* cent, float* nb,
                     void* stream);

/* Cluster sums Sk, Sk2, Sv (32, C, 128) fp32 over the members in position order
 * (inference/ours_fastbuild.py:111-139; = the scatter_add sums of methods_eager.py:549-555). */
int oa_cluster_sums(const void* K, const void* V, int64_t hkv, int64_t Lmax, int64_t C, const int32_t* mem,
                    int64_t mem_stride, const int32_t* cstart, const int32_t* clen, float* Sk, float* Sk2, float* Sv,
                    void* stream);

#ifdef __cplusplus
}
#endif

#endif /* OPENATTENTION_B200_H */
