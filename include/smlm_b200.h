/*
 * C ABI of the B200 product-key-memory (PKM) kernels: libsmlm_b200.so.
 *
 * Each entry point replaces one function of the reference's kernel layer (smlm/kernels.py of
 * re133/sparse-memory-lm) or one torch-op sequence of its PyTorch path; the comment above each declaration
 * names the reference interface (file:line) it stands in for. The Python shims in smlm_b200/kernels.py keep
 * the reference's Python signatures and call these through ctypes.
 *
 * Conventions shared by all entry points:
 *   - All tensor pointers are device pointers (CUDA global memory); sizes are element counts.
 *   - Work is enqueued on `stream` (a cudaStream_t; NULL = legacy default stream) and is asynchronous:
 *     no entry point synchronizes the device or the stream, none allocates device memory.
 *   - Scratch memory comes in through `workspace` / `workspace_bytes`; the matching *_workspace() query
 *     returns the number of bytes needed (a pure host computation).
 *   - Return value: SMLM_OK, or an error code; smlm_last_error() describes the error (thread-local).
 *     SMLM_ERR_INVALID is raised before any launch (shape / dtype / range checks on the host).
 *   - Index range violations found on the device (a row outside [0, rows)) never trap: the lookup is skipped
 *     and SMLM_FLAG_INDEX_RANGE is OR-ed into *status (if status is not NULL).
 *   - Layouts are row-major and contiguous.
 */
#ifndef SMLM_B200_H
#define SMLM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define SMLM_API __attribute__((visibility("default")))
#else
#define SMLM_API
#endif

/* return codes */
#define SMLM_OK 0
#define SMLM_ERR_INVALID 1   /* bad argument, detected on the host before launch */
#define SMLM_ERR_CUDA 2      /* a CUDA runtime call or launch failed */
#define SMLM_ERR_WORKSPACE 3 /* workspace_bytes smaller than the size query's answer */

/* element types */
#define SMLM_F32 0
#define SMLM_BF16 1
#define SMLM_F16 2
#define SMLM_Q4 3 /* packed 4-bit rows (d/2 bytes) + one fp16 scale per row, see smlm_quantize_q4 */
/* index types (row-sharded entry points) */
#define SMLM_I32 4
#define SMLM_I64 5
/* compact optimizer state: int8 first-moment codes, uint8 second-moment codes, one fp32 scale per row each */
#define SMLM_I8 6

/* device status word bits */
#define SMLM_FLAG_INDEX_RANGE 1
#define SMLM_FLAG_TIMEOUT 4 /* a bounded wait inside a kernel gave up; that call's outputs are invalid */

/* flags of smlm_bag_backward_rows: rows whose touched byte is 0 are written, not accumulated (the caller
 * guarantees such rows count as zero, e.g. a RowStore whose untouched rows are never read as data) */
#define SMLM_BWD_FIRST_TOUCH_WRITES 1
/* flags of smlm_bag_backward_rows: deferred row sums (needs SMLM_BWD_FIRST_TOUCH_WRITES, touched and row_sqnorm;
 * acc may be NULL). The call sorts the lookups, writes gw, the row norms and the touched marks, but not the rows:
 * the sorted pairs stay in the workspace, and smlm_lazy_adam_deferred_step (or smlm_bag_rows_materialize) finish
 * them later with the same grad_out, weights and sizes. */
#define SMLM_BWD_DEFER_ROWS 2
/* widest row (values per table row) the row-sparse backward and its optimizer steps take; wider rows return
 * SMLM_ERR_INVALID (the forward bag has no limit) */
#define SMLM_MAX_ROW_WIDTH 512
/* flags of the optimizer steps: leave the consumed accumulator rows unchanged instead of zeroing them (they
 * count as zero once their touched byte is cleared) */
#define SMLM_STEP_KEEP_ACC 1

/* row-wise optimizer kinds (smlm/row_optim.py:21 KINDS) */
#define SMLM_ROWRMS 0
#define SMLM_ROWADAGRAD 1

/* score modes of the fused scoring + selection (smlm_score_select) */
#define SMLM_SCORE_F32_EXACT 0 /* fp32 sub-key scores, sequential fmaf over the half dimension */
#define SMLM_SCORE_BF16 1      /* bf16 operands, fp32 accumulate, scores rounded to bf16 (autocast path) */

/* Library version (major * 10000 + minor * 100 + patch) and the last error of this thread. */
/* Interface version (100 for this header) and the text of the calling thread's last error. No counterpart in the
 * reference: its Python kernel layer raises exceptions where these entry points return a code. */
SMLM_API int smlm_version(void);
SMLM_API const char *smlm_last_error(void);

/* ----------------------------------------------------------------------------------- value bag (gather) */

/* out[n, :] = sum_j weights[n, j] * table[indices[n, j], :], fp32 accumulation in j order.
 * Replaces kernels.py:229 bag_forward (and the aten _embedding_bag forward of sparse_values.py:78).
 * weights: F32 or BF16 (n, k); table: F32 or BF16 (rows, d); out: F32 or BF16 (n, d). */
SMLM_API int smlm_bag_forward(const int64_t *indices, const void *weights, int weights_dtype, const void *table,
                     int table_dtype, int64_t n, int64_t k, int64_t rows, int64_t d, void *out, int out_dtype,
                     int *status, void *stream);

/* Inference bag on an fp32 / bf16 / q4 table with the swilu product fused:
 *   a = sum_j weights[n, j] * table[indices[n, j]]   (q4: codes * per-row fp16 scale)
 *   if pre: a = a * bf16(silu(pre[n]))               (pre: BF16 or F32 (n, d))
 *   out = a (F32) or bf16(a) (BF16).
 * Replaces kernels.py:364 bag_infer. For q4, table is uint8 (rows, d/2) and scales is fp16 (rows,). */
SMLM_API int smlm_bag_infer(const int64_t *indices, const void *weights, int weights_dtype, const void *table,
                   int table_dtype, const void *scales, const void *pre, int pre_dtype, int64_t n, int64_t k,
                   int64_t rows, int64_t d, void *out, int out_dtype, int *status, void *stream);

/* 4-bit row quantisation: per row s = half(w[argmax|w|] / -8) (1 if zero), codes clamp(round(w / s), -8, 7) + 8,
 * byte i of a row = code(col i) | code(col i + d/2) << 4. Replaces kernels.py:280 quantize_q4. d must be even. */
SMLM_API int smlm_quantize_q4(const float *table, int64_t rows, int64_t d, uint8_t *packed, void *scales_f16,
                     void *stream);

/* ------------------------------------------------------------------------ value bag backward (row-sparse) */

/* Scratch bytes of smlm_bag_backward_rows / smlm_shard_bag_backward_rows for these sizes (sort keys and positions,
 * chunk carries), host arithmetic only. The reference's bag_backward_rows (kernels.py:73-88) takes its sort
 * temporaries from the torch allocator; here the caller passes them in. */
SMLM_API size_t smlm_bag_backward_workspace(int64_t n, int64_t k, int64_t rows, int64_t d);

/* Row-sparse backward of the value bag:
 *   gw[n, j] = <grad_out[n], table[indices[n, j]]>
 *   acc[r] += sum over (n, j) with indices[n, j] == r of weights[n, j] * grad_out[n]   (in place)
 *   touched[indices[n, j]] = 1                                                          (in place)
 * The (row, position) pairs are radix-sorted (stable) and each row's run is summed in position order;
 * runs that cross a work chunk are completed by a second pass in chunk order. No float atomics:
 * results are bit-identical from run to run.
 * Replaces kernels.py:73 bag_backward_rows (and sparse_values.py:97-103, the aten per-sample-weight
 * backward + index_put_ accumulation). grad_out: F32/BF16 (n, d) (grad_dtype); weights F32/BF16; table
 * F32/BF16; acc F32. acc == NULL (and touched == NULL): only gw is computed (frozen table,
 * sparse_values.py:118-120). gw == NULL: only acc / touched are updated (table may then be NULL).
 * touched may be NULL (no mark kept). row_sqnorm (optional, fp32 (rows,)): the squared L2 norm of every
 * accumulator row written by this call. flags: SMLM_BWD_FIRST_TOUCH_WRITES. */
SMLM_API int smlm_bag_backward_rows(const void *grad_out, int grad_dtype, const int64_t *indices,
                                    const void *weights, int weights_dtype, const void *table, int table_dtype,
                                    float *acc, uint8_t *touched, float *row_sqnorm, int flags, float *gw,
                                    int64_t n, int64_t k, int64_t rows, int64_t d, void *workspace,
                                    size_t workspace_bytes, int *status, void *stream);

/* Writes the rows of a deferred backward (SMLM_BWD_DEFER_ROWS; every row it touched counts as zero before):
 * acc[row] = the row's sum, exactly what the backward would have written. Same grad_out, weights, sizes and
 * workspace as that backward. No counterpart in the reference (its backward always writes the rows). */
SMLM_API int smlm_bag_rows_materialize(const void *grad_out, int grad_dtype, const void *weights, int weights_dtype,
                                       float *acc, int64_t n, int64_t k, int64_t rows, int64_t d, void *workspace,
                                       size_t workspace_bytes, void *stream);

/* ------------------------------------------------------------------------------- row-sparse optimizers */

/* Scratch bytes of the touched-row compaction that the optimizer steps and smlm_touched_norm run first (the list
 * of touched rows), host arithmetic only. No counterpart in the reference: its steps scan the whole mask
 * (kernels.py:417-433, row_optim.py:179-201). */
SMLM_API size_t smlm_touched_workspace(int64_t rows);

/* Lazy Adam on the rows with touched[r] != 0 (the only rows loaded): with g = acc[r] * scale,
 *   m = m + (1 - b1) (g - m);  v = v b2 + (1 - b2) g g;  p = p + neg_step_size * (m / (sqrt(v) / bc2_sqrt + eps))
 * then acc[r] = 0 and touched[r] = 0. Operation order and fp32 rounding follow the reference's C loop
 * (smlm/host_rows.c:63-80, no contraction into FMA), so results are bit-identical to it.
 * scale = *grad_scale_dev if grad_scale_dev is not NULL, else grad_scale.
 * value_copy (optional, copy_dtype BF16 or F32, (rows, d)): the updated rows are also written there.
 * flags: SMLM_STEP_KEEP_ACC (acc rows are not zeroed).
 * Replaces kernels.py:417 lazy_adam_step (and LazyRowAdam.step's torch path, sparse_values.py:270-305). */
SMLM_API int smlm_lazy_adam_step(float *param, float *exp_avg, float *exp_avg_sq, float *acc, uint8_t *touched,
                                 const float *grad_scale_dev, float grad_scale, int64_t rows, int64_t d,
                                 float one_minus_b1, float b2, float one_minus_b2, float bc2_sqrt, float eps,
                                 float neg_step_size, void *value_copy, int copy_dtype, int flags, void *workspace,
                                 size_t workspace_bytes, void *stream);

/* smlm_lazy_adam_step with the six step scalars read from device memory when the kernel runs: scalars_dev[0..5] =
 * one_minus_b1, b2, one_minus_b2, bc2_sqrt, eps, neg_step_size (fp32), so a training step with several backward
 * passes into one table (the accumulator written, then stepped) can be captured in a CUDA graph; the caller writes
 * each step's scalars before replaying. No counterpart in the reference. */
SMLM_API int smlm_lazy_adam_step_dev(float *param, float *exp_avg, float *exp_avg_sq, float *acc, uint8_t *touched,
                                     const float *grad_scale_dev, float grad_scale, int64_t rows, int64_t d,
                                     const float *scalars_dev, void *value_copy, int copy_dtype, int flags,
                                     void *workspace, size_t workspace_bytes, void *stream);

/* Lazy Adam with compact moments (state_dtype SMLM_BF16: bf16 exp_avg / exp_avg_sq; SMLM_I8: int8 exp_avg codes
 * c with m = sign(c) (c / 127)^2 exp_avg_scale[row], uint8 exp_avg_sq codes u with v = ((u / 255)
 * exp_avg_sq_scale[row])^4, the scales fp32 (rows,)). Per touched row, in fp32 with every operation rounded:
 *   g = acc * grad_scale; m = beta1 m + (1 - beta1) g; v = beta2 v + ((1 - beta2) g) g;
 *   p = p - (step_size m) / (sqrt(v) / bc2_sqrt + eps)      (step_size = lr / (1 - beta1^step),
 *                                                               bc2_sqrt = sqrt(1 - beta2^step))
 * then the moments are stored rounded to nearest even (int8: scales = the row maxima of |m| and v^(1/4), codes
 * round(127 sign(m) sqrt(|m| / m_scale)) and round(255 v^(1/4) / v_scale), a positive v never gets code 0).
 * Touched flags cleared, acc rows zeroed unless SMLM_STEP_KEEP_ACC; value_copy as smlm_lazy_adam_step; unread
 * rows and their state unchanged. Workspace: smlm_touched_workspace(rows).
 * Replaces kernels.py:498-515 lazy_adam_step_lowmem (kernel kernels.py:445-495). */
SMLM_API int smlm_lazy_adam_lowmem_step(float *param, void *exp_avg, void *exp_avg_sq, float *exp_avg_scale,
                                        float *exp_avg_sq_scale, int state_dtype, float *acc, uint8_t *touched,
                                        const float *grad_scale_dev, float grad_scale, int64_t rows, int64_t d,
                                        float beta1, float beta2, float one_minus_b1, float one_minus_b2, float eps,
                                        float step_size, float bc2_sqrt, void *value_copy, int copy_dtype, int flags,
                                        void *workspace, size_t workspace_bytes, void *stream);

/* Row-wise optimizer on the touched rows (smlm/row_optim.py; formulas of host_rows.c:84-117):
 *   q = mean over the row of g^2 (summed in double), g = acc[r] * scale
 *   SMLM_ROWRMS:     v[r] = b2 v[r] + (1 - b2) q;  count[r] += 1;  denom = sqrt(v[r] / (1 - b2^count[r])) + eps
 *   SMLM_ROWADAGRAD: v[r] += q;                                      denom = sqrt(v[r]) + eps
 *   p[r] -= (lr / denom) * g;  acc[r] = 0;  touched[r] = 0.
 * count may be NULL for SMLM_ROWADAGRAD. flags: SMLM_STEP_KEEP_ACC.
 * Replaces RowWiseOptimizer._masked (row_optim.py:179-201). */
/* Lazy Adam fused with the row sums of a deferred backward: each row's sum (the gradient
 * smlm_bag_rows_materialize would have written, in the same summation order) goes straight into the
 * smlm_lazy_adam_step update of that row (same scalars, same operation order: the result is bit-identical to
 * materialising and stepping), touched cleared; the accumulator is never written or read. Same grad_out,
 * weights, sizes and workspace as the deferred backward. Replaces kernels.py:417-433 lazy_adam_step for a
 * RowStore whose rows come from one backward since the last step. */
SMLM_API int smlm_lazy_adam_deferred_step(float *param, float *exp_avg, float *exp_avg_sq, uint8_t *touched,
                                          const void *grad_out, int grad_dtype, const void *weights, int weights_dtype,
                                          const float *grad_scale_dev, float grad_scale, int64_t n, int64_t k,
                                          int64_t rows, int64_t d, float one_minus_b1, float b2, float one_minus_b2,
                                          float bc2_sqrt, float eps, float neg_step_size, void *value_copy,
                                          int copy_dtype, void *workspace, size_t workspace_bytes, void *stream);

/* smlm_lazy_adam_deferred_step with the six step scalars read from device memory when the kernels run:
 * scalars_dev[0..5] = one_minus_b1, b2, one_minus_b2, bc2_sqrt, eps, neg_step_size (fp32). For a training step
 * captured in a CUDA graph: the caller writes each step's scalars (computed as for the by-value call, so the
 * results are the same bits) into that buffer before replaying. No counterpart in the reference. */
SMLM_API int smlm_lazy_adam_deferred_step_dev(float *param, float *exp_avg, float *exp_avg_sq, uint8_t *touched,
                                              const void *grad_out, int grad_dtype, const void *weights,
                                              int weights_dtype, const float *grad_scale_dev, float grad_scale,
                                              int64_t n, int64_t k, int64_t rows, int64_t d, const float *scalars_dev,
                                              void *value_copy, int copy_dtype, void *workspace,
                                              size_t workspace_bytes, void *stream);

/* Row-wise optimizer step over the touched rows (kind SMLM_ROWRMS or SMLM_ROWADAGRAD): g = acc row * clip factor,
 * q = mean of g^2 (summed in double), rowrms v = b2 v + (1 - b2) q with a per-row step count, rowadagrad v += q,
 * then the parameter update; touched rows consumed, others bit-unchanged. Replaces RowWiseOptimizer.step's GPU
 * path (row_optim.py:52-71, 179-201) with the formulas of host_rows.c:82-117. Workspace:
 * smlm_touched_workspace(rows). */
SMLM_API int smlm_rowwise_step(float *param, float *acc, uint8_t *touched, float *v, int32_t *count,
                               const float *grad_scale_dev, float grad_scale, int64_t rows, int64_t d, int kind,
                               float b2, float eps, float lr, int flags, void *workspace, size_t workspace_bytes,
                               void *stream);

/* The row-wise step fused with the row sums of a deferred backward: each row's sum (the gradient
 * smlm_bag_rows_materialize would have written, same summation order) goes straight into the smlm_rowwise_step
 * update of that row (same formulas and rounding: bit-identical to materialising and stepping), touched cleared;
 * no accumulator is written or read. Same grad_out, weights, sizes and workspace as the deferred backward.
 * Replaces RowWiseOptimizer._masked (row_optim.py:179-201) for a RowStore whose rows come from one backward. */
SMLM_API int smlm_rowwise_deferred_step(float *param, uint8_t *touched, float *v, int32_t *count, const void *grad_out,
                                        int grad_dtype, const void *weights, int weights_dtype,
                                        const float *grad_scale_dev, float grad_scale, int64_t n, int64_t k,
                                        int64_t rows, int64_t d, int kind, float b2, float eps, float lr,
                                        void *workspace, size_t workspace_bytes, void *stream);

/* L2 norm of the accumulator over the touched rows, written to *norm_out (device fp32): the reference's
 * acc.norm() (sparse_values.py:143) for an accumulator whose untouched rows count as zero. With row_sqnorm
 * (the per-row squared norms the backward wrote) only 4 bytes per touched row are read, else the rows of acc.
 * Deterministic (fixed partial-sum order). */
SMLM_API int smlm_touched_norm(const float *acc, const float *row_sqnorm, const uint8_t *touched, int64_t rows,
                               int64_t d, float *norm_out, void *workspace, size_t workspace_bytes, void *stream);

/* acc rows whose touched byte is 0 are set to zero: turns "untouched rows count as zero" into actual zeros
 * before an accumulator is handed to code that reads it as a dense tensor (RowStore.acc). No counterpart in the
 * reference, whose accumulator is always dense (sparse_values.py:26-41). */
SMLM_API int smlm_zero_untouched(float *acc, const uint8_t *touched, int64_t rows, int64_t d, void *stream);

/* ------------------------------------------------------------------------- product-key scoring / select */

/* Product-key selection on given sub-key scores s1, s2 (n, h, nk), F32 or BF16:
 * per (n, h): top-knn of each half by (score desc, index asc); the knn x knn pair sums (rounded to the
 * score type, as `s1 + s2` in PyTorch); top-knn of those by (score desc, full index asc), full index
 * = i1 * nk + i2; softmax in fp32. Outputs scores (n, h, knn) in the score type, indices int64, weights F32,
 * in (score desc, index asc) order. 1 <= knn <= 32, knn <= nk <= 65536.
 * Replaces kernels.py:214 pk_select and pkm.py:125-136 get_indices + pkm.py:205-208 softmax. */
SMLM_API int smlm_pk_select(const void *s1, const void *s2, int score_dtype, int64_t n, int64_t h, int64_t nk,
                   int64_t knn, void *scores, int64_t *indices, float *weights, void *stream);

/* Backward of the selection, dense form: dl = w (g_w - sum(w g_w)) + g_scores; ds = dl rounded to the score
 * type; ds1[n, h, i1] = sum of ds over the selected pairs with that i1 (fp32, in selection order, then
 * rounded), ds2 likewise; all other entries zero. grad_w / grad_scores may be NULL.
 * Replaces kernels.py:253-266 PKSelect.backward. */
SMLM_API int smlm_select_backward(const int64_t *indices, const float *weights, const float *grad_w,
                         const void *grad_scores, int score_dtype, int64_t n, int64_t h, int64_t nk, int64_t knn,
                         void *ds1, void *ds2, void *stream);

/* Backward of the selection, sparse form, for the scoring contraction's backward without dense (n, h, nk)
 * gradients. Per (token n, head hh, half c) it emits knn lookups (entry e = ((n h + hh) 2 + c) knn + j, the
 * pair j of the selection) into the keys viewed as (h 2 nk, half): on the first occurrence of a sub-key in the
 * selection, entry_rows[e] = (hh 2 + c) nk + sub-key and entry_weights[e] (score type) = ds1 / ds2 of
 * smlm_select_backward at that sub-key; on its later occurrences entry_rows[e] = -1 and entry_weights[e] = 0.
 * Then, with row_base 0 and shard_rows h 2 nk (the -1 rows are skipped):
 *   dq (viewed (n h 2, half)) = the value bag of the entries over the keys              (smlm_shard_bag_forward)
 *   dkeys = its row-sparse backward with the query halves as grad_out, gw NULL   (smlm_shard_bag_backward_rows)
 * which are the two contractions of the reference's scoring backward restricted to the nonzero gradients.
 * Replaces kernels.py:253-266 PKSelect.backward together with the autograd backward of pkm.py:117-123. */
SMLM_API int smlm_select_grad_entries(const int64_t *indices, const float *weights, const float *grad_w,
                                      const void *grad_scores, int score_dtype, int64_t n, int64_t h, int64_t nk,
                                      int64_t knn, int64_t *entry_rows, void *entry_weights, void *stream);

/* Exact fp32 sub-key scores: s1[n, h, j] = sum_t q[n, h, t] k[h, 0, j, t] and s2 with the second halves,
 * each a sequential fmaf chain over t = 0 .. half-1 (the order a C loop reproduces bit for bit).
 * q: (n, h, 2 half), keys: (h, 2, nk, half). Replaces pkm.py:117-123 subkey_scores in fp32. */
SMLM_API int smlm_subkey_scores_f32(const float *q, const float *keys, int64_t n, int64_t h, int64_t nk, int64_t half,
                           float *s1, float *s2, void *stream);

/* Scratch bytes of smlm_score_select (the per-half top lists of every (token, head)), host arithmetic only. No
 * counterpart in the reference, whose einsum + pk_select path (pkm.py:195-201) allocates through torch. */
SMLM_API size_t smlm_score_select_workspace(int64_t n, int64_t h);

/* Fused scoring + selection under bf16 (the autocast path): q (n, h, 2 half) bf16, keys (h, 2, nk, half) bf16.
 * Per (token, head, half) the sub-key scores are a tensor-core GEMM (tcgen05, bf16 operands, fp32 accumulate,
 * TMA-fed, accumulators in TMEM), rounded to bf16 as the reference's bf16 einsum output; their top-knn
 * (score desc, index asc) is kept in the GEMM epilogue, so the (n, h, nk) score tensors are never written.
 * Then the pairs / final top-knn / softmax of smlm_pk_select. Outputs as smlm_pk_select with bf16 scores.
 * Calls of at most 16 tokens (decoding) with nk a multiple of 256 up to 8192 score on the SIMT cores instead
 * (one fp32 fmaf chain per sub-key, rounded once to bf16) when the workspace holds their lists: the tensor-core
 * pipeline has too little work there to hide its latency. Their scores equal the tensor-core path's up to the
 * order of the fp32 additions (both are within one bf16 step of the reference's einsum).
 * s1_out / s2_out (optional, bf16 (n, h, nk)): the rounded sub-key scores, for checking only.
 * half in {64, 128}; nk % 8 == 0; 1 <= knn <= 32. A kernel-internal wait that gives up raises
 * SMLM_FLAG_TIMEOUT in *status (outputs then invalid); nothing traps.
 * Replaces pkm.py:117-123 subkey_scores (bf16 autocast) + kernels.py:214 pk_select. */
SMLM_API int smlm_score_select(const void *q, const void *keys, int64_t n, int64_t h, int64_t nk, int64_t half,
                               int64_t knn, void *scores, int64_t *indices, float *weights, void *s1_out,
                               void *s2_out, void *workspace, size_t workspace_bytes, int *status, void *stream);

/* Allocation-free variant of smlm_score_select (same inputs, outputs and results; no debug score outputs), for
 * callers that cannot allocate device memory at call time: a host framework that has reserved the GPU's memory
 * in its own pool, or a latency-critical serving loop where cudaMalloc / cudaFree would synchronise the device.
 * No counterpart in the reference. Its scratch is a static device array inside the library, sized for at most
 * SMLM_NOALLOC_MAX_ROWS (token, head) rows (n * h; 8 MiB, held by every GPU that loads the library until the
 * process exits); larger calls return SMLM_ERR_INVALID. The first call on a device looks up that array's device
 * address (cudaGetSymbolAddress) with the device current; make that first call before any stream capture (a
 * first call on a capturing stream returns SMLM_ERR_INVALID). All calls share the one array, so calls that
 * overlap on the GPU (other streams, other threads) race: serialise them. Calls of at most 16 tokens take the
 * same SIMT path as smlm_score_select. Otherwise the key range is split over several CTAs per (token tile, head)
 * as the workspace entry point does, but only as far as the array holds the splits' lists (n * h * splits <=
 * SMLM_NOALLOC_MAX_ROWS): near the row limit the call runs unsplit, so a few hundred tokens at most use fewer
 * SMs than smlm_score_select would. The call allocates nothing: no cudaMalloc /
 * cudaFree, no allocating library routine. */
#define SMLM_NOALLOC_MAX_ROWS 16384
SMLM_API int smlm_score_select_noalloc(const void *q, const void *keys, int64_t n, int64_t h, int64_t nk,
                                       int64_t half, int64_t knn, void *scores, int64_t *indices, float *weights,
                                       int *status, void *stream);

/* ------------------------------------------------------------------------------ row-sharded value table
 * Multi-GPU form of the value bag (no counterpart in the reference, which runs on one device): the table, its
 * accumulator and its optimizer state are split into contiguous row ranges, one per GPU; rank r holds rows
 * [row_base, row_base + shard_rows). Every rank receives all ranks' lookups (global row indices) and serves
 * the ones that fall into its range; lookups of other ranges are skipped without an error. The exchange around
 * these calls (the lookups' all-gather, the partial bags' and weight gradients' all-to-all) runs on NCCL. */

/* out[n] = sum over the lookups j of token n whose row is in this shard, in j order, of
 * weights[n, j] * table_shard[indices[n, j] - row_base] (fp32 accumulation): this shard's partial bag.
 * indices: int32 or int64 global rows (index_dtype SMLM_I32 / SMLM_I64). Tokens with no lookup here get 0. */
SMLM_API int smlm_shard_bag_forward(const void *indices, int index_dtype, int64_t row_base, const void *weights,
                                    int weights_dtype, const void *table_shard, int table_dtype, int64_t n, int64_t k,
                                    int64_t shard_rows, int64_t d, void *out, int out_dtype, void *stream);

/* smlm_bag_backward_rows restricted to this shard's lookups: acc / touched / row_sqnorm are the shard's (local
 * rows), gw[n, j] is the per-sample-weight gradient of lookups in this shard and 0 for the others. Workspace
 * size: smlm_bag_backward_workspace(n, k, shard_rows, d). */
SMLM_API int smlm_shard_bag_backward_rows(const void *grad_out, int grad_dtype, const void *indices, int index_dtype,
                                          int64_t row_base, const void *weights, int weights_dtype,
                                          const void *table_shard, int table_dtype, float *acc, uint8_t *touched,
                                          float *row_sqnorm, int flags, float *gw, int64_t n, int64_t k,
                                          int64_t shard_rows, int64_t d, void *workspace, size_t workspace_bytes,
                                          int *status, void *stream);

/* dst[i] = (...((src[0][i] + src[1][i]) + src[2][i]) ... + src[slots-1][i]) in fp32, src (slots, count)
 * contiguous: the owners' partial results summed in rank order (deterministic). */
SMLM_API int smlm_slot_sum(const float *src, int64_t slots, int64_t count, float *dst, void *stream);

/* ----------------------------------------------- row-sharded exchange through peer memory (NVLink, CUDA IPC)
 * No counterpart in the reference (one device there). The same exchange as the NCCL collectives above, fused
 * into the owner's kernels: every rank owns one exchange
 * block in its HBM (flags, an epoch counter, its lookups bucketed by owner, a receive area for the owners' partial
 * bags and one for the weight gradients), mapped into the other ranks' processes with CUDA IPC (no multicast
 * objects anywhere). Each rank sorts its lookups into per-owner buckets (a counting sort by owner, slot order kept)
 * in its own block; the owner's forward kernel reads only its bucket of each rank over NVLink and stores that
 * rank's partial bag straight into its receive area; the weight-gradient kernel stores each in-shard lookup's
 * gradient straight into the requesting rank's area. Ranks announce progress by writing an epoch into each other's
 * flags after a system-scope fence: the caller's (> 0, the same on every rank), or with epoch 0 the block's own
 * counter, which the forward advances on the device and the backward reuses, so a step captured in a CUDA graph
 * gets a new epoch on every replay. Every wait is bounded (10 s of %globaltimer) and a timeout raises
 * SMLM_FLAG_TIMEOUT in *status (required) and ends every later wait at once. One forward may be outstanding per
 * exchange (its backward runs before the next forward). All ranks call the same entries with the same n, k, n_cap,
 * d, at most 64 ranks. The block is allocated once by smlm_xchg_alloc (the library's only device allocation, made
 * at setup, not per step). */
SMLM_API size_t smlm_xchg_bytes(int world, int64_t n_cap, int64_t k, int64_t d);
/* cudaMalloc of the block (zeroed) and its IPC handle (cudaIpcMemHandle_t, 64 bytes) for the other ranks */
SMLM_API int smlm_xchg_alloc(size_t bytes, void **block, void *ipc_handle);
/* maps another rank's block (cudaIpcOpenMemHandle, peer access enabled); unmap with smlm_xchg_close */
SMLM_API int smlm_xchg_open(const void *ipc_handle, void **block);
SMLM_API int smlm_xchg_close(void *block);
SMLM_API int smlm_xchg_free(void *block);

/* Forward of the sharded bag: buckets and publishes this rank's lookups (idx int32 global rows, -1 for padding,
 * and fp32 weights, (n, k); the owner of row r is r / rows_per_rank), computes this shard's partial bags of every
 * rank's tokens into their receive areas, waits for every owner and writes out (n, d) = the partials summed in
 * owner order, times silu(pre) when pre ((n, d) fp32 / bf16, the swilu projection) is given, as fp32 or bf16
 * (out_dtype). all_idx / all_w ((world n, k), both or neither): the lookups this shard served, in the layout of
 * every rank's lookups stacked (the others -1), for the backward. peers_dev: device array of world block pointers
 * (this rank's own included). d % 4 == 0, d <= 512, table, pre and out 16-byte aligned. */
SMLM_API int smlm_xchg_forward(void *const *peers_dev, void *my_block, int rank, int world, const int32_t *idx,
                               const float *weights, int64_t n, int64_t k, int64_t n_cap, int64_t rows_per_rank,
                               const void *table_shard, int table_dtype, int64_t row_base, int64_t shard_rows,
                               int64_t d, int32_t *all_idx, float *all_w, const void *pre, int pre_dtype, void *out,
                               int out_dtype, int64_t epoch, int *status, void *stream);
/* Backward, owner side: weight gradients of this shard's lookups of every rank (grad_all: the all-gathered
 * output gradients (world n, d), fp32 / bf16) into the requesting ranks' areas. */
SMLM_API int smlm_xchg_backward_gw(void *const *peers_dev, int rank, int world, const void *grad_all, int grad_dtype,
                                   const int32_t *all_idx, int64_t n, int64_t k, int64_t n_cap,
                                   const void *table_shard, int table_dtype, int64_t row_base, int64_t shard_rows,
                                   int64_t d, int64_t epoch, int *status, void *stream);
/* Backward, requester side: waits for every owner's weight gradients and copies them to gw (n, k) fp32. */
SMLM_API int smlm_xchg_collect_gw(void *const *peers_dev, int rank, int world, int64_t n, int64_t k, int64_t n_cap,
                                  int64_t d, float *gw, int64_t epoch, int *status, void *stream);

/* ------------------------------------------------------------------------------------- host-RAM value tables
 * Tables too large for the GPUs' memory stay in host RAM with their gradient accumulator and optimizer state
 * (reference: smlm/host_values.py, smlm/host_optim.py, smlm/host_rows.c). Here those host tensors are page-locked
 * and mapped into the device's address space, and kernels work on the rows a step reads directly over the host
 * link: no CPU loop and no staging copy through the CPU. smlm_lazy_adam_step, smlm_lazy_adam_lowmem_step and
 * smlm_rowwise_step take mapped host pointers for the table, the accumulator, the touched mask and the state as
 * they are; the calls below add what the host path needs besides. d % 4 == 0 (16-byte row accesses). */

/* Page-locks [ptr, ptr + bytes) of host memory and maps it into the current device's address space
 * (cudaHostRegister, mapped and portable); *device_ptr receives the address kernels use. The memory must stay
 * allocated until smlm_host_unregister. No counterpart in the reference (its host rows are read by C loops). */
SMLM_API int smlm_host_register(void *ptr, size_t bytes, void **device_ptr);
SMLM_API int smlm_host_unregister(void *ptr);

/* out[i] (device, (n, d) fp32) = hot[slot[i]] when slot (device int32, may be NULL) has slot[i] >= 0 (the row's
 * HOT copy on the device), else cache[slot2[i]] when slot2 (device int32, may be NULL) has slot2[i] >= 0 (a device
 * copy of the row, e.g. as the previous step updated it), else table[rows[i]] (table: a mapped host table of
 * table_rows rows; rows: device int64, distinct). Out-of-range rows give zeros and SMLM_FLAG_INDEX_RANGE. Replaces
 * HostEmbedding.gather's staging (host_values.py:82-119: indices to the host, a C gather into pinned memory, a
 * copy to the device). */
SMLM_API int smlm_host_rows_gather(const float *table, int64_t table_rows, const int64_t *rows, const int32_t *slot,
                                   const float *hot, const int32_t *slot2, const float *cache, int64_t n, int64_t d,
                                   float *out, int *status, void *stream);

/* table[rows[i]] = values[i] (table: a mapped host table of table_rows rows; rows device int64, distinct; values
 * device (n, d) fp32): the write-back of rows updated on the device. No counterpart in the reference (its row-wise
 * step writes the rows with a C loop, row_optim.py:73-135). */
SMLM_API int smlm_host_rows_scatter(float *table, int64_t table_rows, const int64_t *rows, const float *values,
                                    int64_t n, int64_t d, int *status, void *stream);

/* acc[rows[i]] = acc[rows[i]] + grads[i] and touched[rows[i]] = 1 (acc / touched: mapped host tensors of
 * table_rows rows; grads device (n, d) fp32; rows device int64, distinct), skipping the rows whose skip[i] >= 0
 * (skip may be NULL; HOT rows keep their own accumulator on the device). A row whose touched mark is 0 is written
 * as 0 + grads[i] without reading it, so the optimizer steps may leave stepped rows' accumulators uncleared
 * (SMLM_STEP_KEEP_ACC); touched may be NULL (every row accumulates). row_sqnorm: NULL, or a device fp32 array
 * of table_rows entries that gets each added row's new squared L2 norm (the row_sqnorm input of
 * smlm_touched_norm). Replaces HostEmbedding.accumulate's copy to the host and C scatter-add
 * (host_values.py:121-150, host_rows.c host_rows_add) and HostRowStore.norm's pass over the accumulator rows
 * (host_optim.py:95-107). */
SMLM_API int smlm_host_rows_add(float *acc, uint8_t *touched, float *row_sqnorm, int64_t table_rows,
                                const int64_t *rows, const float *grads, const int32_t *skip, int64_t n, int64_t d,
                                int *status, void *stream);

/* The row-wise step (kind SMLM_ROWRMS / SMLM_ROWADAGRAD; smlm_rowwise_step's formulas, order and rounding) of the
 * distinct rows rows[i] (device int64) with gradient grads[i] (device (n, d) fp32, e.g. a step's row sums kept on
 * the GPU), times the clip factor (*grad_scale_dev when given, else grad_scale); param, v and count may be mapped
 * host memory. current: NULL, or the rows' current values (device (n, d) fp32, equal to param's rows, e.g. the
 * rows the forward gathered), read instead of param, which is then only written. flags: SMLM_ROWS_TO_CURRENT
 * writes the updated rows into current instead of param (param is not touched and may be NULL; the caller writes
 * them back, smlm_host_rows_scatter). Replaces RowWiseOptimizer._step_gacc's chunked copies to the host and C loop
 * (row_optim.py:73-135, host_rows.c host_rows_rowwise). */
#define SMLM_ROWS_TO_CURRENT 1
SMLM_API int smlm_rows_rowwise_step(float *param, int64_t table_rows, const int64_t *rows, const float *grads,
                                    float *current, int64_t n, int64_t d, float *v, int32_t *count, int kind,
                                    float beta2, float eps, float lr, const float *grad_scale_dev, float grad_scale,
                                    int flags, int *status, void *stream);

/* ------------------------------------------------------------------------------------- Engram n-gram rows
 * Row indices of an Engram module's lookups: for position t of sequence b and lookup (order o, head h), the XOR over
 * i < orders[o] of c[b, history + t - i] * mult[o, h, i] (int64), then x ^= x >> 17, row = (x mod rows, floored)
 * + (o * heads + h) * rows. c: (batch, history + t_len) int64 compressed token ids (the history positions first);
 * mult: (n_orders, heads, max_order) int64 device array; orders: n_orders host ints, 1 <= orders[o] <= max_order,
 * orders[o] <= history + 1, n_orders <= 8; out: (batch, t_len, n_orders * heads) int64.
 * Replaces engram.py:63-75 NgramHash.forward (the table lookups themselves are smlm_bag_forward with k = 1). */
SMLM_API int smlm_ngram_rows(const int64_t *c, int64_t batch, int64_t t_len, int history, const int64_t *mult,
                             const int *orders, int n_orders, int heads, int max_order, int64_t rows, int64_t *out,
                             void *stream);

#ifdef __cplusplus
}
#endif

#endif /* SMLM_B200_H */
