/*
 * select_oracle.h -- CPU oracle of loom.cpp's logits->token stage.
 *
 * TEST INFRASTRUCTURE ONLY. This is the checker the CUDA kernels are compared against; it is never
 * linked into, loaded by, or called from the product library. Only the tests, the smoke check and
 * the bench's CPU-baseline / reference legs use it.
 *
 * Each function restates the loom.cpp code it cites (paths relative to the loom.cpp tree). Where
 * loom.cpp has no code (the sampling chain), the function follows the semantics written in
 * include/loom_select.h and shares only the exponential of include/loom_select_math.h, which is part
 * of those semantics.
 *
 * Status codes are those of include/loom_select.h.
 */
#ifndef LOOM_SELECT_ORACLE_H
#define LOOM_SELECT_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Generator::argmax (src/core/generation.cpp:64-74): strict '>' scan from index 0. */
int32_t oracle_argmax(const float* row, int64_t n);

/*
 * argmax_tensor_row (src/core/lua_bridge.cpp:302-330) over a [n_rows, n_vocab] f32 matrix with the
 * given row stride: requested_row < 0 means the last row, hi < 0 means n_vocab, the id is absolute.
 * Returns LOOM_SELECT_EWINDOW for a bad row (:312-314) or window (:315-319).
 */
int oracle_argmax_tensor_row(const float* data, int64_t n_vocab, int64_t n_rows, int64_t row_stride,
                             int64_t requested_row, int64_t lo, int64_t hi, int64_t* out_id);

/* argmax_tensor_rows (src/core/lua_bridge.cpp:343-365): one id per row; EINVAL when empty. */
int oracle_argmax_tensor_rows(const float* data, int64_t n_classes, int64_t n_rows, int64_t row_stride,
                              int32_t* out_ids);

/* The array form of loom.argmax_row (src/core/lua_bridge.cpp:744-758), over doubles. */
int oracle_argmax_row_array(const double* flat, int64_t flat_len, int64_t n_vocab, int64_t row_index,
                            int64_t* out_id);

/* Batched windowed argmax with loom_argmax_rows' argument conventions (f32 or bf16). */
int oracle_argmax_rows(const void* logits, int dtype, int64_t rows, int64_t n_vocab, int64_t row_stride,
                       int64_t lo, int64_t hi, int32_t* out_ids, int nthreads);

/*
 * ctc_greedy_decode (src/core/ctc_decode.cpp:7-31) for one utterance, plus the frame that emitted
 * each token and (optional) the per-frame raw argmax and its log-softmax value. Returns the number
 * of tokens written to out_ids / out_frames (capacity n_frames).
 */
int64_t oracle_ctc_greedy_one(const float* logits, int64_t n_frames, int64_t n_classes, int32_t blank,
                              int32_t* out_ids, int32_t* out_frames, int32_t* out_frame_ids,
                              float* out_frame_logp);

/* Batched form with loom_ctc_greedy's argument conventions. */
int oracle_ctc_greedy(const void* logits, int dtype, int64_t n_utt, int64_t n_frames, int64_t n_classes,
                      int32_t blank, int32_t* out_ids, int32_t* out_frames, int32_t* out_len,
                      int32_t* out_frame_ids, float* out_frame_logp, int nthreads);

/* The sampling chain of loom_sample_rows (semantics in include/loom_select.h), row by row. */
int oracle_sample_rows(const void* logits, int dtype, int64_t rows, int64_t n_vocab, int64_t row_stride,
                       const int32_t* history, int32_t history_len, const float* u, float temperature,
                       float repetition_penalty, int32_t top_k, float top_p, int32_t* out_ids,
                       float* out_prob, float* out_logp, int32_t* out_topk_ids, int nthreads);

/* Shard records with loom_sample_shard_partial's layout, and their merge. */
size_t oracle_shard_record_bytes(int32_t top_k);
int oracle_shard_partial(const void* logits, int dtype, int64_t rows, int64_t shard_vocab, int64_t row_stride,
                         int64_t vocab_offset, int64_t vocab_total, const int32_t* history,
                         int32_t history_len, float temperature, float repetition_penalty, int32_t top_k,
                         void* out_records, int nthreads);
int oracle_shard_merge(const void* records, int32_t n_shards, int64_t rows, const float* u, float temperature,
                       int32_t top_k, float top_p, int32_t* out_ids, float* out_prob, float* out_logp,
                       int32_t* out_topk_ids);

/* loom_exp_d of include/loom_select_math.h, exported so the tests can measure it against libm. */
double oracle_exp_d(double x);

/* Test helper: mismatches of the kernels' division by T (Markstein's method) against x / T, over every
 * x mantissa in [1, 2) and the nT given T values (see select_oracle.c). */
int64_t oracle_div_check(const float* T, int64_t nT, int nthreads, float* bad_x, float* bad_T);

#ifdef __cplusplus
}
#endif

#endif
