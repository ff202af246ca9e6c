/*
 * loom_select.h -- C-ABI of the B200 logits->token stage for loom.cpp.
 *
 * What this replaces in loom.cpp (paths relative to the loom.cpp source tree):
 *
 *   loom_argmax_rows   Generator::read_row + Generator::argmax        src/core/generation.cpp:56-74
 *                      argmax_tensor_row (windowed, absolute id)      src/core/lua_bridge.cpp:302-330
 *                      argmax_tensor_rows (one id per row)            src/core/lua_bridge.cpp:343-365
 *                      behind the Lua bindings loom.argmax_row / loom.argmax_row_range /
 *                      loom.argmax_rows                               src/core/lua_bridge.cpp:729-822
 *   loom_ctc_greedy    ctc_greedy_decode                              src/core/ctc_decode.cpp:7-31
 *                      (declared include/loom/core/ctc_decode.h:13), and the driver's
 *                      loom.argmax_rows + Lua collapse used by loom::audio::transcribe
 *                      (src/core/transcribe.cpp:235-259)
 *   loom_sample_rows   the token selection inside loom::text::generate (src/core/text_generate.cpp:30-85
 *                      -> driver -> src/core/lua_bridge.cpp:729-743). loom.cpp itself only selects
 *                      greedily; the repetition penalty / temperature / top-k / top-p / draw chain has
 *                      no counterpart there and follows the semantics written beside it below.
 *   loom_sample_shard_partial / loom_sample_shard_merge
 *                      the same chain with the vocabulary split across GPUs; no counterpart.
 *   loom_lm_head_argmax
 *                      the text model's last ggml_mul_mat(lm_head, hidden) followed by
 *                      Generator::argmax (src/core/generation.cpp:64-74), fused: the logits stay on chip.
 *
 * Conventions (those of loom.cpp's engine where it has one):
 *   - Every data pointer is DEVICE memory owned by the caller; the library keeps no pointer after a
 *     call returns (loom.cpp's non-owning convention, include/loom/core/backend.h:33-35).
 *   - Calls are stream-ordered on `stream` (a cudaStream_t; NULL is the legacy default stream) and
 *     return as soon as the work is enqueued. Calls never allocate: scratch memory is the caller's
 *     `workspace`, sized by the matching *_workspace_size query and zeroed once with
 *     loom_select_workspace_init before its first use. Kernels leave it zeroed again on success.
 *     One workspace must not be used by two calls that can run at the same time. The one exception
 *     is loom_sample_rows_noalloc, which takes no workspace: it uses a fixed scratch array inside
 *     the library and clears what it needs of it on every call.
 *   - Every function returns an int status (LOOM_SELECT_OK = 0). Argument errors are found on the
 *     host before anything is enqueued. Errors that only the device can see (a history id outside
 *     the vocabulary, a bounded wait that gave up) are recorded in the workspace and returned by
 *     loom_select_read_status. Nothing traps or aborts: loom.cpp turns errors into loom::Error
 *     exceptions (include/loom/loom_errors.h:10); the C++ wrapper in loom_select.hpp does the same
 *     with these codes.
 *   - Row r of a [rows, n_vocab] logits matrix starts at element r * row_stride (row_stride >=
 *     n_vocab), like a ggml tensor's nb[1] / element size.
 *   - dtype: LOOM_SELECT_F32 or LOOM_SELECT_BF16 (bf16 is widened exactly to f32).
 */
#ifndef LOOM_SELECT_H
#define LOOM_SELECT_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__) || defined(__clang__)
#define LOOM_SELECT_API __attribute__((visibility("default")))
#else
#define LOOM_SELECT_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define LOOM_SELECT_OK 0
#define LOOM_SELECT_EINVAL 1     /* null pointer, negative or zero size, row_stride < n_vocab, ... */
#define LOOM_SELECT_EDTYPE 2     /* dtype is not LOOM_SELECT_F32 / LOOM_SELECT_BF16 */
#define LOOM_SELECT_EWINDOW 3    /* id window [lo, hi) empty or outside [0, n_vocab) */
#define LOOM_SELECT_EWORKSPACE 4 /* workspace NULL, too small, or not 256-byte aligned */
#define LOOM_SELECT_ECUDA 5      /* a CUDA runtime call failed */
#define LOOM_SELECT_ETIMEOUT 6   /* device: a bounded wait gave up (the call's outputs are invalid) */
#define LOOM_SELECT_EHISTORY 7   /* device: a history id outside [0, vocabulary) */
#define LOOM_SELECT_EPARAM 8     /* sampling parameter out of its documented range */
#define LOOM_SELECT_ESHAPE 9     /* a size beyond what the kernels support (documented per call) */

/* Element types of a logits buffer. */
#define LOOM_SELECT_F32 0
#define LOOM_SELECT_BF16 1

/* Largest top_k, and longest per-row history, the sampling kernels accept. */
#define LOOM_SELECT_MAX_TOP_K 1024
#define LOOM_SELECT_MAX_HISTORY 1024

/* Returns a static English description of a status code. */
LOOM_SELECT_API const char* loom_select_strerror(int status);

/* ABI version of this header (major * 100 + minor). */
LOOM_SELECT_API int loom_select_abi_version(void);

/*
 * Workspace sizes in bytes for a call with these sizes. The result does not depend on the device,
 * so a workspace sized once serves every call up to these sizes.
 */
LOOM_SELECT_API size_t loom_argmax_workspace_size(int64_t rows, int64_t n_vocab);
LOOM_SELECT_API size_t loom_sample_workspace_size(int64_t rows, int64_t n_vocab, int32_t top_k);
LOOM_SELECT_API size_t loom_ctc_workspace_size(int64_t n_utt, int64_t n_frames);

/* Zeroes `bytes` of workspace on `stream` (once, before the workspace's first use). */
LOOM_SELECT_API int loom_select_workspace_init(void* workspace, size_t workspace_bytes, void* stream);

/*
 * Waits for `stream`, then returns (and clears) the first device-side error recorded in
 * `workspace` by calls enqueued so far: LOOM_SELECT_OK, LOOM_SELECT_EHISTORY or LOOM_SELECT_ETIMEOUT.
 * After LOOM_SELECT_ETIMEOUT the workspace must be re-initialised.
 */
LOOM_SELECT_API int loom_select_read_status(void* workspace, void* stream);

/*
 * Test hook, no loom.cpp counterpart: drives the bounded-wait failure path of the streamed kernels
 * (argmax of long rows, the sampler for top_k <= 128) and of loom_lm_head_argmax (where the withheld
 * stage is the first CTA's K slice number withhold_stage) without any fault. It writes into the
 * workspace header, on `stream`: wait_limit_ns (> 0) replaces the 2 s bound of every wait of those
 * kernels, and withhold_stage >= 0 makes the first CTA's producer leave that stage of its range
 * unissued, so its consumers' waits run out. The next such call records LOOM_SELECT_ETIMEOUT (its
 * outputs are invalid) and every wait still ends. loom_select_workspace_init clears the hook and
 * the state a timed-out call leaves behind; nothing else touches it. Not for production use.
 */
LOOM_SELECT_API int loom_select_test_wait_fault(void* workspace, int64_t wait_limit_ns, int32_t withhold_stage,
                                                void* stream);

/*
 * Greedy argmax of every row over the id window [lo, hi), hi < 0 meaning n_vocab.
 *
 * Replaces Generator::argmax (src/core/generation.cpp:64-74) and the scan inside argmax_tensor_row /
 * argmax_tensor_rows (src/core/lua_bridge.cpp:320-329, :358-362), with the same result on every
 * input: a strict '>' scan from `lo`, so the lowest id wins among equal maxima, -0 equals +0, a NaN
 * at `lo` wins (nothing compares greater than it) and a NaN anywhere else never wins.
 * out_ids[r] is the ABSOLUTE id (lo + offset), as argmax_tensor_row returns.
 * Errors: LOOM_SELECT_EWINDOW for lo < 0, lo >= hi or hi > n_vocab (lua_bridge.cpp:315-319).
 */
LOOM_SELECT_API int loom_argmax_rows(const void* logits, int dtype, int64_t rows, int64_t n_vocab, int64_t row_stride,
                     int64_t lo, int64_t hi, int32_t* out_ids, void* workspace, size_t workspace_bytes,
                     void* stream);

/* Largest number of id windows one loom_argmax_windows call takes. */
#define LOOM_SELECT_MAX_WINDOWS 8

/* Workspace size in bytes for loom_argmax_windows on `rows` rows and `n_windows` windows. */
LOOM_SELECT_API size_t loom_argmax_windows_workspace_size(int64_t rows, int32_t n_windows);

/*
 * Greedy argmax of every row over each of several id windows, in one launch:
 * out_ids[r * n_windows + w] = the ABSOLUTE argmax id of row r over [lo[w], hi[w]), by the
 * loom_argmax_rows rule (strict '>' from lo[w]; a NaN at lo[w] wins; -0 == +0).
 *
 * Replaces n_windows calls per row of argmax_tensor_row (src/core/lua_bridge.cpp:302-330), the scan
 * behind loom.argmax_row_range (lua_bridge.cpp:779-797): Whisper's driver asks one decoder row for its
 * language block and its timestamp block, each a window inside the 51865-id vocabulary.
 * lo and hi are HOST arrays of n_windows (1 .. LOOM_SELECT_MAX_WINDOWS) entries, read during the call;
 * hi[w] < 0 means n_vocab. Errors, before anything is enqueued: LOOM_SELECT_EWINDOW for a window with
 * lo < 0, lo >= hi or hi > n_vocab (lua_bridge.cpp:315-319); LOOM_SELECT_EINVAL for n_windows out of range.
 */
LOOM_SELECT_API int loom_argmax_windows(const void* logits, int dtype, int64_t rows, int64_t n_vocab,
                                        int64_t row_stride, const int64_t* lo, const int64_t* hi, int32_t n_windows,
                                        int32_t* out_ids, void* workspace, size_t workspace_bytes, void* stream);

/* Sampling parameters (passed by pointer to host memory; read during the call). */
typedef struct loom_sample_params {
    float temperature;        /* T > 0, finite; T == 0 selects greedy (loom_argmax_rows semantics) */
    float repetition_penalty; /* r > 0, finite; 1 disables */
    int32_t top_k;            /* 1 <= k <= min(vocabulary, LOOM_SELECT_MAX_TOP_K) */
    float top_p;              /* 0 < p <= 1 */
} loom_sample_params;

/*
 * Fused sampling chain, one token per row. No loom.cpp counterpart (loom.cpp selects greedily only);
 * it stands in for the selection step of loom::text::generate. Semantics, per row x[0..V):
 *   1. penalty: for each DISTINCT id v in history[r*history_len .. +history_len):
 *      x[v] = x[v] > 0 ? x[v] / r : x[v] * r                      (fp32, round to nearest)
 *      an id outside [0, V) records LOOM_SELECT_EHISTORY and makes out_ids[r] = -1.
 *   2. temperature: y[v] = x[v] / T                              (fp32 divide)
 *   3. key: y descending, then id ascending; -0 == +0; NaN below -inf.
 *   4. top-k: the first k ids under that key (out_topk_ids[r*k .. +k] if non-NULL).
 *   5. survivor softmax in double: e_i = loom_survivor_weight(y_i, y_0) (loom_select_math.h),
 *      S_j = e_0 + ... + e_j summed in key order.
 *   6. top-p: n = the smallest n >= 1 with S_{n-1} >= p * S_{k-1}.
 *   7. draw: the first i < n with u[r] * S_{n-1} < S_i, else n - 1.
 *   out_ids[r] = id of survivor i, out_prob[r] = (float)(e_i / S_{n-1}).
 *   out_logp (optional) = y_i - (M + log sum_v exp(y_v - M)) over the whole penalised, tempered row
 *   (M = max y), accurate to 1e-5 relative on the probability scale.
 * With T == 0 the chain is greedy over the penalised row: the loom_argmax_rows rule picks the id,
 * out_prob = 1 and out_logp uses T = 1.
 * history may be NULL when history_len == 0 (history_len <= LOOM_SELECT_MAX_HISTORY, else
 * LOOM_SELECT_ESHAPE). u is one uniform per row in [0, 1).
 */
LOOM_SELECT_API int loom_sample_rows(const void* logits, int dtype, int64_t rows, int64_t n_vocab, int64_t row_stride,
                     const int32_t* history, int32_t history_len, const float* u,
                     const loom_sample_params* params, int32_t* out_ids, float* out_prob, float* out_logp,
                     int32_t* out_topk_ids, void* workspace, size_t workspace_bytes, void* stream);

/*
 * loom_sample_rows for callers that cannot allocate device memory. No counterpart in loom.cpp (nor in
 * this library's other entry points): it exists for hosts whose device memory is all handed out up
 * front -- an engine whose own arena (ggml's backend allocator) sizes one buffer for the whole graph,
 * a serving loop that may not grow its footprint after start-up, a plugin host with no allocation
 * hook -- and so cannot give loom_sample_rows a workspace.
 * Same arguments, checks and results as loom_sample_rows, without the workspace. Its scratch is one
 * fixed device array inside the library (LOOM_SELECT_NOALLOC_SCRATCH_BYTES per device), so:
 *   - top_k is limited to LOOM_SELECT_NOALLOC_MAX_TOP_K; a larger one returns LOOM_SELECT_ESHAPE;
 *   - each call clears the array's status word and tickets itself (a memset on `stream`);
 *   - calls whose work can overlap on the GPU (other streams, other host threads) race on the array:
 *     order them on one stream;
 *   - the first call on a device looks the array up and loads its code there; make it before any
 *     stream capture; the address is kept until the process exits, so do not use this entry point
 *     on a device after cudaDeviceReset there;
 *   - out_status (device int32, may be NULL) receives the call's device-side status
 *     (LOOM_SELECT_EHISTORY, LOOM_SELECT_ETIMEOUT or 0), the word loom_select_read_status reads for
 *     a caller-owned workspace.
 */
#define LOOM_SELECT_NOALLOC_MAX_TOP_K 64
#define LOOM_SELECT_NOALLOC_SCRATCH_BYTES 1106176 /* 256 + 8192 + 16384 + 2048 * (16 + 8 * 64) */

LOOM_SELECT_API int loom_sample_rows_noalloc(const void* logits, int dtype, int64_t rows, int64_t n_vocab,
                             int64_t row_stride, const int32_t* history, int32_t history_len, const float* u,
                             const loom_sample_params* params, int32_t* out_ids, float* out_prob,
                             float* out_logp, int32_t* out_topk_ids, int32_t* out_status, void* stream);

/*
 * Vocabulary-sharded sampling: each GPU owns ids [vocab_offset, vocab_offset + shard_vocab) of a
 * vocabulary of vocab_total ids and runs loom_sample_shard_partial on its [rows, shard_vocab] slice.
 * The per-row records (loom_shard_record_bytes(top_k) bytes each, `rows` records) are then gathered
 * from every shard -- ncclAllGather over NVLink in a multi-GPU job -- into one [n_shards][rows] array,
 * and loom_sample_shard_merge turns them into exactly what loom_sample_rows returns for the whole
 * row. History ids are global; each shard applies the penalty to the ids it owns. T must be > 0.
 * A record holds: int32 count, float m, float s, int32 reserved, then `top_k` pairs (float y,
 * int32 global id) -- the shard's top-k under the chain's key and its partial max / sum-exp.
 */
LOOM_SELECT_API size_t loom_shard_record_bytes(int32_t top_k);

LOOM_SELECT_API int loom_sample_shard_partial(const void* logits, int dtype, int64_t rows, int64_t shard_vocab,
                              int64_t row_stride, int64_t vocab_offset, int64_t vocab_total,
                              const int32_t* history, int32_t history_len, const loom_sample_params* params,
                              void* out_records, void* workspace, size_t workspace_bytes, void* stream);

LOOM_SELECT_API int loom_sample_shard_merge(const void* records, int32_t n_shards, int64_t rows, const float* u,
                            const loom_sample_params* params, int32_t* out_ids, float* out_prob,
                            float* out_logp, int32_t* out_topk_ids, void* stream);

/*
 * Greedy CTC decode of n_utt utterances, each [n_frames, n_classes] row-major and contiguous
 * (utterance u starts at element u * n_frames * n_classes).
 *
 * Replaces ctc_greedy_decode (src/core/ctc_decode.cpp:7-31) with the same result: per-frame argmax
 * by the loom_argmax_rows rule on the RAW logits, then collapse repeats and drop `blank`, with the
 * previous id seeded as blank. For utterance u, out_len[u] tokens are written to
 * out_ids[u*n_frames ..] and, in out_frames, the frame index that emitted each (the first frame of
 * its run; loom.cpp produces no offsets). Optional per-frame outputs ([n_utt * n_frames], NULL to
 * skip): out_frame_ids = the raw argmax (what loom.argmax_rows returns, lua_bridge.cpp:343-365) and
 * out_frame_logp = its log-softmax value, accurate to 1e-5 relative on the probability scale.
 */
LOOM_SELECT_API int loom_ctc_greedy(const void* logits, int dtype, int64_t n_utt, int64_t n_frames, int64_t n_classes,
                    int32_t blank, int32_t* out_ids, int32_t* out_frames, int32_t* out_len,
                    int32_t* out_frame_ids, float* out_frame_logp, void* workspace, size_t workspace_bytes,
                    void* stream);

/*
 * Greedy selection fused into the LM-head GEMM: logits[r, v] = sum_h hidden[r, h] * weight[v, h]
 * (bf16 inputs, f32 tensor-core accumulation) are reduced tile by tile on chip and never written to
 * memory. Replaces ggml's mul_mat(lm_head, hidden) that ends loom.cpp's text models followed by
 * Generator::argmax (src/core/generation.cpp:64-74); the weight layout is ggml's: [n_vocab,
 * hidden_dim] row-major. out_ids[r] follows the loom_argmax_rows rule on those f32 logits (lowest id
 * among equal maxima, a NaN at id 0 wins, a NaN elsewhere never wins); out_logit[r] (NULL to skip) is
 * the winning logit and out_lse[r] (NULL to skip) the row's log-sum-exp, so out_logit - out_lse is
 * the greedy token's log-probability. Requirements: hidden_dim a multiple of 64 (LOOM_SELECT_ESHAPE
 * otherwise), hidden and weight 16-byte aligned with rows packed (row stride = hidden_dim). Device
 * errors (a bounded wait that gave up) are read with loom_select_read_status.
 */
LOOM_SELECT_API size_t loom_lm_head_workspace_size(int64_t rows, int64_t n_vocab);
LOOM_SELECT_API int loom_lm_head_argmax(const void* hidden, const void* weight, int64_t rows, int64_t hidden_dim,
                                        int64_t n_vocab, int32_t* out_ids, float* out_logit, float* out_lse,
                                        void* workspace, size_t workspace_bytes, void* stream);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* LOOM_SELECT_H */
