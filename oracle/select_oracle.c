/*
 * select_oracle.c -- CPU oracle of loom.cpp's logits->token stage.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA kernels, never part of the product library.
 * Built with -ffp-contract=off so that every float / double expression rounds exactly as written.
 * Citations are paths in the loom.cpp source tree.
 */
#include "select_oracle.h"

#include "loom_select.h"
#include "loom_select_math.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------------------------------ */
/* element access                                                                                   */

static inline float widen_bf16(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, sizeof f);
    return f;
}

static inline float load_elem(const void* base, int dtype, int64_t i) {
    if (dtype == LOOM_SELECT_BF16) return widen_bf16(((const uint16_t*)base)[i]);
    return ((const float*)base)[i];
}

/* ------------------------------------------------------------------------------------------------ */
/* greedy argmax                                                                                    */

/* Generator::argmax, src/core/generation.cpp:64-74. */
int32_t oracle_argmax(const float* row, int64_t n) {
    int32_t best = 0;
    float best_val = row[0];
    for (int64_t i = 1; i < n; ++i) {
        if (row[i] > best_val) {
            best_val = row[i];
            best = (int32_t)i;
        }
    }
    return best;
}

/* argmax_tensor_row, src/core/lua_bridge.cpp:302-330 (the f32 check of :304-306 is the caller's). */
int oracle_argmax_tensor_row(const float* data, int64_t n_vocab, int64_t n_rows, int64_t row_stride,
                             int64_t requested_row, int64_t lo, int64_t hi, int64_t* out_id) {
    const int64_t row = requested_row < 0 ? n_rows - 1 : requested_row;
    if (n_vocab <= 0 || row < 0 || row >= n_rows) return LOOM_SELECT_EWINDOW;
    if (hi < 0) hi = n_vocab;
    if (lo < 0 || lo >= hi || hi > n_vocab) return LOOM_SELECT_EWINDOW;
    const int64_t width = hi - lo;
    const float* logits = data + row * row_stride + lo;
    int64_t best = 0;
    for (int64_t i = 1; i < width; ++i) {
        if (logits[i] > logits[best]) best = i;
    }
    *out_id = lo + best;
    return LOOM_SELECT_OK;
}

/* argmax_tensor_rows, src/core/lua_bridge.cpp:343-365. */
int oracle_argmax_tensor_rows(const float* data, int64_t n_classes, int64_t n_rows, int64_t row_stride,
                              int32_t* out_ids) {
    if (n_classes <= 0 || n_rows <= 0) return LOOM_SELECT_EINVAL;
    for (int64_t r = 0; r < n_rows; ++r) {
        const float* row = data + r * row_stride;
        int64_t best = 0;
        for (int64_t i = 1; i < n_classes; ++i) {
            if (row[i] > row[best]) best = i;
        }
        out_ids[r] = (int32_t)best;
    }
    return LOOM_SELECT_OK;
}

/* l_argmax_row's array form, src/core/lua_bridge.cpp:744-758. */
int oracle_argmax_row_array(const double* flat, int64_t flat_len, int64_t n_vocab, int64_t row_index,
                            int64_t* out_id) {
    if (n_vocab == 0 || (row_index + 1) * n_vocab > flat_len) return LOOM_SELECT_EWINDOW;
    const double* row = flat + row_index * n_vocab;
    int64_t best = 0;
    double best_val = row[0];
    for (int64_t i = 1; i < n_vocab; ++i) {
        if (row[i] > best_val) {
            best_val = row[i];
            best = i;
        }
    }
    *out_id = best;
    return LOOM_SELECT_OK;
}

/* ------------------------------------------------------------------------------------------------ */
/* a tiny parallel-for over rows (the oracle is also the timed CPU baseline)                        */

typedef void (*row_fn)(void* ctx, int64_t row);

typedef struct {
    row_fn fn;
    void* ctx;
    int64_t begin, end;
} row_task;

static void* run_rows(void* arg) {
    row_task* t = (row_task*)arg;
    for (int64_t r = t->begin; r < t->end; ++r) t->fn(t->ctx, r);
    return NULL;
}

static void parallel_rows(row_fn fn, void* ctx, int64_t rows, int nthreads) {
    if (nthreads < 1) nthreads = 1;
    if (nthreads > rows) nthreads = (int)(rows > 0 ? rows : 1);
    if (nthreads == 1) {
        for (int64_t r = 0; r < rows; ++r) fn(ctx, r);
        return;
    }
    pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)nthreads);
    row_task* tasks = (row_task*)malloc(sizeof(row_task) * (size_t)nthreads);
    for (int i = 0; i < nthreads; ++i) {
        tasks[i].fn = fn;
        tasks[i].ctx = ctx;
        tasks[i].begin = rows * i / nthreads;
        tasks[i].end = rows * (i + 1) / nthreads;
        pthread_create(&th[i], NULL, run_rows, &tasks[i]);
    }
    for (int i = 0; i < nthreads; ++i) pthread_join(th[i], NULL);
    free(tasks);
    free(th);
}

/* ------------------------------------------------------------------------------------------------ */
/* batched windowed argmax                                                                          */

typedef struct {
    const void* logits;
    int dtype;
    int64_t row_stride, lo, hi;
    int32_t* out;
} argmax_ctx;

static void argmax_row_fn(void* vctx, int64_t r) {
    const argmax_ctx* c = (const argmax_ctx*)vctx;
    const int64_t base = r * c->row_stride;
    int64_t best = c->lo;
    float best_val = load_elem(c->logits, c->dtype, base + c->lo);
    for (int64_t i = c->lo + 1; i < c->hi; ++i) {
        const float v = load_elem(c->logits, c->dtype, base + i);
        if (v > best_val) {
            best_val = v;
            best = i;
        }
    }
    c->out[r] = (int32_t)best;
}

int oracle_argmax_rows(const void* logits, int dtype, int64_t rows, int64_t n_vocab, int64_t row_stride,
                       int64_t lo, int64_t hi, int32_t* out_ids, int nthreads) {
    if (dtype != LOOM_SELECT_F32 && dtype != LOOM_SELECT_BF16) return LOOM_SELECT_EDTYPE;
    if (!logits || !out_ids || rows <= 0 || n_vocab <= 0 || row_stride < n_vocab) return LOOM_SELECT_EINVAL;
    if (hi < 0) hi = n_vocab;
    if (lo < 0 || lo >= hi || hi > n_vocab) return LOOM_SELECT_EWINDOW;
    argmax_ctx c = {logits, dtype, row_stride, lo, hi, out_ids};
    parallel_rows(argmax_row_fn, &c, rows, nthreads);
    return LOOM_SELECT_OK;
}

/* ------------------------------------------------------------------------------------------------ */
/* CTC greedy decode                                                                                */

/* log-softmax value of x[id] over a row, in double, over the non-NaN entries. */
static double row_logsoftmax_at(const float* x, int64_t n, int64_t id) {
    double m = -INFINITY;
    int any = 0;
    for (int64_t i = 0; i < n; ++i) {
        if (x[i] == x[i]) {
            if (!any || x[i] > m) m = x[i];
            any = 1;
        }
    }
    if (!any) return NAN;
    if (isinf(m)) return (double)x[id] - m;
    double s = 0.0;
    for (int64_t i = 0; i < n; ++i) {
        if (x[i] == x[i]) s += exp((double)x[i] - m);
    }
    return (double)x[id] - (m + log(s));
}

/* ctc_greedy_decode, src/core/ctc_decode.cpp:7-31, plus emitting-frame indices. */
int64_t oracle_ctc_greedy_one(const float* logits, int64_t n_frames, int64_t n_classes, int32_t blank,
                              int32_t* out_ids, int32_t* out_frames, int32_t* out_frame_ids,
                              float* out_frame_logp) {
    int64_t n_out = 0;
    int32_t prev = blank; /* seeded with blank, ctc_decode.cpp:23 */
    for (int64_t f = 0; f < n_frames; ++f) {
        const float* frame = logits + f * n_classes;
        int32_t best_id = 0;
        float best_val = frame[0];
        for (int64_t c = 1; c < n_classes; ++c) {
            if (frame[c] > best_val) {
                best_val = frame[c];
                best_id = (int32_t)c;
            }
        }
        if (out_frame_ids) out_frame_ids[f] = best_id;
        if (out_frame_logp) out_frame_logp[f] = (float)row_logsoftmax_at(frame, n_classes, best_id);
        if (best_id != prev && best_id != blank) {
            out_ids[n_out] = best_id;
            out_frames[n_out] = (int32_t)f;
            ++n_out;
        }
        prev = best_id;
    }
    return n_out;
}

typedef struct {
    const void* logits;
    int dtype;
    int64_t n_frames, n_classes;
    int32_t blank;
    int32_t *out_ids, *out_frames, *out_len, *out_frame_ids;
    float* out_frame_logp;
} ctc_ctx;

static void ctc_utt_fn(void* vctx, int64_t u) {
    const ctc_ctx* c = (const ctc_ctx*)vctx;
    const int64_t n = c->n_frames * c->n_classes;
    float* tmp = NULL;
    const float* src;
    if (c->dtype == LOOM_SELECT_BF16) {
        tmp = (float*)malloc(sizeof(float) * (size_t)n);
        for (int64_t i = 0; i < n; ++i) tmp[i] = load_elem(c->logits, c->dtype, u * n + i);
        src = tmp;
    } else {
        src = (const float*)c->logits + u * n;
    }
    c->out_len[u] = (int32_t)oracle_ctc_greedy_one(
        src, c->n_frames, c->n_classes, c->blank, c->out_ids + u * c->n_frames, c->out_frames + u * c->n_frames,
        c->out_frame_ids ? c->out_frame_ids + u * c->n_frames : NULL,
        c->out_frame_logp ? c->out_frame_logp + u * c->n_frames : NULL);
    free(tmp);
}

int oracle_ctc_greedy(const void* logits, int dtype, int64_t n_utt, int64_t n_frames, int64_t n_classes,
                      int32_t blank, int32_t* out_ids, int32_t* out_frames, int32_t* out_len,
                      int32_t* out_frame_ids, float* out_frame_logp, int nthreads) {
    if (dtype != LOOM_SELECT_F32 && dtype != LOOM_SELECT_BF16) return LOOM_SELECT_EDTYPE;
    if (!logits || !out_ids || !out_frames || !out_len || n_utt <= 0 || n_frames <= 0 || n_classes <= 0)
        return LOOM_SELECT_EINVAL;
    ctc_ctx c = {logits, dtype, n_frames, n_classes, blank, out_ids, out_frames, out_len, out_frame_ids,
                 out_frame_logp};
    parallel_rows(ctc_utt_fn, &c, n_utt, nthreads);
    return LOOM_SELECT_OK;
}

/* ------------------------------------------------------------------------------------------------ */
/* sampling chain                                                                                   */

double oracle_exp_d(double x) { return loom_exp_d(x); }

typedef struct {
    uint64_t key;
    float y;
    int32_t id;
} cand;

/* min-heap on key (the root is the worst of the current best k) */
static void heap_sift_down(cand* h, int n, int i) {
    for (;;) {
        int l = 2 * i + 1, r = l + 1, m = i;
        if (l < n && h[l].key < h[m].key) m = l;
        if (r < n && h[r].key < h[m].key) m = r;
        if (m == i) return;
        cand t = h[i];
        h[i] = h[m];
        h[m] = t;
        i = m;
    }
}

static void heap_sift_up(cand* h, int i) {
    while (i > 0) {
        int p = (i - 1) / 2;
        if (h[p].key <= h[i].key) return;
        cand t = h[i];
        h[i] = h[p];
        h[p] = t;
        i = p;
    }
}

static int cand_desc(const void* a, const void* b) {
    const uint64_t ka = ((const cand*)a)->key, kb = ((const cand*)b)->key;
    return ka < kb ? 1 : (ka > kb ? -1 : 0);
}

/* Offer (y, id) to a heap of capacity k holding n entries; returns the new n. */
static int topk_offer(cand* heap, int n, int k, float y, int32_t id) {
    const uint64_t key = loom_rank_key(y, id);
    if (n < k) {
        heap[n].key = key;
        heap[n].y = y;
        heap[n].id = id;
        heap_sift_up(heap, n);
        return n + 1;
    }
    if (key > heap[0].key) {
        heap[0].key = key;
        heap[0].y = y;
        heap[0].id = id;
        heap_sift_down(heap, n, 0);
    }
    return n;
}

/*
 * Steps 5-7 of the chain on survivors already in key order (best first). Every double operation is
 * written out in the order the semantics give, with no contraction (see loom_select_math.h).
 */
static void decide(const cand* top, int k, float top_p, float u, int32_t* out_id, float* out_prob) {
    if (k <= 0) {
        *out_id = -1;
        *out_prob = NAN;
        return;
    }
    double* e = (double*)calloc((size_t)k, sizeof(double));
    double* S = (double*)calloc((size_t)k, sizeof(double));
    const float m = top[0].y;
    for (int i = 0; i < k; ++i) e[i] = loom_survivor_weight(top[i].y, m);
    S[0] = e[0];
    for (int i = 1; i < k; ++i) S[i] = S[i - 1] + e[i];
    const double target = (double)top_p * S[k - 1];
    int n = k;
    for (int j = 0; j < k; ++j) {
        if (S[j] >= target) {
            n = j + 1;
            break;
        }
    }
    const double draw = (double)u * S[n - 1];
    int sel = n - 1;
    for (int i = 0; i < n; ++i) {
        if (draw < S[i]) {
            sel = i;
            break;
        }
    }
    *out_id = top[sel].id;
    *out_prob = (float)(e[sel] / S[n - 1]);
    free(S);
    free(e);
}

/* max over the non-NaN values (-inf when there are none) and the sum of exp(y - max) in double. */
static void lse_partial(const float* y, int64_t n, double* m_out, double* s_out) {
    double m = -INFINITY;
    for (int64_t i = 0; i < n; ++i)
        if (y[i] == y[i] && y[i] > m) m = y[i];
    double s = 0.0;
    if (m != -INFINITY) {
        for (int64_t i = 0; i < n; ++i) {
            if (y[i] != y[i]) continue;
            s += (y[i] == m) ? 1.0 : exp((double)y[i] - m);
        }
    }
    *m_out = m;
    *s_out = s;
}

static int cmp_i32(const void* a, const void* b) {
    const int32_t x = *(const int32_t*)a, y = *(const int32_t*)b;
    return x < y ? -1 : (x > y ? 1 : 0);
}

/*
 * Applies the repetition penalty to x[0..n) for the DISTINCT history ids in [id_lo, id_lo + n);
 * returns LOOM_SELECT_EHISTORY if an id lies outside [0, id_limit).
 */
static int apply_penalty(float* x, int64_t n, int64_t id_lo, int64_t id_limit, const int32_t* hist, int32_t hlen,
                         float r) {
    if (hlen <= 0) return LOOM_SELECT_OK;
    int32_t* h = (int32_t*)malloc(sizeof(int32_t) * (size_t)hlen);
    memcpy(h, hist, sizeof(int32_t) * (size_t)hlen);
    qsort(h, (size_t)hlen, sizeof(int32_t), cmp_i32);
    int status = LOOM_SELECT_OK;
    for (int32_t j = 0; j < hlen; ++j) {
        if (h[j] < 0 || h[j] >= id_limit) {
            status = LOOM_SELECT_EHISTORY;
            break;
        }
    }
    if (status == LOOM_SELECT_OK) {
        for (int32_t j = 0; j < hlen; ++j) {
            if (j > 0 && h[j] == h[j - 1]) continue; /* a set: duplicates apply once */
            const int64_t v = (int64_t)h[j] - id_lo;
            if (v < 0 || v >= n) continue;
            x[v] = x[v] > 0.0f ? x[v] / r : x[v] * r;
        }
    }
    free(h);
    return status;
}

typedef struct {
    const void* logits;
    int dtype;
    int64_t n_vocab, row_stride;
    const int32_t* history;
    int32_t history_len;
    const float* u;
    float T, r, p;
    int32_t k;
    int32_t *out_ids, *out_topk;
    float *out_prob, *out_logp;
    int status; /* first error, written racily but only ever with the same value */
} sample_ctx;

static void sample_row_fn(void* vctx, int64_t row) {
    sample_ctx* c = (sample_ctx*)vctx;
    const int64_t V = c->n_vocab;
    float* x = (float*)malloc(sizeof(float) * (size_t)V);
    for (int64_t i = 0; i < V; ++i) x[i] = load_elem(c->logits, c->dtype, row * c->row_stride + i);
    const int32_t* hist = c->history ? c->history + row * (int64_t)c->history_len : NULL;
    if (apply_penalty(x, V, 0, V, hist, c->history_len, c->r) != LOOM_SELECT_OK) {
        c->status = LOOM_SELECT_EHISTORY;
        c->out_ids[row] = -1;
        c->out_prob[row] = NAN;
        if (c->out_logp) c->out_logp[row] = NAN;
        if (c->out_topk)
            for (int32_t j = 0; j < c->k; ++j) c->out_topk[row * c->k + j] = -1;
        free(x);
        return;
    }
    const int greedy = (c->T == 0.0f);
    if (!greedy)
        for (int64_t i = 0; i < V; ++i) x[i] = x[i] / c->T; /* y = x / T, fp32 divide */
    cand* heap = (cand*)malloc(sizeof(cand) * (size_t)c->k);
    int n = 0;
    for (int64_t i = 0; i < V; ++i) n = topk_offer(heap, n, c->k, x[i], (int32_t)i);
    qsort(heap, (size_t)n, sizeof(cand), cand_desc);
    int32_t id;
    float prob;
    if (greedy) {
        /* the argmax rule: a NaN at id 0 wins, otherwise the best key (lowest id among maxima) */
        id = (x[0] != x[0]) ? 0 : heap[0].id;
        prob = 1.0f;
    } else {
        decide(heap, n, c->p, c->u[row], &id, &prob);
    }
    c->out_ids[row] = id;
    c->out_prob[row] = prob;
    if (c->out_topk)
        for (int32_t j = 0; j < c->k; ++j) c->out_topk[row * c->k + j] = heap[j].id;
    if (c->out_logp) {
        double m, s;
        lse_partial(x, V, &m, &s);
        c->out_logp[row] = (float)((double)x[id] - (m + log(s)));
    }
    free(heap);
    free(x);
}

static int check_params(int64_t vocab, float T, float r, int32_t k, float p) {
    if (!(T >= 0.0f) || isinf(T)) return LOOM_SELECT_EPARAM;
    if (!(r > 0.0f) || isinf(r)) return LOOM_SELECT_EPARAM;
    if (k < 1 || k > LOOM_SELECT_MAX_TOP_K || k > vocab) return LOOM_SELECT_EPARAM;
    if (!(p > 0.0f && p <= 1.0f)) return LOOM_SELECT_EPARAM;
    return LOOM_SELECT_OK;
}

int oracle_sample_rows(const void* logits, int dtype, int64_t rows, int64_t n_vocab, int64_t row_stride,
                       const int32_t* history, int32_t history_len, const float* u, float temperature,
                       float repetition_penalty, int32_t top_k, float top_p, int32_t* out_ids,
                       float* out_prob, float* out_logp, int32_t* out_topk_ids, int nthreads) {
    if (dtype != LOOM_SELECT_F32 && dtype != LOOM_SELECT_BF16) return LOOM_SELECT_EDTYPE;
    if (!logits || !u || !out_ids || !out_prob || rows <= 0 || n_vocab <= 0 || row_stride < n_vocab ||
        history_len < 0 || (history_len > 0 && !history))
        return LOOM_SELECT_EINVAL;
    int st = check_params(n_vocab, temperature, repetition_penalty, top_k, top_p);
    if (st) return st;
    sample_ctx c = {logits, dtype, n_vocab, row_stride, history, history_len, u, temperature, repetition_penalty,
                    top_p, top_k, out_ids, out_topk_ids, out_prob, out_logp, LOOM_SELECT_OK};
    parallel_rows(sample_row_fn, &c, rows, nthreads);
    return c.status;
}

/* ------------------------------------------------------------------------------------------------ */
/* vocabulary shards                                                                                */

size_t oracle_shard_record_bytes(int32_t top_k) { return 16 + 8 * (size_t)top_k; }

typedef struct {
    int32_t count;
    float m, s;
    int32_t reserved;
} shard_head;

typedef struct {
    const void* logits;
    int dtype;
    int64_t shard_vocab, row_stride, vocab_offset, vocab_total;
    const int32_t* history;
    int32_t history_len;
    float T, r;
    int32_t k;
    unsigned char* out;
    int status;
} shard_ctx;

static void shard_row_fn(void* vctx, int64_t row) {
    shard_ctx* c = (shard_ctx*)vctx;
    const int64_t Vs = c->shard_vocab;
    float* x = (float*)malloc(sizeof(float) * (size_t)Vs);
    for (int64_t i = 0; i < Vs; ++i) x[i] = load_elem(c->logits, c->dtype, row * c->row_stride + i);
    const int32_t* hist = c->history ? c->history + row * (int64_t)c->history_len : NULL;
    unsigned char* rec = c->out + (size_t)row * oracle_shard_record_bytes(c->k);
    shard_head* head = (shard_head*)rec;
    if (apply_penalty(x, Vs, c->vocab_offset, c->vocab_total, hist, c->history_len, c->r) != LOOM_SELECT_OK) {
        c->status = LOOM_SELECT_EHISTORY;
        head->count = -1;
        head->m = NAN;
        head->s = NAN;
        head->reserved = 0;
        free(x);
        return;
    }
    for (int64_t i = 0; i < Vs; ++i) x[i] = x[i] / c->T;
    const int k = (int)(c->k < Vs ? c->k : Vs);
    if (k <= 0) {
        free(x);
        return;
    }
    cand* heap = (cand*)malloc(sizeof(cand) * (size_t)k);
    int n = 0;
    for (int64_t i = 0; i < Vs; ++i) n = topk_offer(heap, n, k, x[i], (int32_t)(c->vocab_offset + i));
    qsort(heap, (size_t)n, sizeof(cand), cand_desc);
    double m, s;
    lse_partial(x, Vs, &m, &s);
    head->count = n;
    head->m = (float)m;
    head->s = (float)s;
    head->reserved = 0;
    float* pairs = (float*)(rec + 16);
    for (int j = 0; j < n; ++j) {
        pairs[2 * j] = heap[j].y;
        memcpy(&pairs[2 * j + 1], &heap[j].id, sizeof(int32_t));
    }
    free(heap);
    free(x);
}

int oracle_shard_partial(const void* logits, int dtype, int64_t rows, int64_t shard_vocab, int64_t row_stride,
                         int64_t vocab_offset, int64_t vocab_total, const int32_t* history,
                         int32_t history_len, float temperature, float repetition_penalty, int32_t top_k,
                         void* out_records, int nthreads) {
    if (dtype != LOOM_SELECT_F32 && dtype != LOOM_SELECT_BF16) return LOOM_SELECT_EDTYPE;
    if (!logits || !out_records || rows <= 0 || shard_vocab <= 0 || row_stride < shard_vocab ||
        vocab_offset < 0 || vocab_offset + shard_vocab > vocab_total || history_len < 0 ||
        (history_len > 0 && !history))
        return LOOM_SELECT_EINVAL;
    int st = check_params(vocab_total, temperature, repetition_penalty, top_k, 1.0f);
    if (st) return st;
    if (temperature == 0.0f) return LOOM_SELECT_EPARAM;
    shard_ctx c = {logits, dtype, shard_vocab, row_stride, vocab_offset, vocab_total, history, history_len,
                   temperature, repetition_penalty, top_k, (unsigned char*)out_records, LOOM_SELECT_OK};
    parallel_rows(shard_row_fn, &c, rows, nthreads);
    return c.status;
}

int oracle_shard_merge(const void* records, int32_t n_shards, int64_t rows, const float* u, float temperature,
                       int32_t top_k, float top_p, int32_t* out_ids, float* out_prob, float* out_logp,
                       int32_t* out_topk_ids) {
    (void)temperature;
    if (!records || n_shards <= 0 || rows <= 0 || !u || !out_ids || !out_prob) return LOOM_SELECT_EINVAL;
    if (top_k < 1 || top_k > LOOM_SELECT_MAX_TOP_K || !(top_p > 0.0f && top_p <= 1.0f)) return LOOM_SELECT_EPARAM;
    const size_t rb = oracle_shard_record_bytes(top_k);
    cand* heap = (cand*)malloc(sizeof(cand) * (size_t)top_k);
    int status = LOOM_SELECT_OK;
    for (int64_t row = 0; row < rows; ++row) {
        int n = 0, bad = 0;
        double M = -INFINITY;
        for (int32_t g = 0; g < n_shards; ++g) {
            const shard_head* h = (const shard_head*)((const unsigned char*)records + ((size_t)g * rows + row) * rb);
            if (h->count < 0) bad = 1;
            else if (h->m > M) M = h->m;
        }
        if (bad) {
            status = LOOM_SELECT_EHISTORY;
            out_ids[row] = -1;
            out_prob[row] = NAN;
            if (out_logp) out_logp[row] = NAN;
            if (out_topk_ids)
                for (int32_t j = 0; j < top_k; ++j) out_topk_ids[row * top_k + j] = -1;
            continue;
        }
        double S = 0.0;
        for (int32_t g = 0; g < n_shards; ++g) {
            const unsigned char* rec = (const unsigned char*)records + ((size_t)g * rows + row) * rb;
            const shard_head* h = (const shard_head*)rec;
            if (h->s > 0.0f) S += (double)h->s * ((double)h->m == M ? 1.0 : exp((double)h->m - M));
            const float* pairs = (const float*)(rec + 16);
            for (int32_t j = 0; j < h->count; ++j) {
                int32_t id;
                memcpy(&id, &pairs[2 * j + 1], sizeof id);
                n = topk_offer(heap, n, top_k, pairs[2 * j], id);
            }
        }
        qsort(heap, (size_t)n, sizeof(cand), cand_desc);
        int32_t id;
        float prob;
        decide(heap, n, top_p, u[row], &id, &prob);
        out_ids[row] = id;
        out_prob[row] = prob;
        if (out_topk_ids)
            for (int32_t j = 0; j < top_k; ++j) out_topk_ids[row * top_k + j] = j < n ? heap[j].id : -1;
        if (out_logp) {
            float ysel = 0.0f;
            for (int j = 0; j < n; ++j)
                if (heap[j].id == id) ysel = heap[j].y;
            out_logp[row] = (float)((double)ysel - (M + log(S)));
        }
    }
    free(heap);
    return status;
}

/* ---- check of the kernels' division by T (test infrastructure) ----
 * The log-sum-exp of the sampling kernels divides each logit by T without a divide instruction, by
 * Markstein's method: with inv = fl(1 / T), q0 = fl(x * inv), r = x - T * q0 (exact, one FMA) and
 * q = fl(q0 + r * inv) (one FMA). This counts, for every float mantissa of x in [1, 2) and each given
 * T, the x where q differs from the IEEE quotient x / T. The rounding of x / T depends on the
 * mantissas only (away from overflow and subnormals), so [1, 2) covers every x. */
static float div_markstein(float x, float T, float inv) {
    const float q0 = x * inv;
    const float r = fmaf(-q0, T, x);
    return fmaf(r, inv, q0);
}

typedef struct {
    const float* T;
    int64_t nT, t0, t1;
    int64_t bad;
    float bad_x, bad_T;
} div_job;

static void* div_worker(void* arg) {
    div_job* j = (div_job*)arg;
    for (int64_t t = j->t0; t < j->t1; ++t) {
        const float T = j->T[t];
        const float inv = 1.0f / T;
        for (uint32_t m = 0; m < (1u << 23); ++m) {
            uint32_t bits = 0x3f800000u | m;
            float x;
            memcpy(&x, &bits, sizeof x);
            const float want = x / T;
            const float got = div_markstein(x, T, inv);
            if (memcmp(&want, &got, sizeof want) != 0) {
                if (j->bad == 0) {
                    j->bad_x = x;
                    j->bad_T = T;
                }
                ++j->bad;
            }
        }
    }
    return NULL;
}

int64_t oracle_div_check(const float* T, int64_t nT, int nthreads, float* bad_x, float* bad_T) {
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 64) nthreads = 64;
    pthread_t th[64];
    div_job jobs[64];
    for (int i = 0; i < nthreads; ++i) {
        jobs[i].T = T;
        jobs[i].nT = nT;
        jobs[i].t0 = nT * i / nthreads;
        jobs[i].t1 = nT * (i + 1) / nthreads;
        jobs[i].bad = 0;
        pthread_create(&th[i], NULL, div_worker, &jobs[i]);
    }
    int64_t bad = 0;
    for (int i = 0; i < nthreads; ++i) {
        pthread_join(th[i], NULL);
        if (jobs[i].bad && !bad) {
            *bad_x = jobs[i].bad_x;
            *bad_T = jobs[i].bad_T;
        }
        bad += jobs[i].bad;
    }
    return bad;
}
