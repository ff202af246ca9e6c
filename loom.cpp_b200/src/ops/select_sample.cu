// select_sample.cu -- the fused sampling chain (K2) and the vocabulary-shard merge (K4).
//
// One pass over the logits: rows stream through shared memory, and every element below a threshold
// X is dropped with one compare (X is at most the smallest raw value whose tempered value x / T
// reaches a lower bound of the row's k-th best, so no element of the top-k is ever below it). The few
// elements that reach X become candidates; at the end of a row segment the exact top-k of the
// candidates is ranked into order and the survivor decision runs in double precision on one warp
// (select_topk.cuh), in exactly the oracle's operation order.
//
// Two kernels share the row-segment bookkeeping (records and tickets of split rows, the decision):
//   sample_stream_kernel (top_k <= kWarpMaxK): free-running consumer warps with private candidate
//     buffers, a threshold raised from a sorted list of stage maxima; described at WarpSampleOp.
//   sample_wide_kernel (larger top_k): lockstep stages; each thread marks, in a register bitmask,
//     the vectors of the stage whose maximum reaches X, moves their passing elements into its own
//     slots, and the CTA prunes the candidates to the exact top-k (raising X) when more than
//     k + max(kPruneSlack, k) are held. The first stage of a segment seeds X: each warp sorts its lanes'
//     maxima, and the smallest of the warps' ceil(k / warps)-th largest is reached by k elements.
//
// The repetition penalty touches only the history ids: at the start of a row segment the distinct
// ones inside it go into a shared-memory hash set and a list, and the stream skips set members
// (looked up only for elements that pass X); their penalised values enter separately.
// Bound: HBM bandwidth (4 bytes per f32 logit, 2 per bf16, read once).
#include <atomic>

#include "select_internal.h"
#include "select_rows.cuh"
#include "select_stream.cuh"
#include "select_topk.cuh"

namespace loom_select {

namespace {

constexpr int kSampWarps = 8;
constexpr int kSampNT = kSampWarps * 32;
constexpr int kSampCtasPerSm = kSampleCtasPerSm;  // two independent CTAs per SM overlap their latency-bound phases
constexpr int kSampStages = 2;
constexpr int kSampStageBytes = 32768;
constexpr int kSlots = 4;           // raw candidates a thread holds between prunes
constexpr int kCandCap = 2176;      // candidate rank keys in shared memory
constexpr int kPruneSlack = 64;     // prune at a stage end when more than k + max(this, k) are held
constexpr int kHashSlots = 2048;    // history hash set (load <= 1/2 at kMaxHistory ids)
constexpr int kDecideSlots = 1024;
constexpr uint32_t kPenalisedFlag = 0x80000000u;  // a raw slot holding a history id's raw value
static_assert(kCandCap >= LOOM_SELECT_MAX_TOP_K + kPruneSlack + kSampNT * kSlots, "a prune's keys must fit");
static_assert(LOOM_SELECT_MAX_TOP_K <= kDecideSlots && 2 * kDecideSlots <= kCandCap,
              "decision scratch e[] lives in key slots [1024, 2048)");
static_assert(2 * kMaxHistory <= kHashSlots, "hash set load");
static_assert(kHashSlots == 2048, "hash_slot takes 11 bits");

struct SampleDev {
    float T, r, p;
    int32_t k;
    bool greedy, penalty, lse, shard;
    int64_t vocab_offset, vocab_limit;
    const int32_t* hist;
    int32_t hist_len;
    const float* u;
    int32_t* out_ids;
    float* out_prob;
    float* out_logp;
    int32_t* out_topk;
    unsigned char* shard_out; // [rows] records of loom_shard_record_bytes(k) (pairs)
    unsigned char* recs;      // workspace records [2 * ctas] (keys), see record_slot
    size_t rec_bytes;         // 16 + 8k
    int* tickets;             // [2 * ctas]: a split row's ticket is its first piece's record slot
    int* status;
};

struct RecordHead {
    int32_t count; // -1: the row has a bad history id
    float m;
    float s;
    int32_t reserved;
};

struct SampleShared {
    TopkShared tk;
    int K;         // rank keys held in cand[0, K)
    int fail;      // a thread's slots filled up mid-stage
    int bad;
    int n_uniq;
    uint32_t warm_key;
    float X;
    float thr_y;
    int last;
    int wcnt[kSampWarps];
    LseAcc lse_w[kSampWarps];
    LseAcc seg_lse;
    int nan_tot[kSampWarps];
    int nan_have;
    int32_t sel_id;
    float sel_prob;
    float sel_y;
    unsigned long long key_t;  // warp path: every kept key reaches this (a k-th best key, or a value floor)
    uint32_t x_key;            // warp path: order key of the raw threshold X
    float wq[kSampWarps];      // warp path: per warp, a raw value that ceil(k / warps) of its lanes' maxima reach
    float u_row;               // the segment's row's uniform (loaded when the segment starts)
    int mcnt[32];              // split-row merge: the batch's piece counts (-1: a bad history id)
    LseAcc mpart[32];          // and their log-sum-exp states
};

__device__ __forceinline__ float neg_inf() { return -__int_as_float(0x7f800000); }

__device__ __forceinline__ float penalise(float x, float r) { return x > 0.0f ? __fdiv_rn(x, r) : __fmul_rn(x, r); }

// Descending bitonic sort of one float per lane across the warp.
__device__ __forceinline__ float warp_sort_desc(float v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int size = 2; size <= 32; size <<= 1) {
#pragma unroll
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            const float o = __shfl_xor_sync(0xffffffffu, v, stride);
            const bool lower = (lane & stride) == 0;
            const bool desc = (lane & size) == 0;
            v = (lower == desc) ? fmaxf(v, o) : fminf(v, o);
        }
    }
    return v;
}

template <int kDtype>
__device__ __forceinline__ float smem_elem(const unsigned char* data, int32_t i) {
    if constexpr (kDtype == LOOM_SELECT_BF16) {
        return bf16_bits_to_float(reinterpret_cast<const unsigned short*>(data)[i]);
    } else {
        return reinterpret_cast<const float*>(data)[i];
    }
}

// History hash set: open addressing over global ids, -1 = empty.
__device__ __forceinline__ uint32_t hash_slot(int32_t id) {
    return (static_cast<uint32_t>(id) * 2654435761u) >> (32 - 11);  // 2048 slots
}

__device__ __forceinline__ bool hash_contains(const int32_t* set, int32_t id) {
    uint32_t h = hash_slot(id);
    for (int probe = 0; probe < kHashSlots; ++probe) {
        const int32_t v = set[h];
        if (v == id) return true;
        if (v < 0) return false;
        h = (h + 1) & (kHashSlots - 1);
    }
    return false;
}

// Inserts id; true if it was not there yet.
__device__ __forceinline__ bool hash_insert(int32_t* set, int32_t id) {
    uint32_t h = hash_slot(id);
    for (int probe = 0; probe < kHashSlots; ++probe) {
        const int32_t old = atomicCAS(&set[h], -1, id);
        if (old == -1) return true;
        if (old == id) return false;
        h = (h + 1) & (kHashSlots - 1);
    }
    return false;
}

// Tempers every thread's raw candidates into rank keys after the held ones, keeps the exact top-k,
// sorted, in cand[0, K), raises the threshold to the k-th, and empties the slots. A raw slot with
// kPenalisedFlag is a history id's raw value (penalised here); a raw slot without it that is a
// history id is the stream's copy of that id and is dropped. Every consumer thread calls it with its
// own slot count `qn` (returned as 0); hset is the segment's history set (unused without penalty).
template <int kNT>
__device__ void prune(const SampleDev p, uint64_t* cand, const uint2* slots, const int32_t* hset, int& qn,
                      SampleShared* sh) {
    const int tid = threadIdx.x, lane = tid & 31;
    uint64_t kk[kSlots];
    int nk = 0;
#pragma unroll
    for (int j = 0; j < kSlots; ++j) {
        kk[j] = 0ull;
        if (j < qn) {
            const uint2 e = slots[j * kNT + tid];
            const int32_t id = static_cast<int32_t>(e.y & ~kPenalisedFlag);
            float x = __uint_as_float(e.x);
            bool keep = true;
            if (e.y & kPenalisedFlag) x = penalise(x, p.r);
            else if (p.penalty && hash_contains(hset, id)) keep = false;
            if (keep) {
                const float y = tempered(x, p.T, p.greedy);
                if (y == y) kk[nk++] = loom_rank_key(y, id);  // (NaN never reaches a slot)
            }
        }
    }
    int excl = nk;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const int o = __shfl_up_sync(0xffffffffu, excl, off);
        if (lane >= off) excl += o;
    }
    const int wsum = __shfl_sync(0xffffffffu, excl, 31);
    excl -= nk;
    int base = 0;
    if (lane == 0) base = atomicAdd(&sh->K, wsum);
    base = __shfl_sync(0xffffffffu, base, 0);
#pragma unroll
    for (int j = 0; j < kSlots; ++j)
        if (j < nk) cand[base + excl + j] = kk[j];
    qn = 0;
    group_sync<kNT>();
    const int n = sh->K;
    const int K = topk_select_sorted<kNT, kCandCap>(cand, n, p.k, &sh->tk);
    if (tid == 0) {
        sh->K = K;
        sh->fail = 0;
        if (K == p.k) {
            const float t = rank_key_value(cand[K - 1]);
            if (t > sh->thr_y) {
                sh->thr_y = t;
                sh->X = inverse_threshold_bound(t, p.T, p.greedy);
            }
        }
    }
    group_sync<kNT>();
}

// The K (<= k) best keys of a whole row, sorted: fill up to k with NaN ids when the row has fewer
// than k non-NaN values, then emit the row's result (a decision, or a shard record).
template <int kDtype, int kNT>
__device__ void finalize_row(const SampleDev p, const StreamGeom g, int64_t row, uint64_t* cand, double* e, double* S,
                             int K, LseAcc lse, bool bad, SampleShared* sh) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int kEsz = (kDtype == LOOM_SELECT_BF16) ? 2 : 4;
    const unsigned char* rowp = g.base + row * g.row_stride * kEsz;
    if (bad) {
        if (p.shard) {
            if (tid == 0) {
                RecordHead* h = reinterpret_cast<RecordHead*>(p.shard_out + row * p.rec_bytes);
                h->count = -1;
                h->m = __int_as_float(0x7fc00000);
                h->s = __int_as_float(0x7fc00000);
                h->reserved = 0;
            }
        } else {
            if (tid == 0) {
                p.out_ids[row] = -1;
                p.out_prob[row] = __int_as_float(0x7fc00000);
                if (p.out_logp) p.out_logp[row] = __int_as_float(0x7fc00000);
            }
            if (p.out_topk)
                for (int j = tid; j < p.k; j += kNT) p.out_topk[row * p.k + j] = -1;
        }
        group_sync<kNT>();
        return;
    }
    const int kk = static_cast<int>(p.k < g.width ? p.k : g.width); // a shard may be narrower than k
    if (K < kk) {
        // NaN fill in column order: NaN ranks below everything, lower id first (after the sorted K)
        if (tid == 0) sh->nan_have = K;
        group_sync<kNT>();
        for (int64_t base = 0; base < g.width; base += kNT) {
            const int have = sh->nan_have;
            if (have >= kk) break;
            const int64_t col = base + tid;
            bool isn = false;
            if (col < g.width) {
                const float x = load_global_elem<kDtype>(rowp, col);
                isn = x != x;
            }
            const uint32_t ballot = __ballot_sync(0xffffffffu, isn);
            if (lane == 0) sh->nan_tot[warp] = __popc(ballot);
            group_sync<kNT>();
            int before = 0, total = 0;
            for (int w = 0; w < kSampWarps; ++w) {
                if (w < warp) before += sh->nan_tot[w];
                total += sh->nan_tot[w];
            }
            if (isn) {
                const int pos = have + before + __popc(ballot & ((1u << lane) - 1u));
                if (pos < kk) cand[pos] = loom_rank_key(__int_as_float(0x7fc00000), static_cast<int32_t>(p.vocab_offset + col));
            }
            group_sync<kNT>();
            if (tid == 0) sh->nan_have = have + total;
            group_sync<kNT>();
        }
        K = kk;
    }
    if (p.shard) {
        unsigned char* rec = p.shard_out + row * p.rec_bytes;
        if (tid == 0) {
            RecordHead* h = reinterpret_cast<RecordHead*>(rec);
            h->count = K;
            h->m = lse.m;
            h->s = lse.s;
            h->reserved = 0;
        }
        uint2* pairs = reinterpret_cast<uint2*>(rec + 16);
        for (int j = tid; j < K; j += kNT) {
            const uint64_t key = cand[j];
            pairs[j] = make_uint2(__float_as_uint(rank_key_value(key)), static_cast<uint32_t>(rank_key_id(key)));
        }
        group_sync<kNT>();
        return;
    }
    if (warp == 0) {
        if (p.greedy) {
            if (lane == 0) {
                const float x0 = load_global_elem<kDtype>(rowp, 0);
                if (x0 != x0) {
                    sh->sel_id = static_cast<int32_t>(p.vocab_offset);
                    sh->sel_y = x0;
                } else {
                    sh->sel_id = rank_key_id(cand[0]);
                    sh->sel_y = rank_key_value(cand[0]);
                }
                sh->sel_prob = 1.0f;
            }
        } else {
            decide_warp(cand, K, p.p, sh->u_row, e, S, &sh->sel_id, &sh->sel_prob, &sh->sel_y);
        }
        if (lane == 0) {
            p.out_ids[row] = sh->sel_id;
            p.out_prob[row] = sh->sel_prob;
            if (p.out_logp) {
                const double lp = static_cast<double>(sh->sel_y) -
                                  (static_cast<double>(lse.m) + log(static_cast<double>(lse.s)));
                p.out_logp[row] = static_cast<float>(lp);
            }
        }
    }
    if (p.out_topk)
        for (int j = tid; j < p.k; j += kNT) p.out_topk[row * p.k + j] = rank_key_id(cand[j]);
    group_sync<kNT>();
}

template <int kNT, int kCap, bool kSmallK>
__device__ __forceinline__ int select_best(uint64_t* cand, int n, int k, TopkShared* sh) {
    if constexpr (kSmallK) return topk_select_sorted_small_k<kNT, kCap>(cand, n, k, sh);
    else return topk_select_sorted<kNT, kCap>(cand, n, k, sh);
}

// The end of a row segment, once its K best keys are sorted in cand[0, K): a whole row is finalised
// here; a piece of a split row writes its record and takes the row's ticket, and the CTA that takes
// the last ticket merges every piece's record and finalises the row. cand holds kCap keys.
template <int kDtype, int kNT, int kCap, bool kSmallK>
__device__ void finish_segment(const SampleDev p, const StreamGeom g, const Segment& s, uint64_t* cand, double* e,
                               double* S, int K, LseAcc seg, bool bad, SampleShared* sh) {
    const int tid = threadIdx.x;
    if (s.count == 1) {
        finalize_row<kDtype, kNT>(p, g, s.row, cand, e, S, K, seg, bad, sh);
        return;
    }
    // a piece of a split row: write its record, take a ticket, the last one merges
    unsigned char* rec = p.recs + static_cast<size_t>(record_slot(g, s.first_cta + s.index, s.row)) * p.rec_bytes;
    uint64_t* keys = reinterpret_cast<uint64_t*>(rec + 16);
    for (int j = tid; j < K; j += kNT) keys[j] = cand[j];
    if (tid == 0) {
        RecordHead* h = reinterpret_cast<RecordHead*>(rec);
        h->count = bad ? -1 : K;
        h->m = seg.m;
        h->s = seg.s;
        h->reserved = 0;
    }
    __threadfence();
    group_sync<kNT>();
    if (tid == 0) {
        const int prev = atomicAdd(&p.tickets[record_slot(g, s.first_cta, s.row)], 1);
        sh->last = prev == s.count - 1;
    }
    group_sync<kNT>();
    if (!sh->last) return;
    __threadfence();
    // merge every piece's record, in batches of up to 32 pieces whose loads are in flight together:
    // piece b's k key slots go to cand[have + b k, have + (b + 1) k), those past its count as a
    // filler key (piece index * k + slot + 1: below 2^32, so below every real key, and distinct, as
    // the selection needs); the number of real keys bounds the result
    const int fit = (kCap - p.k) / p.k;
    const int per_batch = fit < 1 ? 1 : (fit > 32 ? 32 : fit);
    int have = 0, real = 0;
    bool any_bad = false;
    LseAcc tot = lse_init();
    for (int j0 = 0; j0 < s.count; j0 += per_batch) {
        const int nb = s.count - j0 < per_batch ? s.count - j0 : per_batch;
        if (have + nb * p.k > kCap) have = select_best<kNT, kCap, kSmallK>(cand, have, p.k, &sh->tk);
        for (int idx = tid; idx < nb * p.k; idx += kNT) {
            const int bb = idx / p.k, i = idx - bb * p.k;
            const unsigned char* r =
                p.recs + static_cast<size_t>(record_slot(g, s.first_cta + j0 + bb, s.row)) * p.rec_bytes;
            const int32_t c = __ldcg(reinterpret_cast<const int32_t*>(r));
            const uint64_t key = __ldcg(reinterpret_cast<const uint64_t*>(r + 16) + i);
            cand[have + idx] = i < c ? key : static_cast<uint64_t>(j0) * p.k + idx + 1;
        }
        if (tid < nb) {
            const unsigned char* r =
                p.recs + static_cast<size_t>(record_slot(g, s.first_cta + j0 + tid, s.row)) * p.rec_bytes;
            sh->mcnt[tid] = __ldcg(reinterpret_cast<const int32_t*>(r));
            sh->mpart[tid].m = __ldcg(reinterpret_cast<const float*>(r) + 1);
            sh->mpart[tid].s = __ldcg(reinterpret_cast<const float*>(r) + 2);
        }
        group_sync<kNT>();
        for (int bb = 0; bb < nb; ++bb) {  // every thread, in the same order: the same results
            const int c = sh->mcnt[bb];
            if (c < 0) {
                any_bad = true;
            } else {
                tot = lse_merge(tot, sh->mpart[bb]);
                real += c;
            }
        }
        have += nb * p.k;
        group_sync<kNT>();  // mcnt / mpart are rewritten by the next batch
    }
    int Kf = select_best<kNT, kCap, kSmallK>(cand, have, p.k, &sh->tk);
    if (Kf > real) Kf = real;
    if (tid == 0) p.tickets[record_slot(g, s.first_cta, s.row)] = 0;
    finalize_row<kDtype, kNT>(p, g, s.row, cand, e, S, Kf, tot, any_bad, sh);
}

template <int kDtype>
struct WideSampleOp {
    static constexpr int kEsz = (kDtype == LOOM_SELECT_BF16) ? 2 : 4;
    static constexpr int kPer = 16 / kEsz;
    static constexpr int kNT = kSampNT;
    StreamGeom g;  // copies: no pointer into the kernel's parameters
    SampleDev p;
    SampleShared* sh;
    uint64_t* cand;
    uint2* slots;   // [kSlots][kNT]: thread t's raw candidates (value bits, global id) at [j][t]
    int32_t* hset;  // history hash set of the segment
    int32_t* uniq;  // its distinct ids, as a list
    double* S;      // decision scratch
    LseAcc lse;
    int qn;         // this thread's raw candidates
    bool first_chunk;

    __device__ const unsigned char* row_ptr(int64_t row) const { return g.base + row * g.row_stride * kEsz; }
    __device__ const int32_t* row_hist(int64_t row) const { return p.hist + row * static_cast<int64_t>(p.hist_len); }

    __device__ __forceinline__ bool is_history(int64_t gid) const {
        return p.penalty && hash_contains(hset, static_cast<int32_t>(gid));
    }

    __device__ void begin_segment(const Segment& s) {
        const int tid = threadIdx.x;
        if (tid == 0) {
            sh->K = 0;
            if (p.u && !p.shard && !p.greedy) sh->u_row = __ldg(p.u + s.row);  // used at the row's end
            sh->fail = 0;
            sh->bad = 0;
            sh->n_uniq = 0;
            sh->X = neg_inf();
            sh->thr_y = neg_inf();
            sh->warm_key = 0xffffffffu;
        }
        lse = lse_init();
        qn = 0;
        first_chunk = true;
        if (p.penalty) {
            int4* h4 = reinterpret_cast<int4*>(hset);
            for (int i = tid; i < kHashSlots / 4; i += kNT) h4[i] = make_int4(-1, -1, -1, -1);
        }
        group_sync<kNT>();
        // validate the whole history; the distinct ids inside this segment go into the set and list
        const int64_t seg_lo = p.vocab_offset + s.j0, seg_hi = p.vocab_offset + s.j1;
        for (int j = tid; j < p.hist_len; j += kNT) {
            const int32_t id = __ldg(row_hist(s.row) + j);
            if (id < 0 || id >= p.vocab_limit) sh->bad = 1;
            else if (p.penalty && id >= seg_lo && id < seg_hi && hash_insert(hset, id))
                uniq[atomicAdd(&sh->n_uniq, 1)] = id;
        }
        group_sync<kNT>();
        // edges: the few elements outside the 16-byte-aligned interior, read from global memory
        const int32_t n_edges = segment_edge_count(s, kEsz);
        if (tid < n_edges) {
            const int64_t col = segment_edge_col(s, kEsz, tid);
            float x = load_global_elem<kDtype>(row_ptr(s.row), col);
            const int32_t gid = static_cast<int32_t>(p.vocab_offset + col);
            if (is_history(gid)) x = penalise(x, p.r);
            const float y = tempered(x, p.T, p.greedy);
            if (p.lse) lse_offer(lse, y);
            if (y == y) cand[atomicAdd(&sh->K, 1)] = loom_rank_key(y, gid);
        }
        group_sync<kNT>();
        if (tid == 0 && sh->bad) record_status(p.status, LOOM_SELECT_EHISTORY);
    }

    __device__ void chunk(const Segment& s, const unsigned char* data, int64_t col0, int32_t n) {
        const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
        const int32_t nvec = n / kPer;
        const uint4* v4 = reinterpret_cast<const uint4*>(data);
        const int64_t gid0 = p.vocab_offset + col0;

        // 1. the history ids this stage holds: pending flagged raw entries, swept with the marks
        //    (entry m of this thread's share of the list is bit m)
        constexpr int kUniqPerThread = (kMaxHistory + kNT - 1) / kNT;
        static_assert(kUniqPerThread <= 32, "pending history entries are one 32-bit word");
        uint32_t pend = 0;
        if (p.penalty) {
            const int nu = sh->n_uniq;
#pragma unroll
            for (int m = 0; m < kUniqPerThread; ++m) {
                const int j = m * kNT + tid;
                if (j < nu) {
                    const int64_t c = static_cast<int64_t>(uniq[j]) - gid0;
                    if (c >= 0 && c < n) {
                        pend |= 1u << m;
                        if (p.lse)
                            lse_offer(lse, tempered(penalise(smem_elem<kDtype>(data, static_cast<int32_t>(c)), p.r),
                                                    p.T, p.greedy));
                    }
                }
            }
        }

        // 2. seed the threshold from the segment's first stage
        if (first_chunk) {
            first_chunk = false;
            float m = neg_inf();
            int64_t at = -1;
            for (int32_t v = tid; v < nvec; v += kNT) {
                Vec16<kDtype> e;
                e.unpack(v4[v]);
#pragma unroll
                for (int q = 0; q < kPer; ++q)
                    if (e.x[q] > m) {
                        m = e.x[q];
                        at = gid0 + static_cast<int64_t>(v) * kPer + q;
                    }
            }
            // a lane whose maximum is a history id vouches for nothing
            if (at >= 0 && is_history(at)) m = neg_inf();
            const float sorted = warp_sort_desc(m);
            const int q = (p.k + kSampWarps - 1) / kSampWarps;
            const float bw = q <= 32 ? __shfl_sync(0xffffffffu, sorted, q - 1) : neg_inf();
            if (lane == 0) atomicMin(&sh->warm_key, loom_order_key(bw));
            group_sync<kNT>();
            if (tid == 0) {
                const float tx = order_key_to_float(sh->warm_key);
                const float ty = tempered(tx, p.T, p.greedy);
                if (ty > sh->thr_y) {
                    sh->thr_y = ty;
                    sh->X = inverse_threshold_bound(ty, p.T, p.greedy);
                }
            }
            group_sync<kNT>();
        }

        // 3. mark: the vectors whose maximum reaches X (all loads in flight at once, no branches)
        constexpr int kVecsPerThread = kSampStageBytes / 16 / kNT;
        static_assert(kVecsPerThread <= 32, "marks are one 32-bit word");
        uint32_t hits = 0;
        {
            const float X = sh->X;
#pragma unroll
            for (int i = 0; i < kVecsPerThread; ++i) {
                const int32_t v = i * kNT + tid;
                if (v < nvec) {
                    Vec16<kDtype> e;
                    e.unpack(v4[v]);
                    float mu = e.x[0];
#pragma unroll
                    for (int q = 1; q < kPer; ++q) mu = fmaxf(mu, e.x[q]);
                    hits |= static_cast<uint32_t>(mu >= X) << i;
                    if (p.lse) {
                        // every element once (history ids are offered in step 1)
#pragma unroll
                        for (int q = 0; q < kPer; ++q)
                            if (!is_history(gid0 + static_cast<int64_t>(v) * kPer + q))
                                lse_offer(lse, tempered(e.x[q], p.T, p.greedy));
                    }
                }
            }
        }

        // 4. sweep: each thread moves its pending history entries, then the passing elements of its
        //    marked vectors, into its slots, element by element. A thread whose slots are full stops
        //    there (its marks, pending bits and element cursor stay) and goes on after the prune.
        // Every round but the last sweeps at least one element per stopped thread, so the bound is
        // never reached; it only guarantees that the loop ends.
        const int max_rounds = (kVecsPerThread * kPer + kUniqPerThread) / kSlots + 3;
        int qpos = 0;  // next element of the first marked vector
        for (int32_t round = 0;; ++round) {
            const float X = sh->X;  // rises at a prune
            bool stopped = false;
            while (pend) {
                if (qn == kSlots) {
                    stopped = true;
                    break;
                }
                const int m = __ffs(pend) - 1;
                const int32_t id = uniq[m * kNT + tid];
                const float x = smem_elem<kDtype>(data, static_cast<int32_t>(id - gid0));
                // with r >= 1 the penalty only lowers a value: one already below X cannot make the top-k
                if (x == x && !(p.r >= 1.0f && x < X))
                    slots[(qn++) * kNT + tid] = make_uint2(__float_as_uint(x), static_cast<uint32_t>(id) | kPenalisedFlag);
                pend &= pend - 1u;
            }
            while (hits && !stopped) {
                const int i = __ffs(hits) - 1;
                const int32_t e0 = (i * kNT + tid) * kPer;  // element index of the vector in the stage
                for (; qpos < kPer; ++qpos) {
                    const float x = smem_elem<kDtype>(data, e0 + qpos);
                    if (x >= X) {
                        if (qn == kSlots) {
                            stopped = true;
                            break;
                        }
                        slots[(qn++) * kNT + tid] = make_uint2(__float_as_uint(x), static_cast<uint32_t>(gid0 + e0 + qpos));
                    }
                }
                if (stopped) break;
                qpos = 0;
                hits &= hits - 1u;
            }
            if (stopped) sh->fail = 1;
            const int wsum = __reduce_add_sync(0xffffffffu, qn);
            if (lane == 0) sh->wcnt[warp] = wsum;
            group_sync<kNT>();
            const bool failed = sh->fail != 0;
            int held = sh->K;
            for (int w = 0; w < kSampWarps; ++w) held += sh->wcnt[w];
            // prune when the held keys exceed k by the slack (at least k: the prune sorts ~k keys)
            if (!failed && held <= p.k + (p.k > kPruneSlack ? p.k : kPruneSlack)) break;
            group_sync<kNT>();
            prune<kNT>(p, cand, slots, hset, qn, sh);
            if (!failed) break;
            if (round > max_rounds) {  // unreachable by construction (see above)
                if (tid == 0) record_status(p.status, LOOM_SELECT_ETIMEOUT);
                break;
            }
        }
    }

    __device__ void end_chunk(const Segment&) {}

    __device__ void end_segment(const Segment& s) {
        const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
        if (p.lse) {
            const LseAcc w = lse_warp_reduce(lse);
            if (lane == 0) sh->lse_w[warp] = w;
        }
        group_sync<kNT>();
        if (tid == 0) {
            LseAcc a = lse_init();
            if (p.lse)
                for (int w = 0; w < kSampWarps; ++w) a = lse_merge(a, sh->lse_w[w]);
            sh->seg_lse = a;
        }
        prune<kNT>(p, cand, slots, hset, qn, sh);  // also syncs
        finish_segment<kDtype, kNT, kCandCap, false>(p, g, s, cand, reinterpret_cast<double*>(cand + kDecideSlots), S, sh->K,
                                             sh->seg_lse, sh->bad != 0, sh);
    }
};

constexpr size_t kWideDynSmem = static_cast<size_t>(kSampStages) * kSampStageBytes + kCandCap * sizeof(uint64_t) +
                                kSlots * kSampNT * sizeof(uint2) + kHashSlots * sizeof(int32_t) +
                                kMaxHistory * sizeof(int32_t) + kDecideSlots * sizeof(double);
static_assert(kWideDynSmem + 4096 <= 232448 / kSampCtasPerSm, "two CTAs per SM must fit the SM's shared memory");

// Lockstep kernel for top_k above the warp path's limit.
template <int kDtype>
__global__ void __launch_bounds__((kSampWarps + 1) * 32, kSampCtasPerSm) sample_wide_kernel(StreamGeom g, SampleDev p) {
    extern __shared__ __align__(128) unsigned char dyn[];
    __shared__ StreamCtl ctl;
    __shared__ SampleShared sh;
    unsigned char* ring = dyn;
    uint64_t* cand = reinterpret_cast<uint64_t*>(dyn + static_cast<size_t>(kSampStages) * kSampStageBytes);
    uint2* slots = reinterpret_cast<uint2*>(cand + kCandCap);
    int32_t* hset = reinterpret_cast<int32_t*>(slots + kSlots * kSampNT);
    int32_t* uniq = hset + kHashSlots;
    double* S = reinterpret_cast<double*>(uniq + kMaxHistory);
    WideSampleOp<kDtype> op{g, p, &sh, cand, slots, hset, uniq, S, lse_init(), 0, true};
    stream_ranges<kSampStages, kSampStageBytes, kSampWarps>(g, op, ring, &ctl, p.status);
}

// ---------------------------------------------------------------------------------------------
// The warp path (top_k <= kWarpMaxK). Consumer warps run free of one another between segment
// boundaries (stream_ranges_warps): no CTA barrier per stage. Each warp appends the raw (value, id)
// pairs that reach the raw threshold X to a buffer of its own, one ballot per step. When the buffer
// is full the warp alone tempers it into rank keys, keeps its best k (a register bitonic sort) and
// raises the CTA's thresholds with shared-memory atomics: key_t, which every kept key reaches, and X,
// the raw bound derived from it. Both only rise, so a warp that reads them late keeps more than it
// needs, never less. What raises them in the common case costs one max per vector: each warp keeps,
// one per lane, a sorted list of the 32 largest "stage maxima" it has seen in the segment (the
// maximum of one lane's elements in one stage: distinct elements, taken at their true, penalised
// value when they are history ids); a lane whose stage maximum beats the list's ceil(k / warps)-th
// entry inserts it (a shuffle and a select). That entry, published now and then, is reached by
// ceil(k / warps) distinct elements of the warp, so the smallest value the warps have published is
// reached by at least k and bounds the k-th best from below. The stream skips history ids' raw values (a hash lookup, only for elements
// that pass X); at the segment end the CTA reads their logits again from global memory (the row has
// just gone through L2), penalises and tempers them, and offers them against the final threshold.
// A segment ends with every warp's best k merged by the whole CTA (exact selection, then the
// decision).

constexpr int kWarpStages = 2;                    // the warp path's ring
constexpr int kWarpStageBytes = 36864;  // 9 vectors per thread; two CTAs per SM leave no room for more
constexpr int kWarpMaxK = 128;                    // the warp path serves top_k up to this
constexpr int kRawCap = 128;                      // raw pairs a warp holds between its prunes
constexpr int kWarpKeyCap = kWarpMaxK + kRawCap;  // a warp's kept keys plus one tempered raw batch
constexpr int kWarpCand = kSampWarps * kRawCap;   // the segment-end gather (aliases the raw buffers)
static_assert(kSampWarps * kWarpMaxK <= kWarpCand, "the warps' best k keys fit the gather");
static_assert(kWarpMaxK <= kSampNT, "the warp path ranks at most one key per thread");
static_assert(kWarpKeyCap <= 256, "a warp sorts at most 8 keys per lane");
static_assert(2 * kWarpMaxK * sizeof(double) <= kSampWarps * kWarpKeyCap * sizeof(uint64_t),
              "decision scratch fits the key buffers");

__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float pos_inf() { return __int_as_float(0x7f800000); }

// (a0, a1) - (m, m), then * (c, c): two packed f32x2 operations, each element rounded as the
// scalar __fsub_rn / __fmul_rn would round it. mm and cc hold (m, m) and (c, c).
__device__ __forceinline__ void sub_mul_f32x2(float a0, float a1, uint64_t mm, uint64_t cc, float& d0, float& d1) {
    uint64_t a, d;
    asm("mov.b64 %0, {%1, %2};" : "=l"(a) : "f"(a0), "f"(a1));
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(mm));
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(d), "l"(cc));
    asm("mov.b64 {%0, %1}, %2;" : "=f"(d0), "=f"(d1) : "l"(d));
}

__device__ __forceinline__ uint64_t f32x2_splat(float v) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %1};" : "=l"(r) : "f"(v));
    return r;
}

constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ uint32_t lanemask_lt() {
    uint32_t m;
    asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
    return m;
}

// Descending bitonic sort of 32 * P keys held P per lane (element j * 32 + lane in a[j]).
template <int P>
__device__ __forceinline__ void warp_sort_keys_desc(uint64_t (&a)[P]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int size = 2; size <= 32 * P; size <<= 1) {
#pragma unroll
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            if (stride >= 32) {
                const int js = stride >> 5;
#pragma unroll
                for (int j = 0; j < P; ++j) {
                    if ((j & js) == 0) {
                        const int j2 = j | js;
                        const bool desc = ((j * 32) & size) == 0;
                        const uint64_t lo = a[j], hi = a[j2];
                        const bool swap = desc ? (lo < hi) : (lo > hi);
                        a[j] = swap ? hi : lo;
                        a[j2] = swap ? lo : hi;
                    }
                }
            } else {
#pragma unroll
                for (int j = 0; j < P; ++j) {
                    const uint64_t o = __shfl_xor_sync(0xffffffffu, a[j], stride);
                    const bool lower = (lane & stride) == 0;
                    const bool desc = ((j * 32 + lane) & size) == 0;
                    const uint64_t big = a[j] > o ? a[j] : o, small = a[j] > o ? o : a[j];
                    a[j] = (lower == desc) ? big : small;
                }
            }
        }
    }
}

template <int P>
__device__ int warp_keep_best_p(uint64_t* w, int n, int k) {
    const int lane = threadIdx.x & 31;
    uint64_t a[P];
#pragma unroll
    for (int j = 0; j < P; ++j) {
        const int i = j * 32 + lane;
        a[j] = i < n ? w[i] : 0ull;  // 0 ranks below every real key
    }
    __syncwarp();
    warp_sort_keys_desc<P>(a);
    const int K = n < k ? n : k;
#pragma unroll
    for (int j = 0; j < P; ++j) {
        const int i = j * 32 + lane;
        if (i < K) w[i] = a[j];
    }
    __syncwarp();
    return K;
}

// Sorts a warp's keys w[0, n) (n <= 256) best-first and keeps the best min(n, k) in w[0, ...).
__device__ int warp_keep_best(uint64_t* w, int n, int k) {
    if (n <= 32) return warp_keep_best_p<1>(w, n, k);
    if (n <= 64) return warp_keep_best_p<2>(w, n, k);
    if (n <= 128) return warp_keep_best_p<4>(w, n, k);
    return warp_keep_best_p<8>(w, n, k);
}

template <int kDtype, bool kLse>
struct WarpSampleOp {
    static constexpr int kEsz = (kDtype == LOOM_SELECT_BF16) ? 2 : 4;
    static constexpr int kPer = 16 / kEsz;
    static constexpr int kNT = kSampNT;
    StreamGeom g;  // copies: no pointer into the kernel's parameters
    SampleDev p;
    SampleShared* sh;
    uint2* raw;         // this warp's raw pairs (value bits, global id) [kRawCap]
    uint64_t* wk;       // this warp's kept keys [kWarpKeyCap]
    uint64_t* cand;     // segment-end gather [kWarpCand] (the raw buffers of all warps)
    uint64_t* keys0;    // all warps' key buffers (decision scratch at a segment end)
    int32_t* hset;      // history hash set of the segment
    int32_t* uniq;      // its distinct ids, as a list
    LseAcc lse;
    int nr;      // raw pairs this warp holds (the same in every lane)
    int nk;      // keys this warp keeps
    int stage;   // stage index within the segment
    float tv;      // this lane's entry of the warp's sorted list of stage maxima (lane i: i-th largest)
    float wv;      // the list's ceil(k / warps)-th entry
    bool pending;  // wv has risen since it was last published
    float lm, ls;     // log-sum-exp of the streamed elements in raw units: max lm, ls = sum of 2^((x - lm) c)
    float c;          // log2(e) / T (log2(e) for greedy rows)
    uint32_t* wflag;  // this warp's 32 words: per lane, which of its vectors of the stage hold a history id

    // One value into the lane's raw-unit log-sum-exp (NaN and -inf add nothing).
    __device__ __forceinline__ void raw_offer(float v) {
        if (v != v || v == neg_inf()) return;
        if (v > lm) {
            ls = ls * ex2_approx(__fmul_rn(__fsub_rn(lm, v), c)) + 1.0f;
            lm = v;
        } else if (v == lm) {
            ls += 1.0f;
        } else {
            ls += ex2_approx(__fmul_rn(__fsub_rn(v, lm), c));
        }
    }

    // Log-sum-exp terms of this lane's vectors of a stage, in raw units. History ids are left out
    // (they enter at their penalised value at the segment end): the warp first flags, from the
    // segment's list of distinct ids, the vectors of its lanes that hold one. A flagged vector goes
    // element by element; every other one costs two float operations and one ex2 per element,
    // after one rescale to the largest of their maxima.
    template <int kV>
    __device__ void lse_stage(const uint4* v4, int32_t nvec, int64_t gid0, const float (&mu)[kV]) {
        const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
        uint32_t fl = 0u;
        const int nu = p.penalty ? sh->n_uniq : 0;
        if (nu > 0) {
            const int64_t n = static_cast<int64_t>(nvec) * kPer;
            for (int j = lane; j < nu; j += 32) {
                const int64_t e = static_cast<int64_t>(uniq[j]) - gid0;
                if (e >= 0 && e < n) {
                    const int32_t v = static_cast<int32_t>(e / kPer);
                    if (((v % kNT) >> 5) == warp) atomicOr(&wflag[v & 31], 1u << (v / kNT));
                }
            }
            __syncwarp();
            fl = wflag[lane];
            wflag[lane] = 0u;
            __syncwarp();
        }
        float smc = neg_inf();
#pragma unroll
        for (int i = 0; i < kV; ++i)
            if (!((fl >> i) & 1u)) smc = fmaxf(smc, mu[i]);  // (a vector past the stage's end has NaN)
        const float mnew = fmaxf(lm, smc);
        if (mnew > lm) {
            ls = ls * ex2_approx(__fmul_rn(__fsub_rn(lm, mnew), c));
            lm = mnew;
        }
        if (lm == pos_inf()) {
#pragma unroll
            for (int i = 0; i < kV; ++i) {
                const int32_t v = i * kNT + tid;
                if (v < nvec && !((fl >> i) & 1u)) {
                    Vec16<kDtype> e;
                    e.unpack(v4[v]);
#pragma unroll
                    for (int q = 0; q < kPer; ++q) ls += e.x[q] == pos_inf() ? 1.0f : 0.0f;
                }
            }
        } else if (lm > neg_inf()) {
            // -inf elements give 2^-inf = 0; a NaN element makes the sum NaN, and only then is the
            // stage summed again with each term guarded
            const float m = lm;
            const uint64_t mm = f32x2_splat(m), cc = f32x2_splat(c);
            float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
            for (int i = 0; i < kV; ++i) {
                const int32_t v = i * kNT + tid;
                if (v < nvec && !((fl >> i) & 1u)) {
                    Vec16<kDtype> e;
                    e.unpack(v4[v]);
#pragma unroll
                    for (int q = 0; q < kPer; q += 2) {
                        float d0, d1;
                        sub_mul_f32x2(e.x[q], e.x[q + 1], mm, cc, d0, d1);
                        s0 += ex2_approx(d0);
                        s1 += ex2_approx(d1);
                    }
                }
            }
            float sum = s0 + s1;
            if (sum != sum) {
                sum = 0.0f;
#pragma unroll
                for (int i = 0; i < kV; ++i) {
                    const int32_t v = i * kNT + tid;
                    if (v < nvec && !((fl >> i) & 1u)) {
                        Vec16<kDtype> e;
                        e.unpack(v4[v]);
#pragma unroll
                        for (int q = 0; q < kPer; ++q)
                            sum += ex2_approx(fmaxf(__fmul_rn(__fsub_rn(e.x[q], m), c), neg_inf()));
                    }
                }
            }
            ls += sum;
        }
        while (fl) {
            const int i = __ffs(fl) - 1;
            fl &= fl - 1u;
            const int32_t v = i * kNT + tid;
            Vec16<kDtype> e;
            e.unpack(v4[v]);
#pragma unroll
            for (int q = 0; q < kPer; ++q)
                if (!is_history(gid0 + static_cast<int64_t>(v) * kPer + q)) raw_offer(e.x[q]);
        }
    }

    __device__ const unsigned char* row_ptr(int64_t row) const { return g.base + row * g.row_stride * kEsz; }
    __device__ const int32_t* row_hist(int64_t row) const { return p.hist + row * static_cast<int64_t>(p.hist_len); }

    __device__ __forceinline__ bool is_history(int64_t gid) const {
        return p.penalty && hash_contains(hset, static_cast<int32_t>(gid));
    }

    __device__ __forceinline__ float threshold_X() const {
        return order_key_to_float(*reinterpret_cast<const volatile uint32_t*>(&sh->x_key));
    }

    // One lane: k kept keys reach `kth`, so the row's k-th best does too.
    __device__ void raise(uint64_t kth) {
        const unsigned long long old = atomicMax(&sh->key_t, static_cast<unsigned long long>(kth));
        if (kth > old) atomicMax(&sh->x_key, loom_order_key(inverse_threshold_bound(rank_key_value(kth), p.T, p.greedy)));
    }

    // One lane: at least k distinct non-history elements have a raw value >= v.
    __device__ void raise_raw(float v) {
        const float t = tempered(v, p.T, p.greedy);
        if (!(t > neg_inf())) return;  // (-inf or NaN: nothing to raise)
        const unsigned long long floor = static_cast<unsigned long long>(loom_order_key(t)) << 32;
        const unsigned long long old = atomicMax(&sh->key_t, floor);
        if (floor > old) atomicMax(&sh->x_key, loom_order_key(inverse_threshold_bound(t, p.T, p.greedy)));
    }

    // Warp-collective: inserts every lane's value c with `take` into the warp's sorted list, and
    // updates wv.
    __device__ __forceinline__ void list_insert(bool take, float c) {
        const int lane = threadIdx.x & 31;
        uint32_t b = __ballot_sync(0xffffffffu, take);
        while (b) {
            const int src = __ffs(b) - 1;
            b &= b - 1u;
            const float ci = __shfl_sync(0xffffffffu, c, src);
            const float up = __shfl_up_sync(0xffffffffu, tv, 1);  // lane i: entry i - 1
            if (!(tv >= ci)) tv = (lane == 0 || up >= ci) ? ci : up;
        }
        const float v = __shfl_sync(0xffffffffu, tv, (p.k + kSampWarps - 1) / kSampWarps - 1);
        if (v > wv) {
            wv = v;
            pending = true;
        }
    }

    // Warp-collective: publishes wv when it has risen and raises the thresholds to the smallest
    // value the warps have published.
    __device__ void publish() {
        if (!pending) return;
        pending = false;
        const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
        if (lane == 0) {
            volatile float* wq = sh->wq;
            wq[warp] = wv;
            float mn = wv;
            for (int w = 0; w < kSampWarps; ++w) mn = fminf(mn, wq[w]);
            raise_raw(mn);
        }
    }

    // Warp-collective: tempers the raw pairs into keys after the kept ones (dropping those under
    // key_t), keeps the best k and, holding k, raises the thresholds to the k-th.
    __device__ void prune() {
        if (nr == 0) return;
        const int lane = threadIdx.x & 31;
        __syncwarp();
        const uint64_t floor = *reinterpret_cast<const volatile unsigned long long*>(&sh->key_t);
        int n = nk;
        for (int base = 0; base < nr; base += 32) {
            const int i = base + lane;
            uint64_t key = 0ull;
            bool keep = false;
            if (i < nr) {
                const uint2 e = raw[i];
                key = loom_rank_key(tempered(__uint_as_float(e.x), p.T, p.greedy), static_cast<int32_t>(e.y));
                keep = key >= floor;
            }
            const uint32_t b = __ballot_sync(0xffffffffu, keep);
            if (keep) wk[n + __popc(b & lanemask_lt())] = key;
            n += __popc(b);
        }
        nr = 0;
        __syncwarp();
        if (n >= p.k) {
            n = warp_keep_best(wk, n, p.k);
            if (lane == 0) raise(wk[p.k - 1]);
        }
        nk = n;
    }

    // Warp-collective: the lanes with `take` append (x, id); a full buffer is pruned first.
    __device__ __forceinline__ void append(bool take, float x, int32_t id) {
        const uint32_t b = __ballot_sync(0xffffffffu, take);
        if (b == 0u) return;
        const int c = __popc(b);
        if (nr + c > kRawCap) prune();
        if (take) raw[nr + __popc(b & lanemask_lt())] = make_uint2(__float_as_uint(x), static_cast<uint32_t>(id));
        nr += c;
    }

    __device__ void begin_segment(const Segment& s) {
        const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
        if (tid == 0) {
            sh->K = 0;
            if (p.u && !p.shard && !p.greedy) sh->u_row = __ldg(p.u + s.row);  // used at the row's end
            sh->bad = 0;
            sh->n_uniq = 0;
            sh->warm_key = 0xffffffffu;
            sh->key_t = 0ull;
            sh->x_key = loom_order_key(neg_inf());
            for (int w = 0; w < kSampWarps; ++w) sh->wq[w] = neg_inf();
        }
        lse = lse_init();
        lm = neg_inf();
        ls = 0.0f;
        nr = 0;
        nk = 0;
        stage = 0;
        tv = neg_inf();
        wv = neg_inf();
        pending = false;
        // this thread's first history id is loaded before the set is cleared (its latency overlaps)
        const int32_t id_first = tid < p.hist_len ? __ldg(row_hist(s.row) + tid) : 0;
        if (p.penalty) {
            int4* h4 = reinterpret_cast<int4*>(hset);
            for (int i = tid; i < kHashSlots / 4; i += kNT) h4[i] = make_int4(-1, -1, -1, -1);
        }
        group_sync<kNT>();
        // validate the whole history; the distinct ids inside this segment go into the set and list
        const int64_t seg_lo = p.vocab_offset + s.j0, seg_hi = p.vocab_offset + s.j1;
        for (int j = tid; j < p.hist_len; j += kNT) {
            const int32_t id = j == tid ? id_first : __ldg(row_hist(s.row) + j);
            if (id < 0 || id >= p.vocab_limit) sh->bad = 1;
            else if (p.penalty && id >= seg_lo && id < seg_hi && hash_insert(hset, id))
                uniq[atomicAdd(&sh->n_uniq, 1)] = id;
        }
        group_sync<kNT>();
        if (tid == 0 && sh->bad) record_status(p.status, LOOM_SELECT_EHISTORY);
        // edges (at most 14 elements outside the 16-byte-aligned interior), read by warp 0
        if (warp == 0) {
            const int32_t n_edges = segment_edge_count(s, kEsz);
            bool take = false;
            float x = 0.0f;
            int32_t gid = 0;
            if (lane < n_edges) {
                const int64_t col = segment_edge_col(s, kEsz, lane);
                x = load_global_elem<kDtype>(row_ptr(s.row), col);
                gid = static_cast<int32_t>(p.vocab_offset + col);
                // a history id enters at the segment end, with the segment's other history ids
                if (!is_history(gid)) {
                    if (p.lse) lse_offer(lse, tempered(x, p.T, p.greedy));
                    take = x == x;
                }
            }
            append(take, x, gid);
        }
    }

    // The first stage of a segment seeds the thresholds (every warp, two CTA barriers): each warp
    // sorts its lanes' maxima (a lane whose maximum is a history id vouches for nothing) and the
    // smallest of the warps' ceil(k / warps)-th largest is a value that at least k elements reach.
    __device__ void warm_up(const uint4* v4, int32_t nvec, int64_t gid0, bool live) {
        const int tid = threadIdx.x, lane = tid & 31;
        float m = neg_inf();
        if (live) {
            int64_t at = -1;
            for (int32_t v = tid; v < nvec; v += kNT) {
                Vec16<kDtype> e;
                e.unpack(v4[v]);
#pragma unroll
                for (int q = 0; q < kPer; ++q)
                    if (e.x[q] > m) {
                        m = e.x[q];
                        at = gid0 + static_cast<int64_t>(v) * kPer + q;
                    }
            }
            if (at >= 0 && is_history(at)) m = neg_inf();
        }
        const float sorted = warp_sort_desc(m);
        tv = sorted;  // the list starts as the first stage's lane maxima
        const int q = (p.k + kSampWarps - 1) / kSampWarps;  // <= 16
        const float bw = __shfl_sync(0xffffffffu, sorted, q - 1);
        wv = bw;
        if (lane == 0) {
            sh->wq[threadIdx.x >> 5] = bw;
            atomicMin(&sh->warm_key, loom_order_key(bw));
        }
        group_sync<kNT>();
        if (tid == 0) {
            const float ty = tempered(order_key_to_float(sh->warm_key), p.T, p.greedy);
            if (ty == ty && ty > neg_inf()) {
                atomicMax(&sh->key_t, static_cast<unsigned long long>(loom_order_key(ty)) << 32);
                atomicMax(&sh->x_key, loom_order_key(inverse_threshold_bound(ty, p.T, p.greedy)));
            }
        }
        group_sync<kNT>();
    }

    __device__ void chunk(const Segment&, const unsigned char* data, int64_t col0, int32_t n, bool live) {
        const int tid = threadIdx.x;
        const int32_t nvec = n / kPer;
        const uint4* v4 = reinterpret_cast<const uint4*>(data);
        const int64_t gid0 = p.vocab_offset + col0;
        const int st = stage++;
        if (st == 0) warm_up(v4, nvec, gid0, live);
        if (!live) return;
        const float X = threshold_X();

        // 2. mark. The common path is one max per element: each vector's maximum mu[i] (NaN for a
        //    vector past the stage's end) and the lane's stage maximum smax; only a lane whose smax
        //    reaches X (rare) turns its mu[i] into marks.
        constexpr int kVecsPerThread = kWarpStageBytes / 16 / kNT;
        static_assert(kVecsPerThread <= 32, "marks are one 32-bit word");
        float mu[kVecsPerThread];
        float smax = neg_inf();
        if (nvec == kVecsPerThread * kNT) {
#pragma unroll
            for (int i = 0; i < kVecsPerThread; ++i) {
                mu[i] = vec_max<kDtype>(v4[i * kNT + tid]);
                smax = fmaxf(smax, mu[i]);
            }
        } else {
#pragma unroll
            for (int i = 0; i < kVecsPerThread; ++i) {
                const int32_t v = i * kNT + tid;
                mu[i] = __int_as_float(0x7fc00000);
                if (v < nvec) mu[i] = vec_max<kDtype>(v4[v]);
                smax = fmaxf(smax, mu[i]);
            }
        }
        if constexpr (kLse) lse_stage<kVecsPerThread>(v4, nvec, gid0, mu);
        uint32_t hits = 0;
        if (smax >= X) {
#pragma unroll
            for (int i = 0; i < kVecsPerThread; ++i) hits |= static_cast<uint32_t>(mu[i] >= X) << i;
        }

        // The warp's list of stage maxima (the first stage's are already in it, from the warm-up).
        // A lane whose maximum beats wv finds the vector holding it (from mu[]) and, with a
        // penalty, checks whether that element is a history id: then it enters at its penalised value.
        if (st > 0 && __any_sync(0xffffffffu, smax > wv)) {
            float c = smax;
            if (p.penalty && smax > wv) {
                int at = 0;
#pragma unroll
                for (int i = kVecsPerThread - 1; i >= 0; --i)
                    if (mu[i] == smax) at = i;
                const int32_t v = at * kNT + tid;
                Vec16<kDtype> e;
                e.unpack(v4[v]);
                int q = 0;
#pragma unroll
                for (int t = kPer - 1; t >= 0; --t)
                    if (e.x[t] == smax) q = t;
                if (is_history(gid0 + static_cast<int64_t>(v) * kPer + q)) c = penalise(smax, p.r);
            }
            list_insert(c > wv, c);
        }
        if (st < 4 || (st & 3) == 3) publish();  // every stage at first, then every fourth at most

        // 3. sweep: one passing element per lane per step, appended by ballot
        if (__any_sync(0xffffffffu, hits != 0u)) {
            uint32_t m = 0u;  // pass bits of the vector this lane is sweeping
            int32_t e0 = 0;   // its first element in the stage
            for (;;) {
                while (m == 0u && hits != 0u) {
                    const int i = __ffs(hits) - 1;
                    hits &= hits - 1u;
                    const int32_t v = i * kNT + tid;
                    Vec16<kDtype> e;
                    e.unpack(v4[v]);
#pragma unroll
                    for (int q = 0; q < kPer; ++q) m |= static_cast<uint32_t>(e.x[q] >= X) << q;
                    e0 = v * kPer;
                }
                const bool has = m != 0u;
                if (!__any_sync(0xffffffffu, has)) break;
                bool take = false;
                float x = 0.0f;
                int32_t id = 0;
                if (has) {
                    const int q = __ffs(m) - 1;
                    m &= m - 1u;
                    x = smem_elem<kDtype>(data, e0 + q);
                    id = static_cast<int32_t>(gid0 + e0 + q);
                    take = !is_history(id);  // a history id's stream value is replaced at the segment end
                }
                append(take, x, id);
            }
        }
    }

    __device__ void end_segment(const Segment& s) {
        const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
        // the first of this lane's history logits, loaded before the prune (its latency overlaps)
        const int nu0 = p.penalty ? sh->n_uniq : 0;
        const int j_first = warp * 32 + lane;
        float x_first = 0.0f;
        if (j_first < nu0)
            x_first = load_global_elem<kDtype>(row_ptr(s.row), static_cast<int64_t>(uniq[j_first]) - p.vocab_offset);
        prune();  // at most k keys per warp, the raw buffer empty
        if (kLse && ls > 0.0f) {
            // the streamed sum, relative to the tempered maximum: 2^((x - lm) c) = e^(x / T - lm / T)
            LseAcc r;
            r.m = tempered(lm, p.T, p.greedy);
            r.s = ls;
            lse = lse_merge(lse, r);
        }
        if (p.penalty) {
            // The segment's distinct history ids with their penalised, tempered values, read from
            // global memory (the row has just streamed through L2), against the final threshold.
            const int nu = sh->n_uniq;
            const uint64_t floor = *reinterpret_cast<const volatile unsigned long long*>(&sh->key_t);
            for (int base = warp * 32; base < nu; base += kNT) {  // warp-uniform trip count
                const int j = base + lane;
                uint64_t key = 0ull;
                bool keep = false;
                if (j < nu) {
                    const int32_t id = uniq[j];
                    const float x = j == j_first ? x_first
                                                 : load_global_elem<kDtype>(row_ptr(s.row),
                                                                            static_cast<int64_t>(id) - p.vocab_offset);
                    const float y = tempered(penalise(x, p.r), p.T, p.greedy);
                    if (p.lse) lse_offer(lse, y);
                    key = loom_rank_key(y, id);
                    keep = y == y && key >= floor;
                }
                const uint32_t b = __ballot_sync(0xffffffffu, keep);
                if (keep) wk[nk + __popc(b & lanemask_lt())] = key;
                nk += __popc(b);
            }
            __syncwarp();
            if (nk > p.k) nk = warp_keep_best(wk, nk, p.k);
        }
        if (p.lse) {
            const LseAcc w = lse_warp_reduce(lse);
            if (lane == 0) sh->lse_w[warp] = w;
        }
        group_sync<kNT>();  // every raw buffer is empty: the gather (which aliases them) is free
        int off = 0;
        if (lane == 0) off = atomicAdd(&sh->K, nk);
        off = __shfl_sync(0xffffffffu, off, 0);
        for (int i = lane; i < nk; i += 32) cand[off + i] = wk[i];
        if (tid == 0) {
            LseAcc a = lse_init();
            if (p.lse)
                for (int w = 0; w < kSampWarps; ++w) a = lse_merge(a, sh->lse_w[w]);
            sh->seg_lse = a;
        }
        group_sync<kNT>();
        const int K = topk_select_sorted_small_k<kNT, kWarpCand>(cand, sh->K, p.k, &sh->tk);
        double* e = reinterpret_cast<double*>(keys0);
        finish_segment<kDtype, kNT, kWarpCand, true>(p, g, s, cand, e, e + kWarpMaxK, K, sh->seg_lse, sh->bad != 0, sh);
    }
};

constexpr size_t kWarpDynSmem = static_cast<size_t>(kWarpStages) * kWarpStageBytes +
                                kSampWarps * kRawCap * sizeof(uint2) + kSampWarps * kWarpKeyCap * sizeof(uint64_t) +
                                kHashSlots * sizeof(int32_t) + kMaxHistory * sizeof(int32_t) +
                                kSampWarps * 32 * sizeof(uint32_t);
static_assert(kWarpDynSmem + 4096 <= 232448 / kSampCtasPerSm, "two CTAs per SM must fit the SM's shared memory");

// kLse: the log-sum-exp is wanted (log-probabilities or shard records), p.lse == kLse.
template <int kDtype, bool kLse>
__global__ void __launch_bounds__((kSampWarps + 1) * 32, kSampCtasPerSm) sample_stream_kernel(StreamGeom g, SampleDev p) {
    extern __shared__ __align__(128) unsigned char dyn[];
    __shared__ StreamCtl ctl;
    __shared__ SampleShared sh;
    unsigned char* ring = dyn;
    uint2* raw_all = reinterpret_cast<uint2*>(dyn + static_cast<size_t>(kWarpStages) * kWarpStageBytes);
    uint64_t* keys_all = reinterpret_cast<uint64_t*>(raw_all + kSampWarps * kRawCap);
    int32_t* hset = reinterpret_cast<int32_t*>(keys_all + kSampWarps * kWarpKeyCap);
    int32_t* uniq = hset + kHashSlots;
    uint32_t* wflag_all = reinterpret_cast<uint32_t*>(uniq + kMaxHistory);
    // (zeroed before the streamer's first barrier; each stage's reader returns its words to zero)
    for (int i = threadIdx.x; i < kSampWarps * 32; i += blockDim.x) wflag_all[i] = 0u;
    const int warp = threadIdx.x >> 5;
    const int w = warp < kSampWarps ? warp : 0;  // the producer warp holds no buffers
    const float c = p.greedy ? kLog2e : __fdiv_rn(kLog2e, p.T);
    WarpSampleOp<kDtype, kLse> op{g,     p,    &sh,  raw_all + w * kRawCap, keys_all + w * kWarpKeyCap,
                                  reinterpret_cast<uint64_t*>(raw_all), keys_all, hset, uniq, lse_init(), 0, 0, 0,
                                  neg_inf(), neg_inf(), false,            // (tv, wv, pending)
                                  neg_inf(), 0.0f, c, wflag_all + w * 32};  // (lm, ls, c, wflag)
    stream_ranges_warps<kWarpStages, kWarpStageBytes, kSampWarps>(g, op, ring, &ctl, p.status);
}

// ---------------------------------------------------------------------------------------------
// K4: merge of the gathered shard records, one CTA per row.

constexpr int kMergeNT = 256;

__global__ void __launch_bounds__(kMergeNT) shard_merge_kernel(const unsigned char* records, int32_t n_shards,
                                                               int64_t rows, size_t rec_bytes, const float* u,
                                                               int32_t k, float top_p, int32_t* out_ids,
                                                               float* out_prob, float* out_logp, int32_t* out_topk) {
    extern __shared__ __align__(16) uint64_t mcand[];
    __shared__ TopkShared tk;
    __shared__ int bad;
    __shared__ int32_t sel_id;
    __shared__ float sel_prob, sel_y;
    __shared__ float m_max;
    const int64_t row = blockIdx.x;
    const int tid = threadIdx.x;
    if (tid == 0) {
        bad = 0;
        float M = neg_inf();
        for (int g = 0; g < n_shards; ++g) {
            const RecordHead* h = reinterpret_cast<const RecordHead*>(records + (static_cast<size_t>(g) * rows + row) * rec_bytes);
            if (h->count < 0) bad = 1;
            else if (h->m > M) M = h->m;
        }
        m_max = M;
    }
    __syncthreads();
    if (bad) {
        if (tid == 0) {
            out_ids[row] = -1;
            out_prob[row] = __int_as_float(0x7fc00000);
            if (out_logp) out_logp[row] = __int_as_float(0x7fc00000);
        }
        if (out_topk)
            for (int j = tid; j < k; j += kMergeNT) out_topk[row * k + j] = -1;
        return;
    }
    int have = 0;
    for (int g = 0; g < n_shards; ++g) {
        const unsigned char* rec = records + (static_cast<size_t>(g) * rows + row) * rec_bytes;
        const int32_t c = reinterpret_cast<const RecordHead*>(rec)->count;
        if (have + c > kCandCap) have = topk_select_sorted<kMergeNT, kCandCap>(mcand, have, k, &tk);
        const uint2* pairs = reinterpret_cast<const uint2*>(rec + 16);
        for (int i = tid; i < c; i += kMergeNT) {
            const uint2 pr = pairs[i];
            mcand[have + i] = loom_rank_key(__uint_as_float(pr.x), static_cast<int32_t>(pr.y));
        }
        have += c;
        __syncthreads();
    }
    const int K = topk_select_sorted<kMergeNT, kCandCap>(mcand, have, k, &tk);
    if (tid < 32) {
        double* e = reinterpret_cast<double*>(mcand + kDecideSlots);
        double* S = reinterpret_cast<double*>(mcand + kCandCap);
        decide_warp(mcand, K, top_p, __ldg(u + row), e, S, &sel_id, &sel_prob, &sel_y);
        if (tid == 0) {
            out_ids[row] = sel_id;
            out_prob[row] = sel_prob;
            if (out_logp) {
                const double M = m_max;
                double S_all = 0.0;
                for (int g = 0; g < n_shards; ++g) {
                    const RecordHead* h = reinterpret_cast<const RecordHead*>(records + (static_cast<size_t>(g) * rows + row) * rec_bytes);
                    if (h->s > 0.0f) S_all += static_cast<double>(h->s) * (static_cast<double>(h->m) == M ? 1.0 : exp(static_cast<double>(h->m) - M));
                }
                out_logp[row] = static_cast<float>(static_cast<double>(sel_y) - (M + log(S_all)));
            }
        }
    }
    if (out_topk)
        for (int j = tid; j < k; j += kMergeNT) out_topk[row * k + j] = j < K ? rank_key_id(mcand[j]) : -1;
}

template <int kDtype>
cudaError_t launch_sample_t(const StreamGeom& g, const SampleDev& p, cudaStream_t stream) {
    static std::atomic<bool> configured[64] = {};  // set once per device, from any host thread
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(sample_stream_kernel<kDtype, false>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kWarpDynSmem));
        if (e != cudaSuccess) return e;
        e = cudaFuncSetAttribute(sample_stream_kernel<kDtype, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(kWarpDynSmem));
        if (e != cudaSuccess) return e;
        e = cudaFuncSetAttribute(sample_wide_kernel<kDtype>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(kWideDynSmem));
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    if (p.k <= kWarpMaxK && p.lse)
        sample_stream_kernel<kDtype, true><<<g.ctas, (kSampWarps + 1) * 32, kWarpDynSmem, stream>>>(g, p);
    else if (p.k <= kWarpMaxK)
        sample_stream_kernel<kDtype, false><<<g.ctas, (kSampWarps + 1) * 32, kWarpDynSmem, stream>>>(g, p);
    else
        sample_wide_kernel<kDtype><<<g.ctas, (kSampWarps + 1) * 32, kWideDynSmem, stream>>>(g, p);
    return cudaGetLastError();
}

}  // namespace

size_t sample_record_bytes(int32_t top_k) { return 16 + 8 * static_cast<size_t>(top_k); }

cudaError_t launch_sample_stream(const SampleLaunch& a, void* workspace, const WsLayout& l, int ctas,
                                 cudaStream_t stream) {
    StreamGeom g;
    g.base = static_cast<const unsigned char*>(a.logits);
    g.rows = a.rows;
    g.width = a.width;
    g.row_stride = a.row_stride;
    g.total = a.rows * a.width;
    g.esz = a.dtype == LOOM_SELECT_BF16 ? 2 : 4;
    g.ctas = ctas;
    unsigned char* ws = static_cast<unsigned char*>(workspace);
    SampleDev p;
    p.T = a.temperature;
    p.r = a.penalty;
    p.p = a.top_p;
    p.k = a.top_k;
    p.greedy = a.temperature == 0.0f;
    p.penalty = a.history_len > 0 && a.penalty != 1.0f;
    p.shard = a.shard_out != nullptr;
    p.lse = p.shard || a.out_logp != nullptr;
    p.vocab_offset = a.vocab_offset;
    p.vocab_limit = a.vocab_limit;
    p.hist = a.history;
    p.hist_len = a.history_len;
    p.u = a.u;
    p.out_ids = a.out_ids;
    p.out_prob = a.out_prob;
    p.out_logp = a.out_logp;
    p.out_topk = a.out_topk;
    p.shard_out = static_cast<unsigned char*>(a.shard_out);
    p.recs = ws + l.records;
    p.rec_bytes = sample_record_bytes(a.top_k);
    p.tickets = reinterpret_cast<int*>(ws + l.tickets);
    p.status = reinterpret_cast<int*>(ws);
    if (a.dtype == LOOM_SELECT_BF16) return launch_sample_t<LOOM_SELECT_BF16>(g, p, stream);
    return launch_sample_t<LOOM_SELECT_F32>(g, p, stream);
}

cudaError_t launch_shard_merge(const void* records, int32_t n_shards, int64_t rows, const float* u, int32_t top_k,
                               float top_p, int32_t* out_ids, float* out_prob, float* out_logp, int32_t* out_topk,
                               cudaStream_t stream) {
    const size_t smem = kCandCap * sizeof(uint64_t) + kDecideSlots * sizeof(double);
    static std::atomic<bool> configured[64] = {};  // set once per device, from any host thread
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        const cudaError_t e =
            cudaFuncSetAttribute(shard_merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    shard_merge_kernel<<<static_cast<unsigned>(rows), kMergeNT, smem, stream>>>(
        static_cast<const unsigned char*>(records), n_shards, rows, sample_record_bytes(top_k), u, top_k, top_p, out_ids,
        out_prob, out_logp, out_topk);
    return cudaGetLastError();
}

}  // namespace loom_select
