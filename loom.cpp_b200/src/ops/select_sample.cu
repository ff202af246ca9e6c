// select_sample.cu -- the fused sampling chain (K2) and the vocabulary-shard merge (K4).
//
// One pass over the logits: rows stream through shared memory (select_stream.cuh). The per-element
// work is a compare without branches: each thread marks, in a register bitmask, which of its
// vectors of the stage (16 bytes each) have a maximum reaching a threshold X. Every element below X
// is strictly worse than k elements already kept (X is at most the smallest raw value whose tempered
// value x / T reaches the current k-th best). At the end of the stage each thread sweeps its few
// marked vectors: the elements that pass go, raw, into the thread's own slots in shared memory (one
// store each; no atomics, no shuffles, no divides).
//
// At the end of a stage, when more than k + kPruneSlack candidates are held, they are tempered with
// an IEEE divide (in parallel), the exact top-k is kept as 64-bit rank keys, and X rises to the k-th.
// The first stage of each row segment seeds X: each warp sorts its lanes' maxima and the smallest of
// the warps' ceil(k / warps)-th largest is a value that at least k elements reach.
//
// The repetition penalty touches only the history ids: at the start of a row segment the distinct
// ones inside it go into a shared-memory hash set and a list. Each stage inserts the listed ids it
// holds with their penalised, tempered values; the stream skips set members (looked up only for
// elements that pass X). So the per-element path carries no penalty work.
//
// At the end of a row the exact top-k is ranked into order and the survivor decision runs in double
// precision on one warp (select_topk.cuh), in exactly the oracle's operation order.
// Bound: HBM bandwidth (4 bytes per f32 logit, 2 per bf16, read once).
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
constexpr int kPruneSlack = 64;     // prune at a stage end when more than k + this many are held
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
__device__ void finalize_row(const SampleDev p, const StreamGeom g, int64_t row, uint64_t* cand, double* S, int K,
                             LseAcc lse, bool bad, SampleShared* sh) {
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
        double* e = reinterpret_cast<double*>(cand + kDecideSlots);
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
            decide_warp(cand, K, p.p, __ldg(p.u + row), e, S, &sh->sel_id, &sh->sel_prob, &sh->sel_y);
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

template <int kDtype>
struct SampleOp {
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
            if (!failed && held <= p.k + kPruneSlack) break;
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
        const int K = sh->K;
        const LseAcc seg = sh->seg_lse;
        const bool bad = sh->bad != 0;
        if (s.count == 1) {
            finalize_row<kDtype, kNT>(p, g, s.row, cand, S, K, seg, bad, sh);
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
        // merge every piece's record
        int have = 0;
        bool any_bad = false;
        LseAcc tot = lse_init();
        for (int j = 0; j < s.count; ++j) {
            const unsigned char* r = p.recs + static_cast<size_t>(record_slot(g, s.first_cta + j, s.row)) * p.rec_bytes;
            const int32_t c = __ldcg(reinterpret_cast<const int32_t*>(r));
            if (c < 0) {
                any_bad = true;
                continue;
            }
            LseAcc part;
            part.m = __ldcg(reinterpret_cast<const float*>(r) + 1);
            part.s = __ldcg(reinterpret_cast<const float*>(r) + 2);
            tot = lse_merge(tot, part);
            if (have + c > kCandCap) have = topk_select_sorted<kNT, kCandCap>(cand, have, p.k, &sh->tk);
            const uint64_t* rk = reinterpret_cast<const uint64_t*>(r + 16);
            for (int i = tid; i < c; i += kNT) cand[have + i] = __ldcg(rk + i);
            have += c;
            group_sync<kNT>();
        }
        const int Kf = topk_select_sorted<kNT, kCandCap>(cand, have, p.k, &sh->tk);
        if (tid == 0) p.tickets[record_slot(g, s.first_cta, s.row)] = 0;
        finalize_row<kDtype, kNT>(p, g, s.row, cand, S, Kf, tot, any_bad, sh);
    }
};

constexpr size_t kSampDynSmem = static_cast<size_t>(kSampStages) * kSampStageBytes + kCandCap * sizeof(uint64_t) +
                                kSlots * kSampNT * sizeof(uint2) + kHashSlots * sizeof(int32_t) +
                                kMaxHistory * sizeof(int32_t) + kDecideSlots * sizeof(double);
static_assert(kSampDynSmem + 4096 <= 232448 / kSampCtasPerSm, "two CTAs per SM must fit the SM's shared memory");

template <int kDtype>
__global__ void __launch_bounds__((kSampWarps + 1) * 32, kSampCtasPerSm) sample_stream_kernel(StreamGeom g, SampleDev p) {
    extern __shared__ __align__(128) unsigned char dyn[];
    __shared__ StreamCtl ctl;
    __shared__ SampleShared sh;
    unsigned char* ring = dyn;
    uint64_t* cand = reinterpret_cast<uint64_t*>(dyn + static_cast<size_t>(kSampStages) * kSampStageBytes);
    uint2* slots = reinterpret_cast<uint2*>(cand + kCandCap);
    int32_t* hset = reinterpret_cast<int32_t*>(slots + kSlots * kSampNT);
    int32_t* uniq = hset + kHashSlots;
    double* S = reinterpret_cast<double*>(uniq + kMaxHistory);
    SampleOp<kDtype> op{g, p, &sh, cand, slots, hset, uniq, S, lse_init(), 0, true};
    stream_ranges<kSampStages, kSampStageBytes, kSampWarps>(g, op, ring, &ctl, p.status);
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
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        const cudaError_t e = cudaFuncSetAttribute(sample_stream_kernel<kDtype>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   static_cast<int>(kSampDynSmem));
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    sample_stream_kernel<kDtype><<<g.ctas, (kSampWarps + 1) * 32, kSampDynSmem, stream>>>(g, p);
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
    static bool configured[64] = {};
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
