// select_topk.cuh -- exact top-k over 64-bit rank keys in shared memory, and the survivor decision.
//
// A candidate is one 64-bit rank key: (order key of the value << 32) | (0xffffffff - id), so a larger
// key ranks first (value descending, id ascending, -0 == +0, NaN lowest) and (value, id) can be read
// back from the key. All routines are CTA-cooperative over kNT threads that synchronise on named
// barrier 1; every thread of the group must call them with the same arguments.
#pragma once

#include "select_device.cuh"

namespace loom_select {

struct TopkShared {
    uint32_t hist[256];
    uint32_t warp_tot[32];
    int sel_count;
    int digit_shift;
    uint32_t need;
    uint32_t eq;
    uint64_t prefix;
};

__device__ __forceinline__ int next_pow2(int n) {
    int p = 1;
    while (p < n) p <<= 1;
    return p;
}

// Radix select: finds the rule that keeps exactly K = min(k, n) of the n keys -- those with
// (key >> shift) >= (prefix >> shift) -- and compacts them to cand[0, K) (in no particular order).
// Keys are distinct (ids are), so the K kept are exactly the K largest.
template <int kNT, int kMaxPerThread>
__device__ int topk_select_compact(uint64_t* cand, int n, int k, TopkShared* sh) {
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    if (n <= k) return n;
    uint64_t prefix = 0;
    uint32_t need = static_cast<uint32_t>(k);
    int shift = 56;
    for (;;) {
        for (int i = tid; i < 256; i += kNT) sh->hist[i] = 0;
        group_sync<kNT>();
        for (int base = 0; base < n; base += kNT) { // uniform trip count: every lane reaches the match
            const int i = base + tid;
            const uint64_t key = i < n ? cand[i] : 0ull;
            const bool match = i < n && ((shift == 56) || ((key ^ prefix) >> (shift + 8)) == 0);
            const uint32_t d = match ? (static_cast<uint32_t>(key >> shift) & 255u) : 256u;
            const uint32_t peers = __match_any_sync(0xffffffffu, d);
            if (match && lane == __ffs(peers) - 1) atomicAdd(&sh->hist[d], static_cast<uint32_t>(__popc(peers)));
        }
        group_sync<kNT>();
        if (tid < 32) {
            // lane l owns digits [8l, 8l+8); find the digit where the count from the top reaches need
            uint32_t c[8];
            uint32_t mine = 0;
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                c[q] = sh->hist[8 * lane + q];
                mine += c[q];
            }
            // suffix sum over lanes (higher lanes hold higher digits)
            uint32_t above = 0; // total of lanes > lane
            uint32_t incl = mine;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const uint32_t o = __shfl_down_sync(0xffffffffu, incl, off);
                if (lane + off < 32) incl += o;
            }
            above = incl - mine;
            // the lane whose range holds the need-th key from the top
            const bool holds = above < need && need <= incl;
            if (holds) {
                uint32_t acc = above;
                int d = 7;
                for (; d >= 0; --d) {
                    if (acc + c[d] >= need) break;
                    acc += c[d];
                }
                sh->prefix = prefix | (static_cast<uint64_t>(8 * lane + d) << shift);
                sh->need = need - acc;
                sh->eq = c[d];
            }
        }
        group_sync<kNT>();
        prefix = sh->prefix;
        need = sh->need;
        const uint32_t eq = sh->eq;
        if (eq == need || shift == 0) break;
        shift -= 8;
        group_sync<kNT>(); // everyone has read sh before the next pass rewrites it
    }
    // compaction: keep (key >> shift) >= (prefix >> shift)
    uint64_t mine[kMaxPerThread];
#pragma unroll
    for (int j = 0; j < kMaxPerThread; ++j) {
        const int i = tid + j * kNT;
        mine[j] = i < n ? cand[i] : 0ull;
    }
    if (tid == 0) sh->sel_count = 0;
    group_sync<kNT>();
    const uint64_t thr = prefix >> shift;
#pragma unroll
    for (int j = 0; j < kMaxPerThread; ++j) {
        const int i = tid + j * kNT;
        const bool keep = i < n && (mine[j] >> shift) >= thr;
        const uint32_t ballot = __ballot_sync(0xffffffffu, keep);
        int base = 0;
        if (lane == 0 && ballot) base = atomicAdd(&sh->sel_count, __popc(ballot));
        base = __shfl_sync(0xffffffffu, base, 0);
        if (keep) cand[base + __popc(ballot & ((1u << lane) - 1u))] = mine[j];
    }
    group_sync<kNT>();
    return k;
}

// Sorts cand[0, n) descending (n <= P, P a power of two; cand must have room for P keys).
template <int kNT>
__device__ void topk_sort_desc(uint64_t* cand, int n, int P) {
    for (int i = n + threadIdx.x; i < P; i += kNT) cand[i] = 0ull; // 0 ranks below every real key
    group_sync<kNT>();
    for (int size = 2; size <= P; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int t = threadIdx.x; t < (P >> 1); t += kNT) {
                const int i = 2 * t - (t & (stride - 1));
                const int j = i + stride;
                const uint64_t a = cand[i], b = cand[j];
                const bool desc = (i & size) == 0;
                if (desc ? (a < b) : (a > b)) {
                    cand[i] = b;
                    cand[j] = a;
                }
            }
            group_sync<kNT>();
        }
    }
}

// Exact rank selection of small sets: each key's rank is the number of larger keys (keys are
// distinct), so the K = min(k, n) largest land, sorted descending, at cand[rank] in [0, K).
// O(n^2 / kNT) compares with broadcast shared-memory reads; n <= kPer * kNT.
template <int kNT, int kPer>
__device__ int topk_rank_sort(uint64_t* cand, int n, int k) {
    const int tid = threadIdx.x;
    uint64_t mine[kPer];
    int rank[kPer];
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
        const int i = tid + j * kNT;
        mine[j] = i < n ? cand[i] : 0ull;
        rank[j] = 0;
    }
    int i = 0;
    const int my_n = tid < n ? n : 0;  // threads that own no key skip the count
    for (; i + 4 <= my_n; i += 4) {
        const uint64_t o0 = cand[i], o1 = cand[i + 1], o2 = cand[i + 2], o3 = cand[i + 3];
#pragma unroll
        for (int j = 0; j < kPer; ++j)
            rank[j] += static_cast<int>(o0 > mine[j]) + static_cast<int>(o1 > mine[j]) + static_cast<int>(o2 > mine[j]) +
                       static_cast<int>(o3 > mine[j]);
    }
    for (; i < my_n; ++i) {
        const uint64_t o = cand[i];
#pragma unroll
        for (int j = 0; j < kPer; ++j) rank[j] += static_cast<int>(o > mine[j]);
    }
    group_sync<kNT>();
    const int K = n < k ? n : k;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
        const int i2 = tid + j * kNT;
        if (i2 < n && rank[j] < K) cand[rank[j]] = mine[j];
    }
    group_sync<kNT>();
    return K;
}

// The K = min(k, n) largest keys of cand[0, n), sorted descending, in cand[0, K). Large sets are
// first cut to k by the radix select; up to kNT keys are then ranked (O(n^2 / kNT) compares, one
// barrier), more are sorted by the bitonic network (O(n log^2 n / kNT), a barrier per pass).
// n <= kCap (the buffer), k <= 1024; cand has room for 1024 keys.
// The same for k <= kNT: a radix cut (when n > 2 kNT), then the ranking.
template <int kNT, int kCap>
__device__ int topk_select_sorted_small_k(uint64_t* cand, int n, int k, TopkShared* sh) {
    if (n > 2 * kNT) n = topk_select_compact<kNT, (kCap + kNT - 1) / kNT>(cand, n, k, sh);
    if (n <= kNT) return topk_rank_sort<kNT, 1>(cand, n, k);
    return topk_rank_sort<kNT, 2>(cand, n, k);
}

template <int kNT, int kCap>
__device__ int topk_select_sorted(uint64_t* cand, int n, int k, TopkShared* sh) {
    static_assert(kCap >= 1024, "the bitonic sort of up to 1024 keys works in place");
    if (n > 2 * kNT) n = topk_select_compact<kNT, (kCap + kNT - 1) / kNT>(cand, n, k, sh);
    if (n <= kNT) return topk_rank_sort<kNT, 1>(cand, n, k);
    if (n > k) n = topk_select_compact<kNT, (kCap + kNT - 1) / kNT>(cand, n, k, sh);
    if (n <= kNT) return topk_rank_sort<kNT, 1>(cand, n, k);
    topk_sort_desc<kNT>(cand, n, next_pow2(n));
    return n;
}


// Monotone map of non-NaN floats to int32 (distinguishes -0 < +0), and back.
__device__ __forceinline__ int32_t float_to_ordinal(float x) {
    const int32_t b = __float_as_int(x);
    return b < 0 ? (b ^ 0x7fffffff) : b;
}
__device__ __forceinline__ float ordinal_to_float(int32_t k) { return __int_as_float(k < 0 ? (k ^ 0x7fffffff) : k); }

__device__ __forceinline__ float tempered(float x, float T, bool greedy) { return greedy ? x : __fdiv_rn(x, T); }

// A float X with tempered(x) < t for every x < X (t not NaN): X is at most the exact inverse
// computed below, so filtering on x >= X drops only elements that tempered(x) < t rules out. It
// starts a few ulps under t * T and checks that tempered(X) < t (then X lies below the exact
// boundary by monotonicity); one or two divides instead of a search.
__device__ inline float inverse_threshold(float t, float T, bool greedy);

__device__ __forceinline__ float inverse_threshold_bound(float t, float T, bool greedy) {
    if (greedy || t == -__int_as_float(0x7f800000)) return t;
    const float guess = __fmul_rn(t, T);
    if (guess == guess && guess != __int_as_float(0x7f800000) && guess != -__int_as_float(0x7f800000)) {
        int64_t o = float_to_ordinal(guess) - 4;
        for (int i = 0; i < 8; ++i, o -= 8) {
            if (o <= float_to_ordinal(-__int_as_float(0x7f800000))) break;
            const float x = ordinal_to_float(static_cast<int32_t>(o));
            if (tempered(x, T, false) < t) return x;  // every x' <= x has tempered(x') < t too
        }
    }
    return inverse_threshold(t, T, greedy);
}

// The smallest float x with tempered(x) >= t (t not NaN): every x below it has tempered(x) < t.
// Division by T > 0 in round-to-nearest is monotone, so a search over ordinals finds it exactly:
// gallop from the estimate t * T to bracket the boundary, then bisect.
__device__ inline float inverse_threshold(float t, float T, bool greedy) {
    if (greedy) return t;
    if (t == -__int_as_float(0x7f800000)) return t;
    // predicate(o) = tempered(ordinal_to_float(o)) >= t; false at -inf (t > -inf), true at +inf
    int64_t lo = float_to_ordinal(-__int_as_float(0x7f800000));
    int64_t hi = float_to_ordinal(__int_as_float(0x7f800000));
    const float guess = __fmul_rn(t, T);
    if (guess == guess) {
        const int64_t a = float_to_ordinal(guess);
        if (a > lo && a < hi) {
            if (tempered(ordinal_to_float(static_cast<int32_t>(a)), T, false) >= t) {
                hi = a;
                for (int64_t step = 1; hi - lo > 1 && step < (int64_t(1) << 32); step <<= 1) {
                    const int64_t b = hi - step;
                    if (b <= lo) break;
                    if (tempered(ordinal_to_float(static_cast<int32_t>(b)), T, false) >= t) {
                        hi = b;
                    } else {
                        lo = b;
                        break;
                    }
                }
            } else {
                lo = a;
                for (int64_t step = 1; hi - lo > 1 && step < (int64_t(1) << 32); step <<= 1) {
                    const int64_t b = lo + step;
                    if (b >= hi) break;
                    if (tempered(ordinal_to_float(static_cast<int32_t>(b)), T, false) >= t) {
                        hi = b;
                        break;
                    }
                    lo = b;
                }
            }
        }
    }
    while (hi - lo > 1) {
        const int64_t mid = lo + ((hi - lo) >> 1);
        if (tempered(ordinal_to_float(static_cast<int32_t>(mid)), T, false) >= t) hi = mid;
        else lo = mid;
    }
    return ordinal_to_float(static_cast<int32_t>(hi));
}

// The survivor decision on keys sorted best-first, by warp 0 only (the other threads skip it):
// weights, sequential prefix sums, top-p cutoff and draw, exactly as the oracle orders them.
// e and S are scratch arrays of K doubles.
__device__ inline void decide_warp(const uint64_t* keys, int K, float top_p, float u, double* e, double* S, int32_t* id_out,
                            float* prob_out, float* y_out) {
    const int lane = threadIdx.x & 31;
    const float m = rank_key_value(keys[0]);
    for (int i = lane; i < K; i += 32) e[i] = loom_survivor_weight(rank_key_value(keys[i]), m);
    __syncwarp();
    if (lane == 0) {
        double acc = e[0];
        S[0] = acc;
        for (int i = 1; i < K; ++i) {
            acc = __dadd_rn(acc, e[i]);
            S[i] = acc;
        }
    }
    __syncwarp();
    const double target = __dmul_rn(static_cast<double>(top_p), S[K - 1]);
    int n = K;
    for (int base = 0; base < K; base += 32) {
        const int j = base + lane;
        const uint32_t hit = __ballot_sync(0xffffffffu, j < K && S[j] >= target);
        if (hit) {
            n = base + __ffs(hit);
            break;
        }
    }
    const double draw = __dmul_rn(static_cast<double>(u), S[n - 1]);
    int sel = n - 1;
    for (int base = 0; base < n; base += 32) {
        const int i = base + lane;
        const uint32_t hit = __ballot_sync(0xffffffffu, i < n && draw < S[i]);
        if (hit) {
            sel = base + __ffs(hit) - 1;
            break;
        }
    }
    if (lane == 0) {
        *id_out = rank_key_id(keys[sel]);
        *prob_out = __double2float_rn(__ddiv_rn(e[sel], S[n - 1]));
        *y_out = rank_key_value(keys[sel]);
    }
    __syncwarp();
}

}  // namespace loom_select
