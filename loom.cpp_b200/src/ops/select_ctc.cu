// select_ctc.cu -- short rows, one warp per row: batched argmax of short rows and greedy CTC (K3).
//
// CTC replaces ctc_greedy_decode (src/core/ctc_decode.cpp:7-31) and the per-frame
// ggml_backend_tensor_get + scan of argmax_tensor_rows (src/core/lua_bridge.cpp:343-365):
//   1. per frame: argmax of the raw logits (strict '>' scan rule, NaN in column 0 wins), optionally
//      its log-softmax value;
//   2. per utterance, once all its frames are done (by the CTA holding it whole, or -- for an
//      utterance split across CTAs -- by the CTA that completes its atomic frame count; nothing
//      waits): keep frame f when id[f] != id[f-1] (id[-1] = blank) and id[f] != blank, then a block
//      scan compacts the kept ids and their frame indices.
// Each persistent CTA owns a contiguous, equal share of the n_utt * n_frames frames.
// Bound: HBM bandwidth (one read of the logits; the per-frame ids are 4 bytes per frame).
#include <cstdint>

#include <atomic>

#include "select_internal.h"
#include "select_rows.cuh"
#include "select_stream.cuh"

namespace loom_select {

namespace {

constexpr int kRowWarps = 8;
constexpr int kRowNT = kRowWarps * 32;

// ----------------------------------------------------------------------------------------------
// batched argmax of short rows

template <int kDtype>
__global__ void __launch_bounds__(kRowNT) rows_argmax_kernel(const unsigned char* base, int64_t rows, int64_t width,
                                                             int64_t stride_bytes, int64_t lo, int32_t* out_ids) {
    const int lane = threadIdx.x & 31;
    const int64_t gw = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t nw = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    for (int64_t r = gw; r < rows; r += nw) {
        const unsigned char* row = base + r * stride_bytes;
        ArgBest best;
        LseAcc lse;
        warp_row_reduce<kDtype, false>(row, width, best, lse);
        if (lane == 0) {
            const float x0 = load_global_elem<kDtype>(row, 0);
            out_ids[r] = static_cast<int32_t>(lo + ((x0 != x0) ? 0 : best.i));
        }
    }
}

// ----------------------------------------------------------------------------------------------
// CTC

constexpr int kMaxUttPerCta = 64;
static_assert(kCtcMaxUtt == kTicketSlots * (kMaxUttPerCta - 2), "CTC utterance bound");

struct CtcShared {
    int n_last;
    int64_t last_utt[kMaxUttPerCta];
    int last_ticket[kMaxUttPerCta]; // -1: the utterance lies wholly in this CTA
    int warp_tot[kRowWarps];
};

// Frames are split evenly: CTA c owns [c * total / G, (c + 1) * total / G).
__device__ __forceinline__ int64_t ctc_range_start(int64_t c, int64_t total, int64_t G) { return c * total / G; }

// Compacts utterance u's kept frames. Called by the whole CTA. Each thread takes kCollapsePer
// consecutive frames (their ids loaded at once), and one block scan per pass places the kept ones.
constexpr int kCollapsePer = 8;

__device__ void ctc_collapse(int64_t u, int64_t n_frames, int32_t blank, const int32_t* frame_ids, int32_t* out_ids,
                             int32_t* out_frames, int32_t* out_len, CtcShared* sh) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const bool act = threadIdx.x < kRowNT;  // a CTA's further warps (a producer) only meet the barriers
    const int32_t* ids = frame_ids + u * n_frames;
    int carry = 0;  // frames kept by the earlier passes (the same in every thread)
    for (int64_t base = 0; base < n_frames; base += static_cast<int64_t>(kRowNT) * kCollapsePer) {
        const int64_t f0 = act ? base + static_cast<int64_t>(threadIdx.x) * kCollapsePer : n_frames + 1;
        int32_t v[kCollapsePer];
        const int32_t prev0 = (f0 == 0 || f0 > n_frames) ? blank : __ldcg(ids + f0 - 1);
#pragma unroll
        for (int j = 0; j < kCollapsePer; ++j) v[j] = f0 + j < n_frames ? __ldcg(ids + f0 + j) : blank;
        uint32_t keep = 0;
#pragma unroll
        for (int j = 0; j < kCollapsePer; ++j) {
            const int32_t prev = j == 0 ? prev0 : v[j - 1];
            keep |= static_cast<uint32_t>(f0 + j < n_frames && v[j] != prev && v[j] != blank) << j;
        }
        const int cnt = __popc(keep);
        int incl = cnt;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int o = __shfl_up_sync(0xffffffffu, incl, off);
            if (lane >= off) incl += o;
        }
        if (lane == 31 && act) sh->warp_tot[warp] = incl;
        __syncthreads();
        int pos = carry + incl - cnt, total = 0;
        for (int w = 0; w < kRowWarps; ++w) {
            const int t = sh->warp_tot[w];
            if (w < warp) pos += t;
            total += t;
        }
#pragma unroll
        for (int j = 0; j < kCollapsePer; ++j) {
            if ((keep >> j) & 1u) {
                out_ids[u * n_frames + pos] = v[j];
                out_frames[u * n_frames + pos] = static_cast<int32_t>(f0 + j);
                ++pos;
            }
        }
        carry += total;
        __syncthreads();  // warp_tot is rewritten by the next pass
    }
    if (threadIdx.x == 0) out_len[u] = carry;
}

// After a CTA's frames [f_lo, f_hi) are all written: collapses the utterances it holds whole, and those
// split across CTAs whose frame count it completes (a ticket per split utterance, at the CTA holding
// its first frame; at most one split utterance starts in any CTA). `start(c)` gives CTA c's first frame.
template <class Start>
__device__ void ctc_finish_cta(int64_t f_lo, int64_t f_hi, int64_t n_utt, int64_t n_frames, int32_t blank,
                               const int32_t* frame_ids, int32_t* out_ids, int32_t* out_frames, int32_t* out_len,
                               int* tickets, CtcShared* sh, Start start) {
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        sh->n_last = 0;
        const int64_t G = gridDim.x;
        if (f_hi > f_lo) {
            const int64_t u0 = f_lo / n_frames, u1 = (f_hi - 1) / n_frames;
            for (int64_t u = u0; u <= u1; ++u) {
                const int64_t a = u * n_frames > f_lo ? u * n_frames : f_lo;
                const int64_t b = (u + 1) * n_frames < f_hi ? (u + 1) * n_frames : f_hi;
                const int n = static_cast<int>(b - a);
                if (n == n_frames) {
                    sh->last_utt[sh->n_last] = u;
                    sh->last_ticket[sh->n_last++] = -1;
                    continue;
                }
                // the CTA holding the utterance's first frame
                const int64_t f = u * n_frames;
                int64_t c = f * G / (n_utt * n_frames);
                if (c >= G) c = G - 1;
                while (c + 1 < G && start(c + 1) <= f) ++c;
                while (c > 0 && start(c) > f) --c;
                const int t = static_cast<int>(c);
                const int prev = atomicAdd(&tickets[t], n);
                if (prev + n == n_frames) {
                    sh->last_utt[sh->n_last] = u;
                    sh->last_ticket[sh->n_last++] = t;
                }
            }
        }
        __threadfence();
    }
    __syncthreads();
    const int n_last = sh->n_last;
    for (int j = 0; j < n_last; ++j) {
        const int64_t u = sh->last_utt[j];
        const int t = sh->last_ticket[j];
        ctc_collapse(u, n_frames, blank, frame_ids, out_ids, out_frames, out_len, sh);
        if (threadIdx.x == 0 && t >= 0) tickets[t] = 0;
    }
}

template <int kDtype, bool kLogp>
__global__ void __launch_bounds__(kRowNT) ctc_kernel(const unsigned char* logits, int64_t n_utt, int64_t n_frames,
                                                     int64_t n_classes, int32_t blank, int32_t* frame_ids,
                                                     float* frame_logp, int32_t* out_ids, int32_t* out_frames,
                                                     int32_t* out_len, int* tickets) {
    constexpr int kEsz = (kDtype == LOOM_SELECT_BF16) ? 2 : 4;
    __shared__ CtcShared sh;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t total = n_utt * n_frames;
    const int64_t f_lo = static_cast<int64_t>(blockIdx.x) * total / gridDim.x;
    const int64_t f_hi = static_cast<int64_t>(blockIdx.x + 1) * total / gridDim.x;
    const int64_t row_bytes = n_classes * kEsz;
    for (int64_t f = f_lo + warp; f < f_hi; f += kRowWarps) {
        const unsigned char* row = logits + f * row_bytes;
        ArgBest best;
        LseAcc lse;
        warp_row_reduce<kDtype, kLogp>(row, n_classes, best, lse);
        if (lane == 0) {
            const float x0 = load_global_elem<kDtype>(row, 0);
            const bool nan0 = x0 != x0;
            frame_ids[f] = nan0 ? 0 : best.i;
            if constexpr (kLogp) {
                const double lp = nan0 ? static_cast<double>(x0)
                                       : static_cast<double>(best.v) -
                                             (static_cast<double>(lse.m) + log(static_cast<double>(lse.s)));
                frame_logp[f] = static_cast<float>(lp);
            }
        }
    }
    ctc_finish_cta(f_lo, f_hi, n_utt, n_frames, blank, frame_ids, out_ids, out_frames, out_len, tickets, &sh,
                   [&](int64_t c) { return ctc_range_start(c, total, gridDim.x); });
}


// ----------------------------------------------------------------------------------------------
// CTC through a ring of bulk copies (K3r). A CTA's frames are one contiguous byte range; eight
// frames of C classes are 8 * C * esz bytes, a multiple of 16 for 2- and 4-byte elements, so when
// every CTA's range starts at a multiple of eight frames of a 16-byte-aligned tensor each stage is
// one legal bulk copy of eight whole frames. A producer warp issues them (cp.async.bulk, mbarrier
// completion, no multicast); consumer warp w reduces frame w of each stage from shared memory. The
// at most seven frames past the last multiple of eight are read from global memory by the last CTA.

constexpr int kRingStages = 3;
constexpr int kRingFrames = kRowWarps;  // one frame per consumer warp and stage
constexpr int kRingThreads = (kRowWarps + 1) * 32;
constexpr int64_t kRingMaxStageBytes = 36864;

struct CtcRingCtl {
    uint64_t full[kRingStages];
    uint64_t empty[kRingStages];
    int abort;
    int issued;
    int waited[kRowWarps];
};

// First frame of CTA c: ranges over the first t8 frames (t8 a multiple of eight) start at multiples
// of eight; the last CTA also holds the frames past t8.
__device__ __forceinline__ int64_t ring_start(int64_t c, int64_t t8, int64_t G, int64_t total) {
    if (c >= G) return total;
    const int64_t p = c * t8 / G;
    return p - p % kRingFrames;
}

template <int kDtype>
__device__ __forceinline__ float smem_frame_elem(const unsigned char* fr, int64_t j) {
    if constexpr (kDtype == LOOM_SELECT_BF16) return bf16_bits_to_float(reinterpret_cast<const unsigned short*>(fr)[j]);
    else return reinterpret_cast<const float*>(fr)[j];
}

template <int kDtype, bool kLogp>
__device__ __forceinline__ void write_frame(int64_t f, ArgBest best, LseAcc lse, bool nan0, int32_t* frame_ids,
                                            float* frame_logp) {
    frame_ids[f] = nan0 ? 0 : best.i;
    if constexpr (kLogp) {
        const double lp = nan0 ? static_cast<double>(__int_as_float(0x7fc00000))
                               : static_cast<double>(best.v) -
                                     (static_cast<double>(lse.m) + log(static_cast<double>(lse.s)));
        frame_logp[f] = static_cast<float>(lp);
    }
}

template <int kDtype, bool kLogp>
__global__ void __launch_bounds__(kRingThreads, 2)
    ctc_ring_kernel(const unsigned char* logits, int64_t n_utt, int64_t n_frames, int64_t n_classes, int32_t blank,
                    int32_t* frame_ids, float* frame_logp, int32_t* out_ids, int32_t* out_frames, int32_t* out_len,
                    int* tickets, int* status) {
    constexpr int kEsz = (kDtype == LOOM_SELECT_BF16) ? 2 : 4;
    extern __shared__ __align__(128) unsigned char ring[];
    __shared__ CtcRingCtl ctl;
    __shared__ CtcShared sh;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t total = n_utt * n_frames;
    const int64_t t8 = total - total % kRingFrames;
    const int64_t G = gridDim.x, c = blockIdx.x;
    const int64_t f_lo = ring_start(c, t8, G, total);
    const int64_t f_ring_hi = c + 1 < G ? ring_start(c + 1, t8, G, total) : t8;
    const int64_t f_hi = c + 1 < G ? f_ring_hi : total;
    const int64_t row_bytes = n_classes * kEsz;
    const uint32_t stage_bytes = static_cast<uint32_t>(kRingFrames * row_bytes);
    const int n_stages = static_cast<int>((f_ring_hi - f_lo) / kRingFrames);

    if (threadIdx.x == 0) {
        for (int i = 0; i < kRingStages; ++i) {
            mbar_init(&ctl.full[i], 1);
            mbar_init(&ctl.empty[i], kRowWarps);
        }
        ctl.abort = 0;
        ctl.issued = 0;
        mbar_fence_init();
    }
    __syncthreads();

    if (warp == kRowWarps) {
        // ---------------- producer ----------------
        int it = 0;
        for (; it < n_stages; ++it) {
            const int slot = it % kRingStages;
            int ok = 1;
            if (lane == 0) {
                ok = mbar_wait_abortable(&ctl.empty[slot], ((it / kRingStages) & 1) ^ 1, status, &ctl.abort) ? 1 : 0;
                if (!ok) {
                    atomicExch(&ctl.abort, 1);
                } else {
                    mbar_arrive_expect_tx(&ctl.full[slot], stage_bytes);
                    bulk_g2s(ring + static_cast<size_t>(slot) * stage_bytes,
                             logits + (f_lo + static_cast<int64_t>(it) * kRingFrames) * row_bytes, stage_bytes,
                             &ctl.full[slot]);
                }
            }
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
        }
        if (lane == 0) ctl.issued = it;
    } else {
        // ---------------- consumers: frame `warp` of each stage ----------------
        int waited = 0;
        for (int it = 0; it < n_stages; ++it) {
            const int slot = it % kRingStages;
            if (!warp_wait_bounded(&ctl.full[slot], (it / kRingStages) & 1, status, &ctl.abort)) {
                if (lane == 0) atomicExch(&ctl.abort, 1);
                break;
            }
            waited = it + 1;
            const unsigned char* fr = ring + static_cast<size_t>(slot) * stage_bytes + warp * row_bytes;
            ArgBest best = arg_init();
            LseAcc lse = lse_init();
            float x0 = 0.0f;
            for (int64_t j = lane; j < n_classes; j += 32) {
                const float x = smem_frame_elem<kDtype>(fr, j);
                if (j == 0) x0 = x;
                arg_offer(best, x, static_cast<int32_t>(j));
                if constexpr (kLogp) lse_offer(lse, x);
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&ctl.empty[slot]);
            const float c0 = __shfl_sync(0xffffffffu, x0, 0);
            best = arg_warp_reduce(best);
            if constexpr (kLogp) lse = lse_warp_reduce(lse);
            if (lane == 0)
                write_frame<kDtype, kLogp>(f_lo + static_cast<int64_t>(it) * kRingFrames + warp, best, lse, c0 != c0,
                                           frame_ids, frame_logp);
        }
        if (lane == 0) ctl.waited[warp] = waited;
        // the frames past t8 (last CTA only), one warp per frame from global memory
        for (int64_t f = f_ring_hi + warp; f < f_hi; f += kRowWarps) {
            const unsigned char* row = logits + f * row_bytes;
            ArgBest best;
            LseAcc lse;
            warp_row_reduce<kDtype, kLogp>(row, n_classes, best, lse);
            const float c0 = load_global_elem<kDtype>(row, 0);
            if (lane == 0) write_frame<kDtype, kLogp>(f, best, lse, c0 != c0, frame_ids, frame_logp);
        }
    }
    __syncthreads();
    // drain: every bulk copy issued has landed before the shared memory goes away
    if (threadIdx.x == 0) {
        int from = ctl.issued;
        for (int w = 0; w < kRowWarps; ++w) from = ctl.waited[w] < from ? ctl.waited[w] : from;
        for (int i = from; i < ctl.issued; ++i)
            if (!mbar_wait_bounded(&ctl.full[i % kRingStages], (i / kRingStages) & 1, status)) break;
    }
    ctc_finish_cta(f_lo, f_hi, n_utt, n_frames, blank, frame_ids, out_ids, out_frames, out_len, tickets, &sh,
                   [&](int64_t cc) { return ring_start(cc, t8, G, total); });
}

}  // namespace

cudaError_t launch_rows_argmax(int dtype, const void* window_base, int64_t rows, int64_t width, int64_t row_stride,
                               int64_t lo, int32_t* out_ids, int sms, cudaStream_t stream) {
    const int64_t want = (rows + kRowWarps - 1) / kRowWarps;
    const int64_t cap = static_cast<int64_t>(sms) * 8;
    const int grid = static_cast<int>(want < cap ? want : cap);
    const unsigned char* base = static_cast<const unsigned char*>(window_base);
    if (dtype == LOOM_SELECT_BF16)
        rows_argmax_kernel<LOOM_SELECT_BF16><<<grid, kRowNT, 0, stream>>>(base, rows, width, row_stride * 2, lo, out_ids);
    else
        rows_argmax_kernel<LOOM_SELECT_F32><<<grid, kRowNT, 0, stream>>>(base, rows, width, row_stride * 4, lo, out_ids);
    return cudaGetLastError();
}

cudaError_t launch_ctc(int dtype, const void* logits, int64_t n_utt, int64_t n_frames, int64_t n_classes,
                       int32_t blank, int32_t* out_ids, int32_t* out_frames, int32_t* out_len, int32_t* frame_ids,
                       float* frame_logp, void* workspace, const WsLayout& l, int sms, cudaStream_t stream) {
    unsigned char* ws = static_cast<unsigned char*>(workspace);
    int* tickets = reinterpret_cast<int*>(ws + l.tickets);
    if (!frame_ids) frame_ids = reinterpret_cast<int32_t*>(ws + l.records);
    const int64_t total = n_utt * n_frames;
    const bool lp = frame_logp != nullptr;
    // the ring: a 16-byte-aligned tensor, eight frames per stage within kRingMaxStageBytes, two CTAs
    // per SM, and no CTA range (at most ceil(t8 / G) + 15 frames) holding more than kMaxUttPerCta - 2
    // whole utterances
    {
        const int esz = dtype == LOOM_SELECT_BF16 ? 2 : 4;
        const int64_t stage = kRingFrames * n_classes * esz;
        const int64_t G = 2 * static_cast<int64_t>(sms);
        const int64_t t8 = total - total % kRingFrames;
        const int64_t max_range = (t8 + G - 1) / G + 2 * kRingFrames;
        if (reinterpret_cast<uintptr_t>(logits) % 16 == 0 && stage <= kRingMaxStageBytes && G <= kTicketSlots &&
            max_range <= (kMaxUttPerCta - 2) * n_frames) {
            const size_t smem = static_cast<size_t>(kRingStages) * static_cast<size_t>(stage);
            static std::atomic<bool> configured[64] = {};  // set once per device, from any host thread
            int dev = 0;
            cudaGetDevice(&dev);
            if (dev >= 0 && dev < 64 && !configured[dev]) {
                const int max_smem = static_cast<int>(kRingStages * kRingMaxStageBytes);
                cudaError_t e = cudaSuccess;
                if ((e = cudaFuncSetAttribute(ctc_ring_kernel<LOOM_SELECT_F32, false>,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem)) != cudaSuccess ||
                    (e = cudaFuncSetAttribute(ctc_ring_kernel<LOOM_SELECT_F32, true>,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem)) != cudaSuccess ||
                    (e = cudaFuncSetAttribute(ctc_ring_kernel<LOOM_SELECT_BF16, false>,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem)) != cudaSuccess ||
                    (e = cudaFuncSetAttribute(ctc_ring_kernel<LOOM_SELECT_BF16, true>,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem)) != cudaSuccess)
                    return e;
                configured[dev] = true;
            }
            const unsigned char* base = static_cast<const unsigned char*>(logits);
            int* status = reinterpret_cast<int*>(ws);
#define LOOM_CTC_RING(DT, LP)                                                                                        \
    ctc_ring_kernel<DT, LP><<<static_cast<int>(G), kRingThreads, smem, stream>>>(base, n_utt, n_frames, n_classes,   \
                                                                                 blank, frame_ids, frame_logp,       \
                                                                                 out_ids, out_frames, out_len,       \
                                                                                 tickets, status)
            if (dtype == LOOM_SELECT_BF16) {
                if (lp) LOOM_CTC_RING(LOOM_SELECT_BF16, true);
                else LOOM_CTC_RING(LOOM_SELECT_BF16, false);
            } else {
                if (lp) LOOM_CTC_RING(LOOM_SELECT_F32, true);
                else LOOM_CTC_RING(LOOM_SELECT_F32, false);
            }
#undef LOOM_CTC_RING
            return cudaGetLastError();
        }
    }
    // otherwise one warp per frame: enough CTAs that none holds more than kMaxUttPerCta - 2 whole
    // utterances, at most one ticket slot per CTA (the caller checked n_utt <= kCtcMaxUtt)
    int64_t grid = static_cast<int64_t>(sms) * 4;
    const int64_t min_grid = (n_utt + kMaxUttPerCta - 3) / (kMaxUttPerCta - 2);
    if (grid < min_grid) grid = min_grid;
    if (grid > kTicketSlots) grid = kTicketSlots;
    if (grid > total) grid = total;
    const unsigned char* base = static_cast<const unsigned char*>(logits);
#define LOOM_CTC_LAUNCH(DT, LP)                                                                                     \
    ctc_kernel<DT, LP><<<static_cast<int>(grid), kRowNT, 0, stream>>>(base, n_utt, n_frames, n_classes, blank,      \
                                                                       frame_ids, frame_logp, out_ids, out_frames, \
                                                                       out_len, tickets)
    if (dtype == LOOM_SELECT_BF16) {
        if (lp) LOOM_CTC_LAUNCH(LOOM_SELECT_BF16, true);
        else LOOM_CTC_LAUNCH(LOOM_SELECT_BF16, false);
    } else {
        if (lp) LOOM_CTC_LAUNCH(LOOM_SELECT_F32, true);
        else LOOM_CTC_LAUNCH(LOOM_SELECT_F32, false);
    }
#undef LOOM_CTC_LAUNCH
    return cudaGetLastError();
}

}  // namespace loom_select
