// select_stream.cuh -- persistent row streaming through shared memory (sm_100a).
//
// The logits of a call are a [rows, width] window of a row-major matrix (row stride `row_stride`
// elements). The flat index space rows*width is cut into `ctas` contiguous ranges of (almost) equal
// size, one per persistent CTA, so every SM reads the same number of bytes whatever the row count.
// A range covers pieces of one or more rows ("segments"). A row cut by a range boundary has several
// segments in different CTAs; each writes a partial result, and the CTA that finishes the row's last
// segment (an atomic ticket per row, no waiting) merges them.
//
// Within a CTA one producer warp streams the 16-byte-aligned interior of each segment into a ring of
// kStages shared-memory stages with bulk copies (cp.async.bulk, completion on an mbarrier), running
// ahead across segment and row boundaries; the consumer warps read stages from shared memory. The
// at most 15 elements of a segment outside its aligned interior ("edges") are read from global
// memory by the consumers. No tensor map, no cluster, no multicast.
#pragma once

#include "select_device.cuh"
#include "select_internal.h"

namespace loom_select {

constexpr int64_t kSplitAlign = kStreamSplitAlign; // range boundaries are multiples of this many elements

struct StreamGeom {
    const unsigned char* base; // element (0, 0) of the window
    int64_t rows;
    int64_t width;      // window width in elements
    int64_t row_stride; // elements between row starts
    int64_t total;      // rows * width
    int32_t esz;        // element size in bytes
    int32_t ctas;       // number of persistent CTAs (ranges)
};

// Start of range c (its end is split_point(c + 1)). With at least as many rows as ranges, ranges are
// whole rows (range c: rows [c * rows / ctas, (c + 1) * rows / ctas)), so no row is split and no
// partial results are merged; otherwise the flat index space is cut into equal pieces.
__host__ __device__ __forceinline__ int64_t split_point(const StreamGeom& g, int64_t c) {
    if (c >= g.ctas) return g.total;
    if (g.rows >= g.ctas) return (c * g.rows / g.ctas) * g.width;
    const int64_t p = c * g.total / g.ctas;
    return p - p % kSplitAlign;
}

// The range that holds flat element e.
__device__ __forceinline__ int64_t range_of(const StreamGeom& g, int64_t e) {
    int64_t c = e * g.ctas / g.total;
    if (c >= g.ctas) c = g.ctas - 1;
    while (c + 1 < g.ctas && split_point(g, c + 1) <= e) ++c;
    while (c > 0 && split_point(g, c) > e) --c;
    return c;
}

struct Segment {
    int64_t row;
    int64_t j0, j1;   // columns [j0, j1) of the window
    int32_t index;    // this segment's index among the row's segments
    int32_t count;    // number of segments of the row
    int64_t first_cta; // the range holding the row's first element (segment j is range first_cta + j)
    // byte geometry
    const unsigned char* a0; // address of column j0
    const unsigned char* A0; // first 16-byte boundary >= a0 (clamped to a1)
    const unsigned char* A1; // last 16-byte boundary <= a1 (>= A0)
    const unsigned char* a1; // address of column j1
    int32_t n_chunks;
};

// Segment of range c in `row`; lo and hi are the range's bounds (split_point(g, c), split_point(g, c + 1)).
// A row that starts at or after lo and ends at or before hi lies wholly in the range (no search).
template <int kStageBytes>
__device__ __forceinline__ Segment make_segment(const StreamGeom& g, int64_t c, int64_t row, int64_t lo, int64_t hi) {
    Segment s;
    const int64_t rs = row * g.width;
    s.row = row;
    s.j0 = (lo > rs ? lo : rs) - rs;
    s.j1 = (hi < rs + g.width ? hi : rs + g.width) - rs;
    if (rs >= lo && rs + g.width <= hi) {
        s.index = 0;
        s.count = 1;
        s.first_cta = c;
    } else {
        const int64_t c0 = range_of(g, rs);
        const int64_t c1 = range_of(g, rs + g.width - 1);
        s.index = static_cast<int32_t>(c - c0);
        s.count = static_cast<int32_t>(c1 - c0 + 1);
        s.first_cta = c0;
    }
    const unsigned char* rowp = g.base + row * g.row_stride * g.esz;
    s.a0 = rowp + s.j0 * g.esz;
    s.a1 = rowp + s.j1 * g.esz;
    const uintptr_t up = (reinterpret_cast<uintptr_t>(s.a0) + 15) & ~uintptr_t(15);
    const uintptr_t dn = reinterpret_cast<uintptr_t>(s.a1) & ~uintptr_t(15);
    if (up < dn) {
        s.A0 = reinterpret_cast<const unsigned char*>(up);
        s.A1 = reinterpret_cast<const unsigned char*>(dn);
    } else {
        s.A0 = s.a1;
        s.A1 = s.a1;
    }
    s.n_chunks = static_cast<int32_t>((s.A1 - s.A0 + kStageBytes - 1) / kStageBytes);
    return s;
}

// Workspace record slot of range c's piece of `row` (a range splits only its first and last row).
__device__ __forceinline__ int64_t record_slot(const StreamGeom& g, int64_t c, int64_t row) {
    return 2 * c + (row == split_point(g, c) / g.width ? 0 : 1);
}

// Edge element e (0 <= e < n_edges) of a segment: its column. Edges are the head [a0, A0) then the
// tail [A1, a1).
__device__ __forceinline__ int32_t segment_edge_count(const Segment& s, int esz) {
    return static_cast<int32_t>(((s.A0 - s.a0) + (s.a1 - s.A1)) / esz);
}

__device__ __forceinline__ int64_t segment_edge_col(const Segment& s, int esz, int32_t e) {
    const int32_t head = static_cast<int32_t>((s.A0 - s.a0) / esz);
    if (e < head) return s.j0 + e;
    return s.j0 + ((s.A1 - s.a0) / esz) + (e - head);
}

// Shared control block of the streamer.
struct StreamCtl {
    uint64_t full[16];
    uint64_t empty[16];
    int abort;
    int issued;
    int consumed;
    int waited[16];  // stream_ranges_warps: stages each consumer warp saw land
    uint64_t limit_ns;  // stream_ranges_warps: the bound of every wait (see WaitFault)
    int withhold;       // stream_ranges_warps: a stage CTA 0 leaves unissued (index + 1), or 0
};

// The persistent CTA body. Consumers are warps [0, kConsumerWarps); warp kConsumerWarps produces.
// Op hooks, all called by every consumer thread (they may use named barrier 1 over the consumers):
//   op.begin_segment(seg)                      before the segment's first chunk (reads its edges)
//   op.chunk(seg, data, col0, n)               n elements of columns [col0, col0 + n) in shared memory
//   op.end_chunk(seg)                          after the chunk, before its stage is released
//   op.end_segment(seg)                        after the segment's last chunk
template <int kStages, int kStageBytes, int kConsumerWarps, class Op>
__device__ void stream_ranges(const StreamGeom g, Op& op, unsigned char* ring, StreamCtl* ctl, int* status) {
    static_assert(kStages <= 16, "ring too deep");
    static_assert(kStageBytes % 16 == 0, "stage must be a multiple of 16 bytes");
    constexpr int kConsumers = kConsumerWarps * 32;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int64_t c = blockIdx.x;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&ctl->full[i], 1);
            mbar_init(&ctl->empty[i], kConsumerWarps);
        }
        ctl->abort = 0;
        ctl->issued = 0;
        ctl->consumed = 0;
        mbar_fence_init();
    }
    __syncthreads();

    const int64_t lo = split_point(g, c), hi = split_point(g, c + 1);
    const int64_t row_first = lo / g.width;
    const int64_t row_last = hi > lo ? (hi - 1) / g.width : row_first - 1;

    if (warp == kConsumerWarps) {
        // ---------------- producer ----------------
        // The whole warp walks the loop (so it reaches the final barrier converged); lane 0 waits
        // and issues, and its decisions are broadcast.
        int it = 0;
        bool stop = false;
        for (int64_t r = row_first; r <= row_last && !stop; ++r) {
            const Segment s = make_segment<kStageBytes>(g, c, r, lo, hi);
            for (int32_t k = 0; k < s.n_chunks; ++k) {
                const int slot = it % kStages;
                const uint32_t parity = ((it / kStages) & 1) ^ 1;
                int ok = 1;
                if (lane == 0) {
                    ok = mbar_wait_bounded(&ctl->empty[slot], parity, status) ? 1 : 0;
                    if (!ok) atomicExch(&ctl->abort, 1);
                    if (*reinterpret_cast<volatile int*>(&ctl->abort)) ok = 0;
                }
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) {
                    stop = true;
                    break;
                }
                if (lane == 0) {
                    const unsigned char* src = s.A0 + static_cast<int64_t>(k) * kStageBytes;
                    const int64_t left = s.A1 - src;
                    const uint32_t bytes = static_cast<uint32_t>(left < kStageBytes ? left : kStageBytes);
                    mbar_arrive_expect_tx(&ctl->full[slot], bytes);
                    bulk_g2s(ring + static_cast<size_t>(slot) * kStageBytes, src, bytes, &ctl->full[slot]);
                }
                __syncwarp();
                ++it;
            }
        }
        if (lane == 0) ctl->issued = it;
    } else {
        // ---------------- consumers ----------------
        int it = 0;
        bool stop = false;
        for (int64_t r = row_first; r <= row_last && !stop; ++r) {
            const Segment s = make_segment<kStageBytes>(g, c, r, lo, hi);
            op.begin_segment(s);
            for (int32_t k = 0; k < s.n_chunks; ++k) {
                const int slot = it % kStages;
                const uint32_t parity = (it / kStages) & 1;
                // every consumer waits itself; the barrier ORs the timeouts so all decide alike
                const bool late = !mbar_wait_bounded(&ctl->full[slot], parity, status);
                if (named_barrier_or(1, kConsumers, late)) {
                    if (threadIdx.x == 0) atomicExch(&ctl->abort, 1);
                    stop = true;
                    break;
                }
                const unsigned char* src = s.A0 + static_cast<int64_t>(k) * kStageBytes;
                const int64_t left = s.A1 - src;
                const int32_t bytes = static_cast<int32_t>(left < kStageBytes ? left : kStageBytes);
                const int esz_log2 = g.esz == 4 ? 2 : 1;  // 4-byte or 2-byte elements
                const int64_t col0 = s.j0 + ((src - s.a0) >> esz_log2);
                op.chunk(s, ring + static_cast<size_t>(slot) * kStageBytes, col0, bytes >> esz_log2);
                op.end_chunk(s);
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&ctl->empty[slot]);
                ++it;
            }
            if (stop) break;
            op.end_segment(s);
        }
        if (threadIdx.x == 0) ctl->consumed = it;
    }
    __syncthreads();
    // Drain: every bulk copy issued must have landed before the CTA's shared memory goes away.
    if (threadIdx.x == 0) {
        for (int i = ctl->consumed; i < ctl->issued; ++i) {
            if (!mbar_wait_bounded(&ctl->full[i % kStages], (i / kStages) & 1, status)) break;
        }
    }
    __syncthreads();
}

// Waits, as a whole warp, for the phase of `bar` with the given parity: every lane polls the barrier
// (so each lane has the barrier's acquire), lane 0's clock and the abort flag decide for the warp.
// False when the wait runs out (recorded as LOOM_SELECT_ETIMEOUT) or another warp has aborted.
__device__ __forceinline__ bool warp_wait_bounded(uint64_t* bar, uint32_t parity, int* status_word, const int* abort,
                                                  uint64_t limit_ns = kWaitLimitNs) {
    if (__all_sync(0xffffffffu, mbar_try_wait(bar, parity))) return true;
    const uint64_t t0 = global_timer_ns();
    for (;;) {
        if (__all_sync(0xffffffffu, mbar_try_wait_sleep(bar, parity))) return true;
        int give_up = 0;
        if ((threadIdx.x & 31) == 0) {
            if (*reinterpret_cast<const volatile int*>(abort)) give_up = 1;
            else if (global_timer_ns() - t0 > limit_ns) give_up = 2;
        }
        give_up = __shfl_sync(0xffffffffu, give_up, 0);
        if (give_up) {
            if (give_up == 2 && (threadIdx.x & 31) == 0) record_status(status_word, LOOM_SELECT_ETIMEOUT);
            return false;
        }
    }
}

// mbar_wait_bounded for one thread that also gives up once another warp has aborted.
__device__ __forceinline__ bool mbar_wait_abortable(uint64_t* bar, uint32_t parity, int* status_word, const int* abort,
                                                    uint64_t limit_ns = kWaitLimitNs) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (;;) {
        if (mbar_try_wait_sleep(bar, parity)) return true;
        if (*reinterpret_cast<const volatile int*>(abort)) return false;
        if (global_timer_ns() - t0 > limit_ns) {
            record_status(status_word, LOOM_SELECT_ETIMEOUT);
            return false;
        }
    }
}

// The persistent CTA body with free-running consumer warps: each consumer warp waits for a stage
// and releases it by itself, so warps drift apart (by up to kStages stages) instead of meeting at a
// barrier every stage. The only CTA-wide barriers are the op's own, in begin_segment, in the first
// chunk of a segment and in end_segment; every consumer warp makes the same sequence of calls.
// A warp whose wait gives up raises the abort flag and goes on "dead": it no longer waits, reads or
// releases stages, but still makes every op call (chunk with live == false), so the op's barriers
// still match; the producer and the other warps see the flag and wind down the same way.
// Op hooks, all called by every consumer thread:
//   op.begin_segment(seg)
//   op.chunk(seg, data, col0, n, live)         live == false: touch no stage data
//   op.end_segment(seg)
template <int kStages, int kStageBytes, int kConsumerWarps, class Op>
__device__ void stream_ranges_warps(const StreamGeom g, Op& op, unsigned char* ring, StreamCtl* ctl, int* status) {
    static_assert(kStages <= 16 && kConsumerWarps <= 16, "control block sizes");
    static_assert(kStageBytes % 16 == 0, "stage must be a multiple of 16 bytes");
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int64_t c = blockIdx.x;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&ctl->full[i], 1);
            mbar_init(&ctl->empty[i], kConsumerWarps);
        }
        ctl->abort = 0;
        ctl->issued = 0;
        ctl->consumed = 0;
        const WaitFault f = read_wait_fault(status);
        ctl->limit_ns = f.limit_ns;
        ctl->withhold = blockIdx.x == 0 ? f.withhold : 0;
        mbar_fence_init();
    }
    __syncthreads();

    const int64_t lo = split_point(g, c), hi = split_point(g, c + 1);
    const int64_t row_first = lo / g.width;
    const int64_t row_last = hi > lo ? (hi - 1) / g.width : row_first - 1;

    if (warp == kConsumerWarps) {
        // ---------------- producer (as in stream_ranges, with abortable waits) ----------------
        int it = 0;
        bool stop = false;
        for (int64_t r = row_first; r <= row_last && !stop; ++r) {
            const Segment s = make_segment<kStageBytes>(g, c, r, lo, hi);
            for (int32_t k = 0; k < s.n_chunks; ++k) {
                const int slot = it % kStages;
                const uint32_t parity = ((it / kStages) & 1) ^ 1;
                int ok = 1;
                if (lane == 0) {
                    ok = mbar_wait_abortable(&ctl->empty[slot], parity, status, &ctl->abort, ctl->limit_ns) ? 1 : 0;
                    if (!ok) atomicExch(&ctl->abort, 1);
                }
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) {
                    stop = true;
                    break;
                }
                if (lane == 0 && it + 1 != ctl->withhold) {  // (the test hook leaves one stage unissued)
                    const unsigned char* src = s.A0 + static_cast<int64_t>(k) * kStageBytes;
                    const int64_t left = s.A1 - src;
                    const uint32_t bytes = static_cast<uint32_t>(left < kStageBytes ? left : kStageBytes);
                    mbar_arrive_expect_tx(&ctl->full[slot], bytes);
                    bulk_g2s(ring + static_cast<size_t>(slot) * kStageBytes, src, bytes, &ctl->full[slot]);
                }
                __syncwarp();
                ++it;
            }
        }
        if (lane == 0) ctl->issued = it;
    } else {
        // ---------------- consumers: one warp at a time ----------------
        int it = 0, waited = 0;
        bool live = true;
        for (int64_t r = row_first; r <= row_last; ++r) {
            const Segment s = make_segment<kStageBytes>(g, c, r, lo, hi);
            op.begin_segment(s);
            for (int32_t k = 0; k < s.n_chunks; ++k) {
                const int slot = it % kStages;
                const uint32_t parity = (it / kStages) & 1;
                if (live) {
                    live = warp_wait_bounded(&ctl->full[slot], parity, status, &ctl->abort, ctl->limit_ns);
                    if (live) waited = it + 1;
                    else if (lane == 0) atomicExch(&ctl->abort, 1);
                }
                const unsigned char* src = s.A0 + static_cast<int64_t>(k) * kStageBytes;
                const int64_t left = s.A1 - src;
                const int32_t bytes = static_cast<int32_t>(left < kStageBytes ? left : kStageBytes);
                const int esz_log2 = g.esz == 4 ? 2 : 1;  // 4-byte or 2-byte elements
                const int64_t col0 = s.j0 + ((src - s.a0) >> esz_log2);
                op.chunk(s, ring + static_cast<size_t>(slot) * kStageBytes, col0, bytes >> esz_log2, live);
                if (live) {
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&ctl->empty[slot]);
                }
                ++it;
            }
            op.end_segment(s);
        }
        if (lane == 0) ctl->waited[warp] = waited;
    }
    __syncthreads();
    // Drain: every bulk copy issued must have landed before the CTA's shared memory goes away. The
    // copies not yet seen by every warp are the last (at most kStages) issued ones.
    if (threadIdx.x == 0) {
        int from = ctl->issued;
        for (int w = 0; w < kConsumerWarps; ++w) from = ctl->waited[w] < from ? ctl->waited[w] : from;
        for (int i = from; i < ctl->issued; ++i) {
            if (i + 1 == ctl->withhold) continue;  // never issued
            if (!mbar_wait_bounded(&ctl->full[i % kStages], (i / kStages) & 1, status, ctl->limit_ns)) break;
        }
    }
    __syncthreads();
}

}  // namespace loom_select
