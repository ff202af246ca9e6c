// select_windows.cu -- argmax over id windows of rows, cut into chunks that any CTA can take (K1w).
//
// Replaces the scan of argmax_tensor_row (src/core/lua_bridge.cpp:320-329) when a caller wants several
// windows of the same rows at once -- Whisper's decoder asks for the language block and the timestamp
// block of one row through loom.argmax_row_range (lua_bridge.cpp:779-797) -- and serves
// loom_argmax_rows for small batches, where the streamed kernel (select_argmax.cu) has too little to
// keep the GPU busy: one decode step is a single 151936-wide row.
//
// Every (row, window) pair is cut into chunks of `chunk` elements; a chunk is one work item, and
// persistent CTAs take items in turn. A CTA reduces its chunk (16-byte loads of the aligned interior,
// scalar loads of the at most 2 x 15 edge bytes) to the best (value, column) under loom.cpp's strict
// '>' rule and merges it into the pair's 64-bit record with atomicMax on its rank key: (order key of
// the value) << 32 | ~column, so the larger value wins and, among equal values, the lower column; NaN
// is never offered. An atomic ticket per pair counts its chunks; the CTA that takes the last one writes
// the absolute id -- the window's first column when that column holds a NaN (nothing compares greater
// than it) -- and returns the record and the ticket to zero, so the workspace is zero between calls.
// Bound: HBM bandwidth (one read of every window) plus one round trip of latency for small calls.
#include <cstdint>

#include "select_internal.h"
#include "select_rows.cuh"

namespace loom_select {

namespace {

constexpr int kWinNT = 256;

struct WinRec {
    unsigned long long key;  // best rank key so far (0: nothing)
    int ticket;              // chunks done
    int pad;
};
static_assert(sizeof(WinRec) == kChunkPairBytes, "pair record size");

struct WinParams {
    const unsigned char* base;
    int64_t row_stride_bytes;
    int64_t rows;
    int32_t n_win;
    int64_t chunk;                       // elements per chunk
    int64_t lo[kArgmaxMaxWindows];
    int64_t hi[kArgmaxMaxWindows];
    int64_t nck[kArgmaxMaxWindows];      // chunks per row of window w
    int64_t item0[kArgmaxMaxWindows + 1];  // first item of window w (items are window-major)
    int32_t* out_ids;                    // [rows][n_win]
    WinRec* recs;                        // [rows][n_win]
};

template <int kDtype>
__global__ void __launch_bounds__(kWinNT) argmax_windows_kernel(const WinParams p) {
    constexpr int kEsz = (kDtype == LOOM_SELECT_BF16) ? 2 : 4;
    constexpr int kPer = 16 / kEsz;
    __shared__ ArgBest red[kWinNT / 32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t n_items = p.item0[p.n_win];
    for (int64_t item = blockIdx.x; item < n_items; item += gridDim.x) {
        int wi = 0;
        while (wi + 1 < p.n_win && item >= p.item0[wi + 1]) ++wi;
        const int64_t local = item - p.item0[wi];
        const int64_t r = local / p.nck[wi];
        const int64_t j = local - r * p.nck[wi];
        const int64_t c_lo = p.lo[wi] + j * p.chunk;
        const int64_t c_hi = c_lo + p.chunk < p.hi[wi] ? c_lo + p.chunk : p.hi[wi];
        const unsigned char* row = p.base + r * p.row_stride_bytes;
        // the chunk's 16-byte-aligned interior [A0, A1) and its edges
        const uintptr_t a0 = reinterpret_cast<uintptr_t>(row) + static_cast<uintptr_t>(c_lo) * kEsz;
        const uintptr_t a1 = reinterpret_cast<uintptr_t>(row) + static_cast<uintptr_t>(c_hi) * kEsz;
        uintptr_t A0 = (a0 + 15) & ~uintptr_t(15), A1 = a1 & ~uintptr_t(15);
        if (A0 >= A1) A0 = A1 = a1;
        const int32_t head = static_cast<int32_t>((A0 - a0) / kEsz);
        const int32_t tail = static_cast<int32_t>((a1 - A1) / kEsz);
        const int64_t nvec = static_cast<int64_t>((A1 - A0) / 16);
        ArgBest b = arg_init();
        constexpr int kU = 4;  // 16-byte loads in flight per thread
        for (int64_t v0 = tid; v0 < nvec; v0 += static_cast<int64_t>(kWinNT) * kU) {
            uint4 raw[kU];
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                const int64_t v = v0 + static_cast<int64_t>(u) * kWinNT;
                if (v < nvec) raw[u] = ldg_stream_v4(reinterpret_cast<const void*>(A0 + v * 16));
            }
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                const int64_t v = v0 + static_cast<int64_t>(u) * kWinNT;
                if (v < nvec) {
                    Vec16<kDtype> e;
                    e.unpack(raw[u]);
                    const int32_t col = static_cast<int32_t>(c_lo + head + v * kPer);
#pragma unroll
                    for (int q = 0; q < kPer; ++q) arg_offer(b, e.x[q], col + q);
                }
            }
        }
        if (tid < head + tail) {
            const int64_t col = tid < head ? c_lo + tid : c_lo + ((A1 - a0) / kEsz) + (tid - head);
            arg_offer(b, load_global_elem<kDtype>(row, col), static_cast<int32_t>(col));
        }
        b = arg_warp_reduce(b);
        if (lane == 0) red[warp] = b;
        __syncthreads();
        if (tid == 0) {
            for (int w = 1; w < kWinNT / 32; ++w) arg_offer(b, red[w].v, red[w].i);
            WinRec* rec = p.recs + r * p.n_win + wi;
            if (b.i != 0x7fffffff)
                atomicMax(&rec->key, static_cast<unsigned long long>(
                                         loom_rank_key(b.v, static_cast<int32_t>(b.i - p.lo[wi]))));
            __threadfence();
            const int prev = atomicAdd(&rec->ticket, 1);
            if (prev == p.nck[wi] - 1) {
                __threadfence();
                const unsigned long long key = atomicAdd(&rec->key, 0ull);
                int64_t id = p.lo[wi];
                const float x_lo = load_global_elem<kDtype>(row, p.lo[wi]);
                if (key != 0ull && x_lo == x_lo) id = p.lo[wi] + rank_key_id(key);
                p.out_ids[r * p.n_win + wi] = static_cast<int32_t>(id);
                rec->key = 0ull;
                rec->ticket = 0;
            }
        }
        __syncthreads();  // red[] is rewritten by the next item
    }
}

// One launch: rows [r0, r0 + rows) of the call, at most kChunkPairs (row, window) pairs.
cudaError_t launch_group(int dtype, const unsigned char* base, int64_t rows, int64_t row_stride_bytes, const int64_t* lo,
                         const int64_t* hi, int32_t n_win, int32_t* out_ids, WinRec* recs, int sms,
                         cudaStream_t stream) {
    WinParams p{};
    p.base = base;
    p.row_stride_bytes = row_stride_bytes;
    p.rows = rows;
    p.n_win = n_win;
    // chunk: enough items to give every SM two, at least 1024 and at most 32768 elements (a multiple
    // of 1024, so a chunk boundary keeps 16-byte alignment wherever the window does)
    int64_t total = 0;
    for (int w = 0; w < n_win; ++w) total += rows * (hi[w] - lo[w]);
    int64_t chunk = total / (2 * static_cast<int64_t>(sms));
    chunk = (chunk + 1023) / 1024 * 1024;
    if (chunk < 1024) chunk = 1024;
    if (chunk > 32768) chunk = 32768;
    p.chunk = chunk;
    p.item0[0] = 0;
    for (int w = 0; w < n_win; ++w) {
        p.lo[w] = lo[w];
        p.hi[w] = hi[w];
        p.nck[w] = (hi[w] - lo[w] + chunk - 1) / chunk;
        p.item0[w + 1] = p.item0[w] + rows * p.nck[w];
    }
    p.out_ids = out_ids;
    p.recs = recs;
    const int64_t items = p.item0[n_win];
    int64_t grid = static_cast<int64_t>(sms) * 8;
    if (grid > items) grid = items;
    if (grid < 1) grid = 1;
    if (dtype == LOOM_SELECT_BF16)
        argmax_windows_kernel<LOOM_SELECT_BF16><<<static_cast<unsigned>(grid), kWinNT, 0, stream>>>(p);
    else
        argmax_windows_kernel<LOOM_SELECT_F32><<<static_cast<unsigned>(grid), kWinNT, 0, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_argmax_windows(int dtype, const void* logits, int64_t rows, int64_t row_stride, const int64_t* lo,
                                  const int64_t* hi, int32_t n_win, int32_t* out_ids, void* workspace,
                                  const WsLayout& l, int sms, cudaStream_t stream) {
    const int esz = dtype == LOOM_SELECT_BF16 ? 2 : 4;
    WinRec* recs = reinterpret_cast<WinRec*>(static_cast<unsigned char*>(workspace) + l.pairs);
    const int64_t per = kChunkPairs / n_win;  // rows per launch
    for (int64_t r0 = 0; r0 < rows; r0 += per) {
        const int64_t n = rows - r0 < per ? rows - r0 : per;
        const cudaError_t e = launch_group(dtype, static_cast<const unsigned char*>(logits) + r0 * row_stride * esz, n,
                                           row_stride * esz, lo, hi, n_win, out_ids + r0 * n_win, recs, sms, stream);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace loom_select
