// select_argmax.cu -- greedy argmax over long rows (K1), streamed through shared memory.
//
// Replaces the host scan of Generator::argmax (src/core/generation.cpp:64-74) and argmax_tensor_row /
// argmax_tensor_rows (src/core/lua_bridge.cpp:320-329, :358-362) for rows too long for one warp.
// Bound: HBM bandwidth (4 or 2 bytes read per element, one compare per element).
#include <atomic>

#include "select_internal.h"
#include "select_rows.cuh"
#include "select_stream.cuh"

namespace loom_select {

namespace {

constexpr int kArgWarps = 8;
constexpr int kArgNT = kArgWarps * 32;
constexpr int kArgStages = 3;  // two CTAs per SM, 96 KB of ring each
constexpr int kArgStageBytes = 32768;

struct ArgRecord {
    float v;
    int32_t i;
};

struct ArgShared {
    ArgBest red[kArgWarps];
    int last;
};

template <int kDtype>
struct ArgmaxOp {
    static constexpr int kEsz = (kDtype == LOOM_SELECT_BF16) ? 2 : 4;
    static constexpr int kPer = 16 / kEsz;
    static constexpr int kU = 4; // vectors per thread per step
    StreamGeom g;  // copies: no pointer into the kernel's parameters
    int64_t lo;
    int32_t* out_ids;
    ArgRecord* records;
    int* tickets;
    ArgShared* sh;
    ArgBest best; // the WARP's best so far: identical in every lane

    __device__ const unsigned char* row_ptr(int64_t row) const { return g.base + row * g.row_stride * kEsz; }

    __device__ void begin_segment(const Segment&) { best = arg_init(); }

    // Steps of kU vectors per thread, columns increasing from step to step. A step can change the
    // warp's best only where some element reaches it (or, before anything is taken, equals -inf);
    // then the lanes' own bests join the warp's in one reduction (value desc, column asc).
    __device__ void chunk(const Segment&, const unsigned char* data, int64_t col0, int32_t n, bool live) {
        constexpr int kNT = kArgNT;
        if (!live) return;
        const int32_t nvec = n / kPer;
        const uint4* v4 = reinterpret_cast<const uint4*>(data);
        const int32_t nsteps = (nvec + kU * kNT - 1) / (kU * kNT);
        for (int32_t step = 0; step < nsteps; ++step) {
            const int32_t v0 = step * kU * kNT + static_cast<int32_t>(threadIdx.x);
            uint4 raw[kU];
            float mu = __int_as_float(0x7fc00000); // NaN: fmaxf skips it
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                const int32_t v = v0 + u * kNT;
                if (v < nvec) {
                    raw[u] = v4[v];
                    mu = fmaxf(mu, vec_max<kDtype>(raw[u]));
                }
            }
            const bool take = mu > best.v || (mu == best.v && best.i == 0x7fffffff);
            if (__any_sync(0xffffffffu, take)) {
                ArgBest b = arg_init();
                if (take) {
#pragma unroll
                    for (int u = 0; u < kU; ++u) {
                        const int32_t v = v0 + u * kNT;
                        if (v < nvec) {
                            const int32_t col = static_cast<int32_t>(col0) + v * kPer;
                            Vec16<kDtype> e;
                            e.unpack(raw[u]);
#pragma unroll
                            for (int q = 0; q < kPer; ++q) arg_offer(b, e.x[q], col + q);
                        }
                    }
                }
                b = arg_warp_reduce(b);
                arg_offer(b, best.v, best.i);
                best = b;
            }
        }
    }

    // The loom.cpp rule on the row's final (value, column): a NaN in column 0 wins.
    __device__ int32_t final_col(int64_t row, ArgBest b) const {
        const float x0 = load_global_elem<kDtype>(row_ptr(row), 0);
        return (x0 != x0) ? 0 : b.i;
    }

    __device__ void end_segment(const Segment& s) {
        const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
        // the edges (outside the aligned interior, at both ends of the columns) join last: the
        // final combine orders by value, then column, whatever the order things were seen in
        ArgBest b = arg_init();
        const int32_t n_edges = segment_edge_count(s, kEsz);
        if (static_cast<int>(threadIdx.x) < n_edges) {
            const int64_t col = segment_edge_col(s, kEsz, threadIdx.x);
            arg_offer(b, load_global_elem<kDtype>(row_ptr(s.row), col), static_cast<int32_t>(col));
        }
        b = arg_warp_reduce(b);
        arg_offer(b, best.v, best.i);
        if (lane == 0) sh->red[warp] = b;
        group_sync<kArgNT>();
        if (threadIdx.x == 0) {
            b = sh->red[0];
            for (int w = 1; w < kArgWarps; ++w) arg_offer(b, sh->red[w].v, sh->red[w].i);
            if (s.count == 1) {
                out_ids[s.row] = static_cast<int32_t>(lo + final_col(s.row, b));
            } else {
                records[record_slot(g, s.first_cta + s.index, s.row)] = ArgRecord{b.v, b.i};
                __threadfence();
                int* ticket = &tickets[record_slot(g, s.first_cta, s.row)];
                const int prev = atomicAdd(ticket, 1);
                if (prev == s.count - 1) {
                    __threadfence();
                    ArgBest m = arg_init();
                    for (int j = 0; j < s.count; ++j) {
                        const ArgRecord* r = records + record_slot(g, s.first_cta + j, s.row);
                        const float v = __ldcg(&r->v);
                        const int32_t i = __ldcg(&r->i);
                        arg_offer(m, v, i);
                    }
                    out_ids[s.row] = static_cast<int32_t>(lo + final_col(s.row, m));
                    *ticket = 0;
                }
            }
        }
        group_sync<kArgNT>();
    }
};

template <int kDtype>
__global__ void __launch_bounds__((kArgWarps + 1) * 32, 2)
    argmax_stream_kernel(StreamGeom g, int64_t lo, int32_t* out_ids, ArgRecord* records, int* tickets, int* status) {
    extern __shared__ __align__(128) unsigned char ring[];
    __shared__ StreamCtl ctl;
    __shared__ ArgShared sh;
    ArgmaxOp<kDtype> op{g, lo, out_ids, records, tickets, &sh, arg_init()};
    stream_ranges_warps<kArgStages, kArgStageBytes, kArgWarps>(g, op, ring, &ctl, status);
}

template <int kDtype>
cudaError_t launch_argmax_stream_t(const StreamGeom& g, int64_t lo, int32_t* out_ids, ArgRecord* records,
                                   int* tickets, int* status, cudaStream_t stream) {
    constexpr size_t smem = static_cast<size_t>(kArgStages) * kArgStageBytes;
    static std::atomic<bool> configured[64] = {};  // set once per device, from any host thread
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        const cudaError_t e = cudaFuncSetAttribute(argmax_stream_kernel<kDtype>,
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    argmax_stream_kernel<kDtype><<<g.ctas, (kArgWarps + 1) * 32, smem, stream>>>(g, lo, out_ids, records, tickets, status);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_argmax_stream(int dtype, const void* window_base, int64_t rows, int64_t width, int64_t row_stride,
                                 int64_t lo, int32_t* out_ids, void* workspace, const WsLayout& l, int ctas,
                                 cudaStream_t stream) {
    StreamGeom g;
    g.base = static_cast<const unsigned char*>(window_base);
    g.rows = rows;
    g.width = width;
    g.row_stride = row_stride;
    g.total = rows * width;
    g.esz = dtype == LOOM_SELECT_BF16 ? 2 : 4;
    g.ctas = ctas;
    unsigned char* ws = static_cast<unsigned char*>(workspace);
    int* status = reinterpret_cast<int*>(ws);
    int* tickets = reinterpret_cast<int*>(ws + l.tickets);
    ArgRecord* records = reinterpret_cast<ArgRecord*>(ws + l.records);
    if (dtype == LOOM_SELECT_BF16)
        return launch_argmax_stream_t<LOOM_SELECT_BF16>(g, lo, out_ids, records, tickets, status, stream);
    return launch_argmax_stream_t<LOOM_SELECT_F32>(g, lo, out_ids, records, tickets, status, stream);
}

}  // namespace loom_select
