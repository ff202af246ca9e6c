// select_rows.cuh -- one warp reduces one short row (a CTC frame, a short classifier row).
//
// The row's 16-byte-aligned interior is read with 128-bit loads (each lane keeps several in flight),
// the at most 2 x 15 bytes outside it with scalar loads, so every access stays inside the row.
// The argmax follows loom.cpp's strict '>' scan (src/core/generation.cpp:64-74,
// src/core/ctc_decode.cpp:9-20): the lowest column wins among equal maxima, NaN never wins except
// at column 0 (checked by the caller's final rule), -0 == +0.
#pragma once

#include "select_device.cuh"

namespace loom_select {

// (value, column) argmax state; column INT32_MAX means "nothing taken yet".
struct ArgBest {
    float v;
    int32_t i;
};

__device__ __forceinline__ ArgBest arg_init() { return {-__int_as_float(0x7f800000), 0x7fffffff}; }

// Take (x, col) if it beats the current best: larger value, or equal value and lower column.
// NaN never beats anything.
__device__ __forceinline__ void arg_offer(ArgBest& b, float x, int32_t col) {
    if (x > b.v || (x == b.v && col < b.i)) {
        b.v = x;
        b.i = col;
    }
}

__device__ __forceinline__ ArgBest arg_warp_reduce(ArgBest b) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, b.v, off);
        const int32_t oi = __shfl_xor_sync(0xffffffffu, b.i, off);
        arg_offer(b, ov, oi);
    }
    return b;
}

// Online log-sum-exp state over the non-NaN values: max m, sum s of exp(x - m).
struct LseAcc {
    float m;
    float s;
};

__device__ __forceinline__ LseAcc lse_init() { return {-__int_as_float(0x7f800000), 0.0f}; }

__device__ __forceinline__ void lse_offer(LseAcc& a, float x) {
    if (x != x || x == -__int_as_float(0x7f800000)) return;
    if (x > a.m) {
        a.s = a.s * __expf(a.m - x) + 1.0f;
        a.m = x;
    } else if (x == a.m) {
        a.s += 1.0f;
    } else {
        a.s += __expf(x - a.m);
    }
}

__device__ __forceinline__ LseAcc lse_merge(LseAcc a, LseAcc b) {
    if (b.s == 0.0f) return a;
    if (a.s == 0.0f) return b;
    if (a.m == b.m) return {a.m, a.s + b.s};
    if (a.m > b.m) return {a.m, a.s + b.s * __expf(b.m - a.m)};
    return {b.m, b.s + a.s * __expf(a.m - b.m)};
}

__device__ __forceinline__ LseAcc lse_warp_reduce(LseAcc a) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        LseAcc o;
        o.m = __shfl_xor_sync(0xffffffffu, a.m, off);
        o.s = __shfl_xor_sync(0xffffffffu, a.s, off);
        a = lse_merge(a, o);
    }
    return a;
}

// Elements of one 16-byte vector as floats.
template <int kDtype>
struct Vec16 {
    static constexpr int kElems = (kDtype == LOOM_SELECT_BF16) ? 8 : 4;
    float x[kElems];
    __device__ __forceinline__ void unpack(uint4 raw) {
        if constexpr (kDtype == LOOM_SELECT_BF16) {
            const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                x[2 * q] = __uint_as_float(w[q] << 16);
                x[2 * q + 1] = __uint_as_float(w[q] & 0xffff0000u);
            }
        } else {
            x[0] = __uint_as_float(raw.x);
            x[1] = __uint_as_float(raw.y);
            x[2] = __uint_as_float(raw.z);
            x[3] = __uint_as_float(raw.w);
        }
    }
};

// Maximum of one 16-byte vector of logits as a float (NaN elements ignored; NaN only if all are
// NaN; -0 and +0 compare equal). bf16 vectors take the maximum of packed pairs (exact in bf16).
template <int kDtype>
__device__ __forceinline__ float vec_max(uint4 raw) {
    if constexpr (kDtype == LOOM_SELECT_BF16) {
        const __nv_bfloat162 a = __hmax2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x),
                                         *reinterpret_cast<const __nv_bfloat162*>(&raw.y));
        const __nv_bfloat162 b = __hmax2(*reinterpret_cast<const __nv_bfloat162*>(&raw.z),
                                         *reinterpret_cast<const __nv_bfloat162*>(&raw.w));
        const __nv_bfloat162 c = __hmax2(a, b);
        return fmaxf(__low2float(c), __high2float(c));
    } else {
        return fmaxf(fmaxf(__uint_as_float(raw.x), __uint_as_float(raw.y)),
                     fmaxf(__uint_as_float(raw.z), __uint_as_float(raw.w)));
    }
}

__device__ __forceinline__ uint4 ldg_stream_v4(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

// Warp-cooperative argmax (and, with kLse, log-sum-exp) of row[0..W). Every lane returns the result.
template <int kDtype, bool kLse>
__device__ __forceinline__ void warp_row_reduce(const unsigned char* row, int64_t W, ArgBest& best, LseAcc& lse) {
    constexpr int kEsz = (kDtype == LOOM_SELECT_BF16) ? 2 : 4;
    constexpr int kPer = 16 / kEsz;
    constexpr int kUnroll = 4;
    const int lane = threadIdx.x & 31;
    best = arg_init();
    lse = lse_init();
    const uintptr_t a0 = reinterpret_cast<uintptr_t>(row);
    const uintptr_t a1 = a0 + static_cast<uintptr_t>(W) * kEsz;
    uintptr_t A0 = (a0 + 15) & ~uintptr_t(15);
    uintptr_t A1 = a1 & ~uintptr_t(15);
    if (A0 >= A1) {
        A0 = a1;
        A1 = a1;
    }
    const int32_t head = static_cast<int32_t>((A0 - a0) / kEsz);
    const int32_t tail = static_cast<int32_t>((a1 - A1) / kEsz);
    const int64_t nvec = static_cast<int64_t>((A1 - A0) / 16);
    const int32_t col_base = head; // column of the first interior element
    // interior, kUnroll loads in flight per lane
    for (int64_t v0 = 0; v0 < nvec; v0 += 32 * kUnroll) {
        uint4 raw[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int64_t v = v0 + u * 32 + lane;
            if (v < nvec) raw[u] = ldg_stream_v4(reinterpret_cast<const void*>(A0 + v * 16));
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int64_t v = v0 + u * 32 + lane;
            if (v < nvec) {
                Vec16<kDtype> e;
                e.unpack(raw[u]);
                const int32_t col = col_base + static_cast<int32_t>(v) * kPer;
#pragma unroll
                for (int q = 0; q < kPer; ++q) {
                    arg_offer(best, e.x[q], col + q);
                    if constexpr (kLse) lse_offer(lse, e.x[q]);
                }
            }
        }
    }
    // edges
    if (lane < head + tail) {
        const int32_t col = lane < head ? lane : static_cast<int32_t>((A1 - a0) / kEsz) + (lane - head);
        const float x = load_global_elem<kDtype>(row, col);
        arg_offer(best, x, col);
        if constexpr (kLse) lse_offer(lse, x);
    }
    best = arg_warp_reduce(best);
    if constexpr (kLse) lse = lse_warp_reduce(lse);
}

}  // namespace loom_select
