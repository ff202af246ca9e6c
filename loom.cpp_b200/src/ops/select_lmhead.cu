// select_lmhead.cu -- greedy selection fused into the LM-head GEMM (sm_100a: TMA + tcgen05 + TMEM).
//
// loom.cpp's text models end in ggml's mul_mat(lm_head, hidden): logits[r, v] = sum_h hidden[r, h] *
// weight[v, h], with the weight stored [n_vocab, hidden_dim] row-major (ggml ne0 = hidden_dim). The
// engine then writes the [rows, n_vocab] logits to memory and Generator::argmax
// (src/core/generation.cpp:64-74) scans them. Here the product is computed tile by tile on the
// tensor cores and reduced before it ever leaves the SM:
//
//   * one persistent CTA per SM walks 128-row x BN-id tiles, BN 256 or 208 (row tile fastest, so the
//     CTAs running at the same time share one weight tile through L2 and the weight is read from HBM
//     about once);
//   * warp 0 streams 64-wide K slices of the hidden and weight tiles into a shared-memory ring of 4-8
//     stages with TMA (2-D tensor maps, 128-byte swizzle, no multicast); warp 1 issues tcgen05.mma
//     (M 128, N BN, K 16, bf16 in, f32 accumulate) into one of two TMEM accumulators;
//   * warps 2-5 drain the other accumulator meanwhile (tcgen05.ld, one row per thread) and reduce each
//     row's BN logits to a record: the tile's maximum, the lowest id reaching it, the sum of
//     exp(logit - maximum) when the log-sum-exp is wanted, and whether column 0 is NaN;
//   * lm_merge_kernel folds a row's records into the greedy id, its logit and the row's log-sum-exp
//     (a warp per row, or the whole block per row for calls of at most 64 rows).
//
// Selection rule (generation.cpp:64-74, a strict '>' scan from id 0): the lowest id among equal
// maxima wins, a NaN at id 0 wins, a NaN anywhere else never wins. The logits themselves are f32 sums
// of exact bf16 products in the tensor cores' order, so they can differ from another GEMM's in the
// last bits; the id is the exact argmax of the logits this kernel computes.
//
// Every mbarrier wait is bounded (kWaitLimitNs, or the workspace test hook's lower bound). A wait
// that runs out records LOOM_SELECT_ETIMEOUT in the workspace, raises the CTA's abort flag, and every
// role winds down: the producer waits (again bounded) for the copies it issued, the MMA warp for the
// MMAs it issued, then TMEM is freed.
#include <cstdint>
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <mutex>

#include "loom_select.h"
#include "select_device.cuh"
#include "select_internal.h"

namespace loom_select {
namespace {

constexpr int kBM = 128;          // rows per tile (MMA M)
constexpr int kBK = 64;           // K slice per stage: 64 bf16 = 128 bytes, one swizzle span
constexpr int kUK = 16;           // K per tcgen05.mma (kind::f16)
constexpr int kThreads = 192;     // warp 0 TMA, warp 1 MMA + TMEM owner, warps 2-5 epilogue
constexpr uint32_t kTmemCols = 512;              // two accumulators, 256 columns apart
constexpr int kAccStride = 256;

// A tile is kBM rows x BN ids; the ring holds as many K slices as fit in shared memory. BN is a
// multiple of 16 (an MMA N for M = 128) and keeps every stage a multiple of 1024 bytes (the 128-byte
// swizzle's repeat).
template <int BN, bool kFewRows>
struct LmTile {
    static_assert(BN % 16 == 0 && BN >= 32 && BN <= 256, "tile width");
    // kFewRows (calls of at most 16 rows, i.e. decoding): the hidden tile is loaded 16 rows high
    // (2 KiB) and the freed shared memory holds more weight stages in flight. The MMA still reads
    // 128 rows of A; rows 16-127 are whatever follows in the stage and only reach TMEM lanes of rows
    // that do not exist, whose results are never read.
    static constexpr int kARows = kFewRows ? 16 : kBM;
    static constexpr uint32_t kTileABytes = uint32_t(kARows) * kBK * 2;
    static constexpr uint32_t kTileBBytes = uint32_t(BN) * kBK * 2;
    static constexpr uint32_t kStageBytes = kTileABytes + kTileBBytes;
    static_assert(kStageBytes % 1024 == 0, "stage alignment");
    static constexpr int kStages = int((227u * 1024u - 2048u) / kStageBytes) < 8 ? int((227u * 1024u - 2048u) / kStageBytes) : 8;
    static_assert(kStages >= 2 && kStageBytes >= kBM * kBK * 2, "the MMA's 128-row A read stays inside its stage");
    static constexpr size_t kSmemBytes = size_t(kStages) * kStageBytes + 256 + 1024;  // ring + barriers + alignment
    // Instruction descriptor, kind::f16: f32 accumulator, bf16 A and B, both K-major, N >> 3, M >> 4.
    static constexpr uint32_t kIdesc =
        (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(BN >> 3) << 17) | (uint32_t(kBM >> 4) << 24);
};

template <int kStages>
struct LmBars {
    uint64_t full[kStages];    // TMA -> MMA
    uint64_t empty[kStages];   // MMA -> TMA
    uint64_t tfull[2];         // MMA -> epilogue
    uint64_t tempty[2];        // epilogue -> MMA (4 arrivals: one per epilogue warp)
    uint64_t drain;            // the MMA warp's final commit
    uint32_t tmem_base;
    int abort;
};

// ---- tcgen05 / TMA wrappers ----

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(x), "r"(y)
        : "memory");
}

// Shared-memory matrix descriptor of a K-major tile written by TMA with the 128-byte swizzle: rows of
// 128 bytes, groups of 8 rows 1024 bytes apart (stride byte offset), descriptor version 1, layout
// type 2 (128-byte swizzle). Stepping K by 16 elements inside the span adds 32 bytes to the start.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= uint64_t((saddr >> 4) & 0x3FFF);
    d |= uint64_t(1) << 16;                    // leading byte offset (unused for swizzled K-major)
    d |= uint64_t((1024 >> 4) & 0x3FFF) << 32; // stride byte offset
    d |= uint64_t(1) << 46;                    // version
    d |= uint64_t(2) << 61;                    // 128-byte swizzle
    return d;
}

__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0; tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
}

__device__ __forceinline__ void tc_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
        "[%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]);
}

template <int W>
__device__ __forceinline__ void tc_ld(uint32_t taddr, float (&v)[W]) {
    if constexpr (W == 32) tc_ld32(taddr, v);
    else tc_ld16(taddr, v);
}

// The running (maximum, lowest id) of one row over W logits at tile columns [c0, c0 + W).
template <int W>
__device__ __forceinline__ void scan_chunk(const float (&v)[W], int c0, int valid, float& bv, int& bi) {
#pragma unroll
    for (int j = 0; j < W; ++j) {
        const int col = c0 + j;
        const float x = v[j];
        if (col < valid && (x > bv || (bi < 0 && x == x))) {
            bv = x;
            bi = col;
        }
    }
}

__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Sum of 2^(v * log2(e) - mb) over the valid columns, two accumulators.
template <int W>
__device__ __forceinline__ void sum_chunk(const float (&v)[W], int c0, int valid, float mb, float& s0, float& s1) {
    const float l2e = 1.4426950408889634f;
#pragma unroll
    for (int j = 0; j < W; j += 2) {
        const int col = c0 + j;
        if (col < valid) s0 += fast_exp2(__fsub_rn(__fmul_rn(v[j], l2e), mb));
        if (col + 1 < valid) s1 += fast_exp2(__fsub_rn(__fmul_rn(v[j + 1], l2e), mb));
    }
}

// Bounded wait that also gives up as soon as another role of the CTA has aborted.
__device__ __forceinline__ bool lm_wait(uint64_t* bar, uint32_t parity, int* status, volatile int* abort_flag,
                                        uint64_t limit_ns) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (;;) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort_flag) return false;
        if (global_timer_ns() - t0 > limit_ns) {
            record_status(status, LOOM_SELECT_ETIMEOUT);
            *abort_flag = 1;
            return false;
        }
    }
}

struct LmArgs {
    int64_t rows, n_vocab;
    int k_blocks;          // hidden_dim / kBK
    int m_tiles, v_tiles;  // tiles along rows and ids
    float4* records;       // [v_tiles][rows]: (max, id bits, sum of exp, col-0 NaN flag)
    int* status;
    int want_lse;
};

template <int BN, bool kFewRows>
__global__ void __launch_bounds__(kThreads, 1)
    lm_head_argmax_kernel(const __grid_constant__ CUtensorMap map_h, const __grid_constant__ CUtensorMap map_w,
                          const LmArgs a) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    using T = LmTile<BN, kFewRows>;
    constexpr uint32_t kTileABytes = T::kTileABytes;
    constexpr int kStages = T::kStages;
    constexpr uint32_t kStageBytes = T::kStageBytes;
    LmBars<kStages>* bars = reinterpret_cast<LmBars<kStages>*>(smem + size_t(kStages) * kStageBytes);
    volatile int* abort_flag = &bars->abort;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // The workspace header's test hook (zero for every normal caller): a lower wait bound, and one
    // K slice that CTA 0's producer leaves unissued so that the MMA warp's wait runs out.
    const WaitFault wf = read_wait_fault(a.status);
    const uint64_t lim = wf.limit_ns;
    const int n_tiles = a.m_tiles * a.v_tiles;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&bars->full[s], 1);
            mbar_init(&bars->empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&bars->tfull[b], 1);
            mbar_init(&bars->tempty[b], 4);
        }
        mbar_init(&bars->drain, 1);
        bars->abort = 0;
        mbar_fence_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&bars->tmem_base)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = bars->tmem_base;

    if (warp == 0) {
        if (lane == 0) {
            // ---- producer: TMA into the ring ----
            int64_t kc = 0;
            const int64_t withheld = (blockIdx.x == 0 && wf.withhold > 0) ? int64_t(wf.withhold) - 1 : -1;
            bool ok = true;
            for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x) {
                const int mt = t % a.m_tiles, vt = t / a.m_tiles;
                for (int kb = 0; kb < a.k_blocks; ++kb, ++kc) {
                    const int s = int(kc % kStages);
                    const int64_t n = kc / kStages;
                    if (n >= 1 && !lm_wait(&bars->empty[s], uint32_t((n - 1) & 1), a.status, abort_flag, lim)) {
                        ok = false;
                        break;
                    }
                    if (kc == withheld) continue;  // test hook only: this slice never arrives
                    unsigned char* st = smem + size_t(s) * kStageBytes;
                    mbar_arrive_expect_tx(&bars->full[s], kStageBytes);
                    tma_load_2d(st, &map_h, kb * kBK, mt * kBM, &bars->full[s]);
                    tma_load_2d(st + kTileABytes, &map_w, kb * kBK, vt * BN, &bars->full[s]);
                }
            }
            // Every copy issued lands before the CTA may exit (on the normal path the MMA warp has
            // consumed them all already and these waits return at once).
            // (A withheld slice was the last use of its stage the producer reached: its next use
            // waits for the MMA warp, which is stuck on the withheld one until the abort.)
            for (int s = 0; s < kStages; ++s) {
                if (kc > s) {
                    int64_t last_kc = s + int64_t(kStages) * ((kc - 1 - s) / kStages);
                    if (last_kc == withheld) last_kc -= kStages;
                    if (last_kc >= 0) mbar_wait_bounded(&bars->full[s], uint32_t((last_kc / kStages) & 1), a.status, lim);
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            // ---- MMA issuer ----
            int64_t kc = 0;
            int i = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x, ++i) {
                const int b = i & 1, u = i >> 1;
                if (u >= 1 && !lm_wait(&bars->tempty[b], uint32_t((u - 1) & 1), a.status, abort_flag, lim)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + uint32_t(b * kAccStride);
                for (int kb = 0; kb < a.k_blocks; ++kb, ++kc) {
                    const int s = int(kc % kStages);
                    const int64_t n = kc / kStages;
                    if (!lm_wait(&bars->full[s], uint32_t(n & 1), a.status, abort_flag, lim)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = smem_addr(smem + size_t(s) * kStageBytes);
                    const uint32_t sb = sa + kTileABytes;
#pragma unroll
                    for (int kk = 0; kk < kBK / kUK; ++kk) {
                        tc_mma(d_tmem, smem_desc_sw128(sa + kk * kUK * 2), smem_desc_sw128(sb + kk * kUK * 2),
                               T::kIdesc, (kb | kk) != 0 ? 1u : 0u);
                    }
                    tc_commit(&bars->empty[s]);
                }
                if (ok) tc_commit(&bars->tfull[b]);
            }
            // All MMAs issued have completed before TMEM is freed.
            tc_commit(&bars->drain);
            mbar_wait_bounded(&bars->drain, 0, a.status, lim);
        }
        __syncwarp();
    } else {
        // ---- epilogue: warps 2-5 read TMEM lanes 32 * (warp % 4) .. + 31, one row per thread ----
        const int q = warp & 3;
        int i = 0;
        for (int t = blockIdx.x; t < n_tiles; t += gridDim.x, ++i) {
            const int mt = t % a.m_tiles, vt = t / a.m_tiles;
            const int b = i & 1, u = i >> 1;
            const bool ok = lm_wait(&bars->tfull[b], uint32_t(u & 1), a.status, abort_flag, lim);
            if (!__all_sync(0xffffffffu, ok)) break;
            tc_fence_after();
            const uint32_t taddr = tmem_base + (uint32_t(q * 32) << 16) + uint32_t(b * kAccStride);
            const int64_t col0 = int64_t(vt) * BN;
            const int valid = a.n_vocab - col0 < BN ? int(a.n_vocab - col0) : BN;
            constexpr int kFull = BN / 32 * 32;  // columns read 32 at a time; the rest (16) at once
            float bv = -INFINITY;
            int bi = -1;
            float nan0 = 0.0f;
            {
                float v[32];
                tc_ld32(taddr, v);
                if (vt == 0 && v[0] != v[0]) nan0 = 1.0f;
                scan_chunk<32>(v, 0, valid, bv, bi);
#pragma unroll 1
                for (int c = 32; c < kFull; c += 32) {
                    tc_ld32(taddr + uint32_t(c), v);
                    scan_chunk<32>(v, c, valid, bv, bi);
                }
                if constexpr (BN % 32 != 0) {
                    float w[16];
                    tc_ld16(taddr + uint32_t(kFull), w);
                    scan_chunk<16>(w, kFull, valid, bv, bi);
                }
            }
            float sum = 0.0f;
            if (a.want_lse) {
                // Every lane makes the same tcgen05.ld calls (they are warp-collective); a lane whose
                // tile part is all NaN sums against 0 and discards the result.
                const float mb = bi >= 0 ? bv * 1.4426950408889634f : 0.0f;
                float s0 = 0.0f, s1 = 0.0f;
                float v[32];
#pragma unroll 1
                for (int c = 0; c < kFull; c += 32) {
                    tc_ld32(taddr + uint32_t(c), v);
                    sum_chunk<32>(v, c, valid, mb, s0, s1);
                }
                if constexpr (BN % 32 != 0) {
                    float w[16];
                    tc_ld16(taddr + uint32_t(kFull), w);
                    sum_chunk<16>(w, kFull, valid, mb, s0, s1);
                }
                sum = bi >= 0 ? s0 + s1 : 0.0f;
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->tempty[b]);
            const int64_t r = int64_t(mt) * kBM + q * 32 + lane;
            if (r < a.rows) {
                a.records[int64_t(vt) * a.rows + r] =
                    make_float4(bv, __int_as_float(bi < 0 ? -1 : int(col0) + bi), sum, nan0);
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols) : "memory");
    }
}

// A row's partial result: maximum, lowest id reaching it (-1: none, every logit NaN), and the sum of
// exp(logit - maximum).
struct LmPart {
    float m;
    int id;
    float s;
};

// A partial sum moved to the maximum M (a part whose maximum is -inf adds nothing below a larger M).
__device__ __forceinline__ float lm_rescale(const LmPart& p, float M) {
    if (p.m == M) return p.s;
    return p.m == -INFINITY ? 0.0f : p.s * expf(p.m - M);
}

// Folds two partial results of one row; the larger maximum wins, the lower id among equal maxima
// (the strict '>' scan of generation.cpp:64-74 in any fold order), sums rescaled to the winner.
__device__ __forceinline__ LmPart lm_fold(LmPart a, LmPart b) {
    if (b.id < 0) return a;
    if (a.id < 0) return b;
    const bool take_b = b.m > a.m || (b.m == a.m && b.id < a.id);
    LmPart r;
    r.m = take_b ? b.m : a.m;
    r.id = take_b ? b.id : a.id;
    r.s = lm_rescale(a, r.m) + lm_rescale(b, r.m);
    return r;
}

__device__ __forceinline__ LmPart lm_shfl_fold(LmPart p) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        LmPart q;
        q.m = __shfl_xor_sync(0xffffffffu, p.m, o);
        q.id = __shfl_xor_sync(0xffffffffu, p.id, o);
        q.s = __shfl_xor_sync(0xffffffffu, p.s, o);
        p = lm_fold(p, q);
    }
    return p;
}

// kTpr threads per row (32: a warp, 8 rows per block; 256: the whole block, for calls of few rows)
// fold the row's tile records in one pass into (id, logit, log-sum-exp).
template <int kTpr>
__global__ void __launch_bounds__(256) lm_merge_kernel(const float4* __restrict__ records, int64_t rows, int v_tiles,
                                                       int want_lse, int32_t* __restrict__ out_ids,
                                                       float* __restrict__ out_logit, float* __restrict__ out_lse) {
    constexpr int kRowsPerBlock = 256 / kTpr;
    const int64_t r = int64_t(blockIdx.x) * kRowsPerBlock + threadIdx.x / kTpr;
    const int li = threadIdx.x % kTpr;
    LmPart p{-INFINITY, -1, 0.0f};
    if (r < rows) {
        for (int t = li; t < v_tiles; t += kTpr) {
            const float4 rec = records[int64_t(t) * rows + r];
            const LmPart q{rec.x, __float_as_int(rec.y), rec.z};
            p = lm_fold(p, q);
        }
    }
    p = lm_shfl_fold(p);
    if constexpr (kTpr == 256) {
        __shared__ LmPart part[8];
        if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = p;
        __syncthreads();
        p = part[0];
#pragma unroll
        for (int w = 1; w < 8; ++w) p = lm_fold(p, part[w]);
    }
    if (li == 0 && r < rows) {
        const bool nan0 = records[r].w != 0.0f;  // tile 0 carries the id-0 NaN flag
        const bool zero = nan0 || p.id < 0;      // a NaN at id 0 (or only NaNs) leaves the scan at id 0
        const float qnan = __int_as_float(0x7fc00000);
        out_ids[r] = zero ? 0 : p.id;
        if (out_logit) out_logit[r] = zero ? qnan : p.m;
        if (out_lse && want_lse) out_lse[r] = zero ? qnan : p.m + logf(p.s);
    }
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link against libcuda).
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

bool make_map(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer, uint32_t box_outer) {
    auto fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {inner * 2};
    const cuuint32_t box[2] = {uint32_t(kBK), box_outer};
    const cuuint32_t estr[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The two tile widths: 256 ids, or 208 when that spreads the tiles over the SMs clearly more evenly
// (151936 ids on one row tile: 594 tiles of 256 leave two SMs a fifth tile, 731 tiles of 208 fill 148
// SMs five times within 1%). The workspace holds records for the narrower one.
constexpr int kWideBN = 256, kNarrowBN = 208;

int64_t v_tiles_of(int64_t n_vocab, int bn) { return (n_vocab + bn - 1) / bn; }

int pick_bn(int64_t m_tiles, int64_t n_vocab, int sms) {
    auto cost = [&](int bn) {
        const int64_t tiles = m_tiles * v_tiles_of(n_vocab, bn);
        return double((tiles + sms - 1) / sms) * bn;
    };
    return cost(kNarrowBN) < 0.97 * cost(kWideBN) ? kNarrowBN : kWideBN;
}

template <int BN, bool kFewRows>
int launch_lm(const void* hidden, const void* weight, const LmArgs& a, int64_t hidden_dim, int sms,
              cudaStream_t stream) {
    using T = LmTile<BN, kFewRows>;
    CUtensorMap map_h, map_w;
    if (!make_map(&map_h, hidden, uint64_t(hidden_dim), uint64_t(a.rows), uint32_t(T::kARows)) ||
        !make_map(&map_w, weight, uint64_t(hidden_dim), uint64_t(a.n_vocab), BN))
        return LOOM_SELECT_ECUDA;
    static std::once_flag attr_once[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return LOOM_SELECT_ECUDA;
    cudaError_t attr_err = cudaSuccess;
    std::call_once(attr_once[dev], [&] {
        attr_err = cudaFuncSetAttribute(lm_head_argmax_kernel<BN, kFewRows>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        int(T::kSmemBytes));
    });
    if (attr_err != cudaSuccess) return LOOM_SELECT_ECUDA;
    const int64_t tiles = int64_t(a.m_tiles) * a.v_tiles;
    const int grid = int(tiles < sms ? tiles : sms);
    lm_head_argmax_kernel<BN, kFewRows><<<grid, kThreads, T::kSmemBytes, stream>>>(map_h, map_w, a);
    return cudaGetLastError() == cudaSuccess ? LOOM_SELECT_OK : LOOM_SELECT_ECUDA;
}

}  // namespace
}  // namespace loom_select

using namespace loom_select;

extern "C" {

LOOM_SELECT_API size_t loom_lm_head_workspace_size(int64_t rows, int64_t n_vocab) {
    if (rows <= 0 || n_vocab <= 0) return 0;
    return ws_layout(sizeof(float4), rows * v_tiles_of(n_vocab, kNarrowBN)).bytes;
}

LOOM_SELECT_API int loom_lm_head_argmax(const void* hidden, const void* weight, int64_t rows, int64_t hidden_dim,
                                        int64_t n_vocab, int32_t* out_ids, float* out_logit, float* out_lse,
                                        void* workspace, size_t workspace_bytes, void* stream) {
    if (!hidden || !weight || !out_ids) return LOOM_SELECT_EINVAL;
    if (rows <= 0 || hidden_dim <= 0 || n_vocab <= 0) return LOOM_SELECT_EINVAL;
    if (hidden_dim % kBK != 0 || rows > (int64_t(1) << 31) - 1 || n_vocab > (int64_t(1) << 31) - 1 ||
        hidden_dim > (int64_t(1) << 20))
        return LOOM_SELECT_ESHAPE;
    if (reinterpret_cast<uintptr_t>(hidden) % 16 != 0 || reinterpret_cast<uintptr_t>(weight) % 16 != 0)
        return LOOM_SELECT_EINVAL;
    const int64_t mt = (rows + kBM - 1) / kBM;
    const int64_t vt_max = v_tiles_of(n_vocab, kNarrowBN);
    if (mt * vt_max > (int64_t(1) << 31) - 1) return LOOM_SELECT_ESHAPE;
    const WsLayout l = ws_layout(sizeof(float4), rows * vt_max);
    if (!workspace || workspace_bytes < l.bytes || reinterpret_cast<uintptr_t>(workspace) % kWsAlign != 0)
        return LOOM_SELECT_EWORKSPACE;
    int st = LOOM_SELECT_OK;
    const int sms = device_sm_count(&st);
    if (st != LOOM_SELECT_OK) return st;

    const int bn = pick_bn(mt, n_vocab, sms);
    LmArgs a;
    a.rows = rows;
    a.n_vocab = n_vocab;
    a.k_blocks = int(hidden_dim / kBK);
    a.m_tiles = int(mt);
    a.v_tiles = int(v_tiles_of(n_vocab, bn));
    a.records = reinterpret_cast<float4*>(static_cast<char*>(workspace) + l.records);
    a.status = static_cast<int*>(workspace);
    a.want_lse = out_lse != nullptr;
    auto s = static_cast<cudaStream_t>(stream);
    const bool few = rows <= 16;
    if (bn == kNarrowBN)
        st = few ? launch_lm<kNarrowBN, true>(hidden, weight, a, hidden_dim, sms, s)
                 : launch_lm<kNarrowBN, false>(hidden, weight, a, hidden_dim, sms, s);
    else
        st = few ? launch_lm<kWideBN, true>(hidden, weight, a, hidden_dim, sms, s)
                 : launch_lm<kWideBN, false>(hidden, weight, a, hidden_dim, sms, s);
    if (st != LOOM_SELECT_OK) return st;
    if (rows <= 64)
        lm_merge_kernel<256><<<unsigned(rows), 256, 0, s>>>(a.records, rows, a.v_tiles, a.want_lse, out_ids, out_logit,
                                                             out_lse);
    else
        lm_merge_kernel<32><<<unsigned((rows + 7) / 8), 256, 0, s>>>(a.records, rows, a.v_tiles, a.want_lse, out_ids,
                                                                    out_logit, out_lse);
    return cudaGetLastError() == cudaSuccess ? LOOM_SELECT_OK : LOOM_SELECT_ECUDA;
}

}  // extern "C"
