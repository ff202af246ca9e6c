// select_device.cuh -- device helpers shared by the logits->token kernels (sm_100a).
//
// mbarrier + bulk-copy (TMA, non-tensor, no multicast) wrappers, bounded waits, the chain's ordering
// keys and element loads. Every wait in these kernels is bounded by the GPU global timer: a wait that
// runs out records LOOM_SELECT_ETIMEOUT in the workspace status word and returns false, and the
// caller winds its work down instead of spinning.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>

#include "loom_select.h"
#include "loom_select_math.h"

namespace loom_select {

// A bounded wait gives up after this long (the whole job normally takes well under a millisecond).
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Test hook in the workspace header (written only by loom_select_test_wait_fault; zero otherwise):
// bytes [8, 16) a wait limit in ns replacing kWaitLimitNs (0: the default), bytes [16, 20) the
// index of one stage that CTA 0's producer of a streamed kernel leaves unissued (0: none; the value
// is the index + 1), so that the consumers' bounded waits run out.
struct WaitFault {
    uint64_t limit_ns;
    int32_t withhold;  // stage index + 1, or 0
};

__device__ __forceinline__ WaitFault read_wait_fault(const int* status_word) {
    WaitFault f;
    const uint64_t lim = *reinterpret_cast<const volatile uint64_t*>(status_word + 2);
    f.limit_ns = lim ? lim : kWaitLimitNs;
    f.withhold = *reinterpret_cast<const volatile int32_t*>(status_word + 4);
    return f;
}

// Records the first device-side error of a call in the workspace status word.
__device__ __forceinline__ void record_status(int* status_word, int code) {
    atomicCAS(status_word, 0, code);
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// try_wait that may suspend the thread until the phase completes, for at most kSuspendHintNs: a
// waiting warp sleeps instead of spinning, so it takes no issue slots from the warps that work.
constexpr uint32_t kSuspendHintNs = 1000000u;

__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, 0, p; }"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity), "r"(kSuspendHintNs)
        : "memory");
    return done != 0;
}

// Waits for the phase of `bar` with the given parity to complete; false (and a recorded timeout)
// if it does not within kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int* status_word,
                                                  uint64_t limit_ns = kWaitLimitNs) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (;;) {
        if (mbar_try_wait_sleep(bar, parity)) return true;
        if (global_timer_ns() - t0 > limit_ns) {
            record_status(status_word, LOOM_SELECT_ETIMEOUT);
            return false;
        }
    }
}

// One bulk copy global -> this CTA's shared memory, completing `bytes` of the barrier's tx count.
// Both addresses 16-byte aligned, bytes a multiple of 16. No multicast.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(smem_dst)),
        "l"(gmem_src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// Orders this thread's generic-proxy shared-memory accesses before later async-proxy (bulk copy)
// writes to the same bytes.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Named barrier among the first `threads` threads of the CTA (id 0 is __syncthreads).
__device__ __forceinline__ void named_barrier(uint32_t id, uint32_t threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Named barrier that also returns, to every participant, the OR of the participants' predicates.
__device__ __forceinline__ bool named_barrier_or(uint32_t id, uint32_t threads, bool pred) {
    uint32_t out;
    asm volatile(
        "{ .reg .pred p, q; setp.ne.u32 p, %1, 0; bar.red.or.pred q, %2, %3, p; selp.u32 %0, 1, 0, q; }"
        : "=r"(out)
        : "r"(static_cast<uint32_t>(pred)), "r"(id), "r"(threads)
        : "memory");
    return out != 0;
}

// Barrier over the kNT consumer threads of a CTA (named barrier 1).
template <int kNT>
__device__ __forceinline__ void group_sync() {
    named_barrier(1, kNT);
}

__device__ __forceinline__ float bf16_bits_to_float(uint32_t h) { return __uint_as_float(h << 16); }

template <int kDtype>
__device__ __forceinline__ float load_global_elem(const void* base, int64_t i) {
    if constexpr (kDtype == LOOM_SELECT_BF16) {
        return bf16_bits_to_float(__ldg(reinterpret_cast<const unsigned short*>(base) + i));
    } else {
        return __ldg(reinterpret_cast<const float*>(base) + i);
    }
}

// Inverse of loom_order_key for non-NaN keys (NaN keys give a NaN); -0 comes back as +0.
__device__ __forceinline__ float order_key_to_float(uint32_t k) {
    const uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
    return __uint_as_float(u);
}

__device__ __forceinline__ float rank_key_value(uint64_t key) {
    return order_key_to_float(static_cast<uint32_t>(key >> 32));
}

__device__ __forceinline__ int32_t rank_key_id(uint64_t key) {
    return static_cast<int32_t>(0xffffffffu - static_cast<uint32_t>(key));
}

}  // namespace loom_select
