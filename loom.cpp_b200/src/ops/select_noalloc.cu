// select_noalloc.cu -- the sampling chain for callers that cannot allocate device memory.
//
// loom_sample_rows takes its scratch from a workspace the caller allocates. Some callers cannot do
// that: an engine whose device memory is all handed out up front by its own arena (ggml's backend
// allocator sizes one buffer for the whole graph), a serving loop that is not allowed to grow its
// device footprint after start-up, or a plugin host that gives its plugins no allocation hook.
// loom_sample_rows_noalloc serves them: the same kernel, with its scratch in one fixed array of this
// file that lives in device memory from the moment the library is loaded on a device until the
// process exits.
//
// The array is shared by every call on a device and keeps the last call's contents: each call first
// clears the part that must start at zero (the status word and the tickets); the records behind them
// are written before they are read. Two calls whose work can overlap on the GPU (different streams,
// or different host threads) race on it.
//
// The first call on a device looks the array's address up (cudaGetSymbolAddress, which also loads this
// file's device code on that device); make that first call before any stream capture. The address is
// kept for the life of the process, so this entry point must not be used on a device after a
// cudaDeviceReset there (the array may come back at another address).
#include <cmath>
#include <mutex>

#include <cuda_runtime.h>

#include "loom_select.h"
#include "select_internal.h"

namespace loom_select {
namespace {

// status word + tickets + the (unused here) pair region + 2 records per CTA of 16 + 8 * 64 bytes: the
// sampler's workspace layout (ws_layout) at top_k 64
constexpr size_t kNoAllocRecordBytes = 16 + 8 * LOOM_SELECT_NOALLOC_MAX_TOP_K;
constexpr size_t kNoAllocTicketBytes = ((kTicketSlots * sizeof(int32_t) + kWsAlign - 1) / kWsAlign) * kWsAlign;
constexpr size_t kNoAllocPairBytes = ((kChunkPairs * kChunkPairBytes + kWsAlign - 1) / kWsAlign) * kWsAlign;
constexpr size_t kNoAllocRecordsBytes =
    ((kNoAllocRecordBytes * kStreamRecordSlots + kWsAlign - 1) / kWsAlign) * kWsAlign;
constexpr size_t kNoAllocScratchBytes = kWsAlign + kNoAllocTicketBytes + kNoAllocPairBytes + kNoAllocRecordsBytes;
static_assert(kNoAllocScratchBytes == LOOM_SELECT_NOALLOC_SCRATCH_BYTES, "header constant out of date");

// The scratch. In host code this name is only a stand-in for the device array: its device address
// comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
void* g_scratch_ptr[kMaxDevices] = {};
std::mutex g_scratch_mutex;

// The device address of the scratch array on the current device, looked up once per device.
int scratch_on_current_device(void** out) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return LOOM_SELECT_ECUDA;
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    if (!g_scratch_ptr[dev]) {
        void* ptr = nullptr;
        if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || !ptr) return LOOM_SELECT_ECUDA;
        g_scratch_ptr[dev] = ptr;
    }
    *out = g_scratch_ptr[dev];
    return LOOM_SELECT_OK;
}

}  // namespace
}  // namespace loom_select

using namespace loom_select;

extern "C" int loom_sample_rows_noalloc(const void* logits, int dtype, int64_t rows, int64_t n_vocab,
                                        int64_t row_stride, const int32_t* history, int32_t history_len,
                                        const float* u, const loom_sample_params* params, int32_t* out_ids,
                                        float* out_prob, float* out_logp, int32_t* out_topk_ids,
                                        int32_t* out_status, void* stream) {
    // the checks of loom_sample_rows, then the size this scratch was made for
    if (dtype != LOOM_SELECT_F32 && dtype != LOOM_SELECT_BF16) return LOOM_SELECT_EDTYPE;
    if (!logits || !u || !out_ids || !out_prob || rows <= 0 || n_vocab <= 0 || row_stride < n_vocab ||
        history_len < 0 || (history_len > 0 && !history) || !params)
        return LOOM_SELECT_EINVAL;
    const float T = params->temperature, r = params->repetition_penalty, p = params->top_p;
    if (!(T >= 0.0f) || std::isinf(T) || !(r > 0.0f) || std::isinf(r) || params->top_k < 1 ||
        params->top_k > LOOM_SELECT_MAX_TOP_K || params->top_k > n_vocab || !(p > 0.0f && p <= 1.0f))
        return LOOM_SELECT_EPARAM;
    if (n_vocab > INT32_MAX || history_len > kMaxHistory) return LOOM_SELECT_ESHAPE;
    if (params->top_k > LOOM_SELECT_NOALLOC_MAX_TOP_K) return LOOM_SELECT_ESHAPE;

    void* scratch = nullptr;
    if (int st = scratch_on_current_device(&scratch)) return st;
    int sms = 0;
    {
        int status = LOOM_SELECT_OK;
        sms = device_sm_count(&status);
        if (status) return status;
    }
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    // the status word and the tickets start at zero for every call (no allocation: a memset)
    if (cudaMemsetAsync(scratch, 0, kWsAlign + kNoAllocTicketBytes, st) != cudaSuccess) return LOOM_SELECT_ECUDA;

    SampleLaunch a{};
    a.dtype = dtype;
    a.logits = logits;
    a.rows = rows;
    a.width = n_vocab;
    a.row_stride = row_stride;
    a.vocab_offset = 0;
    a.vocab_limit = n_vocab;
    a.history = history;
    a.history_len = history_len;
    a.u = u;
    a.temperature = T;
    a.penalty = r;
    a.top_p = p;
    a.top_k = params->top_k;
    a.out_ids = out_ids;
    a.out_prob = out_prob;
    a.out_logp = out_logp;
    a.out_topk = out_topk_ids;
    a.shard_out = nullptr;
    const WsLayout l = ws_layout(sample_record_bytes(params->top_k), kStreamRecordSlots);
    if (l.bytes > kNoAllocScratchBytes) return LOOM_SELECT_ESHAPE;
    // the grid loom_sample_rows would launch for the same call
    const int ctas = sample_ctas(rows, n_vocab, sms);
    if (launch_sample_stream(a, scratch, l, ctas, st) != cudaSuccess) return LOOM_SELECT_ECUDA;
    // the device-side status word (history ids out of range, a timed-out wait) for the caller
    if (out_status && cudaMemcpyAsync(out_status, scratch, sizeof(int32_t), cudaMemcpyDeviceToDevice, st) != cudaSuccess)
        return LOOM_SELECT_ECUDA;
    return LOOM_SELECT_OK;
}
