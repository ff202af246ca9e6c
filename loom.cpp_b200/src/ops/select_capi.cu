// select_capi.cu -- the extern "C" entry points of include/loom_select.h.
//
// Host-side only: argument checks (all before anything is enqueued, mirroring the checks of
// src/core/lua_bridge.cpp:302-319 and :350-353 where loom.cpp has them), workspace layout, the choice
// of kernel and grid, and CUDA error mapping. No allocation, no synchronisation except in
// loom_select_read_status.
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cuda_runtime.h>

#include "loom_select.h"
#include "select_internal.h"

namespace loom_select {

int device_sm_count(int* status) {
    static std::atomic<int> cache[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        *status = LOOM_SELECT_ECUDA;
        return 0;
    }
    if (dev >= 0 && dev < 64) {
        const int c = cache[dev].load(std::memory_order_relaxed);
        if (c > 0) return c;
    }
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) {
        *status = LOOM_SELECT_ECUDA;
        return 0;
    }
    if (dev >= 0 && dev < 64) cache[dev].store(sms, std::memory_order_relaxed);
    return sms;
}

}  // namespace loom_select

using namespace loom_select;

namespace {

// Rows at most this wide are reduced one warp per row; wider rows stream through shared memory.
constexpr int64_t kShortRowMax = 8192;

bool dtype_ok(int dtype) { return dtype == LOOM_SELECT_F32 || dtype == LOOM_SELECT_BF16; }
int esz_of(int dtype) { return dtype == LOOM_SELECT_BF16 ? 2 : 4; }

int check_workspace(const void* ws, size_t have, size_t need) {
    if (!ws || have < need) return LOOM_SELECT_EWORKSPACE;
    if (reinterpret_cast<uintptr_t>(ws) % kWsAlign != 0) return LOOM_SELECT_EWORKSPACE;
    return LOOM_SELECT_OK;
}

int map_cuda(cudaError_t e) { return e == cudaSuccess ? LOOM_SELECT_OK : LOOM_SELECT_ECUDA; }

int check_params(const loom_sample_params* p, int64_t vocab, bool allow_greedy) {
    if (!p) return LOOM_SELECT_EINVAL;
    const float T = p->temperature, r = p->repetition_penalty, pp = p->top_p;
    if (!(T >= 0.0f) || std::isinf(T)) return LOOM_SELECT_EPARAM;
    if (T == 0.0f && !allow_greedy) return LOOM_SELECT_EPARAM;
    if (!(r > 0.0f) || std::isinf(r)) return LOOM_SELECT_EPARAM;
    if (p->top_k < 1 || p->top_k > LOOM_SELECT_MAX_TOP_K || p->top_k > vocab) return LOOM_SELECT_EPARAM;
    if (!(pp > 0.0f && pp <= 1.0f)) return LOOM_SELECT_EPARAM;
    return LOOM_SELECT_OK;
}

size_t sample_ws_bytes(int64_t rows, int32_t top_k) {
    return ws_layout(sample_record_bytes(top_k), kStreamRecordSlots).bytes;
}

}  // namespace

extern "C" {

const char* loom_select_strerror(int status) {
    switch (status) {
        case LOOM_SELECT_OK: return "ok";
        case LOOM_SELECT_EINVAL: return "invalid argument (null pointer, non-positive size or row_stride < n_vocab)";
        case LOOM_SELECT_EDTYPE: return "unsupported dtype (expected LOOM_SELECT_F32 or LOOM_SELECT_BF16)";
        case LOOM_SELECT_EWINDOW: return "id window is not a non-empty sub-range of the row";
        case LOOM_SELECT_EWORKSPACE: return "workspace is NULL, too small or not 256-byte aligned";
        case LOOM_SELECT_ECUDA: return "a CUDA runtime call failed";
        case LOOM_SELECT_ETIMEOUT: return "a bounded device-side wait gave up; outputs are invalid";
        case LOOM_SELECT_EHISTORY: return "a history id lies outside the vocabulary";
        case LOOM_SELECT_EPARAM: return "sampling parameter out of range";
        case LOOM_SELECT_ESHAPE: return "size beyond what the kernels support";
        default: return "unknown status";
    }
}

int loom_select_abi_version(void) { return 100; }

size_t loom_argmax_workspace_size(int64_t rows, int64_t n_vocab) {
    if (rows <= 0 || n_vocab <= 0) return kWsAlign;
    return ws_layout(8, kStreamRecordSlots).bytes;
}

size_t loom_argmax_windows_workspace_size(int64_t rows, int32_t n_windows) {
    if (rows <= 0 || n_windows <= 0) return kWsAlign;
    return ws_layout(0, 0).bytes;  // the fixed regions: status, tickets, pair records
}

int loom_argmax_windows(const void* logits, int dtype, int64_t rows, int64_t n_vocab, int64_t row_stride,
                        const int64_t* lo, const int64_t* hi, int32_t n_windows, int32_t* out_ids, void* workspace,
                        size_t workspace_bytes, void* stream) {
    if (!dtype_ok(dtype)) return LOOM_SELECT_EDTYPE;
    if (!logits || !out_ids || !lo || !hi || rows <= 0 || n_vocab <= 0 || row_stride < n_vocab ||
        n_windows < 1 || n_windows > LOOM_SELECT_MAX_WINDOWS)
        return LOOM_SELECT_EINVAL;
    if (n_vocab > INT32_MAX) return LOOM_SELECT_ESHAPE;
    int64_t wlo[LOOM_SELECT_MAX_WINDOWS], whi[LOOM_SELECT_MAX_WINDOWS];
    for (int32_t w = 0; w < n_windows; ++w) {
        wlo[w] = lo[w];
        whi[w] = hi[w] < 0 ? n_vocab : hi[w];
        if (wlo[w] < 0 || wlo[w] >= whi[w] || whi[w] > n_vocab) return LOOM_SELECT_EWINDOW;
    }
    if (int st = check_workspace(workspace, workspace_bytes, loom_argmax_windows_workspace_size(rows, n_windows)))
        return st;
    int status = LOOM_SELECT_OK;
    const int sms = device_sm_count(&status);
    if (status) return status;
    const WsLayout l = ws_layout(0, 0);
    return map_cuda(launch_argmax_windows(dtype, logits, rows, row_stride, wlo, whi, n_windows, out_ids, workspace, l,
                                          sms, static_cast<cudaStream_t>(stream)));
}

size_t loom_sample_workspace_size(int64_t rows, int64_t n_vocab, int32_t top_k) {
    if (rows <= 0 || n_vocab <= 0 || top_k <= 0) return kWsAlign;
    return sample_ws_bytes(rows, top_k);
}

size_t loom_ctc_workspace_size(int64_t n_utt, int64_t n_frames) {
    if (n_utt <= 0 || n_frames <= 0) return kWsAlign;
    return ws_layout(sizeof(int32_t), n_utt * n_frames).bytes;
}

size_t loom_shard_record_bytes(int32_t top_k) { return top_k > 0 ? sample_record_bytes(top_k) : 0; }

int loom_select_workspace_init(void* workspace, size_t workspace_bytes, void* stream) {
    if (!workspace || workspace_bytes < kWsAlign) return LOOM_SELECT_EWORKSPACE;
    return map_cuda(cudaMemsetAsync(workspace, 0, workspace_bytes, static_cast<cudaStream_t>(stream)));
}

int loom_select_read_status(void* workspace, void* stream) {
    if (!workspace) return LOOM_SELECT_EWORKSPACE;
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    int value = 0;
    if (cudaMemcpyAsync(&value, workspace, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess)
        return LOOM_SELECT_ECUDA;
    if (cudaStreamSynchronize(st) != cudaSuccess) return LOOM_SELECT_ECUDA;
    if (value != 0) {
        if (cudaMemsetAsync(workspace, 0, sizeof(int), st) != cudaSuccess) return LOOM_SELECT_ECUDA;
        if (cudaStreamSynchronize(st) != cudaSuccess) return LOOM_SELECT_ECUDA;
    }
    return value;
}

int loom_select_test_wait_fault(void* workspace, int64_t wait_limit_ns, int32_t withhold_stage, void* stream) {
    if (!workspace) return LOOM_SELECT_EWORKSPACE;
    if (wait_limit_ns <= 0 || withhold_stage < -1) return LOOM_SELECT_EINVAL;
    // the header layout read by read_wait_fault (select_device.cuh): bytes [8, 16) and [16, 20)
    struct {
        uint64_t limit_ns;
        int32_t withhold;
    } hdr{static_cast<uint64_t>(wait_limit_ns), withhold_stage + 1};
    // (pageable source: the copy has read it before this returns)
    return map_cuda(cudaMemcpyAsync(static_cast<unsigned char*>(workspace) + 8, &hdr, 12, cudaMemcpyHostToDevice,
                                    static_cast<cudaStream_t>(stream)));
}

int loom_argmax_rows(const void* logits, int dtype, int64_t rows, int64_t n_vocab, int64_t row_stride, int64_t lo,
                     int64_t hi, int32_t* out_ids, void* workspace, size_t workspace_bytes, void* stream) {
    if (!dtype_ok(dtype)) return LOOM_SELECT_EDTYPE;
    if (!logits || !out_ids || rows <= 0 || n_vocab <= 0 || row_stride < n_vocab) return LOOM_SELECT_EINVAL;
    if (hi < 0) hi = n_vocab;
    if (lo < 0 || lo >= hi || hi > n_vocab) return LOOM_SELECT_EWINDOW;
    if (n_vocab > INT32_MAX) return LOOM_SELECT_ESHAPE;
    const int64_t width = hi - lo;
    if (int st = check_workspace(workspace, workspace_bytes, loom_argmax_workspace_size(rows, n_vocab))) return st;
    int status = LOOM_SELECT_OK;
    const int sms = device_sm_count(&status);
    if (status) return status;
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    const void* base = static_cast<const unsigned char*>(logits) + lo * esz_of(dtype);
    if (width <= kShortRowMax) return map_cuda(launch_rows_argmax(dtype, base, rows, width, row_stride, lo, out_ids, sms, st));
    if (rows * width <= kChunkArgmaxMaxElems) {
        // small batches (a decode step): chunks of the rows spread over every SM
        const WsLayout l = ws_layout(0, 0);
        return map_cuda(launch_argmax_windows(dtype, logits, rows, row_stride, &lo, &hi, 1, out_ids, workspace, l, sms, st));
    }
    const WsLayout l = ws_layout(8, kStreamRecordSlots);
    const int ctas = stream_ctas(rows, width, 2 * sms);  // two argmax CTAs per SM
    return map_cuda(launch_argmax_stream(dtype, base, rows, width, row_stride, lo, out_ids, workspace, l, ctas, st));
}

int loom_sample_rows(const void* logits, int dtype, int64_t rows, int64_t n_vocab, int64_t row_stride,
                     const int32_t* history, int32_t history_len, const float* u, const loom_sample_params* params,
                     int32_t* out_ids, float* out_prob, float* out_logp, int32_t* out_topk_ids, void* workspace,
                     size_t workspace_bytes, void* stream) {
    if (!dtype_ok(dtype)) return LOOM_SELECT_EDTYPE;
    if (!logits || !u || !out_ids || !out_prob || rows <= 0 || n_vocab <= 0 || row_stride < n_vocab ||
        history_len < 0 || (history_len > 0 && !history))
        return LOOM_SELECT_EINVAL;
    if (int st = check_params(params, n_vocab, true)) return st;
    if (n_vocab > INT32_MAX || history_len > kMaxHistory) return LOOM_SELECT_ESHAPE;
    if (int st = check_workspace(workspace, workspace_bytes, sample_ws_bytes(rows, params->top_k))) return st;
    int status = LOOM_SELECT_OK;
    const int sms = device_sm_count(&status);
    if (status) return status;
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
    a.temperature = params->temperature;
    a.penalty = params->repetition_penalty;
    a.top_p = params->top_p;
    a.top_k = params->top_k;
    a.out_ids = out_ids;
    a.out_prob = out_prob;
    a.out_logp = out_logp;
    a.out_topk = out_topk_ids;
    a.shard_out = nullptr;
    const WsLayout l = ws_layout(sample_record_bytes(params->top_k), kStreamRecordSlots);
    return map_cuda(launch_sample_stream(a, workspace, l, sample_ctas(rows, n_vocab, sms),
                                         static_cast<cudaStream_t>(stream)));
}

int loom_sample_shard_partial(const void* logits, int dtype, int64_t rows, int64_t shard_vocab, int64_t row_stride,
                              int64_t vocab_offset, int64_t vocab_total, const int32_t* history, int32_t history_len,
                              const loom_sample_params* params, void* out_records, void* workspace,
                              size_t workspace_bytes, void* stream) {
    if (!dtype_ok(dtype)) return LOOM_SELECT_EDTYPE;
    if (!logits || !out_records || rows <= 0 || shard_vocab <= 0 || row_stride < shard_vocab || vocab_offset < 0 ||
        vocab_offset + shard_vocab > vocab_total || history_len < 0 || (history_len > 0 && !history))
        return LOOM_SELECT_EINVAL;
    if (int st = check_params(params, vocab_total, false)) return st;
    if (vocab_total > INT32_MAX || history_len > kMaxHistory) return LOOM_SELECT_ESHAPE;
    if (int st = check_workspace(workspace, workspace_bytes, sample_ws_bytes(rows, params->top_k))) return st;
    int status = LOOM_SELECT_OK;
    const int sms = device_sm_count(&status);
    if (status) return status;
    SampleLaunch a{};
    a.dtype = dtype;
    a.logits = logits;
    a.rows = rows;
    a.width = shard_vocab;
    a.row_stride = row_stride;
    a.vocab_offset = vocab_offset;
    a.vocab_limit = vocab_total;
    a.history = history;
    a.history_len = history_len;
    a.u = nullptr;
    a.temperature = params->temperature;
    a.penalty = params->repetition_penalty;
    a.top_p = params->top_p;
    a.top_k = params->top_k;
    a.shard_out = out_records;
    const WsLayout l = ws_layout(sample_record_bytes(params->top_k), kStreamRecordSlots);
    return map_cuda(launch_sample_stream(a, workspace, l, sample_ctas(rows, shard_vocab, sms),
                                         static_cast<cudaStream_t>(stream)));
}

int loom_sample_shard_merge(const void* records, int32_t n_shards, int64_t rows, const float* u,
                            const loom_sample_params* params, int32_t* out_ids, float* out_prob, float* out_logp,
                            int32_t* out_topk_ids, void* stream) {
    if (!records || n_shards <= 0 || rows <= 0 || !u || !out_ids || !out_prob) return LOOM_SELECT_EINVAL;
    if (int st = check_params(params, INT32_MAX, false)) return st;
    if (rows > INT32_MAX) return LOOM_SELECT_ESHAPE;
    // the merge holds every shard's candidates of a row in shared memory, pruning as it goes
    return map_cuda(launch_shard_merge(records, n_shards, rows, u, params->top_k, params->top_p, out_ids, out_prob,
                                       out_logp, out_topk_ids, static_cast<cudaStream_t>(stream)));
}

int loom_ctc_greedy(const void* logits, int dtype, int64_t n_utt, int64_t n_frames, int64_t n_classes, int32_t blank,
                    int32_t* out_ids, int32_t* out_frames, int32_t* out_len, int32_t* out_frame_ids,
                    float* out_frame_logp, void* workspace, size_t workspace_bytes, void* stream) {
    if (!dtype_ok(dtype)) return LOOM_SELECT_EDTYPE;
    if (!logits || !out_ids || !out_frames || !out_len || n_utt <= 0 || n_frames <= 0 || n_classes <= 0)
        return LOOM_SELECT_EINVAL;
    if (n_classes > INT32_MAX || n_frames > INT32_MAX || n_utt > kCtcMaxUtt) return LOOM_SELECT_ESHAPE;
    if (int st = check_workspace(workspace, workspace_bytes, loom_ctc_workspace_size(n_utt, n_frames))) return st;
    int status = LOOM_SELECT_OK;
    const int sms = device_sm_count(&status);
    if (status) return status;
    const WsLayout l = ws_layout(sizeof(int32_t), n_utt * n_frames);
    return map_cuda(launch_ctc(dtype, logits, n_utt, n_frames, n_classes, blank, out_ids, out_frames, out_len,
                               out_frame_ids, out_frame_logp, workspace, l, sms, static_cast<cudaStream_t>(stream)));
}

}  // extern "C"
