// select_internal.h -- host-side plumbing shared by the kernel files and the C-ABI (not installed).
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "loom_select.h"

namespace loom_select {

// ---- workspace layout (every region 256-byte aligned) ----
//   [0, 256)              status word (int32) of the device-side error report
//   [256, 256 + 8 KiB)    tickets: kTicketSlots int32 at a FIXED place for every call, zero between
//                         calls (each kernel returns the tickets it used to zero), so calls of any
//                         size and kind can share one workspace
//   [.., + 16 KiB)        pair records of the chunked argmax (kChunkPairs x 16 bytes), also zero
//                         between calls and touched by no other kernel
//   records / frames      per-call scratch, fully written before it is read
constexpr size_t kWsAlign = 256;
inline size_t ws_round(size_t b) { return (b + kWsAlign - 1) / kWsAlign * kWsAlign; }

constexpr int64_t kStreamSplitAlign = 64;
constexpr int64_t kStreamMinRange = 8192;
constexpr int kStreamMaxCtas = 1024;

// A CTA's range splits at most two rows (its first and its last), so a streamed call needs at
// most two partial-result records per CTA: slot 0 for the CTA's first row, slot 1 for its last.
// A split row counts its pieces on the ticket of its first piece's slot.
constexpr int64_t kStreamRecordSlots = 2 * kStreamMaxCtas;
constexpr int64_t kTicketSlots = 2 * kStreamMaxCtas;

// CTC: a CTA holds at most 62 whole utterances and the grid at most kTicketSlots CTAs.
constexpr int64_t kCtcMaxUtt = kTicketSlots * 62;

// The chunked argmax keeps one 16-byte record per (row, window) pair of a launch, at most this many.
constexpr int64_t kChunkPairs = 1024;
constexpr size_t kChunkPairBytes = 16;

struct WsLayout {
    size_t tickets = 0;
    size_t pairs = 0;
    size_t records = 0;
    size_t bytes = 0;
};

inline WsLayout ws_layout(size_t record_bytes, int64_t n_records) {
    WsLayout l;
    l.tickets = kWsAlign;
    l.pairs = l.tickets + ws_round(static_cast<size_t>(kTicketSlots) * sizeof(int32_t));
    l.records = l.pairs + ws_round(static_cast<size_t>(kChunkPairs) * kChunkPairBytes);
    l.bytes = l.records + ws_round(record_bytes * static_cast<size_t>(n_records));
    return l;
}

// CTAs for a streamed call of `rows` rows of `width`: up to `slots` (the resident CTAs), fewer when
// each would get under kStreamMinRange elements. With at least as many rows as CTAs the ranges are
// whole rows (split_point), and the count is chosen so that every CTA gets the same number of rows:
// the slowest CTA sets the time, so r = ceil(rows / slots) rows each over ceil(rows / r) CTAs.
inline int stream_ctas(int64_t rows, int64_t width, int slots) {
    int64_t g = slots;
    if (g > kStreamMaxCtas) g = kStreamMaxCtas;
    const int64_t by_size = rows * width / kStreamMinRange;
    if (g > by_size) g = by_size;
    if (g < 1) g = 1;
    if (rows >= g) {
        const int64_t per = (rows + g - 1) / g;
        g = (rows + per - 1) / per;
    }
    return static_cast<int>(g);
}

// Number of SMs of the current device (cached per device; the cache is safe to fill from several
// host threads at once).
int device_sm_count(int* status);

// Launchers (validated arguments; return a cudaError_t from the launch).
cudaError_t launch_argmax_stream(int dtype, const void* window_base, int64_t rows, int64_t width, int64_t row_stride,
                                 int64_t lo, int32_t* out_ids, void* workspace, const WsLayout& l, int ctas,
                                 cudaStream_t stream);

// Windowed / chunked argmax (select_windows.cu): every (row, window) pair cut into chunks that any CTA
// takes; a 16-byte record per pair in the workspace's pair region (rows in groups of at most
// kChunkPairs pairs per launch). loom_argmax_rows sends calls of at most kChunkArgmaxMaxElems
// elements there.
constexpr int kArgmaxMaxWindows = LOOM_SELECT_MAX_WINDOWS;
constexpr int64_t kChunkArgmaxMaxElems = int64_t(16) << 20;
cudaError_t launch_argmax_windows(int dtype, const void* logits, int64_t rows, int64_t row_stride, const int64_t* lo,
                                  const int64_t* hi, int32_t n_win, int32_t* out_ids, void* workspace,
                                  const WsLayout& l, int sms, cudaStream_t stream);

cudaError_t launch_rows_argmax(int dtype, const void* window_base, int64_t rows, int64_t width, int64_t row_stride,
                               int64_t lo, int32_t* out_ids, int sms, cudaStream_t stream);

cudaError_t launch_ctc(int dtype, const void* logits, int64_t n_utt, int64_t n_frames, int64_t n_classes,
                       int32_t blank, int32_t* out_ids, int32_t* out_frames, int32_t* out_len, int32_t* frame_ids,
                       float* frame_logp, void* workspace, const WsLayout& l, int sms, cudaStream_t stream);

struct SampleLaunch {
    int dtype;
    const void* logits;
    int64_t rows, width, row_stride;
    int64_t vocab_offset, vocab_limit;
    const int32_t* history;
    int32_t history_len;
    const float* u;
    float temperature, penalty, top_p;
    int32_t top_k;
    int32_t* out_ids;
    float* out_prob;
    float* out_logp;
    int32_t* out_topk;
    void* shard_out; // non-NULL: emit shard records instead of decisions
};

constexpr int kMaxHistory = LOOM_SELECT_MAX_HISTORY;
constexpr int kSampleCtasPerSm = 2;  // the sampler runs two CTAs per SM

size_t sample_record_bytes(int32_t top_k);
// The sampler's grid for a call (every sampling entry point launches this one).
inline int sample_ctas(int64_t rows, int64_t width, int sms) { return stream_ctas(rows, width, kSampleCtasPerSm * sms); }
cudaError_t launch_sample_stream(const SampleLaunch& a, void* workspace, const WsLayout& l, int ctas,
                                 cudaStream_t stream);
cudaError_t launch_shard_merge(const void* records, int32_t n_shards, int64_t rows, const float* u, int32_t top_k,
                               float top_p, int32_t* out_ids, float* out_prob, float* out_logp, int32_t* out_topk,
                               cudaStream_t stream);

}  // namespace loom_select
