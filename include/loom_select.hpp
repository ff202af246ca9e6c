// loom_select.hpp -- loom.cpp's host API for token selection, on the B200 kernels.
//
// Header-only C++ over the C-ABI of loom_select.h. Each function keeps the name, the argument
// meaning, the checks and the error text of the loom.cpp function it stands in for, and takes the
// logits where the engine already has them: in device memory (a ggml CUDA tensor's `data`, with
// `nb[1] / sizeof(float)` as the row stride) -- so the per-row device-to-host copy of
// `ggml_backend_tensor_get` disappears.
//
//   loom::select::argmax                 Generator::argmax                src/core/generation.cpp:64-74
//   loom::select::argmax_tensor_row      argmax_tensor_row                src/core/lua_bridge.cpp:302-330
//   loom::select::argmax_tensor_rows     argmax_tensor_rows               src/core/lua_bridge.cpp:343-365
//   loom::select::ctc_greedy_decode      loom::ctc_greedy_decode          src/core/ctc_decode.cpp:7-31
//   loom::select::sample_rows            (the sampling chain; no loom.cpp counterpart)
//
// Errors throw loom::Error -- the engine's own class when include/loom/loom_errors.h is on the
// include path, otherwise a class of the same name and base declared here.
// Unlike the C-ABI, these helpers allocate, but only to grow: each thread keeps one device workspace,
// one device output area and one pinned host area, reused by every later call that fits in them.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <string>
#include <vector>

#include "loom_select.h"

#if __has_include("loom/loom_errors.h")
#include "loom/loom_errors.h"
#else
#include <stdexcept>
namespace loom {
class Error : public std::runtime_error {
public:
    explicit Error(const std::string& what) : std::runtime_error(what) {}
};
}  // namespace loom
#endif

namespace loom {
namespace select {

namespace detail {

inline void check(int status, const std::string& what) {
    if (status != LOOM_SELECT_OK) throw Error(what + ": " + loom_select_strerror(status));
}

inline void check_cuda(cudaError_t e, const std::string& what) {
    if (e != cudaSuccess) throw Error(what + ": " + cudaGetErrorString(e));
}

// Per-thread state of the helpers below: one device workspace (zeroed when it is (re)allocated),
// one device area for a call's outputs and one pinned host area to read them back into. Each grows
// only when a call needs more than it holds, so after the first call of a given size the helpers
// allocate no memory on the device or in pinned host memory. The areas belong to the device that
// was current when they were made; a call on another device makes new ones.
class ThreadState {
public:
    ~ThreadState() { release(); }
    void* workspace(size_t bytes, cudaStream_t stream) {
        on_current_device();
        if (bytes > ws_size_) {
            if (ws_) cudaFree(ws_);
            ws_ = nullptr;
            ws_size_ = 0;
            check_cuda(cudaMalloc(&ws_, bytes), "cudaMalloc(workspace)");
            ws_size_ = bytes;
            check(loom_select_workspace_init(ws_, ws_size_, stream), "loom_select_workspace_init");
        }
        return ws_;
    }
    size_t workspace_size() const { return ws_size_; }
    // Device memory for `bytes` of outputs (256-byte aligned).
    void* device_out(size_t bytes) {
        on_current_device();
        if (bytes > dout_size_) {
            if (dout_) cudaFree(dout_);
            dout_ = nullptr;
            dout_size_ = 0;
            check_cuda(cudaMalloc(&dout_, bytes), "cudaMalloc(outputs)");
            dout_size_ = bytes;
        }
        return dout_;
    }
    // Pinned host memory for `bytes` read back from device_out.
    void* host_out(size_t bytes) {
        if (bytes > hout_size_) {
            if (hout_) cudaFreeHost(hout_);
            hout_ = nullptr;
            hout_size_ = 0;
            check_cuda(cudaMallocHost(&hout_, bytes), "cudaMallocHost(outputs)");
            hout_size_ = bytes;
        }
        return hout_;
    }

private:
    void on_current_device() {
        int dev = -1;
        check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
        if (dev != dev_) {
            release_device();
            dev_ = dev;
        }
    }
    void release_device() {
        if (ws_) cudaFree(ws_);
        if (dout_) cudaFree(dout_);
        ws_ = dout_ = nullptr;
        ws_size_ = dout_size_ = 0;
    }
    void release() {
        release_device();
        if (hout_) cudaFreeHost(hout_);
        hout_ = nullptr;
        hout_size_ = 0;
    }
    void* ws_ = nullptr;
    size_t ws_size_ = 0;
    void* dout_ = nullptr;
    size_t dout_size_ = 0;
    void* hout_ = nullptr;
    size_t hout_size_ = 0;
    int dev_ = -1;
};

inline ThreadState& state() {
    thread_local ThreadState st;
    return st;
}

inline size_t align256(size_t b) { return (b + 255) / 256 * 256; }

// Copies `bytes` of device outputs to the thread's pinned host area and waits for them.
inline const void* read_back(const void* d, size_t bytes, cudaStream_t stream) {
    void* h = state().host_out(bytes > 0 ? bytes : 1);
    if (bytes) {
        check_cuda(cudaMemcpyAsync(h, d, bytes, cudaMemcpyDeviceToHost, stream), "cudaMemcpyAsync");
        check_cuda(cudaStreamSynchronize(stream), "cudaStreamSynchronize");
    }
    return h;
}

}  // namespace detail

// argmax_tensor_row (src/core/lua_bridge.cpp:302-330): the highest-scoring ABSOLUTE id of row
// `requested_row` (negative: the last row) over the id window [lo, hi) (hi < 0: the whole row).
inline int64_t argmax_tensor_row(const float* d_logits, int64_t n_vocab, int64_t n_rows, int64_t row_stride,
                                 int64_t requested_row, const char* fname, int64_t lo = 0, int64_t hi = -1,
                                 cudaStream_t stream = nullptr) {
    const int64_t row = requested_row < 0 ? n_rows - 1 : requested_row;
    if (n_vocab <= 0 || row < 0 || row >= n_rows) {
        throw Error(std::string(fname) + ": row " + std::to_string(requested_row) + " out of range for an output with " +
                    std::to_string(n_rows) + " row(s) of width " + std::to_string(n_vocab));
    }
    if (hi < 0) hi = n_vocab;
    if (lo < 0 || lo >= hi || hi > n_vocab) {
        throw Error(std::string(fname) + ": id window [" + std::to_string(lo) + ", " + std::to_string(hi) +
                    ") is not a non-empty sub-range of this output's " + std::to_string(n_vocab) + " class(es)");
    }
    detail::ThreadState& st = detail::state();
    void* ws = st.workspace(loom_argmax_workspace_size(1, n_vocab), stream);
    int32_t* out = static_cast<int32_t*>(st.device_out(sizeof(int32_t)));
    detail::check(loom_argmax_rows(d_logits + row * row_stride, LOOM_SELECT_F32, 1, n_vocab, n_vocab, lo, hi, out, ws,
                                   st.workspace_size(), stream),
                  fname);
    return *static_cast<const int32_t*>(detail::read_back(out, sizeof(int32_t), stream));
}

// argmax_tensor_rows (src/core/lua_bridge.cpp:343-365): one id per row, in row order, as the Lua
// binding's numbers.
inline std::vector<double> argmax_tensor_rows(const float* d_logits, int64_t n_classes, int64_t n_rows,
                                              int64_t row_stride, const char* fname, cudaStream_t stream = nullptr) {
    if (n_classes <= 0 || n_rows <= 0) {
        throw Error(std::string(fname) + ": output is " + std::to_string(n_classes) + "x" + std::to_string(n_rows) +
                    ", which has no rows to reduce");
    }
    detail::ThreadState& st = detail::state();
    const size_t bytes = static_cast<size_t>(n_rows) * sizeof(int32_t);
    void* ws = st.workspace(loom_argmax_workspace_size(n_rows, n_classes), stream);
    int32_t* out = static_cast<int32_t*>(st.device_out(bytes));
    detail::check(loom_argmax_rows(d_logits, LOOM_SELECT_F32, n_rows, n_classes, row_stride, 0, -1, out, ws,
                                   st.workspace_size(), stream),
                  fname);
    const int32_t* ids = static_cast<const int32_t*>(detail::read_back(out, bytes, stream));
    return std::vector<double>(ids, ids + n_rows);
}

// Generator::argmax (src/core/generation.cpp:64-74) on one device row of n_vocab floats.
inline int32_t argmax(const float* d_row, int64_t n_vocab, cudaStream_t stream = nullptr) {
    return static_cast<int32_t>(argmax_tensor_row(d_row, n_vocab, 1, n_vocab, 0, "argmax", 0, -1, stream));
}

// loom::ctc_greedy_decode (src/core/ctc_decode.cpp:7-31), same signature, logits in device memory.
inline std::vector<int32_t> ctc_greedy_decode(const float* d_logits, int64_t n_frames, int64_t n_classes,
                                              int32_t blank_id, cudaStream_t stream = nullptr) {
    if (n_frames <= 0) return {};
    // device outputs: [len (256 B)] [ids: n_frames] [frames: n_frames]; len and ids come back in one copy
    detail::ThreadState& st = detail::state();
    const size_t ids_bytes = detail::align256(static_cast<size_t>(n_frames) * sizeof(int32_t));
    void* ws = st.workspace(loom_ctc_workspace_size(1, n_frames), stream);
    unsigned char* d = static_cast<unsigned char*>(st.device_out(256 + 2 * ids_bytes));
    int32_t* len = reinterpret_cast<int32_t*>(d);
    int32_t* ids = reinterpret_cast<int32_t*>(d + 256);
    int32_t* frames = reinterpret_cast<int32_t*>(d + 256 + ids_bytes);
    detail::check(loom_ctc_greedy(d_logits, LOOM_SELECT_F32, 1, n_frames, n_classes, blank_id, ids, frames, len, nullptr,
                                  nullptr, ws, st.workspace_size(), stream),
                  "ctc_greedy_decode");
    const unsigned char* h = static_cast<const unsigned char*>(detail::read_back(d, 256 + ids_bytes, stream));
    const int32_t n = *reinterpret_cast<const int32_t*>(h);
    const int32_t* hid = reinterpret_cast<const int32_t*>(h + 256);
    return std::vector<int32_t>(hid, hid + n);
}

struct SampleResult {
    std::vector<int32_t> ids;
    std::vector<float> probs;
};

// The sampling chain (loom_sample_rows) over device logits [rows, n_vocab] (row stride
// row_stride), device history [rows, history_len] and device uniforms [rows]; results on the host.
inline SampleResult sample_rows(const float* d_logits, int64_t rows, int64_t n_vocab, int64_t row_stride,
                                const int32_t* d_history, int32_t history_len, const float* d_u,
                                const loom_sample_params& params, cudaStream_t stream = nullptr) {
    const size_t n = static_cast<size_t>(rows > 0 ? rows : 0);
    const size_t ids_bytes = detail::align256(n * sizeof(int32_t));
    detail::ThreadState& st = detail::state();
    void* ws = st.workspace(loom_sample_workspace_size(rows, n_vocab, params.top_k), stream);
    unsigned char* d = static_cast<unsigned char*>(st.device_out(ids_bytes + n * sizeof(float) + 1));
    int32_t* ids = reinterpret_cast<int32_t*>(d);
    float* probs = reinterpret_cast<float*>(d + ids_bytes);
    detail::check(loom_sample_rows(d_logits, LOOM_SELECT_F32, rows, n_vocab, row_stride, d_history, history_len, d_u,
                                   &params, ids, probs, nullptr, nullptr, ws, st.workspace_size(), stream),
                  "sample_rows");
    const int status = loom_select_read_status(ws, stream);
    if (status != LOOM_SELECT_OK) detail::check(status, "sample_rows");
    const unsigned char* h = static_cast<const unsigned char*>(detail::read_back(d, ids_bytes + n * sizeof(float), stream));
    SampleResult r;
    r.ids.assign(reinterpret_cast<const int32_t*>(h), reinterpret_cast<const int32_t*>(h) + n);
    r.probs.assign(reinterpret_cast<const float*>(h + ids_bytes), reinterpret_cast<const float*>(h + ids_bytes) + n);
    return r;
}

struct GreedyResult {
    std::vector<int32_t> ids;    // per row: the greedy id
    std::vector<float> logit;    // its logit
    std::vector<float> logprob;  // its log-probability (logit - log-sum-exp of the row)
};

// The LM head's ggml_mul_mat(lm_head, hidden) followed by Generator::argmax
// (src/core/generation.cpp:64-74), fused (loom_lm_head_argmax): d_hidden [rows, hidden_dim] and
// d_weight [n_vocab, hidden_dim] are bf16 device arrays with packed rows; the logits are never
// written. Results on the host.
inline GreedyResult lm_head_argmax(const void* d_hidden, const void* d_weight, int64_t rows, int64_t hidden_dim,
                                   int64_t n_vocab, cudaStream_t stream = nullptr) {
    const size_t n = static_cast<size_t>(rows > 0 ? rows : 0);
    const size_t col = detail::align256(n * sizeof(float));
    detail::ThreadState& st = detail::state();
    void* ws = st.workspace(loom_lm_head_workspace_size(rows, n_vocab), stream);
    unsigned char* d = static_cast<unsigned char*>(st.device_out(3 * col + 1));
    int32_t* ids = reinterpret_cast<int32_t*>(d);
    float* logit = reinterpret_cast<float*>(d + col);
    float* lse = reinterpret_cast<float*>(d + 2 * col);
    detail::check(loom_lm_head_argmax(d_hidden, d_weight, rows, hidden_dim, n_vocab, ids, logit, lse, ws,
                                      st.workspace_size(), stream),
                  "lm_head_argmax");
    const int status = loom_select_read_status(ws, stream);
    if (status != LOOM_SELECT_OK) detail::check(status, "lm_head_argmax");
    const unsigned char* h = static_cast<const unsigned char*>(detail::read_back(d, 3 * col, stream));
    GreedyResult r;
    r.ids.assign(reinterpret_cast<const int32_t*>(h), reinterpret_cast<const int32_t*>(h) + n);
    r.logit.assign(reinterpret_cast<const float*>(h + col), reinterpret_cast<const float*>(h + col) + n);
    const float* hl = reinterpret_cast<const float*>(h + 2 * col);
    r.logprob.resize(n);
    for (size_t i = 0; i < n; ++i) r.logprob[i] = r.logit[i] - hl[i];
    return r;
}

}  // namespace select
}  // namespace loom
