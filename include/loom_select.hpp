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
// Unlike the C-ABI, these helpers allocate: each thread keeps one growing device workspace.
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

// A per-thread device workspace, zeroed when (re)allocated.
class Workspace {
public:
    ~Workspace() {
        if (ptr_) cudaFree(ptr_);
    }
    void* get(size_t bytes, cudaStream_t stream) {
        int dev = -1;
        check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
        if (!ptr_ || bytes > size_ || dev != dev_) {
            if (ptr_) cudaFree(ptr_);
            ptr_ = nullptr;
            check_cuda(cudaMalloc(&ptr_, bytes), "cudaMalloc(workspace)");
            size_ = bytes;
            dev_ = dev;
            check(loom_select_workspace_init(ptr_, size_, stream), "loom_select_workspace_init");
        }
        return ptr_;
    }
    size_t size() const { return size_; }

private:
    void* ptr_ = nullptr;
    size_t size_ = 0;
    int dev_ = -1;
};

inline Workspace& workspace() {
    thread_local Workspace ws;
    return ws;
}

template <class T>
class DeviceBuffer {
public:
    explicit DeviceBuffer(size_t n) {
        if (n) check_cuda(cudaMalloc(&p_, n * sizeof(T)), "cudaMalloc");
    }
    ~DeviceBuffer() {
        if (p_) cudaFree(p_);
    }
    DeviceBuffer(const DeviceBuffer&) = delete;
    DeviceBuffer& operator=(const DeviceBuffer&) = delete;
    T* get() const { return p_; }

private:
    T* p_ = nullptr;
};

template <class T>
std::vector<T> to_host(const T* d, size_t n, cudaStream_t stream) {
    std::vector<T> h(n);
    if (n) {
        check_cuda(cudaMemcpyAsync(h.data(), d, n * sizeof(T), cudaMemcpyDeviceToHost, stream), "cudaMemcpyAsync");
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
    detail::DeviceBuffer<int32_t> out(1);
    void* ws = detail::workspace().get(loom_argmax_workspace_size(1, n_vocab), stream);
    detail::check(loom_argmax_rows(d_logits + row * row_stride, LOOM_SELECT_F32, 1, n_vocab, n_vocab, lo, hi, out.get(),
                                   ws, detail::workspace().size(), stream),
                  fname);
    return detail::to_host(out.get(), 1, stream)[0];
}

// argmax_tensor_rows (src/core/lua_bridge.cpp:343-365): one id per row, in row order, as the Lua
// binding's numbers.
inline std::vector<double> argmax_tensor_rows(const float* d_logits, int64_t n_classes, int64_t n_rows,
                                              int64_t row_stride, const char* fname, cudaStream_t stream = nullptr) {
    if (n_classes <= 0 || n_rows <= 0) {
        throw Error(std::string(fname) + ": output is " + std::to_string(n_classes) + "x" + std::to_string(n_rows) +
                    ", which has no rows to reduce");
    }
    detail::DeviceBuffer<int32_t> out(static_cast<size_t>(n_rows));
    void* ws = detail::workspace().get(loom_argmax_workspace_size(n_rows, n_classes), stream);
    detail::check(loom_argmax_rows(d_logits, LOOM_SELECT_F32, n_rows, n_classes, row_stride, 0, -1, out.get(), ws,
                                   detail::workspace().size(), stream),
                  fname);
    const std::vector<int32_t> ids = detail::to_host(out.get(), static_cast<size_t>(n_rows), stream);
    return std::vector<double>(ids.begin(), ids.end());
}

// Generator::argmax (src/core/generation.cpp:64-74) on one device row of n_vocab floats.
inline int32_t argmax(const float* d_row, int64_t n_vocab, cudaStream_t stream = nullptr) {
    return static_cast<int32_t>(argmax_tensor_row(d_row, n_vocab, 1, n_vocab, 0, "argmax", 0, -1, stream));
}

// loom::ctc_greedy_decode (src/core/ctc_decode.cpp:7-31), same signature, logits in device memory.
inline std::vector<int32_t> ctc_greedy_decode(const float* d_logits, int64_t n_frames, int64_t n_classes,
                                              int32_t blank_id, cudaStream_t stream = nullptr) {
    if (n_frames <= 0) return {};
    detail::DeviceBuffer<int32_t> ids(static_cast<size_t>(n_frames)), frames(static_cast<size_t>(n_frames)), len(1);
    void* ws = detail::workspace().get(loom_ctc_workspace_size(1, n_frames), stream);
    detail::check(loom_ctc_greedy(d_logits, LOOM_SELECT_F32, 1, n_frames, n_classes, blank_id, ids.get(), frames.get(),
                                  len.get(), nullptr, nullptr, ws, detail::workspace().size(), stream),
                  "ctc_greedy_decode");
    const int32_t n = detail::to_host(len.get(), 1, stream)[0];
    return detail::to_host(ids.get(), static_cast<size_t>(n), stream);
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
    detail::DeviceBuffer<int32_t> ids(static_cast<size_t>(rows > 0 ? rows : 0));
    detail::DeviceBuffer<float> probs(static_cast<size_t>(rows > 0 ? rows : 0));
    void* ws = detail::workspace().get(loom_sample_workspace_size(rows, n_vocab, params.top_k), stream);
    detail::check(loom_sample_rows(d_logits, LOOM_SELECT_F32, rows, n_vocab, row_stride, d_history, history_len, d_u,
                                   &params, ids.get(), probs.get(), nullptr, nullptr, ws, detail::workspace().size(),
                                   stream),
                  "sample_rows");
    const int st = loom_select_read_status(ws, stream);
    if (st != LOOM_SELECT_OK) detail::check(st, "sample_rows");
    SampleResult r;
    r.ids = detail::to_host(ids.get(), static_cast<size_t>(rows), stream);
    r.probs = detail::to_host(probs.get(), static_cast<size_t>(rows), stream);
    return r;
}

}  // namespace select
}  // namespace loom
