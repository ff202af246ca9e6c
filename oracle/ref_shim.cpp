// ref_shim.cpp -- TEST INFRASTRUCTURE ONLY.
//
// A C entry point around loom.cpp's own ctc_greedy_decode (src/core/ctc_decode.cpp:7-31), which is
// compiled from the loom.cpp source tree where it lies (see the Makefile beside this file) into
// oracle/_ref/. It lets the tests check this directory's restatement, and the committed golden
// fixtures, against the reference's real code.
#include "loom/core/ctc_decode.h"

#include <cstdint>
#include <cstring>
#include <vector>

extern "C" int64_t ref_ctc_greedy_decode(const float* logits, int64_t n_frames, int64_t n_classes,
                                         int32_t blank_id, int32_t* out, int64_t capacity) {
    const std::vector<int32_t> ids = loom::ctc_greedy_decode(logits, n_frames, n_classes, blank_id);
    const int64_t n = static_cast<int64_t>(ids.size());
    std::memcpy(out, ids.data(), sizeof(int32_t) * static_cast<size_t>(n < capacity ? n : capacity));
    return n;
}
