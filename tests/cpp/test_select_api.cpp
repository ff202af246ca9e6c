// test_select_api.cpp -- loom.cpp's selection API (include/loom_select.hpp) on the B200 kernels.
//
// `test_select_api cpu` checks the argument errors, which are raised before any CUDA call, with the
// error text of src/core/lua_bridge.cpp:310-319 and :350-353. `test_select_api gpu` also runs loom.cpp's
// known answers on device memory: tests/ci/test_ctc_decode.cpp:12-38, tests/ci/test_lua_bridge.cpp:139-145
// and the windowed argmax of tests/ci/test_lua_bridge_retained_outputs.cpp:152-174.
// A dependency-free harness in the style of loom.cpp's tests/support/test_util.h; exit 0 = pass.
#include "loom_select.hpp"

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

static int g_checks = 0;
static int g_failures = 0;

#define CHECK(cond)                                                                 \
    do {                                                                            \
        ++g_checks;                                                                 \
        if (!(cond)) {                                                              \
            ++g_failures;                                                           \
            std::fprintf(stderr, "CHECK FAILED at %s:%d: %s\n", __FILE__, __LINE__, #cond); \
        }                                                                           \
    } while (0)

#define CHECK_THROWS(expr, substr)                                                  \
    do {                                                                            \
        ++g_checks;                                                                 \
        bool thrown_ = false;                                                       \
        try {                                                                       \
            (void)(expr);                                                           \
        } catch (const loom::Error& e_) {                                           \
            thrown_ = std::string(e_.what()).find(substr) != std::string::npos;     \
            if (!thrown_) std::fprintf(stderr, "unexpected message: %s\n", e_.what()); \
        }                                                                           \
        if (!thrown_) {                                                             \
            ++g_failures;                                                           \
            std::fprintf(stderr, "CHECK_THROWS FAILED at %s:%d: %s\n", __FILE__, __LINE__, #expr); \
        }                                                                           \
    } while (0)

template <class T>
static T* upload(const std::vector<T>& h) {
    T* d = nullptr;
    if (cudaMalloc(&d, h.size() * sizeof(T)) != cudaSuccess) return nullptr;
    cudaMemcpy(d, h.data(), h.size() * sizeof(T), cudaMemcpyHostToDevice);
    return d;
}

static void cpu_checks() {
    using loom::select::argmax_tensor_row;
    using loom::select::argmax_tensor_rows;
    // a row past the output, an id window past the row, an empty window (lua_bridge.cpp:310-319)
    CHECK_THROWS(argmax_tensor_row(nullptr, 6, 3, 6, 3, "loom.argmax_row"), "out of range");
    CHECK_THROWS(argmax_tensor_row(nullptr, 6, 3, 6, -1, "loom.argmax_row_range", 2, 99),
                 "is not a non-empty sub-range");
    CHECK_THROWS(argmax_tensor_row(nullptr, 6, 3, 6, -1, "loom.argmax_row_range", 3, 3),
                 "is not a non-empty sub-range");
    CHECK_THROWS(argmax_tensor_row(nullptr, 6, 3, 6, -1, "loom.argmax_row_range", -2, 4),
                 "is not a non-empty sub-range");
    CHECK_THROWS(argmax_tensor_row(nullptr, 0, 3, 6, 0, "loom.argmax_row"), "out of range");
    // no rows to reduce (lua_bridge.cpp:350-353)
    CHECK_THROWS(argmax_tensor_rows(nullptr, 0, 5, 0, "loom.argmax_rows"), "which has no rows to reduce");
    CHECK_THROWS(argmax_tensor_rows(nullptr, 4, 0, 4, "loom.argmax_rows"), "which has no rows to reduce");
}

static void gpu_checks() {
    using namespace loom::select;
    // tests/ci/test_ctc_decode.cpp:12-38
    const std::vector<float> l1 = {0, 5, 0, 0, 0, 4, 1, 0, 0, 0, 0, 9, 0, 0, 7, 1,
                                   1, 0, 6, 0, 8, 0, 0, 1, 7, 0, 0, 2, 0, 0, 0, 9};
    float* d1 = upload(l1);
    CHECK((ctc_greedy_decode(d1, 8, 4, 3) == std::vector<int32_t>{1, 2, 0}));
    const std::vector<float> l2 = {0, 0, 0, 9, 0, 5, 0, 0};
    float* d2 = upload(l2);
    CHECK((ctc_greedy_decode(d2, 2, 4, 3) == std::vector<int32_t>{1}));
    const std::vector<float> l3 = {0, 0, 0, 9, 0, 0, 0, 9, 0, 0, 0, 9};
    float* d3 = upload(l3);
    CHECK(ctc_greedy_decode(d3, 3, 4, 3).empty());

    // tests/ci/test_lua_bridge.cpp:139-145: [1,5,2, 9,0,3], n_vocab 3, row 1 -> 0
    const std::vector<float> a = {1, 5, 2, 9, 0, 3};
    float* da = upload(a);
    CHECK(argmax_tensor_row(da, 3, 2, 3, 1, "loom.argmax_row") == 0);
    CHECK(argmax_tensor_row(da, 3, 2, 3, -1, "loom.argmax_row") == 0);
    CHECK(argmax_tensor_row(da, 3, 2, 3, 0, "loom.argmax_row") == 1);
    CHECK((argmax_tensor_rows(da, 3, 2, 3, "loom.argmax_rows") == std::vector<double>{1.0, 0.0}));
    CHECK(argmax(da + 3, 3) == 0);

    // a window that excludes the unrestricted winner returns the window's own best, absolute
    const std::vector<float> w = {0.5f, 4.0f, 1.0f, 2.0f, 3.5f, 0.0f};
    float* dw = upload(w);
    const int64_t full = argmax_tensor_row(dw, 6, 1, 6, -1, "loom.argmax_row_range");
    const int64_t got = argmax_tensor_row(dw, 6, 1, 6, -1, "loom.argmax_row_range", 3, 6);
    CHECK(full == 1);
    CHECK(got == 4);

    // the sampling chain with top-k 1 is the argmax, with probability 1
    const std::vector<float> s = {0.1f, 2.0f, -1.0f, 2.0f, 0.5f, 7.0f, 1.0f, 7.0f};
    float* ds = upload(s);
    const std::vector<float> u = {0.5f, 0.25f};
    float* du = upload(u);
    // row 0 [0.1, 2, -1, 2] with id 1 penalised by 2 (2 -> 1): argmax 3
    // row 1 [0.5, 7, 1, 7]  with id 3 penalised by 2 (7 -> 3.5): argmax 1
    const std::vector<int32_t> hist = {1, 3};
    int32_t* dh = upload(hist);
    loom_sample_params p{1.0f, 2.0f, 1, 1.0f};
    const SampleResult r = sample_rows(ds, 2, 4, 4, dh, 1, du, p);
    CHECK((r.ids == std::vector<int32_t>{3, 1}));
    // a history id outside the vocabulary is a loom::Error
    const std::vector<int32_t> bad = {4, 0};
    int32_t* db = upload(bad);
    CHECK_THROWS(sample_rows(ds, 2, 4, 4, db, 1, du, p), "outside the vocabulary");
    cudaFree(db);
    CHECK(r.probs.size() == 2 && r.probs[0] == 1.0f && r.probs[1] == 1.0f);

    // the LM head fused with the greedy choice: hidden rows e0 and e1 (bf16), a [300, 64] weight that
    // is zero except w[250][0] = 2, w[5][0] = 0.5, w[17][1] = 3 -> ids 250 and 17
    std::vector<uint16_t> hid(2 * 64, 0), wt(300 * 64, 0);
    hid[0] = 0x3F80;       // 1.0
    hid[64 + 1] = 0x3F80;  // 1.0
    wt[250 * 64 + 0] = 0x4000;  // 2.0
    wt[5 * 64 + 0] = 0x3F00;    // 0.5
    wt[17 * 64 + 1] = 0x4040;   // 3.0
    uint16_t* dhid = upload(hid);
    uint16_t* dwt = upload(wt);
    const GreedyResult g = lm_head_argmax(dhid, dwt, 2, 64, 300);
    CHECK((g.ids == std::vector<int32_t>{250, 17}));
    CHECK(g.logit.size() == 2 && g.logit[0] == 2.0f && g.logit[1] == 3.0f);
    const double lp0 = 2.0 - std::log(std::exp(2.0) + std::exp(0.5) + 298.0);
    const double lp1 = 3.0 - std::log(std::exp(3.0) + 299.0);
    CHECK(std::fabs(g.logprob[0] - lp0) < 1e-4 && std::fabs(g.logprob[1] - lp1) < 1e-4);
    cudaFree(dhid);
    cudaFree(dwt);
    for (void* p_ : {static_cast<void*>(d1), static_cast<void*>(d2), static_cast<void*>(d3), static_cast<void*>(da),
                     static_cast<void*>(dw), static_cast<void*>(ds), static_cast<void*>(du), static_cast<void*>(dh)})
        cudaFree(p_);
}

int main(int argc, char** argv) {
    const bool gpu = argc > 1 && std::strcmp(argv[1], "gpu") == 0;
    cpu_checks();
    if (gpu) gpu_checks();
    std::fprintf(stderr, "%d checks, %d failures\n", g_checks, g_failures);
    return g_failures == 0 ? 0 : 1;
}
