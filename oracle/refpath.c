/*
 * refpath.c -- BENCH/TEST INFRASTRUCTURE ONLY: loom.cpp's own host-side selection path, timed.
 *
 * On a CUDA build loom.cpp selects a token by copying logits off the device with
 * ggml_backend_tensor_get (a cudaMemcpy into a host std::vector) and scanning them on one host thread
 * with a strict '>' (src/core/generation.cpp:56-74; src/core/lua_bridge.cpp:302-330, :343-365). These
 * functions do exactly that -- one device-to-host copy into pageable host memory per row (or per frame),
 * then the scan -- so the bench can time the path the kernels replace on the same machine. Nothing in
 * the product links this file.
 *
 *   refpath_greedy_decode       Generator::read_row + Generator::argmax, once per decode step
 *   refpath_argmax_tensor_rows  argmax_tensor_rows: one tensor_get per row, then the scan
 *   refpath_ctc_driver          the CTC driver's path: argmax_tensor_rows per utterance, then the
 *                               collapse of src/core/ctc_decode.cpp:21-29 (keep id != prev && id != blank)
 *
 * Each returns the seconds it took (CLOCK_MONOTONIC), or a negative value when a CUDA call failed.
 */
#define _POSIX_C_SOURCE 199309L
#include <cuda_runtime_api.h>
#include <stdint.h>
#include <stdlib.h>
#include <time.h>

static double now_s(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double)ts.tv_sec + 1e-9 * (double)ts.tv_nsec;
}

/* The scan of generation.cpp:64-74 / lua_bridge.cpp:325-329. */
static int32_t scan(const float* row, int64_t n) {
    int32_t best = 0;
    float best_val = row[0];
    for (int64_t i = 1; i < n; ++i) {
        if (row[i] > best_val) {
            best_val = row[i];
            best = (int32_t)i;
        }
    }
    return best;
}

double refpath_greedy_decode(const float* d_rows, int64_t steps, int64_t n_vocab, int64_t row_stride,
                             int32_t* out_ids) {
    float* host = (float*)malloc((size_t)n_vocab * sizeof(float));
    if (!host) return -1.0;
    const double t0 = now_s();
    for (int64_t s = 0; s < steps; ++s) {
        if (cudaMemcpy(host, d_rows + s * row_stride, (size_t)n_vocab * sizeof(float), cudaMemcpyDeviceToHost) !=
            cudaSuccess) {
            free(host);
            return -2.0;
        }
        out_ids[s] = scan(host, n_vocab);
    }
    const double dt = now_s() - t0;
    free(host);
    return dt;
}

double refpath_argmax_tensor_rows(const float* d, int64_t n_rows, int64_t n_classes, int64_t row_stride,
                                  int32_t* out_ids) {
    float* row = (float*)malloc((size_t)n_classes * sizeof(float));
    if (!row) return -1.0;
    const double t0 = now_s();
    for (int64_t r = 0; r < n_rows; ++r) {
        if (cudaMemcpy(row, d + r * row_stride, (size_t)n_classes * sizeof(float), cudaMemcpyDeviceToHost) !=
            cudaSuccess) {
            free(row);
            return -2.0;
        }
        out_ids[r] = scan(row, n_classes);
    }
    const double dt = now_s() - t0;
    free(row);
    return dt;
}

double refpath_ctc_driver(const float* d, int64_t n_utt, int64_t n_frames, int64_t n_classes, int32_t blank,
                          int32_t* out_ids, int32_t* out_len) {
    float* row = (float*)malloc((size_t)n_classes * sizeof(float));
    int32_t* frame_ids = (int32_t*)malloc((size_t)n_frames * sizeof(int32_t));
    if (!row || !frame_ids) {
        free(row);
        free(frame_ids);
        return -1.0;
    }
    const double t0 = now_s();
    for (int64_t u = 0; u < n_utt; ++u) {
        const float* du = d + u * n_frames * n_classes;
        for (int64_t f = 0; f < n_frames; ++f) {
            if (cudaMemcpy(row, du + f * n_classes, (size_t)n_classes * sizeof(float), cudaMemcpyDeviceToHost) !=
                cudaSuccess) {
                free(row);
                free(frame_ids);
                return -2.0;
            }
            frame_ids[f] = scan(row, n_classes);
        }
        int32_t prev = blank, n = 0;
        for (int64_t f = 0; f < n_frames; ++f) {
            const int32_t id = frame_ids[f];
            if (id != prev && id != blank) out_ids[u * n_frames + n++] = id;
            prev = id;
        }
        out_len[u] = n;
    }
    const double dt = now_s() - t0;
    free(row);
    free(frame_ids);
    return dt;
}
