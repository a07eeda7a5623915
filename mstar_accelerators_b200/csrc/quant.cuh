#pragma once
#include "common.cuh"

namespace mb {

void launch_pack(const float *in, uint8_t *out, int64_t rows, int64_t width, int q4, int preround,
                 int fused, int *flags, cudaStream_t s);
void launch_repack(int q4, const uint8_t *blocks, uint4 *wq, __half *ws, int64_t rows, int64_t nb,
                   int64_t nb_pad, int64_t groups, cudaStream_t s);
void launch_quantize_act(int mode, const float *x, int64_t ldx, int64_t m, int64_t k, int64_t mpad,
                         int64_t nb_pad, uint8_t *xf, float *xs, uint8_t *blocks, int *status,
                         cudaStream_t s);

// Parameters of one fragment-layout GEMV launch (M <= 32 tokens).
struct GemvArgs {
    const uint4 *wq;       // weight fragments
    const __half2 *ws;     // [G][nb_pad][4] half2 scales
    const uint4 *xf;       // activation fragments [nb_pad][mtiles][32]
    const float *xs;       // [nb_pad][mpad]
    int64_t groups, nb_pad, n, m;
    float *out;            // [m][ldo]
    int64_t ldo;
    const float *bias;     // [n] or null
    const float *residual; // [m][ldo] or null
    int flags;
    int32_t *sums;         // debug: [m][n][nb] exact block sums, or null
    int64_t nb;
    // fused readout (argmax) state; keys == null disables it
    unsigned long long *keys;  // [32] running per-token maxima, all zero between calls
    unsigned int *done;        // CTA completion counter, zero between calls
    int64_t *token;            // [m]
    const int64_t *suppressed;
    int64_t suppressed_count;
};

void launch_gemv(int q4, const GemvArgs &a, cudaStream_t s);

}  // namespace mb
