#pragma once
#include "common.cuh"

namespace mb {

void launch_pack(const float *in, uint8_t *out, int64_t rows, int64_t width, int q4, int preround,
                 int fused, int *flags, cudaStream_t s);
void launch_repack(int q4, const uint8_t *blocks, uint4 *wq, __half *ws, int64_t rows, int64_t nb,
                   int64_t nb_pad, int64_t groups, cudaStream_t s);
// fp32 rows -> canonical ggml Q8_0 bytes (the q8cpu_quantize mirror)
void launch_quantize_rows(int mode, const float *x, int64_t ldx, int64_t m, int64_t k, uint8_t *blocks,
                          int *status, cudaStream_t s);
// fp32 rows [-> LayerNorm] -> Q8_0 A fragments + fp32 scales for the GEMV (PDL launch)
void launch_quantize_frag(int mode, const float *x, int64_t ldx, int64_t m, int64_t k, int64_t mpad,
                          int64_t nb_pad, const float *ln_w, const float *ln_b, float ln_eps, uint32_t *xf,
                          float *xs, int *xsum, int *status, cudaStream_t s);

// Parameters of one fragment-layout GEMV launch (M <= 32 tokens).
struct GemvArgs {
    const uint4 *wq;       // weight fragments
    const __half2 *ws;     // [G][nb_pad][4] half2 scales
    int64_t groups, nb, nb_pad, n, m;
    // activations quantized by launch_quantize_frag (global, L2-resident)
    const uint4 *xf;       // [nb_pad][mtiles][32] A fragments
    const float *xs;       // [nb_pad][mpad] fp32 scales
    const int *xsum;       // [nb_pad][mpad] sum of each block's activation quants
    int *status;           // bit 1 (value 2): a bounded pipeline wait timed out
    float *out;            // [m][ldo]
    int64_t ldo;
    const float *bias;     // [n] or null
    const float *residual; // [m][ldo] or null
    int flags;
    const uint16_t *gelu;  // ggml GELU table (gelu_table()), needed with the GELU flag
    int32_t *sums;         // debug: [m][n][nb] exact block sums, or null
    // fused readout (argmax) state; keys == null disables it
    unsigned long long *keys;  // [32] running per-token maxima, all zero between calls
    unsigned int *done;        // CTA completion counter, zero between calls
    int64_t *token;            // [m]
    const int64_t *suppressed;
    int64_t suppressed_count;
    int wpg;                   // warps per row group (set by the launcher)
    int wpg_override;          // > 0 forces a split (tests)
    int ctas_per_sm;           // streamed (unsplit) launches: resident CTAs per SM (0: default)
};

bool gemv_supported(int64_t nb_pad);
void launch_gemv(int q4, const GemvArgs &a, cudaStream_t s);

}  // namespace mb
