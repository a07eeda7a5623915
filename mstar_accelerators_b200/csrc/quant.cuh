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

// Quantizes one 32-element block (lane = element) of token `token` to Q8_0 and
// writes it in the layout of k_quantize_frag: xf [nb_pad][mtiles][32][4 words], xs / xsum [nb_pad][mpad].
template <int MODE>
__device__ __forceinline__ void frag_block(float v, bool live, int64_t b, int token, int mtiles, uint32_t *xf,
                                           float *xs, int *xsum, int *status) {
    const int lane = threadIdx.x & 31;
    if (live && !isfinite(v)) atomicOr(status, 1);
    float amax = fabsf(v);
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float d = __fdiv_rn(amax, 127.0f);
    float id;
    if (MODE == 2) id = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
    else id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    const float sv = __fmul_rn(v, id);
    const int q = MODE == 0 ? int(roundf(sv)) : __float2int_rn(sv);
    const int mt = token / 16, r = token % 16, g = r & 7, hi = r >> 3;
    const int t = (lane & 15) >> 2, half = lane >> 4;
    uint32_t byte = uint32_t(q) & 0xffu;
    uint32_t word = byte;
    word |= __shfl_down_sync(0xffffffffu, byte, 1) << 8;
    word |= __shfl_down_sync(0xffffffffu, byte, 2) << 16;
    word |= __shfl_down_sync(0xffffffffu, byte, 3) << 24;
    if ((lane & 3) == 0) xf[((b * mtiles + mt) * 32 + (4 * g + t)) * 4 + hi + 2 * half] = word;
    int qsum = q;
#pragma unroll
    for (int o = 16; o; o >>= 1) qsum += __shfl_xor_sync(0xffffffffu, qsum, o);
    if (lane == 0) {
        xs[b * mtiles * 16 + token] = __half2float(__float2half_rn(d));
        xsum[b * mtiles * 16 + token] = qsum;
    }
}

// A Q8_0 activation-fragment destination (the layout above) that a producer
// kernel fills for the linear that consumes its output.
struct Q8Frags {
    uint32_t *xf;
    float *xs;
    int *xsum;
    int64_t nb_pad, mpad;
    int mode;  // Q8_0 activation rounding: 0 ref, 1 arm, 2 x86
};

bool gemv_supported(int64_t nb_pad);
// split-K GEMV (Q8_0 weights, n % 32 == 0, m <= 32) that also writes the next
// linear's Q8_0 fragments of its outputs (gemv.cu)
void launch_gemv_frag(GemvArgs a, const Q8Frags &f, cudaStream_t s);
size_t gemv_frag_smem_bytes(int64_t nb_pad, int mt);
void launch_gemv(int q4, const GemvArgs &a, cudaStream_t s);

}  // namespace mb
