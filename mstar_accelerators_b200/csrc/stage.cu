// Operand staging for the tcgen05 GEMM of the encoder graph
// (backends/cpu_ggml/encoder.cpp:400-754):
//   k_stage_rows  (a warp per row, 16-byte vector loads, a Q8_0 block per 8 lanes)
//                 fp32 or fp16 rows [-> LayerNorm] -> Q8_0 -> fp16(q * d): the
//                 activation side of ggml_mul_mat(Q8_0 W, x) after
//                 encoder_norm_affine (encoder.cpp:117-142) or on the fp32
//                 attention output;
//   k_stage_conv_tm / _cm  (a warp per output row, the source tile in shared memory;
//                 k_stage_conv, a warp per Q8_0 block, for sources too wide for it) the
//                 im2col columns of convolution_q8 (encoder.cpp:45-52: kernel 3, padding 1,
//                 column = channel * 3 + tap, K zero-padded to a multiple of 32,
//                 encoder.cpp:551) quantized the same way;
//   k_layer_norm  the final encoder_norm_affine to fp32 (encoder.cpp:725).
// Q8_0 quantization follows ggml quantize_row_q8_0 with the selected rounding
// (ref / ARM / x86); a nonfinite input sets status bit value 1.
#include <cmath>

#include <cuda_bf16.h>

#include "../../include/mstar_b200.h"
#include "gemm.cuh"

namespace mb {

constexpr int STAGE_WARPS = 8;
constexpr int STAGE_MAX_PER_LANE = 48;  // LayerNorm rows keep <= 48 * 32 = 1536 values in registers

template <int MODE>
__device__ __forceinline__ float q8_staged(float v, int *status) {
    if (!isfinite(v) && status) atomicOr(status, 1);
    float amax = fabsf(v);
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float d = __fdiv_rn(amax, 127.0f);
    float id;
    if (MODE == 2) id = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
    else id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    const float sv = __fmul_rn(v, id);
    const int q = MODE == 0 ? int(roundf(sv)) : __float2int_rn(sv);
    return __fmul_rn(float(q), __half2float(__float2half_rn(d)));
}

// Vectorised row staging: lane l of a warp owns the 4 consecutive elements of
// chunk c = i * 32 + l, so one Q8_0 block is 8 consecutive lanes and every
// load / store instruction of the warp covers 128 contiguous elements.
template <bool F16>
__device__ __forceinline__ float4 load4(const void *x, int64_t e) {
    if (F16) {
        const uint2 u = *reinterpret_cast<const uint2 *>(static_cast<const __half *>(x) + e);
        __half2 lo, hi;
        memcpy(&lo, &u.x, 4);
        memcpy(&hi, &u.y, 4);
        const float2 a = __half22float2(lo), b = __half22float2(hi);
        return make_float4(a.x, a.y, b.x, b.y);
    }
    return *reinterpret_cast<const float4 *>(static_cast<const float *>(x) + e);
}

__device__ __forceinline__ void store4(__half *out, int64_t e, float4 v) {
    uint2 u;
    u.x = half2_bits(__floats2half2_rn(v.x, v.y));
    u.y = half2_bits(__floats2half2_rn(v.z, v.w));
    *reinterpret_cast<uint2 *>(out + e) = u;
}

// Q8_0 quantization (ggml quantize_row_q8_0, rounding MODE) of the block held by
// 8 consecutive lanes, 4 values each; returns fp16-exact q * fp16(d) as fp32.
template <int MODE>
__device__ __forceinline__ float4 q8_block8(float4 v, int *status) {
    if (!(isfinite(v.x) && isfinite(v.y) && isfinite(v.z) && isfinite(v.w)) && status) atomicOr(status, 1);
    float amax = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float d = __fdiv_rn(amax, 127.0f);
    float id;
    if (MODE == 2) id = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
    else id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    const float dh = __half2float(__float2half_rn(d));
    auto q = [&](float x) {
        const float sv = __fmul_rn(x, id);
        return __fmul_rn(float(MODE == 0 ? int(roundf(sv)) : __float2int_rn(sv)), dh);
    };
    return make_float4(q(v.x), q(v.y), q(v.z), q(v.w));
}

// The same quantization of a block held by 4 consecutive lanes, 8 values each (v in place).
template <int MODE>
__device__ __forceinline__ void q8_block4(float (&v)[8], int *status) {
    bool finite = true;
    float amax = fabsf(v[0]);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        finite = finite && isfinite(v[i]);
        amax = fmaxf(amax, fabsf(v[i]));
    }
    if (!finite && status) atomicOr(status, 1);
#pragma unroll
    for (int o = 1; o < 4; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float d = __fdiv_rn(amax, 127.0f);
    float id;
    if (MODE == 2) id = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
    else id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    const float dh = __half2float(__float2half_rn(d));
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float sv = __fmul_rn(v[i], id);
        v[i] = __fmul_rn(float(MODE == 0 ? int(roundf(sv)) : __float2int_rn(sv)), dh);
    }
}

constexpr int STAGE_MAX_CHUNKS = STAGE_MAX_PER_LANE / 4;  // float4 chunks a lane keeps for a LayerNorm row
constexpr int STAGE_BATCH = 8;                            // chunk rows in flight per lane without LayerNorm

// ggml_compute_forward_norm_f32 (ggml-cpu/ops.cpp:4094-4137): mean, centred
// variance, y = (x - mean) * (1 / sqrt(var + eps)); then ggml mul and add.
// The sums are warp-reduced (the reference sums sequentially), so the
// normalised value can differ in the last ulp.
template <bool F16>
__device__ __forceinline__ void row_stats4(const void *x, int64_t base, int64_t chunks, float eps,
                                           float4 (&vals)[STAGE_MAX_CHUNKS], float &mean, float &rstd) {
    const int lane = threadIdx.x & 31;
    float sum = 0.0f;
#pragma unroll
    for (int i = 0; i < STAGE_MAX_CHUNKS; ++i) {
        const int64_t c = int64_t(i) * 32 + lane;
        vals[i] = c < chunks ? load4<F16>(x, base + 4 * c) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        sum = __fadd_rn(sum, __fadd_rn(__fadd_rn(vals[i].x, vals[i].y), __fadd_rn(vals[i].z, vals[i].w)));
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float k = float(chunks * 4);
    mean = sum / k;
    float var = 0.0f;
#pragma unroll
    for (int i = 0; i < STAGE_MAX_CHUNKS; ++i) {
        const int64_t c = int64_t(i) * 32 + lane;
        if (c < chunks) {
            const float a = __fsub_rn(vals[i].x, mean), b = __fsub_rn(vals[i].y, mean);
            const float e = __fsub_rn(vals[i].z, mean), f = __fsub_rn(vals[i].w, mean);
            var = __fadd_rn(var, __fadd_rn(__fadd_rn(__fmul_rn(a, a), __fmul_rn(b, b)),
                                           __fadd_rn(__fmul_rn(e, e), __fmul_rn(f, f))));
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) var += __shfl_xor_sync(0xffffffffu, var, o);
    rstd = 1.0f / sqrtf(var / k + eps);
}

__device__ __forceinline__ float norm_affine(float v, float mean, float rstd, float w, float b) {
    return __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v, mean), rstd), w), b);
}

template <int MODE, bool F16, bool LN>
__global__ void __launch_bounds__(STAGE_WARPS * 32)
    k_stage_rows(const void *__restrict__ x, int64_t ldx, int64_t rows, int64_t k, const float *__restrict__ ln_w,
                 const float *__restrict__ ln_b, float eps, __half *__restrict__ out, int64_t ldo,
                 int *__restrict__ status) {
    const int lane = threadIdx.x & 31;
    const int64_t row = int64_t(blockIdx.x) * STAGE_WARPS + (threadIdx.x >> 5);
    if (row >= rows) return;
    const int64_t chunks = k / 4;
    if (LN) {
        float4 vals[STAGE_MAX_CHUNKS];
        float mean, rstd;
        row_stats4<F16>(x, row * ldx, chunks, eps, vals, mean, rstd);
#pragma unroll
        for (int i = 0; i < STAGE_MAX_CHUNKS; ++i) {
            if (int64_t(i) * 32 < chunks) {  // warp-uniform: every lane takes part in the block shuffles
                const int64_t c = int64_t(i) * 32 + lane;
                float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                if (c < chunks) {
                    const float4 w = *reinterpret_cast<const float4 *>(ln_w + 4 * c);
                    const float4 b = *reinterpret_cast<const float4 *>(ln_b + 4 * c);
                    v = make_float4(norm_affine(vals[i].x, mean, rstd, w.x, b.x),
                                    norm_affine(vals[i].y, mean, rstd, w.y, b.y),
                                    norm_affine(vals[i].z, mean, rstd, w.z, b.z),
                                    norm_affine(vals[i].w, mean, rstd, w.w, b.w));
                }
                v = q8_block8<MODE>(v, status);
                if (c < chunks) store4(out, row * ldo + 4 * c, v);
            }
        }
    } else {
        const int64_t crow = (chunks + 31) / 32;
        for (int64_t i0 = 0; i0 < crow; i0 += STAGE_BATCH) {
            float4 v[STAGE_BATCH];
#pragma unroll
            for (int u = 0; u < STAGE_BATCH; ++u) {
                const int64_t c = (i0 + u) * 32 + lane;
                v[u] = c < chunks ? load4<F16>(x, row * ldx + 4 * c) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            }
#pragma unroll
            for (int u = 0; u < STAGE_BATCH; ++u) {
                if (i0 + u < crow) {
                    const int64_t c = (i0 + u) * 32 + lane;
                    const float4 q = q8_block8<MODE>(v[u], status);
                    if (c < chunks) store4(out, row * ldo + 4 * c, q);
                }
            }
        }
    }
}

// Rows without a LayerNorm, eight values per lane (four lanes per Q8_0 block): every
// 32-value block costs one amax butterfly and one pair of divisions for 8 values a lane
// instead of 4, with 4 KB per warp in flight (8 16-byte chunks of fp16 / bf16 rows or
// half as many 32-byte fp32 ones). 16-bit rows need 16-byte aligned rows.
constexpr int ROWS_F32 = 0, ROWS_F16 = 1, ROWS_BF16 = 2;

template <int MODE, int IN>
__global__ void __launch_bounds__(STAGE_WARPS * 32)
    k_stage_rows8(const void *__restrict__ x, int64_t ldx, int64_t rows, int64_t k, __half *__restrict__ out,
                  int64_t ldo, int *__restrict__ status) {
    constexpr bool F16 = IN != ROWS_F32;   // 16-bit rows: one 16-byte load per chunk
    constexpr int BATCH = F16 ? 8 : 4;
    const int lane = threadIdx.x & 31;
    const int64_t row = int64_t(blockIdx.x) * STAGE_WARPS + (threadIdx.x >> 5);
    if (row >= rows) return;   // warp-uniform
    const int chunks = int(k / 8);   // k <= 65536
    const uint4 *src = reinterpret_cast<const uint4 *>(static_cast<const char *>(x) + row * ldx * (F16 ? 2 : 4));
    uint4 *dst = reinterpret_cast<uint4 *>(out + row * ldo);
    for (int i0 = 0; i0 * 32 < chunks; i0 += BATCH) {
        uint4 raw[F16 ? BATCH : 2 * BATCH];   // the loads in flight, converted when quantized
#pragma unroll
        for (int j = 0; j < BATCH; ++j) {
            const int c = (i0 + j) * 32 + lane;
            if constexpr (F16) {
                raw[j] = c < chunks ? src[c] : make_uint4(0u, 0u, 0u, 0u);
            } else {
                raw[2 * j] = c < chunks ? src[2 * c] : make_uint4(0u, 0u, 0u, 0u);
                raw[2 * j + 1] = c < chunks ? src[2 * c + 1] : make_uint4(0u, 0u, 0u, 0u);
            }
        }
#pragma unroll
        for (int j = 0; j < BATCH; ++j) {
            if ((i0 + j) * 32 < chunks) {   // warp-uniform: every lane takes part in the block shuffles
                const int c = (i0 + j) * 32 + lane;
                float v[8];
                if constexpr (F16) {
                    const uint32_t w[4] = {raw[j].x, raw[j].y, raw[j].z, raw[j].w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        float2 f;
                        if constexpr (IN == ROWS_BF16) {
                            __nv_bfloat162 b2;
                            memcpy(&b2, &w[e], 4);
                            f = __bfloat1622float2(b2);
                        } else {
                            __half2 h2;
                            memcpy(&h2, &w[e], 4);
                            f = __half22float2(h2);
                        }
                        v[2 * e] = f.x;
                        v[2 * e + 1] = f.y;
                    }
                } else {
                    const uint32_t w[8] = {raw[2 * j].x,     raw[2 * j].y,     raw[2 * j].z,     raw[2 * j].w,
                                           raw[2 * j + 1].x, raw[2 * j + 1].y, raw[2 * j + 1].z, raw[2 * j + 1].w};
#pragma unroll
                    for (int e = 0; e < 8; ++e) v[e] = __uint_as_float(w[e]);
                }
                q8_block4<MODE>(v, status);
                if (c < chunks) {
                    uint4 o;
                    o.x = half2_bits(__floats2half2_rn(v[0], v[1]));
                    o.y = half2_bits(__floats2half2_rn(v[2], v[3]));
                    o.z = half2_bits(__floats2half2_rn(v[4], v[5]));
                    o.w = half2_bits(__floats2half2_rn(v[6], v[7]));
                    dst[c] = o;
                }
            }
        }
    }
}

template <int MODE>
__global__ void __launch_bounds__(STAGE_WARPS * 32)
    k_stage_conv(const float *__restrict__ src, int time_major, int64_t batch, int64_t channels, int64_t time_in,
                 int64_t time_out, int stride, int64_t k_padded, __half *__restrict__ out, int *__restrict__ status) {
    const int lane = threadIdx.x & 31;
    const int64_t nb = k_padded / QK;
    const int64_t wid = int64_t(blockIdx.x) * STAGE_WARPS + (threadIdx.x >> 5);
    if (wid >= batch * time_out * nb) return;
    const int64_t row = wid / nb, blk = wid % nb;
    const int64_t b = row / time_out, t = row % time_out;
    const int64_t col = blk * 32 + lane;
    float v = 0.0f;
    if (col < 3 * channels) {
        const int64_t c = col / 3, ti = t * stride + col % 3 - 1;
        if (ti >= 0 && ti < time_in)
            v = time_major ? src[(b * time_in + ti) * channels + c] : src[(b * channels + c) * time_in + ti];
    }
    out[row * k_padded + col] = __float2half_rn(q8_staged<MODE>(v, status));
}

// The same columns, a warp per output row and four columns per lane (eight lanes per
// Q8_0 block, as k_stage_rows), read from the source in shared memory so that every
// global load is a whole 16-byte vector of a contiguous run:
//   k_stage_conv_tm: time-major source [batch][time_in][channels]; the warp copies the
//     three source rows its output row needs (zeros outside the input) into its own
//     shared rows [3][channels], then column c * 3 + tap is shared row tap, entry c;
//   k_stage_conv_cm: channel-major source [batch][channels][time_in]; the CTA copies the
//     time span CONV_TILE output rows need of every channel ([channels][span] floats,
//     contiguous runs per channel) and each warp stages CONV_TILE / CONV_WARPS rows.
// Bytes are those of k_stage_conv (the same block quantization of the same values).
constexpr int CONV_WARPS = 4, CONV_TILE = 32;
constexpr int64_t CONV_TM_MAX_CHANNELS = 2048;   // 24 KB of shared rows per warp
constexpr int64_t CONV_CM_MAX_SMEM = 96 * 1024;  // channel-major tile

template <int MODE>
__device__ __forceinline__ void conv_row_out(const float *sm, int64_t cstride, int64_t tstride, int64_t channels,
                                             int64_t k_padded, __half *out_row, int lane, int *status) {
    // column c * 3 + tap of this row is sm[c * cstride + tap * tstride]
    for (int64_t i = 0; i * 128 < k_padded; ++i) {   // warp-uniform: every lane takes part in the block shuffles
        const int64_t col0 = (i * 32 + lane) * 4;
        float e[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int64_t col = col0 + u;
            e[u] = col < 3 * channels ? sm[(col / 3) * cstride + (col % 3) * tstride] : 0.0f;
        }
        const float4 q = q8_block8<MODE>(make_float4(e[0], e[1], e[2], e[3]), status);
        if (col0 < k_padded) store4(out_row, col0, q);
    }
}

template <int MODE>
__global__ void __launch_bounds__(CONV_WARPS * 32)
    k_stage_conv_tm(const float *__restrict__ src, int64_t batch, int64_t channels, int64_t time_in,
                    int64_t time_out, int stride, int64_t k_padded, __half *__restrict__ out,
                    int *__restrict__ status) {
    extern __shared__ __align__(16) float conv_smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t row = int64_t(blockIdx.x) * CONV_WARPS + warp;
    if (row >= batch * time_out) return;   // warp-uniform; no CTA-wide barrier follows
    float *sm = conv_smem + int64_t(warp) * 3 * channels;   // [tap][channels]
    const int64_t b = row / time_out, t = row % time_out;
#pragma unroll
    for (int tap = 0; tap < 3; ++tap) {
        const int64_t ti = t * stride + tap - 1;
        const bool in = ti >= 0 && ti < time_in;
        const float *s = src + (b * time_in + (in ? ti : 0)) * channels;
        if (channels % 4 == 0 && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {   // whole 16-byte vectors
            for (int64_t c4 = lane; c4 < channels / 4; c4 += 32)
                *reinterpret_cast<float4 *>(sm + tap * channels + 4 * c4) =
                    in ? *reinterpret_cast<const float4 *>(s + 4 * c4) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        } else {
            for (int64_t c = lane; c < channels; c += 32) sm[tap * channels + c] = in ? s[c] : 0.0f;
        }
    }
    __syncwarp();
    conv_row_out<MODE>(sm, 1, channels, channels, k_padded, out + row * k_padded, lane, status);
}

template <int MODE>
__global__ void __launch_bounds__(CONV_WARPS * 32)
    k_stage_conv_cm(const float *__restrict__ src, int64_t batch, int64_t channels, int64_t time_in,
                    int64_t time_out, int stride, int64_t k_padded, __half *__restrict__ out,
                    int *__restrict__ status) {
    extern __shared__ __align__(16) float conv_smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t tiles = (time_out + CONV_TILE - 1) / CONV_TILE;
    const int64_t b = blockIdx.x / tiles, t0 = (blockIdx.x % tiles) * CONV_TILE;
    const int64_t span = (CONV_TILE - 1) * stride + 3;   // source times t0 * stride - 1 .. of every channel
    const int64_t first = t0 * stride - 1;
    for (int64_t i = threadIdx.x; i < channels * span; i += blockDim.x) {
        const int64_t c = i / span, j = i % span, ti = first + j;
        conv_smem[i] = ti >= 0 && ti < time_in ? src[(b * channels + c) * time_in + ti] : 0.0f;
    }
    __syncthreads();
    for (int r = warp; r < CONV_TILE; r += CONV_WARPS) {
        const int64_t t = t0 + r;
        if (t >= time_out) break;   // warp-uniform
        conv_row_out<MODE>(conv_smem + int64_t(r) * stride, span, 1, channels, k_padded,
                           out + (b * time_out + t) * k_padded, lane, status);
    }
}

// Attention output rows staged for the output projection straight from the attention's
// [seqs][heads][positions][head_dim] bf16 output (any strides over the first three, head_dim
// contiguous): row s * positions + t is head 0 .. heads-1 of position t of sequence s side by
// side (the transpose and fp32 conversion a torch reshape would first write out), then Q8_0
// blocks as k_stage_rows: a warp per row, eight values per lane (a 16-byte load from one
// head's contiguous run, STAGE_HEADS_BATCH of them in flight), four lanes per block.
constexpr int STAGE_HEADS_BATCH = 8;

template <int MODE>
__global__ void __launch_bounds__(STAGE_WARPS * 32)
    k_stage_heads(const __nv_bfloat16 *__restrict__ att, int64_t seqs, int64_t heads, int64_t positions,
                  int64_t head_dim, int64_t seq_stride, int64_t head_stride, int64_t position_stride,
                  __half *__restrict__ out, int *__restrict__ status) {
    const int lane = threadIdx.x & 31;
    const int64_t row = int64_t(blockIdx.x) * STAGE_WARPS + (threadIdx.x >> 5);
    if (row >= seqs * positions) return;   // warp-uniform
    const int64_t s = row / positions, t = row % positions;
    const int k = int(heads * head_dim), chunks = k / 8, hd = int(head_dim);   // k <= 65536
    const __nv_bfloat16 *base = att + s * seq_stride + t * position_stride;
    __half *dst = out + row * k;
    for (int i0 = 0; i0 * 32 < chunks; i0 += STAGE_HEADS_BATCH) {
        uint4 u[STAGE_HEADS_BATCH];
#pragma unroll
        for (int j = 0; j < STAGE_HEADS_BATCH; ++j) {
            const int c = (i0 + j) * 32 + lane;
            u[j] = make_uint4(0u, 0u, 0u, 0u);
            if (c < chunks) {
                const int h = 8 * c / hd, d = 8 * c - h * hd;
                u[j] = *reinterpret_cast<const uint4 *>(base + h * head_stride + d);
            }
        }
#pragma unroll
        for (int j = 0; j < STAGE_HEADS_BATCH; ++j) {
            if ((i0 + j) * 32 < chunks) {   // warp-uniform: every lane takes part in the block shuffles
                const int c = (i0 + j) * 32 + lane;
                const uint32_t w[4] = {u[j].x, u[j].y, u[j].z, u[j].w};
                float v[8];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    __nv_bfloat162 b2;
                    memcpy(&b2, &w[e], 4);
                    const float2 f = __bfloat1622float2(b2);
                    v[2 * e] = f.x;
                    v[2 * e + 1] = f.y;
                }
                q8_block4<MODE>(v, status);
                if (c < chunks) {
                    uint4 o;
                    o.x = half2_bits(__floats2half2_rn(v[0], v[1]));
                    o.y = half2_bits(__floats2half2_rn(v[2], v[3]));
                    o.z = half2_bits(__floats2half2_rn(v[4], v[5]));
                    o.w = half2_bits(__floats2half2_rn(v[6], v[7]));
                    *reinterpret_cast<uint4 *>(dst + 8 * c) = o;
                }
            }
        }
    }
}

__global__ void __launch_bounds__(STAGE_WARPS * 32)
    k_layer_norm(const float *__restrict__ x, int64_t ldx, int64_t rows, int64_t k, const float *__restrict__ w,
                 const float *__restrict__ bias, float eps, float *__restrict__ out, int64_t ldo) {
    const int lane = threadIdx.x & 31;
    const int64_t row = int64_t(blockIdx.x) * STAGE_WARPS + (threadIdx.x >> 5);
    if (row >= rows) return;
    const int64_t chunks = k / 4;
    float4 vals[STAGE_MAX_CHUNKS];
    float mean, rstd;
    row_stats4<false>(x, row * ldx, chunks, eps, vals, mean, rstd);
#pragma unroll
    for (int i = 0; i < STAGE_MAX_CHUNKS; ++i) {
        const int64_t c = int64_t(i) * 32 + lane;
        if (c < chunks) {
            const float4 g = *reinterpret_cast<const float4 *>(w + 4 * c);
            const float4 b = *reinterpret_cast<const float4 *>(bias + 4 * c);
            *reinterpret_cast<float4 *>(out + row * ldo + 4 * c) =
                make_float4(norm_affine(vals[i].x, mean, rstd, g.x, b.x), norm_affine(vals[i].y, mean, rstd, g.y, b.y),
                            norm_affine(vals[i].z, mean, rstd, g.z, b.z), norm_affine(vals[i].w, mean, rstd, g.w, b.w));
        }
    }
}

template <int MODE>
static void stage_rows_mode(const void *x, int x_f16, int64_t ldx, int64_t rows, int64_t k, const float *ln_w,
                            const float *ln_b, float eps, __half *out, int64_t ldo, int *status, cudaStream_t s) {
    const unsigned grid = unsigned(ceil_div(rows, STAGE_WARPS));
    const int threads = STAGE_WARPS * 32;
    // eight values per lane where the rows allow 16-byte loads and stores (the same bytes)
    const bool wide = ldo % 8 == 0 && uintptr_t(out) % 16 == 0 &&
                      (!x_f16 || (uintptr_t(x) % 16 == 0 && ldx % 8 == 0));
    if (x_f16) {
        if (ln_w) k_stage_rows<MODE, true, true><<<grid, threads, 0, s>>>(x, ldx, rows, k, ln_w, ln_b, eps, out, ldo, status);
        else if (wide) k_stage_rows8<MODE, ROWS_F16><<<grid, threads, 0, s>>>(x, ldx, rows, k, out, ldo, status);
        else k_stage_rows<MODE, true, false><<<grid, threads, 0, s>>>(x, ldx, rows, k, ln_w, ln_b, eps, out, ldo, status);
    } else {
        if (ln_w) k_stage_rows<MODE, false, true><<<grid, threads, 0, s>>>(x, ldx, rows, k, ln_w, ln_b, eps, out, ldo, status);
        else if (wide) k_stage_rows8<MODE, ROWS_F32><<<grid, threads, 0, s>>>(x, ldx, rows, k, out, ldo, status);
        else k_stage_rows<MODE, false, false><<<grid, threads, 0, s>>>(x, ldx, rows, k, ln_w, ln_b, eps, out, ldo, status);
    }
}

void launch_stage_rows(int mode, const void *x, int x_f16, int64_t ldx, int64_t rows, int64_t k, const float *ln_w,
                       const float *ln_b, float ln_eps, __half *out, int64_t ldo, int *status, cudaStream_t s) {
    if (mode == 0) stage_rows_mode<0>(x, x_f16, ldx, rows, k, ln_w, ln_b, ln_eps, out, ldo, status, s);
    else if (mode == 2) stage_rows_mode<2>(x, x_f16, ldx, rows, k, ln_w, ln_b, ln_eps, out, ldo, status, s);
    else stage_rows_mode<1>(x, x_f16, ldx, rows, k, ln_w, ln_b, ln_eps, out, ldo, status, s);
}

void launch_stage_rows_bf16(int mode, const void *x, int64_t rows, int64_t k, __half *out, int *status,
                            cudaStream_t s) {
    const unsigned grid = unsigned(ceil_div(rows, STAGE_WARPS));
    const int threads = STAGE_WARPS * 32;
    if (mode == 0) k_stage_rows8<0, ROWS_BF16><<<grid, threads, 0, s>>>(x, k, rows, k, out, k, status);
    else if (mode == 2) k_stage_rows8<2, ROWS_BF16><<<grid, threads, 0, s>>>(x, k, rows, k, out, k, status);
    else k_stage_rows8<1, ROWS_BF16><<<grid, threads, 0, s>>>(x, k, rows, k, out, k, status);
}

template <int MODE>
static bool launch_stage_conv_rows(const float *src, int time_major, int64_t batch, int64_t channels,
                                   int64_t time_in, int64_t time_out, int stride, int64_t k_padded, __half *out,
                                   int *status, cudaStream_t s) {
    const int threads = CONV_WARPS * 32;
    if (time_major) {
        if (channels > CONV_TM_MAX_CHANNELS) return false;
        const size_t smem = size_t(CONV_WARPS) * 3 * channels * 4;
        cuda_check(cudaFuncSetAttribute(k_stage_conv_tm<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)),
                   "convolution staging shared memory");
        k_stage_conv_tm<MODE><<<unsigned(ceil_div(batch * time_out, CONV_WARPS)), threads, smem, s>>>(
            src, batch, channels, time_in, time_out, stride, k_padded, out, status);
        return true;
    }
    const size_t smem = size_t(channels) * ((CONV_TILE - 1) * stride + 3) * 4;
    if (smem > size_t(CONV_CM_MAX_SMEM)) return false;
    cuda_check(cudaFuncSetAttribute(k_stage_conv_cm<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)),
               "convolution staging shared memory");
    k_stage_conv_cm<MODE><<<unsigned(batch * ceil_div(time_out, CONV_TILE)), threads, smem, s>>>(
        src, batch, channels, time_in, time_out, stride, k_padded, out, status);
    return true;
}

void launch_stage_conv(int mode, const float *src, int time_major, int64_t batch, int64_t channels, int64_t time_in,
                       int64_t time_out, int stride, int64_t k_padded, __half *out, int *status, cudaStream_t s) {
    // row kernels where the source tile fits in shared memory; a warp per block otherwise
    const bool rows = mode == 0   ? launch_stage_conv_rows<0>(src, time_major, batch, channels, time_in, time_out,
                                                                stride, k_padded, out, status, s)
                      : mode == 2 ? launch_stage_conv_rows<2>(src, time_major, batch, channels, time_in, time_out,
                                                                stride, k_padded, out, status, s)
                                  : launch_stage_conv_rows<1>(src, time_major, batch, channels, time_in, time_out,
                                                                stride, k_padded, out, status, s);
    if (rows) return;
    const unsigned grid = unsigned(ceil_div(batch * time_out * (k_padded / QK), STAGE_WARPS));
    const int threads = STAGE_WARPS * 32;
    if (mode == 0)
        k_stage_conv<0><<<grid, threads, 0, s>>>(src, time_major, batch, channels, time_in, time_out, stride, k_padded, out, status);
    else if (mode == 2)
        k_stage_conv<2><<<grid, threads, 0, s>>>(src, time_major, batch, channels, time_in, time_out, stride, k_padded, out, status);
    else
        k_stage_conv<1><<<grid, threads, 0, s>>>(src, time_major, batch, channels, time_in, time_out, stride, k_padded, out, status);
}

void launch_layer_norm(const float *x, int64_t ldx, int64_t rows, int64_t k, const float *w, const float *b, float eps,
                       float *out, int64_t ldo, cudaStream_t s) {
    k_layer_norm<<<unsigned(ceil_div(rows, STAGE_WARPS)), STAGE_WARPS * 32, 0, s>>>(x, ldx, rows, k, w, b, eps, out, ldo);
}

}  // namespace mb

using namespace mb;

extern "C" {

int mstar_b200_stage_rows(const void *x, int32_t x_format, int64_t x_stride, int64_t rows, int64_t width,
                          const float *ln_weight, const float *ln_bias, float ln_eps, void *staged,
                          uint64_t staged_bytes, int32_t rounding, int32_t *status, void *stream, char *error,
                          size_t error_size) {
    try {
        require(x_format == MSTAR_B200_ACT_F32 || x_format == MSTAR_B200_ACT_F16, "staged rows are fp32 or fp16");
        require(rounding >= 0 && rounding <= 2, "unknown Q8_0 activation rounding");
        require(rows >= 1 && rows <= (int64_t(1) << 31) && width >= QK && width % QK == 0 && width <= 65536,
                "invalid staging shape");
        require(x_stride >= width && x_stride % 4 == 0, "row stride must be a multiple of 4 elements");
        require(uintptr_t(x) % (x_format == MSTAR_B200_ACT_F16 ? 8 : 16) == 0, "activation rows must be aligned");
        if (ln_weight) {
            require(ln_bias && std::isfinite(ln_eps) && ln_eps >= 0.0f, "invalid LayerNorm parameters");
            require(width <= int64_t(STAGE_MAX_PER_LANE) * 32, "LayerNorm rows are at most 1536 wide");
            require(uintptr_t(ln_weight) % 16 == 0 && uintptr_t(ln_bias) % 16 == 0, "LayerNorm vectors must be 16-byte aligned");
            check_device(ln_weight, "LayerNorm weight");
            check_device(ln_bias, "LayerNorm bias");
        } else require(!ln_bias, "LayerNorm bias given without its weight");
        const uint64_t esz = x_format == MSTAR_B200_ACT_F16 ? 2 : 4;
        const uint64_t xb = uint64_t((rows - 1) * x_stride + width) * esz;
        const uint64_t ob = uint64_t(rows * width) * 2;
        check_range({x, xb}, xb, esz, "activations");
        check_range({staged, staged_bytes}, ob, 16, "staged operand");
        require(disjoint({x, xb}, {staged, ob}), "staged operand overlaps activations");
        require(status, "missing status word");
        check_device(x, "activations");
        check_device(staged, "staged operand");
        check_device(status, "status word");
        launch_stage_rows(rounding, x, x_format == MSTAR_B200_ACT_F16, x_stride, rows, width, ln_weight, ln_bias, ln_eps,
                          static_cast<__half *>(staged), width, status, as_stream(stream));
        cuda_check(cudaGetLastError(), "staging launch");
        return 0;
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return -1;
    }
}

int mstar_b200_stage_heads(const void *attention, int64_t seqs, int64_t heads, int64_t positions,
                           int64_t head_dim, int64_t seq_stride, int64_t head_stride, int64_t position_stride,
                           void *staged, uint64_t staged_bytes, int32_t rounding, int32_t *status, void *stream,
                           char *error, size_t error_size) {
    try {
        require(rounding >= 0 && rounding <= 2, "unknown Q8_0 activation rounding");
        require(seqs >= 1 && heads >= 1 && positions >= 1 && head_dim >= QK && head_dim % QK == 0 &&
                    seqs * positions <= (int64_t(1) << 31) && heads * head_dim <= 65536,
                "invalid attention layout (head_dim a multiple of 32)");
        require(seq_stride >= 0 && head_stride >= 0 && position_stride >= 0 && seq_stride % 8 == 0 &&
                    head_stride % 8 == 0 && position_stride % 8 == 0,
                "attention strides must be non-negative multiples of 8 elements");
        require(attention && staged && status, "missing staging operand");
        require(uintptr_t(attention) % 16 == 0, "attention output must be 16-byte aligned");
        const uint64_t ab = uint64_t((seqs - 1) * seq_stride + (heads - 1) * head_stride +
                                     (positions - 1) * position_stride + head_dim) * 2;
        const uint64_t ob = uint64_t(seqs * positions * heads * head_dim) * 2;
        check_range({staged, staged_bytes}, ob, 16, "staged operand");
        require(disjoint({attention, ab}, {staged, ob}), "staged operand overlaps the attention output");
        check_device(attention, "attention output");
        check_device(staged, "staged operand");
        check_device(status, "status word");
        const unsigned grid = unsigned(ceil_div(seqs * positions, int64_t(STAGE_WARPS)));
        auto kernel = rounding == 0 ? k_stage_heads<0> : rounding == 2 ? k_stage_heads<2> : k_stage_heads<1>;
        kernel<<<grid, STAGE_WARPS * 32, 0, as_stream(stream)>>>(
            static_cast<const __nv_bfloat16 *>(attention), seqs, heads, positions, head_dim, seq_stride, head_stride,
            position_stride, static_cast<__half *>(staged), status);
        cuda_check(cudaGetLastError(), "attention staging launch");
        return 0;
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return -1;
    }
}

int mstar_b200_stage_conv(const float *source, int32_t time_major, int64_t batch, int64_t channels, int64_t time_in,
                          int32_t stride, int64_t k_padded, void *staged, uint64_t staged_bytes, int32_t rounding,
                          int32_t *status, void *stream, char *error, size_t error_size) {
    try {
        require(rounding >= 0 && rounding <= 2, "unknown Q8_0 activation rounding");
        require(time_major == 0 || time_major == 1, "layout flag is 0 (channel-major) or 1 (time-major)");
        require(stride == 1 || stride == 2, "convolution stride is 1 or 2");
        require(batch >= 1 && batch <= 4096 && channels >= 1 && channels <= 65536 && time_in >= 1 &&
                    time_in <= (int64_t(1) << 24),
                "invalid convolution shape");
        require(k_padded % QK == 0 && k_padded >= 3 * channels && k_padded < 3 * channels + 64,
                "padded K must be 3 * channels rounded up to a multiple of 32 (at most 63 zeros)");
        const int64_t time_out = (time_in + 2 - 3) / stride + 1;
        require(batch * time_out <= (int64_t(1) << 31), "too many convolution rows");
        const uint64_t sb = uint64_t(batch * channels * time_in) * 4;
        const uint64_t ob = uint64_t(batch * time_out * k_padded) * 2;
        check_range({source, sb}, sb, 4, "convolution input");
        check_range({staged, staged_bytes}, ob, 16, "staged operand");
        require(disjoint({source, sb}, {staged, ob}), "staged operand overlaps the input");
        require(status, "missing status word");
        check_device(source, "convolution input");
        check_device(staged, "staged operand");
        check_device(status, "status word");
        launch_stage_conv(rounding, source, time_major, batch, channels, time_in, time_out, stride, k_padded,
                          static_cast<__half *>(staged), status, as_stream(stream));
        cuda_check(cudaGetLastError(), "convolution staging launch");
        return 0;
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return -1;
    }
}

int mstar_b200_layer_norm(const float *x, int64_t x_stride, int64_t rows, int64_t width, const float *weight,
                          const float *bias, float eps, float *out, int64_t out_stride, void *stream, char *error,
                          size_t error_size) {
    try {
        require(rows >= 1 && rows <= (int64_t(1) << 31) && width >= 4 && width % 4 == 0 &&
                    width <= int64_t(STAGE_MAX_PER_LANE) * 32,
                "LayerNorm rows are 4..1536 wide, a multiple of 4");
        require(x_stride >= width && out_stride >= width && x_stride % 4 == 0 && out_stride % 4 == 0,
                "row strides must be multiples of 4 elements");
        require(weight && bias && std::isfinite(eps) && eps >= 0.0f, "invalid LayerNorm parameters");
        require(uintptr_t(x) % 16 == 0 && uintptr_t(out) % 16 == 0 && uintptr_t(weight) % 16 == 0 &&
                    uintptr_t(bias) % 16 == 0,
                "LayerNorm operands must be 16-byte aligned");
        const uint64_t xb = uint64_t((rows - 1) * x_stride + width) * 4;
        const uint64_t ob = uint64_t((rows - 1) * out_stride + width) * 4;
        check_range({x, xb}, xb, 4, "LayerNorm input");
        check_range({out, ob}, ob, 4, "LayerNorm output");
        require(disjoint({x, xb}, {out, ob}), "LayerNorm output overlaps its input");
        check_device(x, "LayerNorm input");
        check_device(out, "LayerNorm output");
        check_device(weight, "LayerNorm weight");
        check_device(bias, "LayerNorm bias");
        launch_layer_norm(x, x_stride, rows, width, weight, bias, eps, out, out_stride, as_stream(stream));
        cuda_check(cudaGetLastError(), "LayerNorm launch");
        return 0;
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return -1;
    }
}

}  // extern "C"
