// Quantizers and layout conversions of libmstar_b200.
//
//  k_pack          logical fp32 weights -> canonical ggml Q8_0 / Q4_0 blocks
//                  (ggml-quants.c:113-147 and :276-297, with the fp16
//                  pre-round of decoder.cpp:307-316 / :816-842)
//  k_repack_q8/q4  canonical blocks -> the B200 fragment layout (common.cuh)
//  k_quantize_act  fp32 activations -> Q8_0 in A-fragment order, with the
//                  three rounding variants of quantize_row_q8_0
//                  (ggml-quants.c:276-297, arch/arm/quants.c:41-75,
//                  arch/x86/quants.c:302-350)
// Every rounding step is an explicit IEEE intrinsic so that the compiler's
// contraction cannot change a byte.
#include "quant.cuh"

namespace mb {

// One thread per 32-element block. flags bit0: nonfinite input, bit1: fp16
// overflow after the pre-round.
__global__ void k_pack(const float *__restrict__ in, uint8_t *__restrict__ out, int64_t rows,
                       int64_t width, int q4, int preround, int fused, int *__restrict__ flags) {
    const int64_t nb = width / QK;
    const int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;
    if (i >= rows * nb) return;
    const float *x = in + i * QK;  // rows are contiguous: block i of the flat array
    float v[QK];
    int bad = 0;
#pragma unroll
    for (int j = 0; j < QK; ++j) {
        float a = x[j];
        if (!isfinite(a)) bad |= 1;
        if (preround) {
            a = __half2float(__float2half_rn(a));
            if (!isfinite(a)) bad |= 2;
        }
        v[j] = a;
    }
    if (bad) atomicOr(flags, bad);
    if (q4) {
        float amax = 0.0f, mx = 0.0f;
#pragma unroll
        for (int j = 0; j < QK; ++j)
            if (amax < fabsf(v[j])) { amax = fabsf(v[j]); mx = v[j]; }
        const float d = __fdiv_rn(mx, -8.0f);
        const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        uint16_t *o16 = reinterpret_cast<uint16_t *>(out + i * Q4_BYTES);  // 2-byte aligned
        o16[0] = __half_as_ushort(__float2half_rn(d));
        uint32_t pair = 0;
#pragma unroll
        for (int j = 0; j < QK / 2; ++j) {
            float t0, t1;
            if (fused) {
                t0 = __fmaf_rn(v[j], id, 8.5f);
                t1 = __fmaf_rn(v[j + 16], id, 8.5f);
            } else {
                t0 = __fadd_rn(__fmul_rn(v[j], id), 8.5f);
                t1 = __fadd_rn(__fmul_rn(v[j + 16], id), 8.5f);
            }
            int q0 = __float2int_rz(t0), q1 = __float2int_rz(t1);
            q0 = q0 > 15 ? 15 : q0;
            q1 = q1 > 15 ? 15 : q1;
            const uint32_t byte = uint32_t(q0 | (q1 << 4)) & 0xffu;
            if (j & 1) o16[1 + j / 2] = uint16_t(pair | (byte << 8));
            else pair = byte;
        }
    } else {
        uint16_t *o16 = reinterpret_cast<uint16_t *>(out + i * Q8_BYTES);  // 2-byte aligned
        float amax = 0.0f;
#pragma unroll
        for (int j = 0; j < QK; ++j) amax = fmaxf(amax, fabsf(v[j]));
        const float d = __fdiv_rn(amax, 127.0f);
        const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        o16[0] = __half_as_ushort(__float2half_rn(d));
#pragma unroll
        for (int j = 0; j < QK; j += 2) {
            const uint32_t q0 = uint32_t(int(roundf(__fmul_rn(v[j], id)))) & 0xffu;
            const uint32_t q1 = uint32_t(int(roundf(__fmul_rn(v[j + 1], id)))) & 0xffu;
            o16[1 + j / 2] = uint16_t(q0 | (q1 << 8));
        }
    }
}

__device__ __forceinline__ uint32_t load4(const uint8_t *p) {
    return uint32_t(p[0]) | (uint32_t(p[1]) << 8) | (uint32_t(p[2]) << 16) | (uint32_t(p[3]) << 24);
}

// One thread per (group, pair, lane).
__global__ void k_repack_q8(const uint8_t *__restrict__ blocks, uint4 *__restrict__ wq, int64_t rows,
                            int64_t nb, int64_t nb_pad, int64_t groups) {
    const int64_t pairs = nb_pad / 2;
    const int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;
    if (i >= groups * pairs * 32) return;
    const int lane = int(i % 32), g = lane >> 2, t = lane & 3;
    const int64_t p = (i / 32) % pairs, G = i / (32 * pairs);
    const int64_t row = G * 8 + g;
    uint32_t w[4] = {0, 0, 0, 0};
    for (int h = 0; h < 2; ++h) {
        const int64_t b = 2 * p + h;
        if (row < rows && b < nb) {
            const uint8_t *qs = blocks + (row * nb + b) * Q8_BYTES + 2;
            w[2 * h] = load4(qs + 4 * t);
            w[2 * h + 1] = load4(qs + 16 + 4 * t);
        }
    }
    wq[i] = make_uint4(w[0], w[1], w[2], w[3]);
}

__global__ void k_repack_q4(const uint8_t *__restrict__ blocks, uint4 *__restrict__ wq, int64_t rows,
                            int64_t nb, int64_t nb_pad, int64_t groups) {
    const int64_t quads = nb_pad / 4;
    const int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;
    if (i >= groups * quads * 32) return;
    const int lane = int(i % 32), g = lane >> 2, t = lane & 3;
    const int64_t q = (i / 32) % quads, G = i / (32 * quads);
    const int64_t row = G * 8 + g;
    uint32_t w[4] = {0x88888888u, 0x88888888u, 0x88888888u, 0x88888888u};  // nibble 8 == value 0
    for (int j = 0; j < 4; ++j) {
        const int64_t b = 4 * q + j;
        if (row < rows && b < nb) w[j] = load4(blocks + (row * nb + b) * Q4_BYTES + 2 + 4 * t);
    }
    wq[i] = make_uint4(w[0], w[1], w[2], w[3]);
}

// ws[G][b][8] fp16 scales; padding rows/blocks get 0.
__global__ void k_repack_scales(const uint8_t *__restrict__ blocks, __half *__restrict__ ws, int64_t rows,
                                int64_t nb, int64_t nb_pad, int64_t groups, int block_bytes) {
    const int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;
    if (i >= groups * nb_pad * 8) return;
    const int r = int(i % 8);
    const int64_t b = (i / 8) % nb_pad, G = i / (8 * nb_pad);
    const int64_t row = G * 8 + r;
    uint16_t h = 0;
    if (row < rows && b < nb) {
        const uint8_t *p = blocks + (row * nb + b) * block_bytes;
        h = uint16_t(p[0]) | uint16_t(uint16_t(p[1]) << 8);
    }
    ws[i] = __ushort_as_half(h);
}

// One warp per (token, block): lane j quantizes element j into canonical
// ggml Q8_0 bytes (the q8cpu_quantize mirror). Tokens are rows here.
template <int MODE>
__global__ void k_quantize_rows(const float *__restrict__ x, int64_t ldx, int64_t m, int64_t k,
                                uint8_t *__restrict__ blocks, int *__restrict__ status) {
    const int lane = threadIdx.x & 31;
    const int64_t nb = k / QK;
    const int64_t wid = (blockIdx.x * int64_t(blockDim.x) + threadIdx.x) >> 5;
    if (wid >= m * nb) return;
    const int64_t token = wid / nb, b = wid % nb;
    const float v = x[token * ldx + b * QK + lane];
    if (!isfinite(v)) atomicOr(status, 1);
    float amax = fabsf(v);
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float d = __fdiv_rn(amax, 127.0f);
    float id;
    if (MODE == 2) id = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
    else id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    const float s = __fmul_rn(v, id);
    const int q = MODE == 0 ? int(roundf(s)) : __float2int_rn(s);
    // 34-byte blocks are 2-byte aligned: even lanes store a pair of quants
    const uint32_t mine = uint32_t(q) & 0xffu;
    const uint32_t next = __shfl_down_sync(0xffffffffu, mine, 1);
    uint16_t *o16 = reinterpret_cast<uint16_t *>(blocks + (token * nb + b) * Q8_BYTES);
    if (!(lane & 1)) o16[1 + lane / 2] = uint16_t(mine | (next << 8));
    if (lane == 0) o16[0] = __half_as_ushort(__float2half_rn(d));
}


// One CTA per token (mpad CTAs): optional LayerNorm of the row (ggml_norm,
// ggml-cpu/ops.cpp:4094-4137, then ggml_mul/ggml_add by the affine), then
// quantize_row_q8_0 with the selected rounding, written in A-fragment order:
//   xf [nb_pad][mtiles][32 lanes][4 words], xs [nb_pad][mpad] fp32 scales.
// Dead tokens (>= m) and padding blocks (>= nb) get zero quants and scales.
// Launched as a programmatic dependent: it waits for the producer of x, then
// lets the consuming GEMV start prefetching its weights.
template <int MODE>
__global__ void __launch_bounds__(256) k_quantize_frag(const float *__restrict__ x, int64_t ldx, int64_t m,
                                                       int64_t k, int64_t mpad, int64_t nb_pad,
                                                       const float *__restrict__ ln_w, const float *__restrict__ ln_b,
                                                       float ln_eps, uint32_t *__restrict__ xf,
                                                       float *__restrict__ xs, int *__restrict__ xsum,
                                                       int *__restrict__ status) {
    pdl_wait();
    pdl_trigger();
    __shared__ float red[2][8];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const int64_t token = blockIdx.x;
    const int64_t nb = k / QK;
    const bool live_token = token < m;
    const float *xr = x + token * ldx;
    float mean = 0.0f, rstd = 1.0f;
    if (ln_w && live_token) {
        float sum = 0.0f;
        for (int64_t i = threadIdx.x; i < k; i += blockDim.x) sum += xr[i];
#pragma unroll
        for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (lane == 0) red[0][warp] = sum;
        __syncthreads();
        sum = 0.0f;
        for (int w = 0; w < nwarps; ++w) sum += red[0][w];
        mean = sum / float(k);
        float var = 0.0f;
        for (int64_t i = threadIdx.x; i < k; i += blockDim.x) {
            const float y = xr[i] - mean;
            var = fmaf(y, y, var);
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) var += __shfl_xor_sync(0xffffffffu, var, o);
        if (lane == 0) red[1][warp] = var;
        __syncthreads();
        var = 0.0f;
        for (int w = 0; w < nwarps; ++w) var += red[1][w];
        rstd = 1.0f / sqrtf(var / float(k) + ln_eps);
    }
    const int64_t mtiles = mpad / 16;
    const int64_t mt = token / 16;
    const int r = int(token % 16), g = r & 7, hi = r >> 3;
    const int t = (lane & 15) >> 2, half = lane >> 4;
    // blocks of this token: all of them (gridDim.y == 1, as the LayerNorm statistics need
    // the whole row), or without a LayerNorm this CTA's share (blocks are independent)
    for (int64_t b = int64_t(blockIdx.y) * nwarps + warp; b < nb_pad; b += int64_t(gridDim.y) * nwarps) {
        const bool live = live_token && b < nb;
        float v = 0.0f;
        if (live) {
            v = xr[b * QK + lane];
            if (ln_w) {
                const int64_t i = b * QK + lane;
                v = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v, mean), rstd), __ldg(ln_w + i)), __ldg(ln_b + i));
            }
            if (!isfinite(v)) atomicOr(status, 1);
        }
        float amax = fabsf(v);
#pragma unroll
        for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const float d = __fdiv_rn(amax, 127.0f);
        float id;
        if (MODE == 2) id = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
        else id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        const float sv = __fmul_rn(v, id);
        const int q = MODE == 0 ? int(roundf(sv)) : __float2int_rn(sv);
        // gather 4 consecutive quants into the word owned by lane (4t + j) / 4
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
            xs[b * mpad + token] = __half2float(__float2half_rn(d));
            xsum[b * mpad + token] = qsum;
        }
    }
}

// The same result as k_quantize_frag, one warp per query row: the lanes load
// the whole row at once (task t = elements 128 t .. 128 t + 127, one float4
// per lane, so lane l holds elements 128 t + 4 l + c), and the LayerNorm sums
// are formed in k_quantize_frag's order from registers: element e belongs to
// its thread e mod VT (VT = 128 or 256 threads), which is thread
// 128 (t mod VT/128) + 4 l + c, so each of those threads' running sums over t
// is local to lane l; its warp reduction (butterfly over the thread's lane
// bits 4..0) becomes a butterfly over lane bits 2..0 then over c, and the
// warps' totals are added in thread order. Each lane then quantizes its four
// elements of one block per task (block maxima over 8 lanes; one division per
// lane for the row's blocks), so its four quants are one fragment word.
constexpr int QW_MAX_TASKS = 12;  // rows up to 1536 wide
constexpr int QW_WARPS = 2;

template <int MODE, int NCH>
__global__ void __launch_bounds__(QW_WARPS * 32) k_quantize_frag_warp(
    const float *__restrict__ x, int64_t ldx, int64_t m, int64_t k, int64_t mpad, int64_t nb_pad,
    const float *__restrict__ ln_w, const float *__restrict__ ln_b, float ln_eps, uint32_t *__restrict__ xf,
    float *__restrict__ xs, int *__restrict__ xsum, int *__restrict__ status) {
    const int lane = threadIdx.x & 31;
    const int64_t q = int64_t(blockIdx.x) * QW_WARPS + (threadIdx.x >> 5);
    const int nb = int(k / QK), j = lane & 7, sb = lane >> 3;
    // narrow rows: the LayerNorm weights are parameters, not the previous kernel's output,
    // so they are loaded before waiting on it (their latency hides behind its tail)
    constexpr bool PRE_LN = NCH <= 4;
    float4 pw[PRE_LN ? NCH : 1], pb[PRE_LN ? NCH : 1];
    if (PRE_LN && ln_w && q < m) {
#pragma unroll
        for (int t = 0; t < (PRE_LN ? NCH : 1); ++t)
            if (4 * t + sb < nb) {
                pw[t] = __ldg(reinterpret_cast<const float4 *>(ln_w + 128 * t + 4 * lane));
                pb[t] = __ldg(reinterpret_cast<const float4 *>(ln_b + 128 * t + 4 * lane));
            }
    }
    pdl_wait();
    pdl_trigger();
    if (q >= mpad) return;  // warp-uniform
    const bool live_row = q < m;
    const float *xr = x + q * ldx;
    float4 v[NCH];
#pragma unroll
    for (int t = 0; t < NCH; ++t) {
        v[t] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (live_row && 4 * t + sb < nb) v[t] = *reinterpret_cast<const float4 *>(xr + 128 * t + 4 * lane);
    }
    if (ln_w && live_row) {
        constexpr int SL = NCH >= 8 ? 2 : 1;  // used only when VT = 256 (k >= 1024 needs NCH >= 8)
        const int slabs = k >= 1024 ? 2 : 1;
        auto stats = [&](auto term, float &total) {
            float p[SL][4];
#pragma unroll
            for (int s2 = 0; s2 < SL; ++s2)
#pragma unroll
                for (int c = 0; c < 4; ++c) p[s2][c] = 0.0f;
#pragma unroll
            for (int t = 0; t < NCH; ++t) {
                if (4 * t + sb >= nb) continue;  // elements past the row: no term
                const int s2 = SL == 2 ? (t & (slabs - 1)) : 0;
                p[s2][0] = term(p[s2][0], v[t].x);
                p[s2][1] = term(p[s2][1], v[t].y);
                p[s2][2] = term(p[s2][2], v[t].z);
                p[s2][3] = term(p[s2][3], v[t].w);
            }
            float tot[SL];
#pragma unroll
            for (int s2 = 0; s2 < SL; ++s2) {
#pragma unroll
                for (int o = 4; o; o >>= 1)  // thread lane bits 4, 3, 2 = this lane's bits 2, 1, 0
#pragma unroll
                    for (int c = 0; c < 4; ++c) p[s2][c] += __shfl_xor_sync(0xffffffffu, p[s2][c], o);
                float r[4];
#pragma unroll
                for (int c = 0; c < 4; ++c) r[c] = p[s2][c] + p[s2][c ^ 2];  // thread lane bit 1
                tot[s2] = r[0] + r[1];                                         // thread lane bit 0
            }
            float sum = 0.0f;  // the thread warps' totals in order: warp 4 s2 + (lane >> 3)
#pragma unroll
            for (int s2 = 0; s2 < SL; ++s2) {
                if (s2 >= slabs) break;
#pragma unroll
                for (int w = 0; w < 4; ++w) sum += __shfl_sync(0xffffffffu, tot[s2], 8 * w);
            }
            total = sum;
        };
        float sum, var;
        stats([](float acc, float e) { return acc + e; }, sum);
        const float mean = sum / float(k);
        stats([mean](float acc, float e) { const float y = e - mean; return fmaf(y, y, acc); }, var);
        const float rstd = 1.0f / sqrtf(var / float(k) + ln_eps);
#pragma unroll
        for (int t = 0; t < NCH; ++t) {
            if (4 * t + sb >= nb) continue;
            const int64_t e = 128 * t + 4 * lane;
            const float4 w = PRE_LN ? pw[PRE_LN ? t : 0] : __ldg(reinterpret_cast<const float4 *>(ln_w + e));
            const float4 c = PRE_LN ? pb[PRE_LN ? t : 0] : __ldg(reinterpret_cast<const float4 *>(ln_b + e));
            auto nf = [&](float xv, float ww, float bb) {
                return __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(xv, mean), rstd), ww), bb);
            };
            v[t] = make_float4(nf(v[t].x, w.x, c.x), nf(v[t].y, w.y, c.y), nf(v[t].z, w.z, c.z), nf(v[t].w, w.w, c.w));
        }
    }
    if (live_row) {
        bool finite = true;
#pragma unroll
        for (int t = 0; t < NCH; ++t)
            if (4 * t + sb < nb)
                finite = finite && isfinite(v[t].x) && isfinite(v[t].y) && isfinite(v[t].z) && isfinite(v[t].w);
        if (!finite) atomicOr(status, 1);
    }
    float amax[NCH];
#pragma unroll
    for (int t = 0; t < NCH; ++t) amax[t] = fmaxf(fmaxf(fabsf(v[t].x), fabsf(v[t].y)), fmaxf(fabsf(v[t].z), fabsf(v[t].w)));
#pragma unroll
    for (int o = 1; o < 8; o <<= 1)
#pragma unroll
        for (int t = 0; t < NCH; ++t) amax[t] = fmaxf(amax[t], __shfl_xor_sync(0xffffffffu, amax[t], o));
    // one division per lane: lane L for blocks L and L + 32 (block b = 4 t + sub-block)
    constexpr int NB2 = (4 * NCH + 31) / 32;
    float my_id[NB2];
#pragma unroll
    for (int h = 0; h < NB2; ++h) {
        const int b = 32 * h + lane;
        float mine = 0.0f;
#pragma unroll
        for (int t = 0; t < NCH; ++t) {
            const float mt = __shfl_sync(0xffffffffu, amax[t], 8 * (b & 3));
            if ((b >> 2) == t) mine = mt;
        }
        const float d = __fdiv_rn(mine, 127.0f);
        if (MODE == 2) my_id[h] = mine != 0.0f ? __fdiv_rn(127.0f, mine) : 0.0f;
        else my_id[h] = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        if (b < nb_pad) xs[b * mpad + q] = __half2float(__float2half_rn(d));
    }
    const int64_t mtiles = mpad / 16, mt = q / 16;
    const int r = int(q % 16), g = r & 7, hi = r >> 3;
#pragma unroll
    for (int t = 0; t < NCH; ++t) {
        const int b = 4 * t + sb;
        const float id = __shfl_sync(0xffffffffu, my_id[(4 * t) / 32 + 0], (4 * t + sb) & 31);
        auto quant = [&](float xv) -> int {
            const float sv = __fmul_rn(xv, id);
            return MODE == 0 ? int(roundf(sv)) : __float2int_rn(sv);
        };
        const int q0 = quant(v[t].x), q1 = quant(v[t].y), q2 = quant(v[t].z), q3 = quant(v[t].w);
        int qs = q0 + q1 + q2 + q3;
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) qs += __shfl_xor_sync(0xffffffffu, qs, o);
        if (b >= nb_pad) continue;
        const uint32_t word = (uint32_t(q0) & 0xffu) | ((uint32_t(q1) & 0xffu) << 8) | ((uint32_t(q2) & 0xffu) << 16) |
                              ((uint32_t(q3) & 0xffu) << 24);
        // word j holds elements 4j..4j+3: fragment lane 4g + (j & 3), register hi + 2 * (j >> 2)
        xf[((b * mtiles + mt) * 32 + 4 * g + (j & 3)) * 4 + hi + 2 * (j >> 2)] = word;
        if (j == 0) xsum[b * mpad + q] = qs;
    }
}

// ------------------------------------------------------------------ launchers
void launch_pack(const float *in, uint8_t *out, int64_t rows, int64_t width, int q4, int preround,
                 int fused, int *flags, cudaStream_t s) {
    const int64_t n = rows * (width / QK);
    if (!n) return;
    k_pack<<<unsigned(ceil_div(n, 128)), 128, 0, s>>>(in, out, rows, width, q4, preround, fused, flags);
}

void launch_repack(int q4, const uint8_t *blocks, uint4 *wq, __half *ws, int64_t rows, int64_t nb,
                   int64_t nb_pad, int64_t groups, cudaStream_t s) {
    const int64_t lanes = groups * (nb_pad / (q4 ? 4 : 2)) * 32;
    if (q4) k_repack_q4<<<unsigned(ceil_div(lanes, 256)), 256, 0, s>>>(blocks, wq, rows, nb, nb_pad, groups);
    else k_repack_q8<<<unsigned(ceil_div(lanes, 256)), 256, 0, s>>>(blocks, wq, rows, nb, nb_pad, groups);
    const int64_t n = groups * nb_pad * 8;
    k_repack_scales<<<unsigned(ceil_div(n, 256)), 256, 0, s>>>(blocks, ws, rows, nb, nb_pad, groups,
                                                               q4 ? Q4_BYTES : Q8_BYTES);
}

void launch_quantize_rows(int mode, const float *x, int64_t ldx, int64_t m, int64_t k, uint8_t *blocks,
                          int *status, cudaStream_t s) {
    const int64_t threads = m * (k / QK) * 32;
    const unsigned grid = unsigned(ceil_div(threads, 256));
    if (mode == 0) k_quantize_rows<0><<<grid, 256, 0, s>>>(x, ldx, m, k, blocks, status);
    else if (mode == 2) k_quantize_rows<2><<<grid, 256, 0, s>>>(x, ldx, m, k, blocks, status);
    else k_quantize_rows<1><<<grid, 256, 0, s>>>(x, ldx, m, k, blocks, status);
}

template <int MODE, int NCH>
static void quantize_warp_nch(cudaLaunchConfig_t &cfg, const float *x, int64_t ldx, int64_t m, int64_t k,
                              int64_t mpad, int64_t nb_pad, const float *ln_w, const float *ln_b, float ln_eps,
                              uint32_t *xf, float *xs, int *xsum, int *status) {
    cudaLaunchKernelEx(&cfg, k_quantize_frag_warp<MODE, NCH>, x, ldx, m, k, mpad, nb_pad, ln_w, ln_b, ln_eps, xf,
                       xs, xsum, status);
}

template <int MODE>
static void quantize_warp_mode(int nch, cudaLaunchConfig_t &cfg, const float *x, int64_t ldx, int64_t m,
                               int64_t k, int64_t mpad, int64_t nb_pad, const float *ln_w, const float *ln_b,
                               float ln_eps, uint32_t *xf, float *xs, int *xsum, int *status) {
#define QW_CASE(N)                                                                                          \
    case N:                                                                                                 \
        quantize_warp_nch<MODE, N>(cfg, x, ldx, m, k, mpad, nb_pad, ln_w, ln_b, ln_eps, xf, xs, xsum, status); \
        break;
    switch (nch) {
        QW_CASE(1) QW_CASE(2) QW_CASE(3) QW_CASE(4) QW_CASE(5) QW_CASE(6)
        QW_CASE(7) QW_CASE(8) QW_CASE(9) QW_CASE(10) QW_CASE(11) QW_CASE(12)
    }
#undef QW_CASE
}

static void launch_quantize_warp(int mode, int nch, cudaLaunchConfig_t &cfg, const float *x, int64_t ldx, int64_t m,
                                 int64_t k, int64_t mpad, int64_t nb_pad, const float *ln_w, const float *ln_b,
                                 float ln_eps, uint32_t *xf, float *xs, int *xsum, int *status) {
    if (mode == 0) quantize_warp_mode<0>(nch, cfg, x, ldx, m, k, mpad, nb_pad, ln_w, ln_b, ln_eps, xf, xs, xsum, status);
    else if (mode == 2) quantize_warp_mode<2>(nch, cfg, x, ldx, m, k, mpad, nb_pad, ln_w, ln_b, ln_eps, xf, xs, xsum, status);
    else quantize_warp_mode<1>(nch, cfg, x, ldx, m, k, mpad, nb_pad, ln_w, ln_b, ln_eps, xf, xs, xsum, status);
}

void launch_quantize_frag(int mode, const float *x, int64_t ldx, int64_t m, int64_t k, int64_t mpad,
                          int64_t nb_pad, const float *ln_w, const float *ln_b, float ln_eps, uint32_t *xf,
                          float *xs, int *xsum, int *status, cudaStream_t s) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(unsigned(mpad));
    cfg.blockDim = dim3(k >= 1024 ? 256 : 128);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const int64_t nch = (k / QK + 3) / 4;
    if (nch <= QW_MAX_TASKS && uintptr_t(x) % 16 == 0 && ldx % 4 == 0 &&
        (!ln_w || (uintptr_t(ln_w) % 16 == 0 && uintptr_t(ln_b) % 16 == 0))) {
        cfg.gridDim = dim3(unsigned(ceil_div(mpad, QW_WARPS)));
        cfg.blockDim = dim3(QW_WARPS * 32);
        launch_quantize_warp(mode, int(nch), cfg, x, ldx, m, k, mpad, nb_pad, ln_w, ln_b, ln_eps, xf, xs, xsum,
                             status);
        return;
    }
    // without a LayerNorm, 8 blocks per CTA over a second grid dimension: a wide row (o_proj's
    // 4096 at 32 queries) no longer leaves most SMs idle while 32 CTAs walk 128 blocks each
    if (!ln_w) {
        cfg.blockDim = dim3(256);
        cfg.gridDim = dim3(unsigned(mpad), unsigned(ceil_div(nb_pad, 8)));
    }
    auto kernel = mode == 0 ? k_quantize_frag<0> : mode == 2 ? k_quantize_frag<2> : k_quantize_frag<1>;
    cudaLaunchKernelEx(&cfg, kernel, x, ldx, m, k, mpad, nb_pad, ln_w, ln_b, ln_eps, xf, xs, xsum, status);
}

}  // namespace mb
