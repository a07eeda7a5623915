// Decode-shape block-quantized linear (M <= 32 tokens), HBM-streaming.
//
// One warp owns one 8-row group at a time and walks all of its K blocks in
// order: every lane issues one 16-byte streaming load per chunk (2 Q8_0 or 4
// Q4_0 blocks of its rows), the chunk's mma.m16n8k32 s8 instructions produce
// the exact int32 block dots, and each lane folds them into fp32 in ggml's
// generic block order (ggml-cpu/quants.c:451-480 for Q8_0:
// sumf += sumi*(dw*dx); quants.c:225-258 for Q4_0: sumf += sumi*dw*dx) with
// explicit IEEE roundings, so the result is bit-identical to the reference's
// generic vec_dot. Activations come pre-quantized in A-fragment order and are
// read through L1 (every warp of an SM shares them).
//
// Fused epilogues: bias, ggml GELU (fp16 table form) or erf GELU, residual
// add; and for the vocab readout, suppression, the first-index / NaN-first
// argmax (decoder.cpp:686-696) reduced per warp, per CTA, then across CTAs
// through 64-bit atomics; the last CTA to finish writes the tokens and resets
// the shared state for the next call.
#include "quant.cuh"

namespace mb {

constexpr int GEMV_THREADS = 256;
constexpr int CHUNKS_IN_FLIGHT = 4;

template <int MT, bool Q4, bool READOUT, bool SUMS>
__global__ void __launch_bounds__(GEMV_THREADS) k_gemv(const GemvArgs a) {
    constexpr int BPC = Q4 ? 4 : 2;  // blocks per 16-byte chunk
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, t = lane & 3;
    const int wpb = GEMV_THREADS / 32;
    const int64_t chunks = a.nb_pad / BPC;
    const int64_t mpad = MT * 16;
    unsigned long long best[MT][2];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) best[mt][0] = best[mt][1] = 0ull;

    for (int64_t G = int64_t(blockIdx.x) * wpb + warp; G < a.groups; G += int64_t(gridDim.x) * wpb) {
        float acc[MT][4];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) acc[mt][0] = acc[mt][1] = acc[mt][2] = acc[mt][3] = 0.0f;
        const uint4 *wp = a.wq + G * chunks * 32 + lane;
        const __half2 *sp = a.ws + G * a.nb_pad * 4 + t;
        for (int64_t c0 = 0; c0 < chunks; c0 += CHUNKS_IN_FLIGHT) {
            uint4 w[CHUNKS_IN_FLIGHT];
            __half2 sc[CHUNKS_IN_FLIGHT][BPC];
#pragma unroll
            for (int u = 0; u < CHUNKS_IN_FLIGHT; ++u) {
                if (c0 + u < chunks) {
                    w[u] = ldg_stream(wp + (c0 + u) * 32);
#pragma unroll
                    for (int j = 0; j < BPC; ++j) sc[u][j] = __ldg(sp + ((c0 + u) * BPC + j) * 4);
                }
            }
#pragma unroll
            for (int u = 0; u < CHUNKS_IN_FLIGHT; ++u) {
                if (c0 + u >= chunks) break;
#pragma unroll
                for (int j = 0; j < BPC; ++j) {
                    const int64_t b = (c0 + u) * BPC + j;
                    uint32_t b0, b1;
                    if (Q4) unpack_q4(word(w[u], j), b0, b1);
                    else {
                        b0 = word(w[u], 2 * j);
                        b1 = word(w[u], 2 * j + 1);
                    }
                    const float2 dw = __half22float2(sc[u][j]);
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt) {
                        const uint4 av = __ldg(a.xf + (b * MT + mt) * 32 + lane);
                        int d[4];
                        mma_s8(d, av, b0, b1);
                        const float dx0 = __ldg(a.xs + b * mpad + mt * 16 + g);
                        const float dx1 = __ldg(a.xs + b * mpad + mt * 16 + g + 8);
                        if (SUMS) {
#pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                const int64_t m = mt * 16 + g + 8 * (i >> 1), n = G * 8 + 2 * t + (i & 1);
                                if (m < a.m && n < a.n && b < a.nb) a.sums[(m * a.n + n) * a.nb + b] = d[i];
                            }
                        }
                        if (Q4) {
                            acc[mt][0] = __fadd_rn(acc[mt][0], __fmul_rn(__fmul_rn(__int2float_rn(d[0]), dw.x), dx0));
                            acc[mt][1] = __fadd_rn(acc[mt][1], __fmul_rn(__fmul_rn(__int2float_rn(d[1]), dw.y), dx0));
                            acc[mt][2] = __fadd_rn(acc[mt][2], __fmul_rn(__fmul_rn(__int2float_rn(d[2]), dw.x), dx1));
                            acc[mt][3] = __fadd_rn(acc[mt][3], __fmul_rn(__fmul_rn(__int2float_rn(d[3]), dw.y), dx1));
                        } else {
                            acc[mt][0] = __fadd_rn(acc[mt][0], __fmul_rn(__int2float_rn(d[0]), __fmul_rn(dw.x, dx0)));
                            acc[mt][1] = __fadd_rn(acc[mt][1], __fmul_rn(__int2float_rn(d[1]), __fmul_rn(dw.y, dx0)));
                            acc[mt][2] = __fadd_rn(acc[mt][2], __fmul_rn(__int2float_rn(d[2]), __fmul_rn(dw.x, dx1)));
                            acc[mt][3] = __fadd_rn(acc[mt][3], __fmul_rn(__int2float_rn(d[3]), __fmul_rn(dw.y, dx1)));
                        }
                    }
                }
            }
        }
        // epilogue: lane (g, t) owns tokens g, g+8 of each m-tile and columns 2t, 2t+1
#pragma unroll
        for (int mt = 0; mt < (SUMS ? 0 : MT); ++mt) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int64_t m = mt * 16 + g + 8 * (i >> 1), n = G * 8 + 2 * t + (i & 1);
                if (m >= a.m || n >= a.n) continue;
                float v = acc[mt][i];
                if (a.flags & 1) v = __fadd_rn(v, __ldg(a.bias + n));
                if (a.flags & 2) v = gelu_ggml(v);
                else if (a.flags & 8) v = gelu_erf(v);
                if (a.flags & 4) v = __fadd_rn(__ldg(a.residual + m * a.ldo + n), v);
                if (READOUT) {
                    for (int64_t s = 0; s < a.suppressed_count; ++s)
                        if (__ldg(a.suppressed + s) == n) v = -INFINITY;
                    const unsigned long long key = argmax_key(v, uint32_t(n));
                    best[mt][i >> 1] = key > best[mt][i >> 1] ? key : best[mt][i >> 1];
                }
                a.out[m * a.ldo + n] = v;
            }
        }
    }

    if (READOUT) {
        __shared__ unsigned long long cta_best[32];
        __shared__ bool last;
        if (threadIdx.x < 32) cta_best[threadIdx.x] = 0ull;
        __syncthreads();
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                unsigned long long k = best[mt][h];
                for (int o = 1; o <= 2; o <<= 1) {
                    const unsigned long long other = __shfl_xor_sync(0xffffffffu, k, o);
                    k = other > k ? other : k;
                }
                if (t == 0 && k) atomicMax(&cta_best[mt * 16 + g + 8 * h], k);
            }
        __syncthreads();
        if (threadIdx.x < a.m && cta_best[threadIdx.x]) atomicMax(a.keys + threadIdx.x, cta_best[threadIdx.x]);
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) last = atomicAdd(a.done, 1u) == gridDim.x - 1;
        __syncthreads();
        if (last) {
            __threadfence();
            if (threadIdx.x < a.m) {
                const unsigned long long k = atomicExch(a.keys + threadIdx.x, 0ull);
                a.token[threadIdx.x] = int64_t(0xFFFFFFFFu - uint32_t(k & 0xFFFFFFFFull));
            }
            if (threadIdx.x == 0) *a.done = 0u;
        }
    }
}

template <int MT, bool Q4>
static void launch_variant(const GemvArgs &a, cudaStream_t s, int sm_count) {
    const int wpb = GEMV_THREADS / 32;
    const int64_t want = ceil_div(a.groups, wpb);
    // Enough CTAs to fill every SM several times; warps loop over the rest.
    const int64_t cap = int64_t(sm_count) * 8;
    const unsigned grid = unsigned(want < cap ? want : cap);
    if (a.sums) k_gemv<MT, Q4, false, true><<<grid, GEMV_THREADS, 0, s>>>(a);
    else if (a.keys) k_gemv<MT, Q4, true, false><<<grid, GEMV_THREADS, 0, s>>>(a);
    else k_gemv<MT, Q4, false, false><<<grid, GEMV_THREADS, 0, s>>>(a);
}

void launch_gemv(int q4, const GemvArgs &a, cudaStream_t s) {
    static int sm_count = 0;
    if (!sm_count) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sm_count, cudaDevAttrMultiProcessorCount, dev);
        if (sm_count <= 0) sm_count = 148;
    }
    const int mt = a.m <= 16 ? 1 : 2;
    if (q4) {
        if (mt == 1) launch_variant<1, true>(a, s, sm_count);
        else launch_variant<2, true>(a, s, sm_count);
    } else {
        if (mt == 1) launch_variant<1, false>(a, s, sm_count);
        else launch_variant<2, false>(a, s, sm_count);
    }
}

}  // namespace mb
