#pragma once
// Device pieces shared by the decode GEMV kernels (gemv.cu) and the
// persistent decode-step kernel (step.cu).
#include "common.cuh"

namespace mb {

// Exact int32 block dots of one m16n8 tile. Q4_0: nibbles n are multiplied
// unsigned and sum((n - 8) x) = sum(n x) - 8 sum(x) with the block's
// activation quant sums of rows g and g+8 (xsum_g[0], xsum_g[8]).
template <bool Q4>
__device__ __forceinline__ void mma_q(int (&d)[4], const uint4 &a, uint32_t b0, uint32_t b1, const int *xsum_g) {
    if (Q4) {
        mma_s8u8(d, a, b0, b1);
        const int s0 = 8 * xsum_g[0], s1 = 8 * xsum_g[8];
        d[0] -= s0;
        d[1] -= s0;
        d[2] -= s1;
        d[3] -= s1;
    } else {
        mma_s8(d, a, b0, b1);
    }
}

// Per-block fp32 terms of one m16n8 tile: rows g (c0, c1) and g+8 (c2, c3)
// with ggml's generic rounding order (see the file comment).
template <bool Q4>
__device__ __forceinline__ void block_terms(const int (&d)[4], float2 dw, float dx0, float dx1, bool hi,
                                            float2 &lo_t, float2 &hi_t) {
    const float2 i01 = i2f2(d[0], d[1]);
    if (Q4) lo_t = mul2(mul2(i01, dw), make_float2(dx0, dx0));
    else lo_t = mul2(i01, mul2(dw, make_float2(dx0, dx0)));
    if (hi) {
        const float2 i23 = i2f2(d[2], d[3]);
        if (Q4) hi_t = mul2(mul2(i23, dw), make_float2(dx1, dx1));
        else hi_t = mul2(i23, mul2(dw, make_float2(dx1, dx1)));
    }
}

// Reduce a per-token argmax key across the 4 lanes sharing row g, then one
// shared-memory atomic per (warp, token).
__device__ __forceinline__ void reduce_best(unsigned long long best, unsigned long long *slot, int t) {
#pragma unroll
    for (int o = 1; o <= 2; o <<= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
    }
    if (t == 0 && best) atomicMax(slot, best);
}


}  // namespace mb
