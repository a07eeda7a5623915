// Thinker attention prologue after the QKV projection, in one launch: per-head
// QK RMSNorm, the prepared (M)RoPE rotation and the KV-cache write.
//
// Arithmetic of the reference's fused op (implementations/qwen3_omni/amd/
// qknorm_rope.py:9-53, bf16 boundaries, no fused multiply-add):
//   x = fp32(bf16 head row of 128), r = 1 / sqrt(sum(x^2) / 128 + eps)
//   n = bf16((x * r) * w)                          (w: q_norm or k_norm weight)
//   rot = rotate_half(n): rot[d] = -n[d + 64] for d < 64, n[d - 64] after
//   a = n * cos[t], b = rot * sin[t]  (each rounded to bf16 when round_products)
//   y = bf16(a + b)
// cos / sin are the token's prepared rows [128] (the MRoPE sections already
// interleaved by the caller, as for the reference op). q heads go to out_q; k
// heads go to k_cache at the token's slot, and (when v is given) the token's v
// heads are copied to v_cache at the same slot (the KV write of the code
// predictor's prologue, cp_kernels.py:16-58). One warp per four heads of a token,
// four elements of a head per lane; the rotation partner is lane ^ 16. The sum of squares is a
// fixed butterfly in fp32, so a result can sit one bf16 step from another
// summation order's where it lands on a rounding boundary.
#include <cmath>

#include <cuda_bf16.h>

#include "../../include/mstar_b200.h"
#include "common.cuh"

namespace mb {

constexpr int QK_HEAD_DIM = 128;
constexpr int QK_WARPS = 8;
constexpr int QK_HEADS_PER_WARP = 4;

struct QkArgs {
    const void *q, *k, *v;               // [T, heads, 128] bf16 (or fp32) rows with strides (elements)
    int64_t q_s0, q_s1, k_s0, k_s1, v_s0, v_s1;
    const __nv_bfloat16 *qw, *kw;        // [128]
    const __nv_bfloat16 *cos, *sin;      // [T, 128] rows
    int64_t cs0, ss0;
    int64_t tokens;
    int qh, kh;
    float eps;
    int round_products;
    __nv_bfloat16 *out_q;                // [T, qh, 128] contiguous
    __nv_bfloat16 *k_cache, *v_cache;    // [slots, kh, 128] contiguous rows of slot stride
    int64_t cache_s0;                    // elements between slots
    const int64_t *slots;                // [T] slot of each token (k / v destination row)
    int64_t num_slots;
    int *status;                         // bit value 1: a slot outside [0, num_slots) (token skipped)
};

__device__ __forceinline__ float bf(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ void bf16x4(const __nv_bfloat16 *p, float (&f)[4]) {
    const uint2 u = *reinterpret_cast<const uint2 *>(p);   // 8-byte aligned (checked by the entry point)
    __nv_bfloat162 lo, hi;
    memcpy(&lo, &u.x, 4);
    memcpy(&hi, &u.y, 4);
    const float2 a = __bfloat1622float2(lo), b = __bfloat1622float2(hi);
    f[0] = a.x, f[1] = a.y, f[2] = b.x, f[3] = b.y;
}

// Four consecutive elements of a q / k / v row as bf16: loaded as they are, or, for fp32
// rows (the projection's fp32 output), rounded to bf16 to nearest even on the way in,
// which is the .to(bfloat16) the op would otherwise run first.
template <bool F32>
__device__ __forceinline__ uint2 load_head4(const void *base, int64_t e) {
    if constexpr (F32) {
        const float4 f = *reinterpret_cast<const float4 *>(static_cast<const float *>(base) + e);
        const __nv_bfloat162 lo = __floats2bfloat162_rn(f.x, f.y), hi = __floats2bfloat162_rn(f.z, f.w);
        uint2 u;
        memcpy(&u.x, &lo, 4);
        memcpy(&u.y, &hi, 4);
        return u;
    } else {
        return *reinterpret_cast<const uint2 *>(static_cast<const __nv_bfloat16 *>(base) + e);
    }
}

// A warp takes QK_HEADS_PER_WARP heads of one token: their rows are loaded together
// (one load per lane and head) and the token's cos / sin rows once for all of them.
template <bool F32>
__global__ void __launch_bounds__(QK_WARPS * 32) k_qknorm_rope(const QkArgs a) {
    const int lane = threadIdx.x & 31;
    const int heads = a.qh + a.kh;
    const int groups = (heads + QK_HEADS_PER_WARP - 1) / QK_HEADS_PER_WARP;
    const int64_t item = int64_t(blockIdx.x) * QK_WARPS + (threadIdx.x >> 5);
    if (item >= a.tokens * groups) return;   // warp-uniform
    const int64_t t = item / groups;
    const int h0 = int(item % groups) * QK_HEADS_PER_WARP;
    const int d0 = 4 * lane;
    uint2 xr[QK_HEADS_PER_WARP], vr[QK_HEADS_PER_WARP];
#pragma unroll
    for (int j = 0; j < QK_HEADS_PER_WARP; ++j) {
        const int h = h0 + j;
        xr[j] = make_uint2(0u, 0u);
        vr[j] = make_uint2(0u, 0u);
        if (h < a.qh) {
            xr[j] = load_head4<F32>(a.q, t * a.q_s0 + int64_t(h) * a.q_s1 + d0);
        } else if (h < heads) {
            xr[j] = load_head4<F32>(a.k, t * a.k_s0 + int64_t(h - a.qh) * a.k_s1 + d0);
            if (a.v) vr[j] = load_head4<F32>(a.v, t * a.v_s0 + int64_t(h - a.qh) * a.v_s1 + d0);
        }
    }
    float c[4], s[4], wq[4], wk[4];
    bf16x4(a.cos + t * a.cs0 + d0, c);
    bf16x4(a.sin + t * a.ss0 + d0, s);
    bf16x4(a.qw + d0, wq);
    bf16x4(a.kw + d0, wk);
    int64_t slot = 0;
    bool slot_ok = true;
    if (h0 + QK_HEADS_PER_WARP > a.qh) {   // the group holds k heads
        slot = a.slots ? a.slots[t] : t;
        slot_ok = slot >= 0 && slot < a.num_slots;
        if (!slot_ok && lane == 0 && a.status) atomicOr(a.status, 1);
    }
    const float sign = lane < 16 ? -1.0f : 1.0f;
#pragma unroll
    for (int j = 0; j < QK_HEADS_PER_WARP; ++j) {
        const int h = h0 + j;
        if (h >= heads) break;   // warp-uniform
        const bool is_q = h < a.qh;
        float x[4];
        {
            __nv_bfloat162 lo, hi;
            memcpy(&lo, &xr[j].x, 4);
            memcpy(&hi, &xr[j].y, 4);
            const float2 p = __bfloat1622float2(lo), q = __bfloat1622float2(hi);
            x[0] = p.x, x[1] = p.y, x[2] = q.x, x[3] = q.y;
        }
        float ss = __fadd_rn(__fadd_rn(__fmul_rn(x[0], x[0]), __fmul_rn(x[1], x[1])),
                             __fadd_rn(__fmul_rn(x[2], x[2]), __fmul_rn(x[3], x[3])));
#pragma unroll
        for (int o = 16; o; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
        const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, float(QK_HEAD_DIM)), a.eps)));
        float n[4], p[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) n[i] = bf(__fmul_rn(__fmul_rn(x[i], r), is_q ? wq[i] : wk[i]));
#pragma unroll
        for (int i = 0; i < 4; ++i) p[i] = __shfl_xor_sync(0xffffffffu, n[i], 16);  // element d +- 64
        __align__(8) __nv_bfloat16 y[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float av = __fmul_rn(n[i], c[i]), bv = __fmul_rn(sign * p[i], s[i]);
            if (a.round_products) {
                av = bf(av);
                bv = bf(bv);
            }
            y[i] = __float2bfloat16_rn(__fadd_rn(av, bv));
        }
        if (is_q) {
            *reinterpret_cast<uint2 *>(a.out_q + (t * a.qh + h) * QK_HEAD_DIM + d0) =
                *reinterpret_cast<const uint2 *>(y);
            continue;
        }
        if (!slot_ok) continue;
        const int64_t at = slot * a.cache_s0 + int64_t(h - a.qh) * QK_HEAD_DIM + d0;
        *reinterpret_cast<uint2 *>(a.k_cache + at) = *reinterpret_cast<const uint2 *>(y);
        if (a.v) *reinterpret_cast<uint2 *>(a.v_cache + at) = vr[j];
    }
}

}  // namespace mb

using namespace mb;

extern "C" {

static int qknorm_rope_impl(bool f32, const void *q, int64_t q_s0, int64_t q_s1, const void *k, int64_t k_s0, int64_t k_s1,
                           const void *v, int64_t v_s0, int64_t v_s1, const void *q_weight, const void *k_weight,
                           const void *cos, int64_t cos_s0, const void *sin, int64_t sin_s0, int64_t tokens,
                           int32_t q_heads, int32_t kv_heads, int32_t head_dim, float eps, int32_t round_products,
                           void *out_q, void *k_cache, void *v_cache, int64_t cache_slot_stride,
                           const int64_t *slots, int64_t num_slots, int32_t *status, void *stream, char *error,
                           size_t error_size) {
    try {
        require(head_dim == QK_HEAD_DIM, "head_dim must be 128");
        require(tokens >= 0 && q_heads >= 1 && kv_heads >= 1 && q_heads + kv_heads <= 1024, "invalid head counts");
        require(std::isfinite(eps) && eps >= 0.0f, "invalid RMSNorm epsilon");
        require(q && k && q_weight && k_weight && cos && sin && out_q && k_cache, "missing prologue operand");
        require(!v == !v_cache, "v and v_cache come together");
        require(q_s1 >= QK_HEAD_DIM && k_s1 >= QK_HEAD_DIM && q_s0 >= q_s1 * q_heads && k_s0 >= k_s1 * kv_heads &&
                    cos_s0 >= QK_HEAD_DIM && sin_s0 >= QK_HEAD_DIM,
                "row strides smaller than the rows");
        require(cache_slot_stride >= int64_t(kv_heads) * QK_HEAD_DIM && num_slots >= 1, "invalid KV cache layout");
        require(slots || num_slots >= tokens, "without a slot table the cache needs a slot per token");
        const int64_t strides[] = {q_s0, q_s1, k_s0, k_s1, cos_s0, sin_s0, cache_slot_stride};
        for (int64_t st : strides) require(st % 4 == 0, "strides must keep 8-byte alignment");
        if (v) {
            require(v_s1 >= QK_HEAD_DIM && v_s0 >= v_s1 * kv_heads, "v row strides smaller than the rows");
            require(v_s0 % 4 == 0 && v_s1 % 4 == 0, "strides must keep 8-byte alignment");
            require(uintptr_t(v) % 8 == 0 && uintptr_t(v_cache) % 8 == 0, "prologue tensors must be 8-byte aligned");
        }
        const void *ptrs[] = {q, k, out_q, k_cache, cos, sin, q_weight, k_weight};
        for (const void *p : ptrs) require(uintptr_t(p) % 8 == 0, "prologue tensors must be 8-byte aligned");
        if (f32) require(uintptr_t(q) % 16 == 0 && uintptr_t(k) % 16 == 0 && uintptr_t(v) % 16 == 0,
                         "fp32 q / k / v rows must be 16-byte aligned");
        check_device(q, "q");
        check_device(out_q, "out_q");
        check_device(k_cache, "k_cache");
        if (tokens == 0) return 0;
        QkArgs a{};
        a.q = q;
        a.k = k;
        a.v = v;
        a.q_s0 = q_s0; a.q_s1 = q_s1; a.k_s0 = k_s0; a.k_s1 = k_s1; a.v_s0 = v_s0; a.v_s1 = v_s1;
        a.qw = static_cast<const __nv_bfloat16 *>(q_weight);
        a.kw = static_cast<const __nv_bfloat16 *>(k_weight);
        a.cos = static_cast<const __nv_bfloat16 *>(cos);
        a.sin = static_cast<const __nv_bfloat16 *>(sin);
        a.cs0 = cos_s0; a.ss0 = sin_s0;
        a.tokens = tokens; a.qh = q_heads; a.kh = kv_heads;
        a.eps = eps;
        a.round_products = round_products ? 1 : 0;
        a.out_q = static_cast<__nv_bfloat16 *>(out_q);
        a.k_cache = static_cast<__nv_bfloat16 *>(k_cache);
        a.v_cache = static_cast<__nv_bfloat16 *>(v_cache);
        a.cache_s0 = cache_slot_stride;
        a.slots = slots;
        a.num_slots = num_slots;
        a.status = status;
        const int64_t items = tokens * ceil_div(q_heads + kv_heads, QK_HEADS_PER_WARP);
        auto kernel = f32 ? k_qknorm_rope<true> : k_qknorm_rope<false>;
        kernel<<<unsigned(ceil_div(items, QK_WARPS)), QK_WARPS * 32, 0, as_stream(stream)>>>(a);
        cuda_check(cudaGetLastError(), "QK norm / RoPE launch");
        return 0;
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return -1;
    }
}

int mstar_b200_qknorm_rope(const void *q, int64_t q_s0, int64_t q_s1, const void *k, int64_t k_s0, int64_t k_s1,
                           const void *v, int64_t v_s0, int64_t v_s1, const void *q_weight, const void *k_weight,
                           const void *cos, int64_t cos_s0, const void *sin, int64_t sin_s0, int64_t tokens,
                           int32_t q_heads, int32_t kv_heads, int32_t head_dim, float eps, int32_t round_products,
                           void *out_q, void *k_cache, void *v_cache, int64_t cache_slot_stride,
                           const int64_t *slots, int64_t num_slots, int32_t *status, void *stream, char *error,
                           size_t error_size) {
    return qknorm_rope_impl(false, q, q_s0, q_s1, k, k_s0, k_s1, v, v_s0, v_s1, q_weight, k_weight, cos, cos_s0, sin,
                            sin_s0, tokens, q_heads, kv_heads, head_dim, eps, round_products, out_q, k_cache, v_cache,
                            cache_slot_stride, slots, num_slots, status, stream, error, error_size);
}

int mstar_b200_qknorm_rope_f32(const void *q, int64_t q_s0, int64_t q_s1, const void *k, int64_t k_s0, int64_t k_s1,
                               const void *v, int64_t v_s0, int64_t v_s1, const void *q_weight, const void *k_weight,
                               const void *cos, int64_t cos_s0, const void *sin, int64_t sin_s0, int64_t tokens,
                               int32_t q_heads, int32_t kv_heads, int32_t head_dim, float eps, int32_t round_products,
                               void *out_q, void *k_cache, void *v_cache, int64_t cache_slot_stride,
                               const int64_t *slots, int64_t num_slots, int32_t *status, void *stream, char *error,
                               size_t error_size) {
    return qknorm_rope_impl(true, q, q_s0, q_s1, k, k_s0, k_s1, v, v_s0, v_s1, q_weight, k_weight, cos, cos_s0, sin,
                            sin_s0, tokens, q_heads, kv_heads, head_dim, eps, round_products, out_q, k_cache, v_cache,
                            cache_slot_stride, slots, num_slots, status, stream, error, error_size);
}

}  // extern "C"
