// The thinker layer's RMSNorm in one launch (transformers'
// Qwen3OmniMoeThinkerTextRMSNorm, the reference's layer norms at
// implementations/qwen3_omni/amd/thinker_model.py:106-148):
//   h = fp32(x); r = rsqrtf(mean(h^2) + eps); n = bf16(h * r); y = bf16(w * n)
// (the bf16 weight times the bf16 normalised row, rounded to bf16). One warp per
// row, eight bf16 per 16-byte load; the sum of squares is a per-lane fp32 sum then a
// warp butterfly, so the mean can differ from torch's reduction order in the last
// bit (and y, rarely, by one bf16 step). y is written as bf16 and, when asked, as
// fp32 (the same values; the Q8_0 linears' fp32 input, saving a conversion pass).
// Also the layer's bf16 residual add of an fp32 projection output in one pass.
#include <cmath>

#include <cuda_bf16.h>

#include "../../include/mstar_b200.h"
#include "common.cuh"

namespace mb {

constexpr int RMS_WARPS = 8;
constexpr int RMS_MAX_VEC = 16;   // 16-byte vectors per lane: rows up to 4096 wide

__global__ void __launch_bounds__(RMS_WARPS * 32)
    k_rms_norm(const __nv_bfloat16 *__restrict__ x, int64_t ldx, int64_t rows, int64_t width,
               const __nv_bfloat16 *__restrict__ w, float eps, __nv_bfloat16 *__restrict__ y, int64_t ldy,
               float *__restrict__ y32, int64_t ldy32) {
    const int lane = threadIdx.x & 31;
    const int64_t row = int64_t(blockIdx.x) * RMS_WARPS + (threadIdx.x >> 5);
    if (row >= rows) return;
    const int64_t vecs = width / 8;
    uint4 v[RMS_MAX_VEC];
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < RMS_MAX_VEC; ++i) {
        const int64_t c = int64_t(i) * 32 + lane;
        v[i] = c < vecs ? *reinterpret_cast<const uint4 *>(x + row * ldx + 8 * c) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int i = 0; i < RMS_MAX_VEC; ++i) {
        const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&v[i]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 f = __bfloat1622float2(h[j]);
            ss = __fadd_rn(ss, __fmul_rn(f.x, f.x));
            ss = __fadd_rn(ss, __fmul_rn(f.y, f.y));
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
    const float r = rsqrtf(__fadd_rn(__fdiv_rn(ss, float(width)), eps));
#pragma unroll
    for (int i = 0; i < RMS_MAX_VEC; ++i) {
        const int64_t c = int64_t(i) * 32 + lane;
        if (c >= vecs) break;
        const uint4 wv = *reinterpret_cast<const uint4 *>(w + 8 * c);
        const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&v[i]);
        const __nv_bfloat162 *wh = reinterpret_cast<const __nv_bfloat162 *>(&wv);
        uint4 o;
        __nv_bfloat162 *oh = reinterpret_cast<__nv_bfloat162 *>(&o);
        float of[8];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 f = __bfloat1622float2(h[j]);
            const float2 wf = __bfloat1622float2(wh[j]);
            const float n0 = __bfloat162float(__float2bfloat16_rn(__fmul_rn(f.x, r)));
            const float n1 = __bfloat162float(__float2bfloat16_rn(__fmul_rn(f.y, r)));
            oh[j] = __floats2bfloat162_rn(__fmul_rn(wf.x, n0), __fmul_rn(wf.y, n1));
            const float2 back = __bfloat1622float2(oh[j]);
            of[2 * j] = back.x;
            of[2 * j + 1] = back.y;
        }
        *reinterpret_cast<uint4 *>(y + row * ldy + 8 * c) = o;
        if (y32) {
            float4 *dst = reinterpret_cast<float4 *>(y32 + row * ldy32 + 8 * c);
            dst[0] = make_float4(of[0], of[1], of[2], of[3]);
            dst[1] = make_float4(of[4], of[5], of[6], of[7]);
        }
    }
}

// out = bf16(fp32(x) + fp32(bf16(v))): torch's bf16 residual add of a projection computed
// in fp32 and returned in bf16 (x + o_proj(att) of the thinker layer), eight values per
// thread.
__global__ void __launch_bounds__(256)
    k_residual_add_bf16(const __nv_bfloat16 *__restrict__ x, const float *__restrict__ v, int64_t n,
                        __nv_bfloat16 *__restrict__ out) {
    const int64_t i = (int64_t(blockIdx.x) * 256 + threadIdx.x) * 8;
    if (i >= n) return;
    const uint4 xv = *reinterpret_cast<const uint4 *>(x + i);
    const float4 a = *reinterpret_cast<const float4 *>(v + i), b = *reinterpret_cast<const float4 *>(v + i + 4);
    const float vv[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    const __nv_bfloat162 *xh = reinterpret_cast<const __nv_bfloat162 *>(&xv);
    uint4 o;
    __nv_bfloat162 *oh = reinterpret_cast<__nv_bfloat162 *>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float2 xf = __bfloat1622float2(xh[j]);
        const float p0 = __bfloat162float(__float2bfloat16_rn(vv[2 * j]));
        const float p1 = __bfloat162float(__float2bfloat16_rn(vv[2 * j + 1]));
        oh[j] = __floats2bfloat162_rn(__fadd_rn(xf.x, p0), __fadd_rn(xf.y, p1));
    }
    *reinterpret_cast<uint4 *>(out + i) = o;
}

}  // namespace mb

using namespace mb;

extern "C" {

int mstar_b200_rms_norm(const void *x, int64_t x_stride, int64_t rows, int64_t width, const void *weight, float eps,
                        void *out, int64_t out_stride, float *out_f32, int64_t out_f32_stride, void *stream,
                        char *error, size_t error_size) {
    try {
        require(rows >= 1 && rows <= (int64_t(1) << 31), "invalid row count");
        require(width >= 8 && width % 8 == 0 && width <= int64_t(RMS_MAX_VEC) * 32 * 8,
                "RMSNorm rows are 8..4096 wide, a multiple of 8");
        require(x && weight && out, "missing RMSNorm operand");
        require(std::isfinite(eps) && eps >= 0.0f, "invalid epsilon");
        require(x_stride >= width && out_stride >= width && x_stride % 8 == 0 && out_stride % 8 == 0,
                "row strides must be multiples of 8 elements");
        require(uintptr_t(x) % 16 == 0 && uintptr_t(weight) % 16 == 0 && uintptr_t(out) % 16 == 0,
                "RMSNorm operands must be 16-byte aligned");
        if (out_f32)
            require(out_f32_stride >= width && out_f32_stride % 4 == 0 && uintptr_t(out_f32) % 16 == 0,
                    "fp32 output must be 16-byte aligned with a stride of whole 16-byte vectors");
        check_device(x, "RMSNorm input");
        check_device(out, "RMSNorm output");
        k_rms_norm<<<unsigned(ceil_div(rows, RMS_WARPS)), RMS_WARPS * 32, 0, as_stream(stream)>>>(
            static_cast<const __nv_bfloat16 *>(x), x_stride, rows, width, static_cast<const __nv_bfloat16 *>(weight),
            eps, static_cast<__nv_bfloat16 *>(out), out_stride, out_f32, out_f32_stride);
        cuda_check(cudaGetLastError(), "RMSNorm launch");
        return 0;
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return -1;
    }
}

int mstar_b200_residual_add_bf16(const void *x, const float *v, int64_t n, void *out, void *stream, char *error,
                                 size_t error_size) {
    try {
        require(n >= 0 && n % 8 == 0, "element count must be a multiple of 8");
        require(x && v && out, "missing residual operand");
        require(uintptr_t(x) % 16 == 0 && uintptr_t(v) % 16 == 0 && uintptr_t(out) % 16 == 0,
                "residual operands must be 16-byte aligned");
        if (n == 0) return 0;
        check_device(x, "residual input");
        check_device(v, "projection output");
        check_device(out, "residual output");
        k_residual_add_bf16<<<unsigned(ceil_div(n / 8, 256)), 256, 0, as_stream(stream)>>>(
            static_cast<const __nv_bfloat16 *>(x), v, n, static_cast<__nv_bfloat16 *>(out));
        cuda_check(cudaGetLastError(), "residual add launch");
        return 0;
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return -1;
    }
}

}  // extern "C"
