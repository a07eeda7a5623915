// Tensor / expert parallelism of the Qwen3-Omni thinker layer over the GPUs of
// one node, with plain peer loads and stores into symmetric device buffers (no
// NCCL, no multicast). Every rank holds the whole bf16 residual stream x
// [T][hidden] in its own peer-visible buffer; rows are split into owner ranges.
//
//   * attention is column-parallel by heads; o_proj is row-parallel (its K = the
//     rank's heads): every rank writes its fp32 partial product [T][hidden] into
//     its own peer-visible buffer. k_thinker_reduce: the owner of a row sums the
//     W partials in rank order, rounds the sum to bf16 (the projection's output
//     dtype), adds it to the residual row in fp32 and rounds to bf16 (torch's
//     bf16 add: x + o_proj(att)), and stores the new row into every rank's x.
//   * the MoE experts are expert-parallel: every rank routes all T tokens (the
//     router sees identical rows everywhere), runs its own experts' rows and
//     leaves them, with each (token, slot) pair's row index, in its peer-visible
//     buffers. k_thinker_combine: the owner of a token reads each slot's expert
//     row from the rank holding that expert, sums the slots in slot order in
//     fp32 (moe_sum_reduce, implementations/qwen3_omni/amd/thinker_moe.py:75-81),
//     rounds to bf16, adds the residual as above and stores the new row into every
//     rank's x. The slot order and the per-row expert GEMM outputs are those of
//     one GPU, so the combined rows are bit-identical to the single-GPU layer.
// One thread per 8 columns of a row: per rank a 32-byte (fp32) or 16-byte (bf16)
// load, 16-byte stores; a warp covers 256 columns of one row.
#include "../../include/mstar_b200.h"
#include "common.cuh"

#include <cuda_bf16.h>

namespace mb {

constexpr int TT_THREADS = 256;
constexpr int TT_MAX_WORLD = 8;
constexpr int TT_MAX_TOPK = 8;

__device__ __forceinline__ void bf16x8_to_f32(const uint4 &u, float *f) {
    const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 t = __bfloat1622float2(h[i]);
        f[2 * i] = t.x;
        f[2 * i + 1] = t.y;
    }
}

// new row = bf16(float(x) + float(bf16(v))), 8 columns, into every rank's x
__device__ __forceinline__ void residual_store(const float *v, __nv_bfloat16 *const *x_ptrs, int rank, int world,
                                               int64_t off) {
    const uint4 xr = *reinterpret_cast<const uint4 *>(x_ptrs[rank] + off);
    float xf[8];
    bf16x8_to_f32(xr, xf);
    uint4 o;
    __nv_bfloat162 *oh = reinterpret_cast<__nv_bfloat162 *>(&o);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float a = __fadd_rn(xf[2 * i], __bfloat162float(__float2bfloat16_rn(v[2 * i])));
        const float b = __fadd_rn(xf[2 * i + 1], __bfloat162float(__float2bfloat16_rn(v[2 * i + 1])));
        oh[i] = __floats2bfloat162_rn(a, b);
    }
#pragma unroll
    for (int p = 0; p < TT_MAX_WORLD; ++p)
        if (p < world) *reinterpret_cast<uint4 *>(x_ptrs[p] + off) = o;
}

__global__ void __launch_bounds__(TT_THREADS)
    k_thinker_reduce(const float *const *parts, __nv_bfloat16 *const *x_ptrs, int rank, int world, int64_t owned,
                     int64_t width, int64_t row0) {
    const int64_t groups = width / 8;
    const int64_t idx = int64_t(blockIdx.x) * TT_THREADS + threadIdx.x;
    if (idx >= owned * groups) return;
    const int64_t off = (row0 + idx / groups) * width + 8 * (idx % groups);
    float4 lo[TT_MAX_WORLD], hi[TT_MAX_WORLD];
#pragma unroll
    for (int p = 0; p < TT_MAX_WORLD; ++p)  // every rank's loads in flight before the sum
        if (p < world) {
            lo[p] = *reinterpret_cast<const float4 *>(parts[p] + off);
            hi[p] = *reinterpret_cast<const float4 *>(parts[p] + off + 4);
        }
    float v[8] = {lo[0].x, lo[0].y, lo[0].z, lo[0].w, hi[0].x, hi[0].y, hi[0].z, hi[0].w};
#pragma unroll
    for (int p = 1; p < TT_MAX_WORLD; ++p)
        if (p < world) {
            v[0] = __fadd_rn(v[0], lo[p].x);
            v[1] = __fadd_rn(v[1], lo[p].y);
            v[2] = __fadd_rn(v[2], lo[p].z);
            v[3] = __fadd_rn(v[3], lo[p].w);
            v[4] = __fadd_rn(v[4], hi[p].x);
            v[5] = __fadd_rn(v[5], hi[p].y);
            v[6] = __fadd_rn(v[6], hi[p].z);
            v[7] = __fadd_rn(v[7], hi[p].w);
        }
    residual_store(v, x_ptrs, rank, world, off);
}

__global__ void __launch_bounds__(TT_THREADS)
    k_thinker_combine(const __nv_bfloat16 *const *y_ptrs, const int32_t *const *inv_ptrs, int64_t y_rows,
                      const int32_t *__restrict__ ids, int experts_per_rank, int experts_total, int top_k,
                      __nv_bfloat16 *const *x_ptrs, int rank, int world, int64_t owned, int64_t hidden, int64_t row0,
                      int *status) {
    const int64_t groups = hidden / 8;
    const int64_t idx = int64_t(blockIdx.x) * TT_THREADS + threadIdx.x;
    if (idx >= owned * groups) return;
    const int64_t t = row0 + idx / groups, col = 8 * (idx % groups);
    int owner[TT_MAX_TOPK];
    int32_t row[TT_MAX_TOPK];
#pragma unroll
    for (int s = 0; s < TT_MAX_TOPK; ++s) {  // every slot's row index in flight first
        owner[s] = -1;
        row[s] = -1;
        if (s < top_k) {
            const int id = ids[t * top_k + s];
            if (id >= 0 && id < experts_total) {
                owner[s] = id / experts_per_rank;
                row[s] = inv_ptrs[owner[s]][t * top_k + s];
            }
        }
    }
    uint4 u[TT_MAX_TOPK];
#pragma unroll
    for (int s = 0; s < TT_MAX_TOPK; ++s) {
        u[s] = make_uint4(0u, 0u, 0u, 0u);
        if (s < top_k && owner[s] >= 0 && row[s] >= 0) {
            if (row[s] < y_rows) u[s] = *reinterpret_cast<const uint4 *>(y_ptrs[owner[s]] + int64_t(row[s]) * hidden + col);
            else if (col == 0) atomicOr(status, 64);
        }
    }
    float v[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int s = 0; s < TT_MAX_TOPK; ++s)
        if (s < top_k && owner[s] >= 0 && row[s] >= 0 && row[s] < y_rows) {
            float f[8];
            bf16x8_to_f32(u[s], f);
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = __fadd_rn(v[i], f[i]);
        }
    residual_store(v, x_ptrs, rank, world, t * hidden + col);
}

}  // namespace mb

using namespace mb;

extern "C" {

int mstar_b200_thinker_reduce(const float *const *part_ptrs, void *const *x_ptrs, int32_t rank, int32_t world,
                              int64_t owned, int64_t width, int64_t row0, void *stream, char *error,
                              size_t error_size) {
    try {
        require(world >= 1 && world <= TT_MAX_WORLD && rank >= 0 && rank < world, "invalid rank / world");
        require(owned >= 0 && row0 >= 0 && width >= 8 && width % 8 == 0, "invalid owned rows or width");
        require(part_ptrs && x_ptrs, "missing reduction operand");
        check_device(part_ptrs, "partial pointer array");
        check_device(x_ptrs, "x pointer array");
        if (owned == 0) return 0;
        const int64_t threads = owned * (width / 8);
        k_thinker_reduce<<<unsigned(ceil_div(threads, TT_THREADS)), TT_THREADS, 0, as_stream(stream)>>>(
            part_ptrs, reinterpret_cast<__nv_bfloat16 *const *>(x_ptrs), rank, world, owned, width, row0);
        cuda_check(cudaGetLastError(), "thinker reduction launch");
        return 0;
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return -1;
    }
}

int mstar_b200_thinker_combine(const void *const *y_ptrs, const int32_t *const *inv_ptrs, int64_t y_rows,
                               const int32_t *topk_ids, int32_t experts_per_rank, int32_t experts_total,
                               int32_t top_k, void *const *x_ptrs, int32_t rank, int32_t world, int64_t owned,
                               int64_t hidden, int64_t row0, int32_t *status, void *stream, char *error,
                               size_t error_size) {
    try {
        require(world >= 1 && world <= TT_MAX_WORLD && rank >= 0 && rank < world, "invalid rank / world");
        require(top_k >= 1 && top_k <= TT_MAX_TOPK, "top_k outside 1..8");
        require(experts_per_rank >= 1 && int64_t(experts_per_rank) * world == experts_total,
                "experts must split evenly over the ranks");
        require(owned >= 0 && row0 >= 0 && hidden >= 8 && hidden % 8 == 0 && y_rows >= 0,
                "invalid combine geometry");
        require(y_ptrs && inv_ptrs && topk_ids && x_ptrs && status, "missing combine operand");
        for (const void *p : {(const void *)y_ptrs, (const void *)inv_ptrs, (const void *)topk_ids,
                              (const void *)x_ptrs, (const void *)status})
            check_device(p, "combine operand");
        if (owned == 0) return 0;
        const int64_t threads = owned * (hidden / 8);
        k_thinker_combine<<<unsigned(ceil_div(threads, TT_THREADS)), TT_THREADS, 0, as_stream(stream)>>>(
            reinterpret_cast<const __nv_bfloat16 *const *>(y_ptrs), inv_ptrs, y_rows, topk_ids, experts_per_rank,
            experts_total, top_k, reinterpret_cast<__nv_bfloat16 *const *>(x_ptrs), rank, world, owned, hidden,
            row0, status);
        cuda_check(cudaGetLastError(), "thinker combine launch");
        return 0;
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return -1;
    }
}

}  // extern "C"
