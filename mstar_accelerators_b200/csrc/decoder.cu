// Non-linear pieces of the Whisper decoder step that sit between the
// block-quantized linears: token + position embedding (ggml_get_rows + add,
// backends/cpu_ggml/decoder.cpp:513-518) and attention over the fp16 KV planes
// (ggml_flash_attn_ext with scale 1/sqrt(head_dim), decoder.cpp:504-511), with
// the new self-attention K/V rows appended first (ggml_set_rows,
// decoder.cpp:566-567). Attention math is fp32 (scores, online softmax,
// weighted sum); K/V are stored fp16 like the reference's F16 plain storage.
#include "../../include/mstar_b200.h"
#include "quant.cuh"

namespace mb {

// x[r] = tok[ids[r]] * scale + pos[positions[r]]  (rows r < n, width d)
__global__ void k_embed(const float *__restrict__ tok, const float *__restrict__ pos, const int64_t *__restrict__ ids,
                        const int64_t *__restrict__ positions, float scale, float *__restrict__ x, int64_t n,
                        int64_t d, int64_t vocab, int64_t npos, int *__restrict__ status) {
    const int64_t r = blockIdx.x;
    if (r >= n) return;
    const int64_t id = ids[r], p = positions[r];
    if (id < 0 || id >= vocab || p < 0 || p >= npos) {
        if (threadIdx.x == 0) atomicOr(status, 4);
        for (int64_t i = threadIdx.x; i < d; i += blockDim.x) x[r * d + i] = 0.0f;
        return;
    }
    for (int64_t i = threadIdx.x; i < d; i += blockDim.x) {
        float v = tok[id * d + i];
        if (scale != 1.0f) v = __fmul_rn(v, scale);
        x[r * d + i] = __fadd_rn(v, pos[p * d + i]);
    }
}

constexpr int ATT_THREADS = 128;
constexpr int ATT_WARPS = ATT_THREADS / 32;
constexpr int HEAD_DIM = 64;
constexpr int MAX_Q = 4;

// One CTA per (sequence b, head h). Queries q_i (i < NQ) of sequence b sit at
// positions begin_b + i; the CTA first appends their K/V rows (when given) to
// the sequence's fp16 planes, then attends query i over keys [0, len_i) with
// len_i = causal ? begin_b + i + 1 : kv_len_b.
//   q:    [b][NQ][q_stride] fp32, head h at column h*64
//   k/v new rows (optional): same layout as q with their own column offset
//   planes: kc/vc [seq][capacity][heads*64] fp16; seq index = shared ? 0 : b
//   out:  [b][NQ][out_stride] fp32, head h at column h*64
// Scores: one thread per key (64-wide dot from one 128-byte K row). Softmax:
// block reductions. Weighted sum: warp w owns a contiguous key range, lane l
// owns dims 2l, 2l+1 (one coalesced half2 per key row), then the four warps'
// partial sums are added in shared memory.
template <int NQ>
__global__ void __launch_bounds__(ATT_THREADS) k_attend(
    const float *__restrict__ q, int64_t q_stride, const float *__restrict__ knew, const float *__restrict__ vnew,
    int64_t kv_stride, __half *__restrict__ kc, __half *__restrict__ vc, int64_t capacity, int heads,
    const int64_t *__restrict__ begin, const int64_t *__restrict__ kv_len, int causal, int shared,
    float *__restrict__ out, int64_t out_stride, float scale, int *__restrict__ status) {
    extern __shared__ float scores[];  // [NQ][capacity]
    __shared__ float qs[NQ][HEAD_DIM];
    __shared__ float red[NQ][ATT_WARPS];
    __shared__ float2 part[ATT_WARPS][NQ][32];
    const int b = blockIdx.x / heads, h = blockIdx.x % heads;
    const int width = heads * HEAD_DIM;
    const int64_t seq = shared ? 0 : b;
    const int64_t b0 = begin ? begin[b] : 0;
    __half *kp = kc + seq * capacity * width + h * HEAD_DIM;
    __half *vp = vc + seq * capacity * width + h * HEAD_DIM;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    if (knew) {  // append the new rows at positions b0 .. b0+NQ-1
        if (b0 < 0 || b0 + NQ > capacity) {
            if (tid == 0) atomicOr(status, 8);
            return;
        }
        for (int i = tid; i < NQ * HEAD_DIM; i += ATT_THREADS) {
            const int qi = i / HEAD_DIM, dd = i % HEAD_DIM;
            const int64_t src = (int64_t(b) * NQ + qi) * kv_stride + h * HEAD_DIM + dd;
            kp[(b0 + qi) * width + dd] = __float2half_rn(knew[src]);
            vp[(b0 + qi) * width + dd] = __float2half_rn(vnew[src]);
        }
    }
    for (int i = tid; i < NQ * HEAD_DIM; i += ATT_THREADS) {
        const int qi = i / HEAD_DIM, dd = i % HEAD_DIM;
        qs[qi][dd] = q[(int64_t(b) * NQ + qi) * q_stride + h * HEAD_DIM + dd];
    }
    __syncthreads();
    const int64_t total = causal ? b0 + NQ : kv_len[b];
    if (total < 1 || total > capacity) {
        if (tid == 0) atomicOr(status, 8);
        return;
    }
    for (int64_t j = tid; j < total; j += ATT_THREADS) {
        const uint4 *krow = reinterpret_cast<const uint4 *>(kp + j * width);
        float acc[NQ];
#pragma unroll
        for (int qi = 0; qi < NQ; ++qi) acc[qi] = 0.0f;
#pragma unroll
        for (int c = 0; c < HEAD_DIM / 8; ++c) {
            const uint4 raw = krow[c];
            const __half2 *h2 = reinterpret_cast<const __half2 *>(&raw);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float2 kv = __half22float2(h2[e]);
#pragma unroll
                for (int qi = 0; qi < NQ; ++qi)
                    acc[qi] = fmaf(qs[qi][8 * c + 2 * e + 1], kv.y, fmaf(qs[qi][8 * c + 2 * e], kv.x, acc[qi]));
            }
        }
#pragma unroll
        for (int qi = 0; qi < NQ; ++qi) {
            const int64_t len = causal ? b0 + qi + 1 : total;
            scores[qi * capacity + j] = j < len ? acc[qi] * scale : -INFINITY;
        }
    }
    __syncthreads();
    float mx[NQ], inv[NQ];
#pragma unroll
    for (int qi = 0; qi < NQ; ++qi) {
        float m = -INFINITY;
        for (int64_t j = tid; j < total; j += ATT_THREADS) m = fmaxf(m, scores[qi * capacity + j]);
#pragma unroll
        for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0) red[qi][warp] = m;
    }
    __syncthreads();
#pragma unroll
    for (int qi = 0; qi < NQ; ++qi) {
        float m = red[qi][0];
#pragma unroll
        for (int w = 1; w < ATT_WARPS; ++w) m = fmaxf(m, red[qi][w]);
        mx[qi] = m;
    }
    __syncthreads();
#pragma unroll
    for (int qi = 0; qi < NQ; ++qi) {
        float sum = 0.0f;
        for (int64_t j = tid; j < total; j += ATT_THREADS) {
            const float e = __expf(scores[qi * capacity + j] - mx[qi]);
            scores[qi * capacity + j] = e;
            sum += e;
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (lane == 0) red[qi][warp] = sum;
    }
    __syncthreads();
#pragma unroll
    for (int qi = 0; qi < NQ; ++qi) {
        float sum = 0.0f;
#pragma unroll
        for (int w = 0; w < ATT_WARPS; ++w) sum += red[qi][w];
        inv[qi] = 1.0f / sum;
    }
    // weighted sum over this warp's key range
    const int64_t per = (total + ATT_WARPS - 1) / ATT_WARPS;
    const int64_t j0 = warp * per, j1 = j0 + per < total ? j0 + per : total;
    float2 o[NQ];
#pragma unroll
    for (int qi = 0; qi < NQ; ++qi) o[qi] = make_float2(0.0f, 0.0f);
    const __half2 *vcol = reinterpret_cast<const __half2 *>(vp) + lane;
    int64_t j = j0;
    for (; j + 4 <= j1; j += 4) {
        float2 v4[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) v4[u] = __half22float2(vcol[(j + u) * (width / 2)]);
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int qi = 0; qi < NQ; ++qi) {
                const float p = scores[qi * capacity + j + u];
                o[qi].x = fmaf(p, v4[u].x, o[qi].x);
                o[qi].y = fmaf(p, v4[u].y, o[qi].y);
            }
    }
    for (; j < j1; ++j) {
        const float2 v = __half22float2(vcol[j * (width / 2)]);
#pragma unroll
        for (int qi = 0; qi < NQ; ++qi) {
            const float p = scores[qi * capacity + j];
            o[qi].x = fmaf(p, v.x, o[qi].x);
            o[qi].y = fmaf(p, v.y, o[qi].y);
        }
    }
#pragma unroll
    for (int qi = 0; qi < NQ; ++qi) part[warp][qi][lane] = o[qi];
    __syncthreads();
    for (int i = tid; i < NQ * 32; i += ATT_THREADS) {
        const int qi = i / 32, l = i % 32;
        float2 acc = part[0][qi][l];
#pragma unroll
        for (int w = 1; w < ATT_WARPS; ++w) {
            acc.x += part[w][qi][l].x;
            acc.y += part[w][qi][l].y;
        }
        float *dst = out + (int64_t(b) * NQ + qi) * out_stride + h * HEAD_DIM + 2 * l;
        dst[0] = acc.x * inv[qi];
        dst[1] = acc.y * inv[qi];
    }
}

// K/V planes from projected rows: kc/vc[seq][r][:] = fp16(src[r][k_off / v_off + :]) + bias
__global__ void k_fill_kv(const float *__restrict__ src, int64_t src_stride, int64_t k_off, int64_t v_off,
                          const float *__restrict__ kbias, const float *__restrict__ vbias, __half *__restrict__ kc,
                          __half *__restrict__ vc, int64_t rows, int64_t width) {
    const int64_t r = blockIdx.x;
    if (r >= rows) return;
    for (int64_t i = threadIdx.x; i < width; i += blockDim.x) {
        float kv = src[r * src_stride + k_off + i], vv = src[r * src_stride + v_off + i];
        if (kbias) kv = __fadd_rn(kv, kbias[i]);
        if (vbias) vv = __fadd_rn(vv, vbias[i]);
        kc[r * width + i] = __float2half_rn(kv);
        vc[r * width + i] = __float2half_rn(vv);
    }
}

}  // namespace mb

using namespace mb;

extern "C" {

int mstar_b200_embed(const float *token_table, int64_t vocab, const float *position_table, int64_t positions_count,
                     int64_t width, const int64_t *ids, const int64_t *positions, int64_t rows, float scale,
                     float *x, int32_t *status, void *stream, char *error, size_t error_size) {
    try {
        require(token_table && position_table && ids && positions && x && status, "missing embedding operand");
        require(rows > 0 && width > 0 && vocab > 0 && positions_count > 0, "invalid embedding shape");
        cudaStream_t s = as_stream(stream);
        k_embed<<<unsigned(rows), 128, 0, s>>>(token_table, position_table, ids, positions, scale, x, rows, width,
                                               vocab, positions_count, status);
        cuda_check(cudaGetLastError(), "embedding launch");
        return 0;
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return -1;
    }
}

int mstar_b200_attend(const float *q, int64_t q_stride, const float *k_new, const float *v_new, int64_t kv_stride,
                      void *k_plane, void *v_plane, int64_t capacity, int32_t heads, int32_t head_dim,
                      int32_t batch, int32_t queries, const int64_t *begin, const int64_t *kv_length, int32_t causal,
                      int32_t shared, float *out, int64_t out_stride, float scale, int32_t *status, void *stream,
                      char *error, size_t error_size) {
    try {
        require(head_dim == HEAD_DIM, "attention head_dim must be 64");
        require(queries >= 1 && queries <= MAX_Q && batch >= 1 && heads >= 1, "invalid attention geometry");
        require(capacity >= 1 && capacity <= 4096, "attention capacity outside 1..4096");
        require(q && k_plane && v_plane && out && status, "missing attention operand");
        require(causal ? (begin != nullptr) : (kv_length != nullptr), "attention lengths missing");
        require(!k_new == !v_new, "new K and V rows must be given together");
        require(uintptr_t(k_plane) % 16 == 0 && uintptr_t(v_plane) % 16 == 0, "KV planes must be 16-byte aligned");
        const size_t smem = size_t(queries) * capacity * sizeof(float);
        require(smem <= 200 * 1024, "attention score tile exceeds shared memory");
        static bool configured = false;
        if (!configured) {
            cudaFuncSetAttribute(k_attend<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
            cudaFuncSetAttribute(k_attend<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
            cudaFuncSetAttribute(k_attend<3>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
            cudaFuncSetAttribute(k_attend<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
            configured = true;
        }
        cudaStream_t s = as_stream(stream);
        auto kernel = queries == 1 ? k_attend<1> : queries == 2 ? k_attend<2> : queries == 3 ? k_attend<3> : k_attend<4>;
        kernel<<<unsigned(batch * heads), ATT_THREADS, smem, s>>>(
            q, q_stride, k_new, v_new, kv_stride, static_cast<__half *>(k_plane), static_cast<__half *>(v_plane),
            capacity, heads, begin, kv_length, causal, shared, out, out_stride, scale, status);
        cuda_check(cudaGetLastError(), "attention launch");
        return 0;
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return -1;
    }
}

int mstar_b200_fill_kv(const float *projected, int64_t stride, int64_t k_offset, int64_t v_offset,
                       const float *k_bias, const float *v_bias, void *k_plane, void *v_plane, int64_t rows,
                       int64_t width, void *stream, char *error, size_t error_size) {
    try {
        require(projected && k_plane && v_plane && rows > 0 && width > 0, "invalid KV fill");
        cudaStream_t s = as_stream(stream);
        k_fill_kv<<<unsigned(rows), 128, 0, s>>>(projected, stride, k_offset, v_offset, k_bias, v_bias,
                                                 static_cast<__half *>(k_plane), static_cast<__half *>(v_plane), rows,
                                                 width);
        cuda_check(cudaGetLastError(), "KV fill launch");
        return 0;
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return -1;
    }
}

}  // extern "C"
