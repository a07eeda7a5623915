// Tensor parallelism across GPUs of one node: the row-parallel reduction of the
// Whisper encoder's out_proj / fc2 (the reference's TP layout: fc1 rows and fc2
// columns sharded, partial products summed, bias added once,
// accelerations/whisper/cpu_tp2/decoder_all_reduce.py:64-90), done with plain
// peer loads and stores over NVLink into symmetric device buffers (no NCCL, no
// multicast):
//   * every rank's row-parallel GEMM writes its fp32 partial product [M][N]
//     into its own peer-visible buffer (local HBM, the GEMM's normal epilogue);
//   * k_tp_barrier: every rank raises a generation counter in every peer's
//     flag array and waits (bounded) for all peers' counters;
//   * k_tp_reduce: each owner of a row range pulls the W partial rows with
//     coalesced peer loads, sums them in rank order, adds the bias, then the
//     residual (x = x + (sum + b), encoder_bias_residual order), keeps its rows,
//     and optionally LayerNorm-stages the new rows (Q8_0 -> fp16(q * d)) with
//     coalesced peer stores into every rank's staged operand, which is the
//     all-gather the next column-parallel GEMM needs.
// Remote reads and writes are whole 512-byte warp segments; a row-per-thread
// push of the partials from the GEMM epilogue instead splits every row into
// 16-byte remote stores.
// Where the buffers are also bound to an NVLink multicast object (NVSwitch
// NVLS), k_tp_reduce<MODE, true> reads each owned row's sum over all ranks with
// one multimem.ld_reduce per 16 bytes (the switch adds the W partials, so an
// owner receives M/W rows instead of (W-1) M/W rows of partials) and writes the
// staged rows to every rank with one multimem.st (the switch replicates them).
// The switch's fp32 addition order is its own, so the sum may differ from the
// rank-order sum in the last bit.
#include <cmath>

#include "../../include/mstar_b200.h"
#include "gemm.cuh"

namespace mb {

constexpr int TP_WARPS = 8;
constexpr int TP_MAX_CHUNKS = 12;  // float4 chunks per lane: rows up to 1536 wide
constexpr int TP_MAX_WORLD = 8;
constexpr long long TP_SPIN_LIMIT = 1ll << 26;  // polls (with 100 ns sleeps) before a barrier gives up

__global__ void k_tp_barrier(int *const *flags, int *mine, int rank, int world, int *counter, int *status,
                             long long limit) {
    const int p = threadIdx.x;
    __shared__ int gen;
    if (p == 0) {  // this rank's barrier count (device-resident, so captured graphs replay correctly)
        gen = *counter + 1;
        *counter = gen;
    }
    __syncthreads();
    const int generation = gen;
    __threadfence_system();  // everything this stream wrote before the barrier is visible first
    if (p < world) {
        int *dst = flags[p] + rank;
        asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(dst), "r"(generation) : "memory");
    }
    __syncthreads();
    if (p < world) {
        long long n = 0;
        int v = 0;
        for (;;) {
            asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(mine + p) : "memory");
            if (v - generation >= 0) break;
            if (++n > limit) {
                atomicOr(status, 16);
                break;
            }
            __nanosleep(100);
        }
    }
}

__device__ __forceinline__ float4 mc_ld_reduce_add(const float *p) {
    float4 v;
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p)
                 : "memory");
    return v;
}
__device__ __forceinline__ void mc_store8(void *p, uint2 u) {
    asm volatile("multimem.st.relaxed.sys.global.v2.f16x2 [%0], {%1, %2};" ::"l"(p), "r"(u.x), "r"(u.y) : "memory");
}

// One warp per owned row. parts[p]: rank p's [M][n] fp32 partial product, or
// (MC) mc_part: the partial buffer's multicast address; x: [owned][n] fp32
// residual rows of this owner (updated in place); staged[p]: rank p's staged
// operand, or (MC) mc_staged: its multicast address.
template <int MODE, bool MC>
__global__ void __launch_bounds__(TP_WARPS * 32)
    k_tp_reduce(const float *const *parts, const float *mc_part, int world, int64_t owned, int64_t n,
                const float *__restrict__ bias, float *__restrict__ x, const float *__restrict__ ln_w,
                const float *__restrict__ ln_b, float eps, __half *const *staged, __half *mc_staged, int64_t row0,
                int *status) {
    const int lane = threadIdx.x & 31;
    const int64_t r = int64_t(blockIdx.x) * TP_WARPS + (threadIdx.x >> 5);
    if (r >= owned) return;
    const int64_t chunks = n / 4;
    float4 v[TP_MAX_CHUNKS];
    float sum = 0.0f;
#pragma unroll
    for (int i = 0; i < TP_MAX_CHUNKS; ++i) {
        const int64_t c = int64_t(i) * 32 + lane;
        v[i] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (c < chunks) {
            float4 acc;
            if (MC) {
                acc = mc_ld_reduce_add(mc_part + (row0 + r) * n + 4 * c);
            } else {
                acc = *reinterpret_cast<const float4 *>(parts[0] + (row0 + r) * n + 4 * c);
                for (int s = 1; s < world; ++s) {
                    const float4 p = *reinterpret_cast<const float4 *>(parts[s] + (row0 + r) * n + 4 * c);
                    acc.x = __fadd_rn(acc.x, p.x);
                    acc.y = __fadd_rn(acc.y, p.y);
                    acc.z = __fadd_rn(acc.z, p.z);
                    acc.w = __fadd_rn(acc.w, p.w);
                }
            }
            const float4 b = *reinterpret_cast<const float4 *>(bias + 4 * c);
            float4 *xr = reinterpret_cast<float4 *>(x + r * n + 4 * c);
            const float4 res = *xr;
            v[i] = make_float4(__fadd_rn(res.x, __fadd_rn(acc.x, b.x)), __fadd_rn(res.y, __fadd_rn(acc.y, b.y)),
                               __fadd_rn(res.z, __fadd_rn(acc.z, b.z)), __fadd_rn(res.w, __fadd_rn(acc.w, b.w)));
            *xr = v[i];
            sum = __fadd_rn(sum, __fadd_rn(__fadd_rn(v[i].x, v[i].y), __fadd_rn(v[i].z, v[i].w)));
        }
    }
    if (!ln_w) return;
    // LayerNorm of the new row (ggml_compute_forward_norm_f32 + mul + add), Q8_0, fp16(q * d)
#pragma unroll
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float mean = sum / float(n);
    float var = 0.0f;
#pragma unroll
    for (int i = 0; i < TP_MAX_CHUNKS; ++i) {
        const int64_t c = int64_t(i) * 32 + lane;
        if (c < chunks) {
            const float a = __fsub_rn(v[i].x, mean), b = __fsub_rn(v[i].y, mean);
            const float e = __fsub_rn(v[i].z, mean), f = __fsub_rn(v[i].w, mean);
            var = __fadd_rn(var, __fadd_rn(__fadd_rn(__fmul_rn(a, a), __fmul_rn(b, b)),
                                           __fadd_rn(__fmul_rn(e, e), __fmul_rn(f, f))));
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) var += __shfl_xor_sync(0xffffffffu, var, o);
    const float rstd = 1.0f / sqrtf(var / float(n) + eps);
#pragma unroll
    for (int i = 0; i < TP_MAX_CHUNKS; ++i) {
        if (int64_t(i) * 32 >= chunks) break;  // warp-uniform
        const int64_t c = int64_t(i) * 32 + lane;
        float4 y = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (c < chunks) {
            const float4 w = *reinterpret_cast<const float4 *>(ln_w + 4 * c);
            const float4 b = *reinterpret_cast<const float4 *>(ln_b + 4 * c);
            auto nf = [&](float t, float ww, float bb) {
                return __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(t, mean), rstd), ww), bb);
            };
            y = make_float4(nf(v[i].x, w.x, b.x), nf(v[i].y, w.y, b.y), nf(v[i].z, w.z, b.z), nf(v[i].w, w.w, b.w));
        }
        if (!(isfinite(y.x) && isfinite(y.y) && isfinite(y.z) && isfinite(y.w))) atomicOr(status, 1);
        float amax = fmaxf(fmaxf(fabsf(y.x), fabsf(y.y)), fmaxf(fabsf(y.z), fabsf(y.w)));
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const float d = __fdiv_rn(amax, 127.0f);
        float id;
        if (MODE == 2) id = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
        else id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        const float dh = __half2float(__float2half_rn(d));
        auto q = [&](float t) {
            const float sv = __fmul_rn(t, id);
            return __fmul_rn(float(MODE == 0 ? int(roundf(sv)) : __float2int_rn(sv)), dh);
        };
        if (c < chunks) {
            uint2 u;
            u.x = half2_bits(__floats2half2_rn(q(y.x), q(y.y)));
            u.y = half2_bits(__floats2half2_rn(q(y.z), q(y.w)));
            if (MC) mc_store8(mc_staged + (row0 + r) * n + 4 * c, u);
            else
                for (int p = 0; p < world; ++p)
                    *reinterpret_cast<uint2 *>(staged[p] + (row0 + r) * n + 4 * c) = u;
        }
    }
}

template <bool MC>
static void launch_tp_reduce(const float *const *parts, const float *mc_part, int world, int64_t owned, int64_t width,
                             const float *bias, float *x, const float *ln_w, const float *ln_b, float eps,
                             __half *const *staged, __half *mc_staged, int64_t row0, int rounding, int *status,
                             cudaStream_t s) {
    const unsigned grid = unsigned(ceil_div(owned, TP_WARPS));
    if (rounding == 0)
        k_tp_reduce<0, MC><<<grid, TP_WARPS * 32, 0, s>>>(parts, mc_part, world, owned, width, bias, x, ln_w, ln_b,
                                                         eps, staged, mc_staged, row0, status);
    else if (rounding == 2)
        k_tp_reduce<2, MC><<<grid, TP_WARPS * 32, 0, s>>>(parts, mc_part, world, owned, width, bias, x, ln_w, ln_b,
                                                         eps, staged, mc_staged, row0, status);
    else
        k_tp_reduce<1, MC><<<grid, TP_WARPS * 32, 0, s>>>(parts, mc_part, world, owned, width, bias, x, ln_w, ln_b,
                                                         eps, staged, mc_staged, row0, status);
}

}  // namespace mb

using namespace mb;

extern "C" {

int mstar_b200_tp_barrier(int32_t *const *flag_ptrs, int32_t *my_flags, int32_t rank, int32_t world,
                          int32_t *counter, int32_t *status, void *stream, char *error, size_t error_size) {
    try {
        require(world >= 1 && world <= TP_MAX_WORLD && rank >= 0 && rank < world, "invalid rank / world");
        require(flag_ptrs && my_flags && counter && status, "missing barrier operand");
        const long long limit = wait_limits().tp_barrier > 0 ? wait_limits().tp_barrier : TP_SPIN_LIMIT;
        k_tp_barrier<<<1, 32, 0, as_stream(stream)>>>(flag_ptrs, my_flags, rank, world, counter, status, limit);
        cuda_check(cudaGetLastError(), "barrier launch");
        return 0;
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return -1;
    }
}

int mstar_b200_tp_reduce(const float *const *part_ptrs, int32_t world, int64_t owned, int64_t width,
                         const float *bias, float *x, const float *ln_weight, const float *ln_bias, float ln_eps,
                         void *const *staged_ptrs, int64_t row0, int32_t rounding, int32_t *status, void *stream,
                         char *error, size_t error_size) {
    try {
        require(world >= 1 && world <= TP_MAX_WORLD, "invalid world size");
        require(owned >= 0 && row0 >= 0, "invalid owned rows");
        require(width >= 4 && width % 32 == 0 && width <= 4 * 32 * TP_MAX_CHUNKS, "width must be 32..1536, /32");
        require(part_ptrs && bias && x && status, "missing reduction operand");
        require(uintptr_t(x) % 16 == 0 && uintptr_t(bias) % 16 == 0, "reduction operands must be 16-byte aligned");
        require(rounding >= 0 && rounding <= 2, "unknown Q8_0 activation rounding");
        if (ln_weight) {
            require(ln_bias && staged_ptrs && std::isfinite(ln_eps) && ln_eps >= 0.0f, "invalid LayerNorm staging");
            require(uintptr_t(ln_weight) % 16 == 0 && uintptr_t(ln_bias) % 16 == 0, "LayerNorm vectors unaligned");
        }
        check_device(x, "owned rows");
        if (owned == 0) return 0;
        launch_tp_reduce<false>(part_ptrs, nullptr, world, owned, width, bias, x, ln_weight, ln_bias, ln_eps,
                                reinterpret_cast<__half *const *>(staged_ptrs), nullptr, row0, rounding, status,
                                as_stream(stream));
        cuda_check(cudaGetLastError(), "reduction launch");
        return 0;
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return -1;
    }
}

int mstar_b200_tp_reduce_multicast(const float *mc_part, int32_t world, int64_t owned, int64_t width,
                                   const float *bias, float *x, const float *ln_weight, const float *ln_bias,
                                   float ln_eps, void *mc_staged, int64_t row0, int32_t rounding, int32_t *status,
                                   void *stream, char *error, size_t error_size) {
    try {
        require(world >= 1 && world <= TP_MAX_WORLD, "invalid world size");
        require(owned >= 0 && row0 >= 0, "invalid owned rows");
        require(width >= 4 && width % 32 == 0 && width <= 4 * 32 * TP_MAX_CHUNKS, "width must be 32..1536, /32");
        require(mc_part && bias && x && status, "missing reduction operand");
        require(uintptr_t(mc_part) % 16 == 0, "multicast partial buffer must be 16-byte aligned");
        require(uintptr_t(x) % 16 == 0 && uintptr_t(bias) % 16 == 0, "reduction operands must be 16-byte aligned");
        require(rounding >= 0 && rounding <= 2, "unknown Q8_0 activation rounding");
        if (ln_weight) {
            require(ln_bias && mc_staged && std::isfinite(ln_eps) && ln_eps >= 0.0f, "invalid LayerNorm staging");
            require(uintptr_t(mc_staged) % 16 == 0, "multicast staged buffer must be 16-byte aligned");
            require(uintptr_t(ln_weight) % 16 == 0 && uintptr_t(ln_bias) % 16 == 0, "LayerNorm vectors unaligned");
        }
        check_device(x, "owned rows");
        if (owned == 0) return 0;
        launch_tp_reduce<true>(nullptr, mc_part, world, owned, width, bias, x, ln_weight, ln_bias, ln_eps, nullptr,
                               static_cast<__half *>(mc_staged), row0, rounding, status, as_stream(stream));
        cuda_check(cudaGetLastError(), "reduction launch");
        return 0;
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return -1;
    }
}

}  // extern "C"
