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
// The fused form (the default of the tensor-parallel encoder) has no pull and no
// barrier before the reduction: the row-parallel GEMM's epilogue stores each
// partial tile straight into its owner's receive slot over NVLink and raises the
// owner's arrival counter of those 32 rows (GEMM_OUT_PUSH in gemm.cu), so the
// transfer runs under the GEMM's MMAs; k_tp_reduce_recv waits per 32-row group for
// every rank's arrivals and sums the slots in rank order (bit-identical to the
// pulled reduction).
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

// The reduction of one owned row r (one warp): v = x[r] + (sum + bias) with the sum over
// slots s = 0 .. slots-1, in that order, of `part(s, c)` (float4 chunk c of slot s's
// partial row), x[r] updated in place; with ln_w, the new row LayerNorm-ed, Q8_0-quantized (MODE rounding) and stored
// as fp16(q * d) into every rank's staged operand (peer stores, or one multicast store).
template <int MODE, bool MC_STORE, class Part>
__device__ __forceinline__ void tp_reduce_row(const Part &part, int slots, int lane, int64_t r, int64_t n,
                                              const float *__restrict__ bias, float *__restrict__ x,
                                              const float *__restrict__ ln_w, const float *__restrict__ ln_b, float eps,
                                              __half *const *staged, __half *mc_staged, int world, int64_t grow,
                                              int *status) {
    const int64_t chunks = n / 4;
    float4 v[TP_MAX_CHUNKS];
    float sum = 0.0f;
    // passes over the row's chunks, each with all of its loads in flight at once: slot by
    // slot (rank order) the partial sums, then bias and residual, then the stores of the
    // new row (a store to x or a per-chunk loop over the slots between the loads would make
    // the row a chain of memory round trips)
#pragma unroll
    for (int i = 0; i < TP_MAX_CHUNKS; ++i) {
        const int64_t c = int64_t(i) * 32 + lane;
        v[i] = c < chunks ? part(0, c) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
    for (int s = 1; s < slots; ++s) {
#pragma unroll
        for (int i = 0; i < TP_MAX_CHUNKS; ++i) {
            const int64_t c = int64_t(i) * 32 + lane;
            if (c < chunks) {
                const float4 p = part(s, c);
                v[i] = make_float4(__fadd_rn(v[i].x, p.x), __fadd_rn(v[i].y, p.y), __fadd_rn(v[i].z, p.z),
                                   __fadd_rn(v[i].w, p.w));
            }
        }
    }
#pragma unroll
    for (int i = 0; i < TP_MAX_CHUNKS; ++i) {
        const int64_t c = int64_t(i) * 32 + lane;
        if (c < chunks) {
            const float4 b = *reinterpret_cast<const float4 *>(bias + 4 * c);
            const float4 res = *reinterpret_cast<const float4 *>(x + r * n + 4 * c);
            v[i] = make_float4(__fadd_rn(res.x, __fadd_rn(v[i].x, b.x)), __fadd_rn(res.y, __fadd_rn(v[i].y, b.y)),
                               __fadd_rn(res.z, __fadd_rn(v[i].z, b.z)), __fadd_rn(res.w, __fadd_rn(v[i].w, b.w)));
        }
    }
#pragma unroll
    for (int i = 0; i < TP_MAX_CHUNKS; ++i) {
        const int64_t c = int64_t(i) * 32 + lane;
        if (c < chunks) {
            *reinterpret_cast<float4 *>(x + r * n + 4 * c) = v[i];
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
            if (MC_STORE) mc_store8(mc_staged + grow * n + 4 * c, u);
            else
                for (int p = 0; p < world; ++p) *reinterpret_cast<uint2 *>(staged[p] + grow * n + 4 * c) = u;
        }
    }
}

// One warp per owned row, partials pulled after a barrier. parts[p]: rank p's [M][n] fp32
// partial product, or (MC) mc_part: the partial buffer's multicast address; x: [owned][n]
// fp32 residual rows of this owner (updated in place); staged[p]: rank p's staged
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
    const int64_t grow = row0 + r;
    auto part = [&](int s, int64_t c) {
        if (MC) return mc_ld_reduce_add(mc_part + grow * n + 4 * c);   // the switch sums the ranks
        return *reinterpret_cast<const float4 *>(parts[s] + grow * n + 4 * c);
    };
    tp_reduce_row<MODE, MC>(part, MC ? 1 : world, lane, r, n, bias, x, ln_w, ln_b, eps, staged, mc_staged, world, grow,
                            status);
}

// The owner's side of pushed partials: one warp per owned row, TP_WARPS rows per CTA.
// recv: this owner's receive buffer [world][own_rows][n] (slot p written by rank p's GEMM
// epilogue); counters[g]: arrivals for rows 32g .. 32g + 31, counters[own_rows / 32]: the
// kernel's own count of finished CTAs. One thread per CTA waits (bounded: status bit value
// 16) until its rows' group holds all `expected` arrivals; the warps then sum the slots in
// rank order (the same order as the pulled reduction) and finish the rows. The last CTA
// to finish clears the arrival counters and its own count for the next pushed GEMM, which
// no rank starts before the barrier that follows this reduction.
template <int MODE, bool MC_STORE>
__global__ void __launch_bounds__(TP_WARPS * 32)
    k_tp_reduce_recv(const float *__restrict__ recv, int *counters, int expected, long long limit, int world,
                     int64_t owned, int64_t own_rows, int64_t n, const float *__restrict__ bias, float *__restrict__ x,
                     const float *__restrict__ ln_w, const float *__restrict__ ln_b, float eps, __half *const *staged,
                     __half *mc_staged, int64_t row0, int *status) {
    __shared__ int arrived;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t first = int64_t(blockIdx.x) * TP_WARPS;   // a CTA's rows lie in one 32-row group
    if (threadIdx.x == 0) {
        long long polls = 0;
        int v = 0;
        for (;;) {
            asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(counters + first / 32) : "memory");
            if (v >= expected) break;
            if (++polls > limit) {
                atomicOr(status, 16);
                break;
            }
            __nanosleep(100);
        }
        arrived = v >= expected;
    }
    __syncthreads();
    const int64_t r = first + warp;
    if (arrived && r < owned) {
        auto part = [&](int s, int64_t c) {
            return *reinterpret_cast<const float4 *>(recv + (int64_t(s) * own_rows + r) * n + 4 * c);
        };
        tp_reduce_row<MODE, MC_STORE>(part, world, lane, r, n, bias, x, ln_w, ln_b, eps, staged, mc_staged, world,
                                      row0 + r, status);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int *done = counters + own_rows / 32;
        __threadfence();
        if (atomicAdd(done, 1) == int(gridDim.x) - 1) {   // every CTA has consumed its group
            for (int64_t g = 0; g < (owned + 31) / 32; ++g) counters[g] = 0;
            *done = 0;
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

static void launch_tp_reduce_recv(const float *recv, int *counters, int expected, long long limit, int world,
                                  int64_t owned, int64_t own_rows, int64_t width, const float *bias, float *x,
                                  const float *ln_w, const float *ln_b, float eps, __half *const *staged,
                                  __half *mc_staged, int64_t row0, int rounding, int *status, cudaStream_t s) {
    static_assert(32 % TP_WARPS == 0, "a CTA's rows must lie in one 32-row group");
    const unsigned grid = unsigned(ceil_div(owned, TP_WARPS));
    auto k = mc_staged ? (rounding == 0   ? k_tp_reduce_recv<0, true>
                          : rounding == 2 ? k_tp_reduce_recv<2, true>
                                          : k_tp_reduce_recv<1, true>)
                       : (rounding == 0   ? k_tp_reduce_recv<0, false>
                          : rounding == 2 ? k_tp_reduce_recv<2, false>
                                          : k_tp_reduce_recv<1, false>);
    k<<<grid, TP_WARPS * 32, 0, s>>>(recv, counters, expected, limit, world, owned, own_rows, width, bias, x, ln_w,
                                     ln_b, eps, staged, mc_staged, row0, status);
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

int mstar_b200_tp_reduce_recv(const float *recv, int32_t *counters, int32_t world, int64_t owned, int64_t owner_rows,
                              int64_t width, const float *bias, float *x, const float *ln_weight,
                              const float *ln_bias, float ln_eps, void *const *staged_ptrs, void *mc_staged,
                              int64_t row0, int32_t rounding, int32_t *status, void *stream, char *error,
                              size_t error_size) {
    try {
        require(world >= 1 && world <= TP_MAX_WORLD, "invalid world size");
        require(owner_rows > 0 && owner_rows % 32 == 0, "owner rows must be a positive multiple of 32");
        require(owned >= 0 && owned <= owner_rows && row0 >= 0, "invalid owned rows");
        require(width >= 32 && width % 32 == 0 && width <= 4 * 32 * TP_MAX_CHUNKS, "width must be 32..1536, /32");
        require(recv && counters && bias && x && status, "missing reduction operand");
        require(uintptr_t(recv) % 16 == 0 && uintptr_t(x) % 16 == 0 && uintptr_t(bias) % 16 == 0,
                "reduction operands must be 16-byte aligned");
        require(rounding >= 0 && rounding <= 2, "unknown Q8_0 activation rounding");
        if (ln_weight) {
            require(ln_bias && (staged_ptrs || mc_staged) && std::isfinite(ln_eps) && ln_eps >= 0.0f,
                    "invalid LayerNorm staging");
            require(uintptr_t(ln_weight) % 16 == 0 && uintptr_t(ln_bias) % 16 == 0, "LayerNorm vectors unaligned");
            require(uintptr_t(mc_staged) % 16 == 0, "multicast staged buffer must be 16-byte aligned");
        }
        check_device(recv, "receive buffer");
        check_device(x, "owned rows");
        if (owned == 0) return 0;
        const long long limit = wait_limits().tp_barrier > 0 ? wait_limits().tp_barrier : TP_SPIN_LIMIT;
        launch_tp_reduce_recv(recv, counters, world * push_arrivals_per_rank(width), limit, world, owned, owner_rows,
                              width, bias, x, ln_weight, ln_bias, ln_eps,
                              reinterpret_cast<__half *const *>(staged_ptrs), static_cast<__half *>(mc_staged), row0,
                              rounding, status, as_stream(stream));
        cuda_check(cudaGetLastError(), "reduction launch");
        return 0;
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return -1;
    }
}

}  // extern "C"
