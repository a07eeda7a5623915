// Exact Q8_0 GEMM on the int8 tensor pipe: every 32-element block's integer dot
// is one tcgen05.mma kind::i8 (M = 128, N = 128, K = 32, s8 x s8 -> s32) into a
// fresh TMEM accumulator, and the epilogue warps fold the blocks in ggml's
// generic order, out = sum over blocks b of float(sumi_b) * (d_w,b * d_x,b), one
// fp32 rounding per product and per addition (ggml-cpu/quants.c:451-480, the
// oracle's generic mul_mat) -- so the result is bit-identical to the decode
// GEMV's and to the oracle's for every row count. The rescale has to leave the
// tensor pipe (the block-scaled MMA kinds take power-of-two or e4m3 scales, not
// Q8_0's fp16 ones), so this path runs at the CUDA cores' rate for those
// operations; the fp16-staged GEMM (gemm.cu) is the throughput path.
//
// Operands: weights as int8 [N][K] (each block's 32 quants) with fp32 scales
// [nb][N_pad] (fp16 d widened; N_pad = N rounded up to 128, zero padded);
// activations as int8 [M][K] with fp32 scales [M][nb] (the Q8_0 quantization of
// each fp32 row with the selected rounding, its d rounded through fp16).
// Kernel: persistent, one CTA per SM over 128 x 128 tiles, 10 warps: warp 0 TMA
// producer (int8 boxes of 128 bytes = 4 blocks of K, 128B swizzle, 4-stage ring),
// warp 1 one thread issuing one MMA per block into a ring of four 128-column
// TMEM slots, warps 2-17 epilogue (four per TMEM lane quarter, 32 columns each):
// tcgen05.ld the block's sums, release the slot, fold in fp32. Every wait is
// bounded (status bit value 2).
#include <cuda.h>
#include <cudaTypedefs.h>

#include "../../include/mstar_b200.h"
#include "gemm.cuh"
#include "tcgen05.cuh"

namespace mb {

constexpr int EX_BM = 128, EX_BN = 128, EX_BKB = 128;  // K bytes per stage: 4 Q8_0 blocks
constexpr int EX_STAGES = 4;
constexpr int EX_A_BYTES = EX_BM * EX_BKB, EX_B_BYTES = EX_BN * EX_BKB;
constexpr int EX_STAGE_BYTES = EX_A_BYTES + EX_B_BYTES;
constexpr int EX_SLOTS = 4;                 // TMEM accumulators of 128 columns
constexpr int EX_EPI_WARPS = 16;
constexpr int EX_THREADS = 64 + 32 * EX_EPI_WARPS;
constexpr int EX_GROUP_M = 8;
// instruction descriptor: D s32 (bits 4-5 = 2), A and B signed 8-bit (bits 7-9, 10-12 = 1),
// K-major, N >> 3 at bits 17-22, M >> 4 at bits 24-28
constexpr uint32_t EX_IDESC = (2u << 4) | (1u << 7) | (1u << 10) | (uint32_t(EX_BN >> 3) << 17) |
                              (uint32_t(EX_BM >> 4) << 24);
constexpr size_t EX_SMEM = size_t(EX_STAGES) * EX_STAGE_BYTES + 1024 + 256;

struct ExactArgs {
    int64_t M, N, K, nb, n_pad;
    const float *x_scale;   // [M][nb]
    const float *w_scale;   // [nb][n_pad]
    const float *bias;      // [N] or null
    float *out;             // [M][ldo]
    int64_t ldo;
    int *status;
};

__device__ __forceinline__ void umma_i8(uint32_t tmem, uint64_t da, uint64_t db) {
    asm volatile("{ .reg .pred p; setp.ne.b32 p, 0, 0; tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p; }"
                 ::"r"(tmem), "l"(da), "l"(db), "r"(EX_IDESC)
                 : "memory");
}

// exact int -> float for |i| < 2^22 (a block dot is at most 32 * 127 * 127 < 2^19)
__device__ __forceinline__ float i2f_exact(uint32_t bits) {
    return __fsub_rn(__int_as_float(int(bits) + 0x4B400000), 12582912.0f);
}

__global__ void __launch_bounds__(EX_THREADS, 1)
    k_gemm_q8_exact(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb, const ExactArgs a) {
    extern __shared__ __align__(1024) unsigned char ex_smem[];
    unsigned char *base = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(ex_smem) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(base + EX_STAGES * EX_STAGE_BYTES);
    uint64_t *empty = full + EX_STAGES;
    uint64_t *blk_full = empty + EX_STAGES;
    uint64_t *blk_empty = blk_full + EX_SLOTS;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(blk_empty + EX_SLOTS);
    __shared__ int failed;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t nb = a.nb;
    const int kt = int((nb + 3) / 4);
    const int64_t tiles_n = (a.N + EX_BN - 1) / EX_BN, tiles_m = (a.M + EX_BM - 1) / EX_BM;
    const int64_t tiles = tiles_n * tiles_m;
    auto tile_coords = [&](int64_t tile, int64_t &m0, int64_t &n0) {
        const int64_t per_group = int64_t(EX_GROUP_M) * tiles_n;
        const int64_t first_m = (tile / per_group) * EX_GROUP_M;
        const int64_t gsz = tiles_m - first_m < EX_GROUP_M ? tiles_m - first_m : EX_GROUP_M;
        const int64_t r = tile % per_group;
        m0 = (first_m + r % gsz) * EX_BM;
        n0 = (r / gsz) * EX_BN;
    };
    if (threadIdx.x == 0) {
        failed = 0;
        for (int s = 0; s < EX_STAGES; ++s) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, 1);
        }
        for (int b = 0; b < EX_SLOTS; ++b) {
            mbar_init(blk_full + b, 1);
            mbar_init(blk_empty + b, EX_EPI_WARPS);
        }
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                     "r"(512)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            int64_t it = 0;
            for (int64_t tile = blockIdx.x; tile < tiles && !failed; tile += gridDim.x) {
                int64_t m0, n0;
                tile_coords(tile, m0, n0);
                for (int i = 0; i < kt; ++i, ++it) {
                    const int s = int(it % EX_STAGES);
                    if (!mbar_wait_bounded(empty + s, uint32_t(((it / EX_STAGES) & 1) ^ 1))) {
                        atomicOr(&failed, 1);
                        break;
                    }
                    unsigned char *sa = base + s * EX_STAGE_BYTES;
                    mbar_expect_tx(full + s, EX_STAGE_BYTES);
                    tma_load_2d(sa, &ta, i * EX_BKB, int(m0), full + s);
                    tma_load_2d(sa + EX_A_BYTES, &tb, i * EX_BKB, int(n0), full + s);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            int64_t it = 0, blk = 0;
            for (int64_t tile = blockIdx.x; tile < tiles && !failed; tile += gridDim.x) {
                for (int i = 0; i < kt && !failed; ++i, ++it) {
                    const int s = int(it % EX_STAGES);
                    if (!mbar_wait_bounded(full + s, uint32_t((it / EX_STAGES) & 1))) {
                        atomicOr(&failed, 1);
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = smem_addr(base + s * EX_STAGE_BYTES);
                    const uint64_t da = sw128_desc(sa), db = sw128_desc(sa + EX_A_BYTES);
                    for (int kk = 0; kk < 4 && int64_t(i) * 4 + kk < nb; ++kk, ++blk) {
                        const int slot = int(blk % EX_SLOTS);
                        if (!mbar_wait_bounded(blk_empty + slot, uint32_t(((blk / EX_SLOTS) & 1) ^ 1))) {
                            atomicOr(&failed, 1);
                            break;
                        }
                        tc_fence_after();
                        // K = 32 bytes per MMA: +32 B in the swizzled 128-byte rows
                        umma_i8(tmem + uint32_t(slot * EX_BN), da + uint64_t(2 * kk), db + uint64_t(2 * kk));
                        umma_commit(blk_full + slot);
                    }
                    umma_commit(empty + s);
                }
            }
        }
    } else {
        const int q = warp & 3;
        const int c0 = ((warp - 2) / 4) * 32;   // first of this warp's 32 columns
        int64_t blk = 0;
        for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
            int64_t m0, n0;
            tile_coords(tile, m0, n0);
            const int64_t row = m0 + 32 * q + lane;
            const bool live = row < a.M;
            float acc[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) acc[j] = 0.0f;
            bool ok = true;
            for (int64_t b = 0; b < nb; ++b, ++blk) {
                const int slot = int(blk % EX_SLOTS);
                if (!mbar_wait_bounded(blk_full + slot, uint32_t((blk / EX_SLOTS) & 1))) {
                    atomicOr(&failed, 1);
                    ok = false;
                    break;
                }
                tc_fence_after();
                uint32_t r[32];
                tmem_ld32(tmem + (uint32_t(32 * q) << 16) + uint32_t(slot * EX_BN + c0), r);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(blk_empty + slot);   // the slot is free for the next block
                const float dx = live ? __ldg(a.x_scale + row * nb + b) : 0.0f;
                const float4 *ws = reinterpret_cast<const float4 *>(a.w_scale + b * a.n_pad + n0 + c0);
#pragma unroll
                for (int j = 0; j < 32; j += 4) {
                    const float4 w4 = __ldg(ws + j / 4);
                    acc[j] = __fadd_rn(acc[j], __fmul_rn(i2f_exact(r[j]), __fmul_rn(w4.x, dx)));
                    acc[j + 1] = __fadd_rn(acc[j + 1], __fmul_rn(i2f_exact(r[j + 1]), __fmul_rn(w4.y, dx)));
                    acc[j + 2] = __fadd_rn(acc[j + 2], __fmul_rn(i2f_exact(r[j + 2]), __fmul_rn(w4.z, dx)));
                    acc[j + 3] = __fadd_rn(acc[j + 3], __fmul_rn(i2f_exact(r[j + 3]), __fmul_rn(w4.w, dx)));
                }
            }
            if (!ok) break;
            if (live) {
                float *o = a.out + row * a.ldo + n0 + c0;
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const int64_t n = n0 + c0 + j;
                    if (n < a.N) o[j] = a.bias ? __fadd_rn(acc[j], a.bias[n]) : acc[j];
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (threadIdx.x == 0 && failed && a.status) atomicOr(a.status, 2);
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512) : "memory");
    }
}

// canonical Q8_0 blocks [N][nb] -> int8 quants [N][K] and fp32 scales [nb][n_pad]
__global__ void k_exact_weights(const uint8_t *__restrict__ blocks, int64_t n, int64_t nb, int64_t n_pad,
                                int8_t *__restrict__ wq, float *__restrict__ ws) {
    const int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;   // one thread per (row, block)
    if (i >= n_pad * nb) return;
    const int64_t r = i / nb, b = i % nb;
    if (r >= n) {
        ws[b * n_pad + r] = 0.0f;
        return;
    }
    const uint8_t *blk = blocks + (r * nb + b) * Q8_BYTES;
    ws[b * n_pad + r] = __half2float(__ushort_as_half(uint16_t(blk[0]) | uint16_t(uint16_t(blk[1]) << 8)));
    // the block's quants are only 2-byte aligned: byte copies
    for (int j = 0; j < QK; ++j) wq[r * nb * QK + b * QK + j] = int8_t(blk[2 + j]);
}

// fp32 rows -> Q8_0 quantization (selected rounding) as int8 quants [M][K] and the
// fp16-rounded scale of every block as fp32 [M][nb]; one warp per (row, block)
template <int MODE>
__global__ void k_exact_activations(const float *__restrict__ x, int64_t ldx, int64_t m, int64_t k,
                                    int8_t *__restrict__ xq, float *__restrict__ xs, int *__restrict__ status) {
    const int lane = threadIdx.x & 31;
    const int64_t nb = k / QK;
    const int64_t wid = (blockIdx.x * int64_t(blockDim.x) + threadIdx.x) >> 5;
    if (wid >= m * nb) return;
    const int64_t row = wid / nb, b = wid % nb;
    const float v = x[row * ldx + b * QK + lane];
    if (!isfinite(v) && status) atomicOr(status, 1);
    float amax = fabsf(v);
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float d = __fdiv_rn(amax, 127.0f);
    float id;
    if (MODE == 2) id = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
    else id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    const float sv = __fmul_rn(v, id);
    xq[row * k + b * QK + lane] = int8_t(MODE == 0 ? int(roundf(sv)) : __float2int_rn(sv));
    if (lane == 0) xs[row * nb + b] = __half2float(__float2half_rn(d));
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_i8() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult qr{};
        cuda_check(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &qr),
                   "cuTensorMapEncodeTiled lookup");
        require(p && qr == cudaDriverEntryPointSuccess, "cuTensorMapEncodeTiled is unavailable");
        fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

static void make_i8_map(CUtensorMap *map, const void *ptr, int64_t rows, int64_t k) {
    require(uintptr_t(ptr) % 16 == 0 && k % 16 == 0, "int8 GEMM operand must be 16-byte aligned with 16-byte rows");
    const cuuint64_t dims[2] = {cuuint64_t(k), cuuint64_t(rows)};
    const cuuint64_t strides[1] = {cuuint64_t(k)};
    const cuuint32_t box[2] = {cuuint32_t(EX_BKB), cuuint32_t(128)};
    const cuuint32_t estride[2] = {1, 1};
    const CUresult r = encode_i8()(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(ptr), dims, strides, box,
                                   estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    require(r == CUDA_SUCCESS, "tensor map encoding failed");
}

}  // namespace mb

using namespace mb;

extern "C" {

int64_t mstar_b200_q8_exact_pad(int64_t rows) { return rows > 0 ? (rows + EX_BN - 1) / EX_BN * EX_BN : 0; }

int mstar_b200_q8_exact_weights(const void *blocks, uint64_t bytes, int64_t rows, int64_t width, void *weights_i8,
                                float *scales, void *stream, char *error, size_t error_size) {
    try {
        require(rows >= 1 && width >= 32 && width % 32 == 0, "invalid weight shape");
        const int64_t nb = width / QK;
        require(bytes == uint64_t(rows) * nb * Q8_BYTES, "weight bytes differ from rows * width / 32 * 34");
        require(blocks && weights_i8 && scales, "missing weight operand");
        check_device(blocks, "weights");
        check_device(weights_i8, "int8 weights");
        check_device(scales, "weight scales");
        const int64_t n_pad = mstar_b200_q8_exact_pad(rows);
        const int64_t items = n_pad * nb;
        k_exact_weights<<<unsigned(ceil_div(items, 256)), 256, 0, as_stream(stream)>>>(
            static_cast<const uint8_t *>(blocks), rows, nb, n_pad, static_cast<int8_t *>(weights_i8), scales);
        cuda_check(cudaGetLastError(), "weight preparation launch");
        return 0;
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return -1;
    }
}

int mstar_b200_q8_exact_activations(const float *x, int64_t x_stride, int64_t rows, int64_t width, int32_t rounding,
                                    void *x_i8, float *scales, int32_t *status, void *stream, char *error,
                                    size_t error_size) {
    try {
        require(rows >= 1 && width >= 32 && width % 32 == 0 && x_stride >= width, "invalid activation shape");
        require(rounding >= 0 && rounding <= 2, "unknown Q8_0 activation rounding");
        require(x && x_i8 && scales, "missing activation operand");
        check_device(x, "activations");
        const int64_t threads = rows * (width / QK) * 32;
        const unsigned grid = unsigned(ceil_div(threads, 256));
        auto *xq = static_cast<int8_t *>(x_i8);
        cudaStream_t s = as_stream(stream);
        if (rounding == 0) k_exact_activations<0><<<grid, 256, 0, s>>>(x, x_stride, rows, width, xq, scales, status);
        else if (rounding == 2) k_exact_activations<2><<<grid, 256, 0, s>>>(x, x_stride, rows, width, xq, scales, status);
        else k_exact_activations<1><<<grid, 256, 0, s>>>(x, x_stride, rows, width, xq, scales, status);
        cuda_check(cudaGetLastError(), "activation quantization launch");
        return 0;
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return -1;
    }
}

int mstar_b200_gemm_q8_exact(const void *x_i8, const float *x_scales, int64_t rows, const void *w_i8,
                             const float *w_scales, int64_t out_features, int64_t width, const float *bias,
                             float *out, int64_t out_stride, int32_t *status, void *stream, char *error,
                             size_t error_size) {
    try {
        require(mstar_b200_capability() == 1, "sm_100a device capability is unavailable");
        require(rows >= 1 && out_features >= 1 && width >= 32 && width % 32 == 0 && out_stride >= out_features,
                "invalid GEMM shape");
        require(x_i8 && x_scales && w_i8 && w_scales && out, "missing GEMM operand");
        require(uintptr_t(w_scales) % 16 == 0, "weight scales must be 16-byte aligned");
        check_device(x_i8, "int8 activations");
        check_device(w_i8, "int8 weights");
        check_device(out, "output");
        static bool configured = false;
        if (!configured) {
            cuda_check(cudaFuncSetAttribute(k_gemm_q8_exact, cudaFuncAttributeMaxDynamicSharedMemorySize, int(EX_SMEM)),
                       "exact GEMM shared-memory attribute");
            configured = true;
        }
        CUtensorMap ta, tb;
        make_i8_map(&ta, x_i8, rows, width);
        make_i8_map(&tb, w_i8, out_features, width);
        ExactArgs a{};
        a.M = rows;
        a.N = out_features;
        a.K = width;
        a.nb = width / QK;
        a.n_pad = mstar_b200_q8_exact_pad(out_features);
        a.x_scale = x_scales;
        a.w_scale = w_scales;
        a.bias = bias;
        a.out = out;
        a.ldo = out_stride;
        a.status = status;
        int dev = 0, sms = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (sms <= 0) sms = 148;
        const int64_t tiles = ceil_div(out_features, EX_BN) * ceil_div(rows, EX_BM);
        const unsigned grid = unsigned(tiles < sms ? tiles : sms);
        k_gemm_q8_exact<<<grid, EX_THREADS, EX_SMEM, as_stream(stream)>>>(ta, tb, a);
        cuda_check(cudaGetLastError(), "exact GEMM launch");
        return 0;
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return -1;
    }
}

}  // extern "C"
