// Prefill / encoder shapes (M >> 32 rows): tcgen05 GEMM over the block-
// quantized operands dequantized to fp16 (the "dequant staging" form of the
// Q8_0 contraction): A = fp16(x_q * d_x) with x_q, d_x the Q8_0 activation
// quantization of ggml quantize_row_q8_0 (selected rounding), B = fp16(w_q * d_w)
// from the canonical weight blocks. The block-quantized values are preserved up
// to one fp16 rounding of each product of a quant and its scale; the
// contraction accumulates in fp32 in TMEM, so results match ggml's mul_mat to
// reorder + fp16-rounding tolerance (the decode GEMV keeps the exact integer
// path).
//
// Kernel: persistent (one CTA per SM walking 128 x 256 output tiles), 18 warps:
//   warp 0  TMA producer: 2-D tiled bulk tensor copies (128B swizzle) of the
//           A (128 x 64) and B (256 x 64) K-slices into a 4-stage ring (3 stages
//           when the epilogue applies GELU: the fourth stage's room holds
//           ggml's fp16 GELU table);
//   warp 1  allocates 512 TMEM columns (two fp32 accumulators of 256 columns);
//           one thread issues tcgen05.mma kind::f16 (M=128, N=256, K=16) into
//           the free accumulator, commits each stage back to the producer and
//           each finished tile to the epilogue;
//   warps 2-17 epilogue: four warps per TMEM lane quarter (warp % 4), each
//           taking a quarter of the 256 columns: tcgen05.ld 32x32b.x32
//           (one thread = one row x 32 columns = one Q8_0 block), bias / GELU /
//           residual, then fp32 or fp16 stores, or the block's Q8_0
//           quantization stored as fp16(q * d) (the next GEMM's staged A
//           operand); then release the accumulator, so tile i's epilogue
//           overlaps tile i+1's MMAs. The epilogue is the long pole of the GELU /
//           Q8_0-staging shapes (about 30 instructions per output before packing),
//           so it has four warps per scheduler to hide its latencies.
// Above 128 rows the CTA-pair kernel (k_gemm_pair) takes over with the same
// warp roles and epilogue.
// Every mbarrier wait is bounded; a timeout sets status bit value 2 and the
// CTA skips to the end (TMEM is still released).
#include <cuda.h>
#include <cudaTypedefs.h>

#include "../../include/mstar_b200.h"
#include "gemm.cuh"
#include "tcgen05.cuh"

namespace mb {

constexpr int GEMM_BM = 128, GEMM_BN = 256, GEMM_BK = 64;
constexpr int GEMM_A_BYTES = GEMM_BM * GEMM_BK * 2;
constexpr int GEMM_B_BYTES = GEMM_BN * GEMM_BK * 2;
constexpr int GEMM_STAGE_BYTES = GEMM_A_BYTES + GEMM_B_BYTES;
constexpr int GEMM_EPI_WARPS = 16;  // four warps per TMEM lane quarter, each owning a quarter of the columns
constexpr int GEMM_THREADS = 64 + 32 * GEMM_EPI_WARPS;
constexpr int GEMM_GROUP_M = 8;
constexpr uint32_t GEMM_TMEM_COLS = 512;  // two 256-column fp32 accumulators
// instruction descriptor: D f32 (bits 4-5 = 1), A/B f16 (0), K-major A and B,
// N >> 3 at bits 17-22, M >> 4 at bits 24-28
constexpr uint32_t GEMM_IDESC = (1u << 4) | (uint32_t(GEMM_BN >> 3) << 17) | (uint32_t(GEMM_BM >> 4) << 24);
// Shared memory: the operand ring, then barriers, then (GELU variant) ggml's
// GELU table; the GELU variant gives one ring stage to the table.
template <int STAGES, bool GELU_TABLE>
constexpr size_t gemm_smem_bytes() {
    return size_t(STAGES) * GEMM_STAGE_BYTES + 1024 + 256 + (GELU_TABLE ? GELU_TABLE_BYTES : 0);
}

// The residual rows a thread's epilogue will read for tile (m0, n0): requested into
// L2 while the epilogue still waits for that tile's MMAs, so the residual read
// does not stall on DRAM latency (one 128-byte line per 32-column block).
__device__ __forceinline__ void prefetch_residual(const GemmArgs &a, int64_t row, int64_t n0, int c0, int chunks) {
    if (!a.residual || row >= a.M) return;
    const int64_t rrow_i = a.res_period ? row % a.res_period : row;
    const float *base = a.residual + rrow_i * a.ldr + n0;
    for (int c = c0; c < c0 + chunks; ++c)
        if (n0 + c * 32 < a.N) asm volatile("prefetch.global.L2 [%0];" ::"l"(base + c * 32));
}

// Epilogue of one row's 32-column block (one Q8_0 block of the output): bias, GELU,
// residual, then the output mode. `r` holds the fp32 accumulators of columns
// nc .. nc + 31 of output row `orow_i` (residual row `rrow_i`).
template <bool GELU_TABLE>
__device__ __forceinline__ void epilogue_block(const GemmArgs &a, const uint32_t (&r)[32], int64_t orow_i,
                                               int64_t rrow_i, int64_t nc, const uint16_t *gelu_smem) {
    void *const obase = a.out;
    const float *rrow = a.residual ? a.residual + rrow_i * a.ldr : nullptr;
    if (nc + 32 <= a.N) {
        // whole 32-column block: bias, activation, residual, then the output mode
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
        if (a.flags & 1) {
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
                const float4 bb = *reinterpret_cast<const float4 *>(a.bias + nc + j);
                v[j] = __fadd_rn(v[j], bb.x); v[j + 1] = __fadd_rn(v[j + 1], bb.y);
                v[j + 2] = __fadd_rn(v[j + 2], bb.z); v[j + 3] = __fadd_rn(v[j + 3], bb.w);
            }
        }
        if (GELU_TABLE && (a.flags & 2)) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = gelu_ggml(v[j], gelu_smem);
        } else if (a.flags & 8) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = gelu_erf(v[j]);
        }
        if (a.flags & 4) {
            if ((reinterpret_cast<uintptr_t>(rrow + nc) & 15) == 0) {
#pragma unroll
                for (int j = 0; j < 32; j += 4) {
                    const float4 rr = *reinterpret_cast<const float4 *>(rrow + nc + j);
                    v[j] = __fadd_rn(rr.x, v[j]); v[j + 1] = __fadd_rn(rr.y, v[j + 1]);
                    v[j + 2] = __fadd_rn(rr.z, v[j + 2]); v[j + 3] = __fadd_rn(rr.w, v[j + 3]);
                }
            } else {
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] = __fadd_rn(rrow[nc + j], v[j]);
            }
        }
        if (a.out_mode == GEMM_OUT_F32) {
            float *o = static_cast<float *>(obase) + orow_i * a.ldo + nc;
            if ((reinterpret_cast<uintptr_t>(o) & 15) == 0) {
#pragma unroll
                for (int j = 0; j < 32; j += 4)
                    *reinterpret_cast<float4 *>(o + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
            } else {
#pragma unroll
                for (int j = 0; j < 32; ++j) o[j] = v[j];
            }
        } else {
            if (a.out_mode == GEMM_OUT_Q8) {
                // amax as ggml takes it (fmaxf skips a NaN); a NaN-propagating max flags any
                // nonfinite input of the block in one instruction per element
                float amax = 0.0f, bad = 0.0f;
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    amax = fmaxf(amax, fabsf(v[j]));
                    asm("max.NaN.f32 %0, %0, %1;" : "+f"(bad) : "f"(fabsf(v[j])));
                }
                if (!isfinite(bad) && a.status) atomicOr(a.status, 1);
                const float d = __fdiv_rn(amax, 127.0f);
                const float id = a.rounding == 2 ? (amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f)
                                                 : (d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f);
                const float dh = __half2float(__float2half_rn(d));
                if (a.rounding == 0) {   // roundf: half away from zero
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] = __fmul_rn(float(int(roundf(__fmul_rn(v[j], id)))), dh);
                } else {
                    // round to nearest even without the conversion pipe: |x * id| <= 127.5 < 2^22,
                    // so adding 1.5 * 2^23 (unit in the last place 1) rounds it to an integer in one
                    // scalar IEEE add and subtracting gives it back exactly
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const float t = __fsub_rn(__fadd_rn(__fmul_rn(v[j], id), 12582912.0f), 12582912.0f);
                        v[j] = __fmul_rn(t, dh);
                    }
                }
            }
            __half *o = static_cast<__half *>(obase) + orow_i * a.ldo + nc;
            if ((reinterpret_cast<uintptr_t>(o) & 15) == 0) {
#pragma unroll
                for (int j = 0; j < 32; j += 8) {
                    uint4 pk;
                    pk.x = half2_bits(__floats2half2_rn(v[j], v[j + 1]));
                    pk.y = half2_bits(__floats2half2_rn(v[j + 2], v[j + 3]));
                    pk.z = half2_bits(__floats2half2_rn(v[j + 4], v[j + 5]));
                    pk.w = half2_bits(__floats2half2_rn(v[j + 6], v[j + 7]));
                    *reinterpret_cast<uint4 *>(o + j) = pk;
                }
            } else {
#pragma unroll
                for (int j = 0; j < 32; ++j) o[j] = __float2half_rn(v[j]);
            }
        }
    } else {
        // ragged last block (fp32 / fp16 output only; Q8_0 staging needs N % 32 == 0)
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            const int64_t n = nc + j;
            if (n < a.N) {
                float v = __uint_as_float(r[j]);
                if (a.flags & 1) v = __fadd_rn(v, a.bias[n]);
                if (GELU_TABLE && (a.flags & 2)) v = gelu_ggml(v, gelu_smem);
                else if (a.flags & 8) v = gelu_erf(v);
                if (a.flags & 4) v = __fadd_rn(rrow[n], v);
                if (a.out_mode == GEMM_OUT_F32) static_cast<float *>(obase)[orow_i * a.ldo + n] = v;
                else static_cast<__half *>(obase)[orow_i * a.ldo + n] = __float2half_rn(v);
            }
        }
    }
}

template <int GEMM_STAGES, bool GELU_TABLE>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    k_gemm_f16(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb, const GemmArgs a) {
    extern __shared__ __align__(1024) unsigned char gemm_smem[];
    unsigned char *base = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(gemm_smem) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(base + GEMM_STAGES * GEMM_STAGE_BYTES);
    uint64_t *empty = full + GEMM_STAGES;
    uint64_t *acc_full = empty + GEMM_STAGES;   // [2] MMA -> epilogue
    uint64_t *acc_empty = acc_full + 2;         // [2] epilogue -> MMA (one arrival per epilogue warp)
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + 2);
    uint16_t *gelu_smem = reinterpret_cast<uint16_t *>(base + GEMM_STAGES * GEMM_STAGE_BYTES + 256);
    __shared__ int failed;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (GELU_TABLE)
        for (int i = threadIdx.x; i < int(GELU_TABLE_BYTES / 16); i += blockDim.x)
            reinterpret_cast<uint4 *>(gelu_smem)[i] = __ldg(reinterpret_cast<const uint4 *>(a.gelu) + i);
    const int kt = int((a.K + GEMM_BK - 1) / GEMM_BK);
    const int64_t tiles_n = (a.N + GEMM_BN - 1) / GEMM_BN, tiles_m = (a.M + GEMM_BM - 1) / GEMM_BM;
    const int64_t tiles = tiles_n * tiles_m;
    // grouped order: groups of GEMM_GROUP_M row tiles, n fastest inside a group,
    // so the tiles in flight at once touch a few A row panels and all of B,
    // both of which stay in L2 while the fp32 output streams past
    auto tile_coords = [&](int64_t tile, int64_t &m0, int64_t &n0) {
        const int64_t per_group = int64_t(GEMM_GROUP_M) * tiles_n;
        const int64_t first_m = (tile / per_group) * GEMM_GROUP_M;
        const int64_t gsz = tiles_m - first_m < GEMM_GROUP_M ? tiles_m - first_m : GEMM_GROUP_M;
        const int64_t r = tile % per_group;
        m0 = (first_m + r % gsz) * GEMM_BM;
        n0 = (r / gsz) * GEMM_BN;
    };

    if (threadIdx.x == 0) {
        failed = 0;
        for (int s = 0; s < GEMM_STAGES; ++s) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(acc_full + b, 1);
            mbar_init(acc_empty + b, GEMM_EPI_WARPS);
        }
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                     "r"(GEMM_TMEM_COLS)
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
                    const int s = int(it % GEMM_STAGES);
                    if (!mbar_wait_bounded(empty + s, uint32_t(((it / GEMM_STAGES) & 1) ^ 1))) {
                        atomicOr(&failed, 1);
                        break;
                    }
                    unsigned char *sa = base + s * GEMM_STAGE_BYTES;
                    mbar_expect_tx(full + s, GEMM_STAGE_BYTES);
                    tma_load_2d(sa, &ta, i * GEMM_BK, int(m0), full + s);
                    tma_load_2d(sa + GEMM_A_BYTES, &tb, i * GEMM_BK, int(n0), full + s);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            int64_t it = 0, local = 0;
            for (int64_t tile = blockIdx.x; tile < tiles && !failed; tile += gridDim.x, ++local) {
                const int buf = int(local & 1);
                // wait until the epilogue has drained this accumulator buffer (use local/2 - 1)
                if (!mbar_wait_bounded(acc_empty + buf, uint32_t(((local >> 1) & 1) ^ 1))) {
                    atomicOr(&failed, 1);
                    break;
                }
                tc_fence_after();
                const uint32_t acc = tmem + uint32_t(buf * GEMM_BN);
                for (int i = 0; i < kt; ++i, ++it) {
                    const int s = int(it % GEMM_STAGES);
                    if (!mbar_wait_bounded(full + s, uint32_t((it / GEMM_STAGES) & 1))) {
                        atomicOr(&failed, 1);
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = smem_addr(base + s * GEMM_STAGE_BYTES);
                    const uint64_t da = sw128_desc(sa), db = sw128_desc(sa + GEMM_A_BYTES);
#pragma unroll
                    for (int kk = 0; kk < GEMM_BK / 16; ++kk)   // K=16 per MMA: +32 B in the swizzled row
                        umma_f16(acc, da + uint64_t(2 * kk), db + uint64_t(2 * kk), GEMM_IDESC, (i | kk) != 0);
                    umma_commit(empty + s);
                }
                umma_commit(acc_full + buf);
            }
        }
    } else {
        const int q = warp & 3;  // TMEM lane quarter this warp may read
        const int c0 = ((warp - 2) / 4) * (GEMM_BN / 32 / (GEMM_EPI_WARPS / 4));  // first 32-column chunk it owns
        int64_t local = 0;
        for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++local) {
            const int buf = int(local & 1);
            int64_t m0, n0;
            tile_coords(tile, m0, n0);
            const int64_t row = m0 + 32 * q + lane;
            prefetch_residual(a, row, n0, c0, GEMM_BN / 32 / (GEMM_EPI_WARPS / 4));
            if (!mbar_wait_bounded(acc_full + buf, uint32_t((local >> 1) & 1))) {
                atomicOr(&failed, 1);
                break;
            }
            tc_fence_after();
            const int64_t orow_i = a.seg_rows ? (row / a.seg_rows) * a.out_seg_rows + row % a.seg_rows : row;
            const int64_t rrow_i = a.res_period ? row % a.res_period : row;
            for (int c = c0; c < c0 + GEMM_BN / 32 / (GEMM_EPI_WARPS / 4); ++c) {
                uint32_t r[32];
                tmem_ld32(tmem + (uint32_t(32 * q) << 16) + uint32_t(buf * GEMM_BN + c * 32), r);
                if (row < a.M) epilogue_block<GELU_TABLE>(a, r, orow_i, rrow_i, n0 + c * 32, gelu_smem);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty + buf);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (threadIdx.x == 0 && failed && a.status) atomicOr(a.status, 2);
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(GEMM_TMEM_COLS)
                     : "memory");
    }
}

// CTA-pair GEMM (cta_group::2) ----------------------------------------------------
// Two CTAs of a cluster compute one 256 x 256 output tile: each loads its own
// 128 rows of A and 128 of the tile's 256 rows of B (32 KB per stage instead of
// 48 KB per CTA for the same MMA work), the leader issues tcgen05.mma
// cta_group::2 (M = 256, N = 256, K = 16) reading both CTAs' shared memory, and
// each CTA's TMEM receives its own 128 rows, which its own epilogue warps drain
// (the same per-row epilogue as the single-CTA kernel). Barriers:
//   full[s]    leader only: the leader producer's expect_tx arrival plus both
//              CTAs' TMA bytes (each load names the leader's barrier);
//   empty[s]   both CTAs: the leader's MMA commit arrives on both (multicast
//              commit; no load uses multicast);
//   acc_full   both CTAs: the same multicast commit after a tile's last MMA;
//   acc_empty  leader only: one arrival per epilogue warp of both CTAs.
// Every wait is bounded; a timeout sets status bit value 2. Both CTAs meet at a
// cluster barrier before any remote arrival and again before they exit.
constexpr int PAIR_A_BYTES = GEMM_BM * GEMM_BK * 2;          // this CTA's 128 rows of A
constexpr int PAIR_B_BYTES = (GEMM_BN / 2) * GEMM_BK * 2;    // this CTA's 128 of the tile's 256 rows of B
constexpr int PAIR_STAGE_BYTES = PAIR_A_BYTES + PAIR_B_BYTES;
constexpr int PAIR_BM = 2 * GEMM_BM;                          // output rows per CTA pair
constexpr int PAIR_GROUP_M = 4;                               // pair row tiles per group (1024 rows)
// instruction descriptor: D f32, A/B f16, K-major, N = 256, M = 256 (the pair)
constexpr uint32_t PAIR_IDESC = (1u << 4) | (uint32_t(GEMM_BN >> 3) << 17) | (uint32_t(PAIR_BM >> 4) << 24);
// Epilogue forms of the pair kernel: EPI_ROWS, one thread = one row x one 32-column block
// stored from registers (every output mode); EPI_PUSH, the partial product delivered to
// its owner (GEMM_OUT_PUSH); EPI_F32T, fp32 output with bias / residual where every
// global access of the epilogue is coalesced. The last two re-lay each warp's 32 x 32 fp32
// block through shared memory (row stride 36 floats: conflict-free 16-byte writes by row
// and reads by column), so one load or store instruction covers four whole 128-byte row
// segments instead of 32 rows of 16 bytes each (which makes the fp32 residual stream of
// the out_proj / fc2 shapes bound by load/store wavefronts, not by DRAM).
// The 32 x 32 block is unpadded (4 KB per warp, so the ring keeps five stages); its 16-byte
// chunks are XOR-swizzled by row, which keeps both access patterns conflict-free.
constexpr int EPI_ROWS = 0, EPI_PUSH = 1, EPI_F32T = 2;
constexpr size_t PUSH_STAGE_BYTES = size_t(GEMM_EPI_WARPS) * 32 * 32 * 4;
// float offset of 16-byte chunk c4 (0..7) of row r in a warp's swizzled 32 x 32 block
__device__ __forceinline__ int blk_at(int r, int c4) { return r * 32 + ((c4 ^ (r & 7)) << 2); }
template <int STAGES, bool GELU_TABLE, int EPI = EPI_ROWS>
constexpr size_t pair_smem_bytes() {
    return size_t(STAGES) * PAIR_STAGE_BYTES + 1024 + 256 + (GELU_TABLE ? GELU_TABLE_BYTES : 0) +
           (EPI != EPI_ROWS ? PUSH_STAGE_BYTES : 0);
}

// One warp's 32 rows x 32 columns of a pushed partial product: registers (one row per
// lane) -> shared memory -> owner's receive slot, four rows of 128 bytes per store.
__device__ __forceinline__ void push_block(const GemmArgs &a, const uint32_t (&r)[32], float *st, int lane,
                                           int64_t row_base, int64_t nc) {
#pragma unroll
    for (int j = 0; j < 32; j += 4)
        *reinterpret_cast<float4 *>(st + blk_at(lane, j >> 2)) = make_float4(
            __uint_as_float(r[j]), __uint_as_float(r[j + 1]), __uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
    __syncwarp();
    // N is a multiple of 32: a block is wholly inside or outside; rows at or past M (the
    // last tile's padding) have no owner (owner_rows * world >= M is checked on the host)
    if (nc < a.N && row_base < a.M) {
        const int owner = int(row_base / a.push_rows);   // a 32-row group never straddles two owners
        float *slot = a.push_out[owner] + (int64_t(a.push_rank) * a.push_rows + (row_base - owner * a.push_rows)) * a.N;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int rr = i * 4 + (lane >> 3), col = (lane & 7) * 4;
            if (row_base + rr < a.M)
                *reinterpret_cast<float4 *>(slot + int64_t(rr) * a.N + nc + col) =
                    *reinterpret_cast<const float4 *>(st + blk_at(rr, lane & 7));
        }
    }
    __syncwarp();
}

// EPI_F32T, first half: the residual rows of one warp's 32 x 32 block copied into its
// swizzled shared block, four 128-byte row segments per instruction (cp.async, issued
// before the block's TMEM load so the copy overlaps it; no registers held).
__device__ __forceinline__ void f32t_residual(const GemmArgs &a, float *st, int lane, int64_t row_base, int64_t nc) {
    if (!(a.flags & 4) || nc >= a.N) return;   // warp-uniform
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int rr = i * 4 + (lane >> 3);
        const int64_t row = row_base + rr;
        const int64_t rrow = a.res_period ? row % a.res_period : row;
        // rows past M copy nothing (zero source bytes) from a clamped, valid address
        const float *src = a.residual + (row < a.M ? rrow : 0) * a.ldr + nc + (lane & 7) * 4;
        cp_async16(st + blk_at(rr, lane & 7), src, row < a.M ? 16 : 0);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
}

// EPI_F32T, second half: bias, the residual from the shared block, then the fp32 rows
// stored four 128-byte row segments at a time.
__device__ __forceinline__ void f32t_block(const GemmArgs &a, const uint32_t (&r)[32], float *st, int lane,
                                           int64_t row_base, int64_t nc) {
    if (nc >= a.N) return;   // warp-uniform: N is a multiple of 32
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
    if (a.flags & 1) {
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
            const float4 bb = *reinterpret_cast<const float4 *>(a.bias + nc + j);
            v[j] = __fadd_rn(v[j], bb.x); v[j + 1] = __fadd_rn(v[j + 1], bb.y);
            v[j + 2] = __fadd_rn(v[j + 2], bb.z); v[j + 3] = __fadd_rn(v[j + 3], bb.w);
        }
    }
    if (a.flags & 4) {
        asm volatile("cp.async.wait_group 0;" ::: "memory");
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
            const float4 rr = *reinterpret_cast<const float4 *>(st + blk_at(lane, j >> 2));
            v[j] = __fadd_rn(rr.x, v[j]); v[j + 1] = __fadd_rn(rr.y, v[j + 1]);
            v[j + 2] = __fadd_rn(rr.z, v[j + 2]); v[j + 3] = __fadd_rn(rr.w, v[j + 3]);
        }
        __syncwarp();
    }
#pragma unroll
    for (int j = 0; j < 32; j += 4)
        *reinterpret_cast<float4 *>(st + blk_at(lane, j >> 2)) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int rr = i * 4 + (lane >> 3), col = (lane & 7) * 4;
        const int64_t row = row_base + rr;
        if (row < a.M) {
            const int64_t orow = a.seg_rows ? (row / a.seg_rows) * a.out_seg_rows + row % a.seg_rows : row;
            *reinterpret_cast<float4 *>(static_cast<float *>(a.out) + orow * a.ldo + nc + col) =
                *reinterpret_cast<const float4 *>(st + blk_at(rr, lane & 7));
        }
    }
    __syncwarp();
}

template <int STAGES, bool GELU_TABLE, int EPI = EPI_ROWS>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(GEMM_THREADS, 1)
    k_gemm_pair(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb, const GemmArgs a) {
    extern __shared__ __align__(1024) unsigned char gemm_smem[];
    unsigned char *base = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(gemm_smem) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(base + STAGES * PAIR_STAGE_BYTES);
    uint64_t *empty = full + STAGES;
    uint64_t *acc_full = empty + STAGES;   // [2]
    uint64_t *acc_empty = acc_full + 2;    // [2] (the leader's counts both CTAs' epilogue warps)
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + 2);
    uint16_t *gelu_smem = reinterpret_cast<uint16_t *>(base + STAGES * PAIR_STAGE_BYTES + 256);
    __shared__ int failed;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    if (GELU_TABLE)
        for (int i = threadIdx.x; i < int(GELU_TABLE_BYTES / 16); i += blockDim.x)
            reinterpret_cast<uint4 *>(gelu_smem)[i] = __ldg(reinterpret_cast<const uint4 *>(a.gelu) + i);
    const int kt = int((a.K + GEMM_BK - 1) / GEMM_BK);
    const int64_t tiles_n = (a.N + GEMM_BN - 1) / GEMM_BN, tiles_m = (a.M + PAIR_BM - 1) / PAIR_BM;
    const int64_t tiles = tiles_n * tiles_m;
    const int64_t cluster = blockIdx.x >> 1, clusters = gridDim.x >> 1;
    auto tile_coords = [&](int64_t tile, int64_t &m0, int64_t &n0) {  // grouped order, as the single-CTA kernel
        const int64_t per_group = int64_t(PAIR_GROUP_M) * tiles_n;
        const int64_t first_m = (tile / per_group) * PAIR_GROUP_M;
        const int64_t gsz = tiles_m - first_m < PAIR_GROUP_M ? tiles_m - first_m : PAIR_GROUP_M;
        const int64_t r = tile % per_group;
        int64_t mi = first_m + r % gsz;
        if (EPI == EPI_PUSH) {
            // owner-interleaved row tiles: the k-th W-tuple of row tiles takes the k-th tile of
            // each owner's share (the tail past W * P in order), so every wave stores to all
            // owners at once and the NVLink stores overlap the MMAs instead of the local and
            // the remote halves of the kernel running one after the other
            const int64_t owners = (a.M + a.push_rows - 1) / a.push_rows;
            const int64_t share = tiles_m / owners;
            if (mi < owners * share) mi = (mi % owners) * share + mi / owners;
        }
        m0 = mi * PAIR_BM;
        n0 = (r / gsz) * GEMM_BN;
    };

    if (threadIdx.x == 0) {
        failed = 0;
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(acc_full + b, 1);
            mbar_init(acc_empty + b, 2 * GEMM_EPI_WARPS);
        }
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                     "r"(GEMM_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    cluster_sync();   // both CTAs' barriers exist before any load or arrival names them
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            int64_t it = 0;
            for (int64_t tile = cluster; tile < tiles && !failed; tile += clusters) {
                int64_t m0, n0;
                tile_coords(tile, m0, n0);
                const int row = int(m0) + int(rank) * GEMM_BM, col = int(n0) + int(rank) * (GEMM_BN / 2);
                for (int i = 0; i < kt; ++i, ++it) {
                    const int s = int(it % STAGES);
                    if (!mbar_wait_bounded(empty + s, uint32_t(((it / STAGES) & 1) ^ 1))) {
                        atomicOr(&failed, 1);
                        break;
                    }
                    unsigned char *sa = base + s * PAIR_STAGE_BYTES;
                    if (leader) mbar_expect_tx(full + s, 2 * PAIR_STAGE_BYTES);
                    const uint32_t bar = cluster_smem(full + s, 0);
                    tma_load_2d_pair(sa, &ta, i * GEMM_BK, row, bar);
                    tma_load_2d_pair(sa + PAIR_A_BYTES, &tb, i * GEMM_BK, col, bar);
                }
            }
        }
    } else if (warp == 1) {
        if (leader && lane == 0) {
            int64_t it = 0, local = 0;
            for (int64_t tile = cluster; tile < tiles && !failed; tile += clusters, ++local) {
                const int buf = int(local & 1);
                if (!mbar_wait_bounded(acc_empty + buf, uint32_t(((local >> 1) & 1) ^ 1))) {
                    atomicOr(&failed, 1);
                    break;
                }
                tc_fence_after();
                const uint32_t acc = tmem + uint32_t(buf * GEMM_BN);
                for (int i = 0; i < kt; ++i, ++it) {
                    const int s = int(it % STAGES);
                    if (!mbar_wait_bounded(full + s, uint32_t((it / STAGES) & 1))) {
                        atomicOr(&failed, 1);
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = smem_addr(base + s * PAIR_STAGE_BYTES);
                    const uint64_t da = sw128_desc(sa), db = sw128_desc(sa + PAIR_A_BYTES);
#pragma unroll
                    for (int kk = 0; kk < GEMM_BK / 16; ++kk)
                        umma_f16_pair(acc, da + uint64_t(2 * kk), db + uint64_t(2 * kk), PAIR_IDESC, (i | kk) != 0);
                    umma_commit_pair(empty + s);
                }
                umma_commit_pair(acc_full + buf);
            }
        }
    } else {
        const int q = warp & 3;
        const int c0 = ((warp - 2) / 4) * (GEMM_BN / 32 / (GEMM_EPI_WARPS / 4));
        const uint32_t leader_acc_empty[2] = {cluster_smem(acc_empty, 0), cluster_smem(acc_empty + 1, 0)};
        int64_t local = 0;
        bool stored_all = true;
        for (int64_t tile = cluster; tile < tiles; tile += clusters, ++local) {
            const int buf = int(local & 1);
            int64_t m0, n0;
            tile_coords(tile, m0, n0);
            const int64_t row = m0 + int64_t(rank) * GEMM_BM + 32 * q + lane;
            if (EPI != EPI_PUSH) prefetch_residual(a, row, n0, c0, GEMM_BN / 32 / (GEMM_EPI_WARPS / 4));
            if (!mbar_wait_bounded(acc_full + buf, uint32_t((local >> 1) & 1))) {
                atomicOr(&failed, 1);
                stored_all = false;
                break;
            }
            tc_fence_after();
            if (EPI == EPI_F32T) {
                const int64_t row_base = row - lane;
                float *st = reinterpret_cast<float *>(gelu_smem) + (warp - 2) * (32 * 32);
                for (int c = c0; c < c0 + GEMM_BN / 32 / (GEMM_EPI_WARPS / 4); ++c) {
                    f32t_residual(a, st, lane, row_base, n0 + c * 32);
                    uint32_t r[32];
                    tmem_ld32(tmem + (uint32_t(32 * q) << 16) + uint32_t(buf * GEMM_BN + c * 32), r);
                    f32t_block(a, r, st, lane, row_base, n0 + c * 32);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster_relaxed(leader_acc_empty[buf]);
                continue;
            }
            if (EPI == EPI_PUSH) {
                const int64_t row_base = row - lane;
                float *st = reinterpret_cast<float *>(gelu_smem) + (warp - 2) * (32 * 32);
                for (int c = c0; c < c0 + GEMM_BN / 32 / (GEMM_EPI_WARPS / 4); ++c) {
                    uint32_t r[32];
                    tmem_ld32(tmem + (uint32_t(32 * q) << 16) + uint32_t(buf * GEMM_BN + c * 32), r);
                    push_block(a, r, st, lane, row_base, n0 + c * 32);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster_relaxed(leader_acc_empty[buf]);
                continue;
            }
            const int64_t orow_i = a.seg_rows ? (row / a.seg_rows) * a.out_seg_rows + row % a.seg_rows : row;
            const int64_t rrow_i = a.res_period ? row % a.res_period : row;
            for (int c = c0; c < c0 + GEMM_BN / 32 / (GEMM_EPI_WARPS / 4); ++c) {
                uint32_t r[32];
                tmem_ld32(tmem + (uint32_t(32 * q) << 16) + uint32_t(buf * GEMM_BN + c * 32), r);
                if (row < a.M) epilogue_block<GELU_TABLE>(a, r, orow_i, rrow_i, n0 + c * 32, gelu_smem);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster_relaxed(leader_acc_empty[buf]);
        }
        if (EPI == EPI_PUSH) {
            // every lane's stores of every tile reach their owners before the arrivals that
            // publish them: one system-scope fence per warp (a fence per tile stalls the
            // epilogue on a remote round trip while the MMAs wait for the accumulator)
            // (after a timed-out wait nothing is published: the owners' bounded waits run out)
            __threadfence_system();
            __syncwarp();
            if (lane == 0 && stored_all) {
                for (int64_t tile = cluster; tile < tiles; tile += clusters) {
                    int64_t m0, n0;
                    tile_coords(tile, m0, n0);
                    const int64_t row_base = m0 + int64_t(rank) * GEMM_BM + 32 * q;
                    if (row_base >= a.M) continue;
                    const int owner = int(row_base / a.push_rows);
                    int *flag = a.push_flags[owner] + (row_base - owner * a.push_rows) / 32;
                    // relaxed: the fence above already orders every store before these
                    // (a release per arrival would fence the system again each time)
                    asm volatile("red.relaxed.sys.global.add.s32 [%0], %1;" ::"l"(flag), "r"(1) : "memory");
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();   // no CTA leaves while its partner may still signal its barriers
    if (threadIdx.x == 0 && failed && a.status) atomicOr(a.status, 2);
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(GEMM_TMEM_COLS)
                     : "memory");
    }
}

// fp16 dequantized operands ---------------------------------------------------
// weights: canonical Q8_0 / Q4_0 blocks [rows][nb] -> fp16(q * d) [rows][K]
__global__ void k_dequant_weights(const uint8_t *__restrict__ blocks, __half *__restrict__ out, int64_t rows,
                                  int64_t nb, int q4) {
    const int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;  // one thread per element
    if (i >= rows * nb * QK) return;
    const int64_t r = i / (nb * QK), k = i % (nb * QK), b = k / QK, j = k % QK;
    const uint8_t *blk = blocks + (r * nb + b) * (q4 ? Q4_BYTES : Q8_BYTES);
    const float d = __half2float(__ushort_as_half(uint16_t(blk[0]) | uint16_t(uint16_t(blk[1]) << 8)));
    int q;
    if (q4) q = (j < 16 ? (blk[2 + j] & 0x0F) : (blk[2 + j - 16] >> 4)) - 8;
    else q = int8_t(blk[2 + j]);
    out[i] = __float2half_rn(__fmul_rn(float(q), d));
}

// activations: fp32 rows -> Q8_0 quantization (selected rounding) -> fp16(q * d)
template <int MODE>
__global__ void k_dequant_act(const float *__restrict__ x, int64_t ldx, int64_t m, int64_t k,
                              __half *__restrict__ out, int *__restrict__ status) {
    const int lane = threadIdx.x & 31;
    const int64_t nb = k / QK;
    const int64_t wid = (blockIdx.x * int64_t(blockDim.x) + threadIdx.x) >> 5;
    if (wid >= m * nb) return;
    const int64_t token = wid / nb, b = wid % nb;
    const float v = x[token * ldx + b * QK + lane];
    if (!isfinite(v) && status) atomicOr(status, 1);
    float amax = fabsf(v);
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float d = __fdiv_rn(amax, 127.0f);
    float id;
    if (MODE == 2) id = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
    else id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    const float sv = __fmul_rn(v, id);
    const int q = MODE == 0 ? int(roundf(sv)) : __float2int_rn(sv);
    const float dh = __half2float(__float2half_rn(d));
    out[token * k + b * QK + lane] = __float2half_rn(__fmul_rn(float(q), dh));
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        cuda_check(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q),
                   "cuTensorMapEncodeTiled lookup");
        require(p && q == cudaDriverEntryPointSuccess, "cuTensorMapEncodeTiled is unavailable");
        fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// 2-D fp16 tensor map over a row-major [rows][k] matrix, box = 64 x box_rows, 128B swizzle
void make_fp16_map(CUtensorMap *map, const void *ptr, int64_t rows, int64_t k, int box_rows) {
    require(uintptr_t(ptr) % 16 == 0 && (k * 2) % 16 == 0, "GEMM operand must be 16-byte aligned with 16-byte rows");
    const cuuint64_t dims[2] = {cuuint64_t(k), cuuint64_t(rows)};
    const cuuint64_t strides[1] = {cuuint64_t(k * 2)};
    const cuuint32_t box[2] = {cuuint32_t(GEMM_BK), cuuint32_t(box_rows)};
    const cuuint32_t estride[2] = {1, 1};
    const CUresult r = encode_fn()(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(ptr), dims, strides,
                                   box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    require(r == CUDA_SUCCESS, "tensor map encoding failed");
}

void launch_dequant_weights(const uint8_t *blocks, __half *out, int64_t rows, int64_t nb, int q4, cudaStream_t s) {
    const int64_t n = rows * nb * QK;
    k_dequant_weights<<<unsigned(ceil_div(n, 256)), 256, 0, s>>>(blocks, out, rows, nb, q4);
}

void launch_dequant_act(int mode, const float *x, int64_t ldx, int64_t m, int64_t k, __half *out, int *status,
                        cudaStream_t s) {
    const int64_t threads = m * (k / QK) * 32;
    const unsigned grid = unsigned(ceil_div(threads, 256));
    if (mode == 0) k_dequant_act<0><<<grid, 256, 0, s>>>(x, ldx, m, k, out, status);
    else if (mode == 2) k_dequant_act<2><<<grid, 256, 0, s>>>(x, ldx, m, k, out, status);
    else k_dequant_act<1><<<grid, 256, 0, s>>>(x, ldx, m, k, out, status);
}

// Pair kernel shapes: 6 stages (192 KB) without GELU, 4 stages + the 75 KB GELU table with it,
// 5 stages + the 64 KB block staging of the push and coalesced fp32 epilogues.
constexpr int PAIR_STAGES = 6, PAIR_STAGES_GELU = 4, PAIR_STAGES_PUSH = 5, PAIR_STAGES_F32T = 5;
static_assert(pair_smem_bytes<PAIR_STAGES_F32T, false, EPI_F32T>() + 64 <= 232448 &&
                  pair_smem_bytes<PAIR_STAGES, false>() + 64 <= 232448 &&
                  pair_smem_bytes<PAIR_STAGES_GELU, true>() + 64 <= 232448,
              "pair GEMM shared memory exceeds 227 KB per CTA");

void launch_gemm(const CUtensorMap &ta, const CUtensorMap &tb, const CUtensorMap &tb_pair, const GemmArgs &a,
                 cudaStream_t s) {
    static bool configured = false;
    static int pair_clusters = 0, pair_clusters_gelu = 0, pair_clusters_push = 0, pair_clusters_f32t = 0;
    if (!configured) {
        cuda_check(cudaFuncSetAttribute(k_gemm_f16<4, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        int(gemm_smem_bytes<4, false>())),
                   "GEMM shared-memory attribute");
        cuda_check(cudaFuncSetAttribute(k_gemm_f16<3, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        int(gemm_smem_bytes<3, true>())),
                   "GEMM shared-memory attribute");
        cuda_check(cudaFuncSetAttribute(k_gemm_pair<PAIR_STAGES, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        int(pair_smem_bytes<PAIR_STAGES, false>())),
                   "pair GEMM shared-memory attribute");
        cuda_check(cudaFuncSetAttribute(k_gemm_pair<PAIR_STAGES_GELU, true>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        int(pair_smem_bytes<PAIR_STAGES_GELU, true>())),
                   "pair GEMM shared-memory attribute");
        cuda_check(cudaFuncSetAttribute(k_gemm_pair<PAIR_STAGES_PUSH, false, EPI_PUSH>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        int(pair_smem_bytes<PAIR_STAGES_PUSH, false, EPI_PUSH>())),
                   "pair GEMM shared-memory attribute");
        cuda_check(cudaFuncSetAttribute(k_gemm_pair<PAIR_STAGES_F32T, false, EPI_F32T>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        int(pair_smem_bytes<PAIR_STAGES_F32T, false, EPI_F32T>())),
                   "pair GEMM shared-memory attribute");
        // persistent grid: as many CTA pairs as can be resident at once
        auto clusters = [](const void *fn, size_t smem) {
            cudaLaunchConfig_t cfg{};
            cfg.gridDim = dim3(2, 1, 1);
            cfg.blockDim = dim3(GEMM_THREADS, 1, 1);
            cfg.dynamicSmemBytes = smem;
            cfg.numAttrs = 0;   // the kernel's own cluster dimensions (2, 1, 1) apply
            int n = 0;
            cuda_check(cudaOccupancyMaxActiveClusters(&n, fn, &cfg), "pair GEMM occupancy");
            return n;
        };
        pair_clusters = clusters(reinterpret_cast<const void *>(k_gemm_pair<PAIR_STAGES, false>),
                                 pair_smem_bytes<PAIR_STAGES, false>());
        pair_clusters_gelu = clusters(reinterpret_cast<const void *>(k_gemm_pair<PAIR_STAGES_GELU, true>),
                                      pair_smem_bytes<PAIR_STAGES_GELU, true>());
        pair_clusters_push = clusters(reinterpret_cast<const void *>(k_gemm_pair<PAIR_STAGES_PUSH, false, EPI_PUSH>),
                                      pair_smem_bytes<PAIR_STAGES_PUSH, false, EPI_PUSH>());
        pair_clusters_f32t = clusters(reinterpret_cast<const void *>(k_gemm_pair<PAIR_STAGES_F32T, false, EPI_F32T>),
                                      pair_smem_bytes<PAIR_STAGES_F32T, false, EPI_F32T>());
        require(pair_clusters > 0 && pair_clusters_gelu > 0 && pair_clusters_push > 0 && pair_clusters_f32t > 0,
                "pair GEMM cannot be resident");
        configured = true;
    }
    static int sms = 0;
    if (!sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (sms <= 0) sms = 148;
    }
    if (a.out_mode == GEMM_OUT_PUSH) {
        // partial products to their owners: CTA pairs only (callers pass more than 128 rows)
        require(a.M > GEMM_BM && a.flags == 0, "pushed partial products need > 128 rows and no epilogue flags");
        const int64_t tiles = ceil_div(a.N, GEMM_BN) * ceil_div(a.M, PAIR_BM);
        const unsigned grid = unsigned(2 * (tiles < pair_clusters_push ? tiles : pair_clusters_push));
        k_gemm_pair<PAIR_STAGES_PUSH, false, EPI_PUSH>
            <<<grid, GEMM_THREADS, pair_smem_bytes<PAIR_STAGES_PUSH, false, EPI_PUSH>(), s>>>(ta, tb_pair, a);
        return;
    }
    if (a.M > GEMM_BM) {
        const int64_t tiles = ceil_div(a.N, GEMM_BN) * ceil_div(a.M, PAIR_BM);
        const bool gelu = (a.flags & 2) != 0;
        // fp32 rows without the GELU table and with a short K (the epilogue-bound shapes, e.g.
        // out_proj: 1280): the coalesced epilogue, where every row segment it touches is 16-byte
        // aligned. With a long K the MMAs dominate and the re-lay's shared-memory traffic costs
        // them more than the coalescing saves (fc2, K = 5120: 276 us against 262 us).
        const bool aligned = uintptr_t(a.out) % 16 == 0 && a.ldo % 4 == 0 &&
                             (!(a.flags & 4) || (uintptr_t(a.residual) % 16 == 0 && a.ldr % 4 == 0)) &&
                             (!(a.flags & 1) || uintptr_t(a.bias) % 16 == 0);
        const bool f32t = !gelu && a.out_mode == GEMM_OUT_F32 && a.N % 32 == 0 && a.K <= 2048 && aligned;
        const int64_t resident = gelu ? pair_clusters_gelu : f32t ? pair_clusters_f32t : pair_clusters;
        const unsigned grid = unsigned(2 * (tiles < resident ? tiles : resident));
        if (f32t)
            k_gemm_pair<PAIR_STAGES_F32T, false, EPI_F32T>
                <<<grid, GEMM_THREADS, pair_smem_bytes<PAIR_STAGES_F32T, false, EPI_F32T>(), s>>>(ta, tb_pair, a);
        else if (gelu)
            k_gemm_pair<PAIR_STAGES_GELU, true><<<grid, GEMM_THREADS, pair_smem_bytes<PAIR_STAGES_GELU, true>(), s>>>(
                ta, tb_pair, a);
        else
            k_gemm_pair<PAIR_STAGES, false><<<grid, GEMM_THREADS, pair_smem_bytes<PAIR_STAGES, false>(), s>>>(
                ta, tb_pair, a);
        return;
    }
    const int64_t tiles = ceil_div(a.N, GEMM_BN) * ceil_div(a.M, GEMM_BM);
    const unsigned grid = unsigned(tiles < sms ? tiles : sms);  // persistent: one CTA per SM
    if (a.flags & 2) k_gemm_f16<3, true><<<grid, GEMM_THREADS, gemm_smem_bytes<3, true>(), s>>>(ta, tb, a);
    else k_gemm_f16<4, false><<<grid, GEMM_THREADS, gemm_smem_bytes<4, false>(), s>>>(ta, tb, a);
}

}  // namespace mb
