// Qwen3-Omni thinker MoE expert FFN on B200.
//
// Reference semantics (rohanchanani/mstar_accelerators):
//  router  ConsistentBF16Router.forward (implementations/qwen3_omni/amd/
//          router_consistency.py:54-62): logits = bf16(x . Wr^T) (fp32
//          accumulation), p = softmax_fp32(logits), top-k, w /= sum(w).
//  experts SmallTokenThinkerMoE (thinker_moe.py:17-105): per (token, slot)
//          g = bf16(x . w_gate), u = bf16(x . w_up), act = bf16(g * sigmoid(g)),
//          mid = bf16(act * u); y_s = bf16((mid . w_down) * w_s);
//          out = bf16(sum over slots s = 0..k-1 of fp32(y_s)), in slot order.
//  layout  w1 [E][2I][H] (gate rows [0, I), up rows [I, 2I)), w2 [E][H][I]
//          (preparation.py:13-36; thinker_moe.py:57-66).
// Q8_0 variant (no counterpart in the reference, composed from its pieces):
// expert weights are Q8_0 blocks; x and mid are Q8_0-quantized per 32-block
// (quantize_row_q8_0, selected rounding) before each contraction; the bf16
// rounding points above are kept.
//
// B200 pipeline for T tokens (all on one stream, no host synchronisation):
//  k_router      CTA per 16 tokens: logits, softmax, top-k, renorm
//  k_moe_count / k_moe_plan / k_moe_scatter
//                counting sort of the T*k (token, slot) pairs by expert and a
//                device-side work list of 128-row tiles per expert
//  k_moe_gather  permuted activation rows (bf16 copy, or Q8_0 quantize ->
//                fp16 dequant for the Q8_0 variant)
//  k_moe_gemm<SWIGLU>  grouped tcgen05 GEMM x_perm . w1^T with gate/up rows
//                interleaved per 256-row tile, so one epilogue thread holds a
//                row's gate and up values and writes mid (bf16, or Q8_0
//                quantized -> fp16 for the Q8_0 variant)
//  k_moe_gemm<DOWN>    grouped GEMM mid . w2^T, epilogue y = bf16(acc * w_slot)
//  k_moe_combine out[t] = bf16(sum_s fp32(y[pair(t, s)])) in slot order
// Operands of one MMA always share their type (both bf16 or both fp16).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>

#include <atomic>
#include <memory>

#include "../../include/mstar_b200.h"
#include "gemm.cuh"
#include "tcgen05.cuh"

namespace mb {

// 2 + 16 warps: the TMA producer, the MMA issuer and four epilogue warps per TMEM lane
// quarter, each taking a quarter of a tile's columns (the SwiGLU epilogue's exp and
// bf16 roundings and the down epilogue's 16-byte row stores have four warps per
// scheduler to hide their latencies)
constexpr int MOE_EPI_WARPS = 16;
constexpr int MOE_BM = 128, MOE_BN = 256, MOE_BK = 64, MOE_STAGES = 4, MOE_THREADS = 64 + 32 * MOE_EPI_WARPS;
constexpr int MOE_A_BYTES = MOE_BM * MOE_BK * 2, MOE_B_BYTES = MOE_BN * MOE_BK * 2;
constexpr int MOE_STAGE_BYTES = MOE_A_BYTES + MOE_B_BYTES;
constexpr size_t MOE_SMEM = size_t(MOE_STAGES) * MOE_STAGE_BYTES + 1024 + 256;
constexpr int MOE_MAX_TOPK = 8;
constexpr int ROUTER_TOKENS = 16;

__device__ __forceinline__ float bf16r(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// ------------------------------------------------------------------ router
// Logits: CTA of WARPS warps per (16 tokens, WARPS * EPW experts). The 16 token rows sit
// in shared memory as bf16; warp w owns experts e0 .. e0 + EPW - 1 and its lanes stream
// their rows with 16-byte loads, accumulating 16 fp32 dots per expert that are then
// reduced across the warp. Per (token, expert) the order of the sums is the same for
// every CTA shape: lane l's fused multiply-adds over chunks l, l + 32, ... and within a
// chunk its eight elements, then the butterfly. EPW > 1 (prefill) reads each token
// chunk from shared memory once for EPW experts; decode uses one expert per warp and 8
// warps, so 32 tokens still spread over 32 CTAs. Output logits[t][e] = bf16(dot)
// (F.linear's output dtype).
template <int WARPS, int EPW>
__global__ void __launch_bounds__(WARPS * 32) k_router_logits(const __nv_bfloat16 *__restrict__ x,
                                                        const __nv_bfloat16 *__restrict__ wr, int T, int H, int E,
                                                        float *__restrict__ logits) {
    extern __shared__ __align__(16) __nv_bfloat16 xs[];  // [ROUTER_TOKENS][H]
    const int t0 = blockIdx.x * ROUTER_TOKENS;
    const int nt = T - t0 < ROUTER_TOKENS ? T - t0 : ROUTER_TOKENS;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int vec = H / 8;  // uint4 per row
    for (int i = threadIdx.x; i < ROUTER_TOKENS * vec; i += blockDim.x) {
        const int tt = i / vec, c = i % vec;
        reinterpret_cast<uint4 *>(xs)[i] =
            tt < nt ? reinterpret_cast<const uint4 *>(x + int64_t(t0 + tt) * H)[c] : make_uint4(0, 0, 0, 0);
    }
    __syncthreads();
    const int e0 = (blockIdx.y * WARPS + warp) * EPW;
    if (e0 >= E) return;
    float acc[EPW][ROUTER_TOKENS];
#pragma unroll
    for (int q = 0; q < EPW; ++q)
#pragma unroll
        for (int i = 0; i < ROUTER_TOKENS; ++i) acc[q][i] = 0.0f;
    constexpr int UNROLL = EPW == 1 ? 4 : 1;   // one expert: its row's weight loads in flight together
#pragma unroll UNROLL
    for (int c = lane; c < vec; c += 32) {
        float wf[EPW][8];
#pragma unroll
        for (int q = 0; q < EPW; ++q) {
            const uint4 wv = e0 + q < E ? __ldg(reinterpret_cast<const uint4 *>(wr + int64_t(e0 + q) * H) + c)
                                        : make_uint4(0, 0, 0, 0);
            const __nv_bfloat162 *w2 = reinterpret_cast<const __nv_bfloat162 *>(&wv);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float2 f = __bfloat1622float2(w2[j]);
                wf[q][2 * j] = f.x;
                wf[q][2 * j + 1] = f.y;
            }
        }
#pragma unroll
        for (int tt = 0; tt < ROUTER_TOKENS; ++tt) {
            const uint4 xv = reinterpret_cast<const uint4 *>(xs + tt * H)[c];
            const __nv_bfloat162 *x2 = reinterpret_cast<const __nv_bfloat162 *>(&xv);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float2 f = __bfloat1622float2(x2[j]);
#pragma unroll
                for (int q = 0; q < EPW; ++q)
                    acc[q][tt] = fmaf(f.y, wf[q][2 * j + 1], fmaf(f.x, wf[q][2 * j], acc[q][tt]));
            }
        }
    }
#pragma unroll
    for (int q = 0; q < EPW; ++q) {
#pragma unroll
        for (int tt = 0; tt < ROUTER_TOKENS; ++tt) {
#pragma unroll
            for (int o = 16; o; o >>= 1) acc[q][tt] += __shfl_xor_sync(0xffffffffu, acc[q][tt], o);
        }
        if (lane < nt && e0 + q < E) {
            float v = acc[q][0];
#pragma unroll
            for (int tt = 1; tt < ROUTER_TOKENS; ++tt)
                if (lane == tt) v = acc[q][tt];
            logits[int64_t(t0 + lane) * E + e0 + q] = bf16r(v);
        }
    }
}

// One warp per token: softmax in fp32, top-k by repeated argmax (lower index
// wins ties), optional renormalisation.
__global__ void k_router_topk(const float *__restrict__ logits, int T, int E, int topk, int renorm,
                              float *__restrict__ topk_w, int32_t *__restrict__ topk_ids) {
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (t >= T) return;
    constexpr int MAXV = 8;  // E <= 256
    float v[MAXV];
    const float *row = logits + int64_t(t) * E;
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
        const int j = lane + 32 * i;
        v[i] = j < E ? row[j] : -INFINITY;
        mx = fmaxf(mx, v[i]);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.0f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i)
        if (lane + 32 * i < E) sum += expf(v[i] - mx);
#pragma unroll
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
#pragma unroll
    for (int i = 0; i < MAXV; ++i) v[i] = lane + 32 * i < E ? expf(v[i] - mx) / sum : -INFINITY;
    float chosen = 0.0f, total = 0.0f;
    int chosen_id = 0;
    for (int r = 0; r < topk; ++r) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
#pragma unroll
        for (int i = 0; i < MAXV; ++i) {
            const int j = lane + 32 * i;
            if (j < E && (v[i] > bv || (v[i] == bv && j < bi))) { bv = v[i]; bi = j; }
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
        if (lane == r) { chosen = bv; chosen_id = bi; }
        total += bv;
#pragma unroll
        for (int i = 0; i < MAXV; ++i)
            if (lane + 32 * i == bi) v[i] = -INFINITY;
    }
    if (lane < topk) {
        topk_w[int64_t(t) * topk + lane] = renorm ? chosen / total : chosen;
        topk_ids[int64_t(t) * topk + lane] = chosen_id;
    }
}

// ------------------------------------------------------------------ permutation
struct MoePlan {
    int *counts;      // [E]
    int *offsets;     // [E]
    int *cursor;      // [E]
    int *tiles;       // [max_tiles][3]: expert, row_start, row_end (permuted rows)
    int *num_tiles;   // [1]
    int *perm;        // [P] permuted position -> pair (token * k + slot); valid below *valid
    int *inv;         // [P] pair -> permuted position, -1 for a pair with an expert id outside [0, E)
    int *valid;       // [1] pairs with a valid expert id (the permuted rows in use)
};

// The handle holds experts [e0, e0 + E) of e_total (all of them without expert
// parallelism): an id outside [0, e_total) sets status bit value 4, an id of
// another rank's expert is skipped silently; both contribute nothing here.
__global__ void k_moe_count(const int32_t *__restrict__ ids, int P, int E, int e0, int e_total,
                            int *__restrict__ counts, int *__restrict__ status) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= P) return;
    const int id = ids[i];
    if (id < 0 || id >= e_total) {
        atomicOr(status, 4);
        return;
    }
    const int e = id - e0;
    if (e >= 0 && e < E) atomicAdd(counts + e, 1);
}

// single CTA: exclusive scans of the counts and of the 128-row tile counts
// (one thread, in shared memory), then every expert's offsets, cursor and tile
// entries written in parallel; the tile list is in expert order, cut at max_tiles
__global__ void k_moe_plan(MoePlan p, int E, int max_tiles) {
    __shared__ int cnt[1024], off[1024], toff[1024];
    const int tid = threadIdx.x;
    for (int e = tid; e < E; e += blockDim.x) cnt[e] = p.counts[e];
    __syncthreads();
    if (tid == 0) {
        int o = 0, t = 0;
        for (int e = 0; e < E; ++e) {
            off[e] = o;
            toff[e] = t;
            o += cnt[e];
            t += (cnt[e] + MOE_BM - 1) / MOE_BM;
        }
        *p.num_tiles = t < max_tiles ? t : max_tiles;
        *p.valid = o;
    }
    __syncthreads();
    for (int e = tid; e < E; e += blockDim.x) {
        p.offsets[e] = off[e];
        p.cursor[e] = 0;
        const int mt = (cnt[e] + MOE_BM - 1) / MOE_BM;
        for (int j = 0; j < mt && toff[e] + j < max_tiles; ++j) {
            const int tile = toff[e] + j;
            p.tiles[3 * tile] = e;
            p.tiles[3 * tile + 1] = off[e] + j * MOE_BM;
            const int end = off[e] + (j + 1) * MOE_BM;
            p.tiles[3 * tile + 2] = end < off[e] + cnt[e] ? end : off[e] + cnt[e];
        }
    }
}

__global__ void k_moe_scatter(const int32_t *__restrict__ ids, int P, int E, int e0, int e_total, MoePlan p) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= P) return;
    const int id = ids[i], e = id - e0;
    if (id < 0 || id >= e_total || e < 0 || e >= E) {  // invalid (status bit 4 already set) or not held here
        p.inv[i] = -1;
        return;
    }
    const int pos = p.offsets[e] + atomicAdd(p.cursor + e, 1);
    p.perm[pos] = i;
    p.inv[i] = pos;
}

// permuted activation rows: row pos <- x[perm[pos] / k]
// q8: quantize each 32-block (selected rounding) of fp32(x) and store fp16(q * d)
__global__ void k_moe_gather(const __nv_bfloat16 *__restrict__ x, const int *__restrict__ perm,
                             const int *__restrict__ valid, int P, int H, int topk, int q8, int rounding,
                             void *__restrict__ xp) {
    const int pos = blockIdx.x;
    if (pos >= P || pos >= *valid) return;
    const int64_t t = perm[pos] / topk;
    const __nv_bfloat16 *src = x + t * H;
    if (!q8) {
        __nv_bfloat16 *dst = static_cast<__nv_bfloat16 *>(xp) + int64_t(pos) * H;
        for (int i = threadIdx.x; i < H; i += blockDim.x) dst[i] = src[i];
        return;
    }
    __half *dst = static_cast<__half *>(xp) + int64_t(pos) * H;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    for (int b = warp; b < H / QK; b += nwarps) {
        const float v = __bfloat162float(src[b * QK + lane]);
        float amax = fabsf(v);
#pragma unroll
        for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const float d = __fdiv_rn(amax, 127.0f);
        float id;
        if (rounding == 2) id = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
        else id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        const float sv = __fmul_rn(v, id);
        const int q = rounding == 0 ? int(roundf(sv)) : __float2int_rn(sv);
        dst[b * QK + lane] = __float2half_rn(__fmul_rn(float(q), __half2float(__float2half_rn(d))));
    }
}

// k_moe_gather with 16-byte row pieces (rows 16-byte aligned, H a multiple of 128), one
// uint4 per thread and pass: bf16 token rows, or (Q8_0 experts) the tokens' rows already
// staged as fp16(q * d), the same 2-byte elements.
__global__ void __launch_bounds__(256) k_moe_gather_vec(const void *__restrict__ x, const int *__restrict__ perm,
                                                        const int *__restrict__ valid, int P, int H, int topk,
                                                        void *__restrict__ xp) {
    const int pos = blockIdx.x;
    if (pos >= P || pos >= *valid) return;
    const int64_t t = perm[pos] / topk;
    const uint4 *s4 = reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(x) + t * H);
    uint4 *d4 = reinterpret_cast<uint4 *>(static_cast<uint16_t *>(xp) + int64_t(pos) * H);
    for (int i = threadIdx.x; i < H / 8; i += blockDim.x) d4[i] = s4[i];
}

// k_moe_combine with 8 outputs per thread (y and out 16-byte aligned, H a multiple of 8)
__global__ void k_moe_combine_vec(const __nv_bfloat16 *__restrict__ y, const int *__restrict__ inv, int T, int H,
                                  int topk, __nv_bfloat16 *__restrict__ out) {
    const int t = blockIdx.x;
    if (t >= T) return;
    int rows[MOE_MAX_TOPK];
    for (int s = 0; s < topk; ++s) rows[s] = inv[t * topk + s];
    for (int n8 = threadIdx.x; n8 < H / 8; n8 += blockDim.x) {
        float acc[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
        for (int s = 0; s < topk; ++s) {
            if (rows[s] < 0) continue;
            const uint4 v = *reinterpret_cast<const uint4 *>(y + int64_t(rows[s]) * H + 8 * n8);
            const __nv_bfloat16 *b = reinterpret_cast<const __nv_bfloat16 *>(&v);
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i] = __fadd_rn(acc[i], __bfloat162float(b[i]));
        }
        uint4 o;
        __nv_bfloat16 *ob = reinterpret_cast<__nv_bfloat16 *>(&o);
#pragma unroll
        for (int i = 0; i < 8; ++i) ob[i] = __float2bfloat16_rn(acc[i]);
        *reinterpret_cast<uint4 *>(out + int64_t(t) * H + 8 * n8) = o;
    }
}

// out[t][n] = bf16(sum_s fp32(y[inv[t*k + s]][n])) in slot order
__global__ void k_moe_combine(const __nv_bfloat16 *__restrict__ y, const int *__restrict__ inv, int T, int H, int topk,
                              __nv_bfloat16 *__restrict__ out) {
    const int t = blockIdx.x;
    if (t >= T) return;
    int rows[MOE_MAX_TOPK];
    for (int s = 0; s < topk; ++s) rows[s] = inv[t * topk + s];
    for (int n = threadIdx.x; n < H; n += blockDim.x) {
        float acc = 0.0f;
        for (int s = 0; s < topk; ++s)
            if (rows[s] >= 0) acc = __fadd_rn(acc, __bfloat162float(y[int64_t(rows[s]) * H + n]));
        out[int64_t(t) * H + n] = __float2bfloat16_rn(acc);
    }
}

// Same slot-ordered sum over caller-given rows (expert parallelism: the rows
// come back from their owners in send order); a row outside [0, y_rows) adds
// nothing.
__global__ void k_moe_combine_rows(const __nv_bfloat16 *__restrict__ y, int64_t y_rows, const int *__restrict__ rows,
                                   int T, int H, int topk, __nv_bfloat16 *__restrict__ out) {
    const int t = blockIdx.x;
    if (t >= T) return;
    int r[MOE_MAX_TOPK];
    for (int s = 0; s < topk; ++s) r[s] = rows[int64_t(t) * topk + s];
    for (int n = threadIdx.x; n < H; n += blockDim.x) {
        float acc = 0.0f;
        for (int s = 0; s < topk; ++s)
            if (r[s] >= 0 && r[s] < y_rows) acc = __fadd_rn(acc, __bfloat162float(y[int64_t(r[s]) * H + n]));
        out[int64_t(t) * H + n] = __float2bfloat16_rn(acc);
    }
}

// k_moe_combine_rows with 8 outputs per thread (y and out 16-byte aligned, H a multiple of 8)
__global__ void k_moe_combine_rows_vec(const __nv_bfloat16 *__restrict__ y, int64_t y_rows,
                                       const int *__restrict__ rows, int T, int H, int topk,
                                       __nv_bfloat16 *__restrict__ out) {
    const int t = blockIdx.x;
    if (t >= T) return;
    int r[MOE_MAX_TOPK];
    for (int s = 0; s < topk; ++s) r[s] = rows[int64_t(t) * topk + s];
    for (int c = threadIdx.x; c < H / 8; c += blockDim.x) {
        float acc[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
        for (int s = 0; s < topk; ++s) {
            if (r[s] < 0 || r[s] >= y_rows) continue;
            const uint4 v = reinterpret_cast<const uint4 *>(y + int64_t(r[s]) * H)[c];
            const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&v);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float2 f = __bfloat1622float2(h[j]);
                acc[2 * j] = __fadd_rn(acc[2 * j], f.x);
                acc[2 * j + 1] = __fadd_rn(acc[2 * j + 1], f.y);
            }
        }
        uint4 o;
        __nv_bfloat162 *oh = reinterpret_cast<__nv_bfloat162 *>(&o);
#pragma unroll
        for (int j = 0; j < 4; ++j) oh[j] = __floats2bfloat162_rn(acc[2 * j], acc[2 * j + 1]);
        reinterpret_cast<uint4 *>(out + int64_t(t) * H)[c] = o;
    }
}

// ------------------------------------------------------------------ expert-parallel dispatch
// Send order of the T*k (token, slot) pairs for W expert-owning ranks: the
// pairs grouped by owning rank d = clamp(floor(id / per), 0, W - 1), in pair
// order inside a rank (a stable counting sort). One CTA of 32 warps. Pass 1
// counts the pairs per rank with warp ballots. Pass 2 walks the pairs in
// rounds of 1024: each pair's place among its warp's pairs for the same rank
// comes from a ballot, the warps' counts become offsets through one warp-level
// scan per rank, and the pair's send position (inverse), local expert id and
// routing weight bits (pairs) are written. meta [W][2] = (pairs for rank d,
// 1 if any id lies outside [0, E)).
constexpr int EP_THREADS = 1024, EP_MAX_RANKS = 32;

__device__ __forceinline__ int ep_rank_of(int id, int per, int W) {
    if (id < 0) return 0;
    const int d = id / per;
    return d < W ? d : W - 1;
}

__global__ void __launch_bounds__(EP_THREADS) k_ep_plan(const int32_t *__restrict__ ids,
                                                        const float *__restrict__ w, int P, int per, int E, int W,
                                                        int64_t *__restrict__ meta, int32_t *__restrict__ pairs,
                                                        int32_t *__restrict__ inverse) {
    __shared__ int warp_off[32][EP_MAX_RANKS + 1];
    __shared__ int base[EP_MAX_RANKS];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const unsigned below = (1u << lane) - 1u;
    if (tid < EP_MAX_RANKS) base[tid] = 0;
    __syncthreads();
    int mine = 0, bad = 0;  // lane d of a warp counts that warp's pairs for rank d
    for (int r0 = 0; r0 < P; r0 += EP_THREADS) {
        const int p = r0 + tid;
        int d = -1;
        if (p < P) {
            const int id = ids[p];
            bad |= id < 0 || id >= E;
            d = ep_rank_of(id, per, W);
        }
        for (int dd = 0; dd < W; ++dd) {
            const unsigned m = __ballot_sync(0xffffffffu, d == dd);
            if (lane == dd) mine += __popc(m);
        }
    }
    if (lane < W) atomicAdd(&base[lane], mine);
    bad = __syncthreads_or(bad);
    if (tid == 0) {  // totals -> meta, and the exclusive scan over ranks as running offsets
        int o = 0;
        for (int d = 0; d < W; ++d) {
            const int c = base[d];
            meta[2 * d] = c;
            meta[2 * d + 1] = bad ? 1 : 0;
            base[d] = o;
            o += c;
        }
    }
    __syncthreads();
    for (int r0 = 0; r0 < P; r0 += EP_THREADS) {
        const int p = r0 + tid;
        int id = 0, d = -1;
        if (p < P) {
            id = ids[p];
            d = ep_rank_of(id, per, W);
        }
        int place = 0, count = 0;
        for (int dd = 0; dd < W; ++dd) {
            const unsigned m = __ballot_sync(0xffffffffu, d == dd);
            if (d == dd) place = __popc(m & below);
            if (lane == dd) count = __popc(m);
        }
        if (lane < W) warp_off[warp][lane] = count;
        __syncthreads();
        if (warp < W) {  // warp d: offsets of the 32 warps' pairs for rank d
            const int c = warp_off[lane][warp];
            int incl = c;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += v;
            }
            const int start = base[warp];
            warp_off[lane][warp] = start + incl - c;
            __syncwarp();
            if (lane == 31) base[warp] = start + incl;
        }
        __syncthreads();
        if (d >= 0) {
            const int pos = warp_off[warp][d] + place;
            inverse[p] = pos;
            pairs[2 * pos] = id - d * per;
            pairs[2 * pos + 1] = __float_as_int(w[p]);
        }
        __syncthreads();  // warp_off is rewritten by the next round
    }
}

// rows[inverse[p]] = x[p / k]; vec: 16-byte pieces (x and rows 16-byte aligned, H a multiple of 8)
__global__ void __launch_bounds__(256) k_ep_rows(const __nv_bfloat16 *__restrict__ x,
                                                 const int32_t *__restrict__ inverse, int P, int H, int topk,
                                                 int vec, __nv_bfloat16 *__restrict__ rows) {
    const int p = blockIdx.x;
    if (p >= P) return;
    const __nv_bfloat16 *src = x + int64_t(p / topk) * H;
    __nv_bfloat16 *dst = rows + int64_t(inverse[p]) * H;
    if (vec) {
        for (int i = threadIdx.x; i < H / 8; i += blockDim.x)
            reinterpret_cast<uint4 *>(dst)[i] = reinterpret_cast<const uint4 *>(src)[i];
    } else {
        for (int i = threadIdx.x; i < H; i += blockDim.x) dst[i] = src[i];
    }
}

// ------------------------------------------------------------------ grouped GEMM
struct MoeGemmArgs {
    const int *tiles;      // [num_tiles][3]
    const int *num_tiles;
    int n_tiles;           // 256-wide output tiles per expert (w rows / 256)
    int w_rows;            // rows of one expert's weight matrix (2I or H)
    int K;
    // SWIGLU epilogue: mid [P][I] bf16 (or fp16 Q8_0-dequantized when q8)
    void *mid;
    int I;
    int q8, rounding;
    // DOWN epilogue: y [P][H] bf16 = bf16(acc * topk_w[perm[row]])
    __nv_bfloat16 *y;
    const float *topk_w;
    const int *perm;
    int *status;
};

constexpr int MOE_SWIGLU = 0, MOE_DOWN = 1;

__device__ __forceinline__ float silu_bf16(float g) {
    // act = bf16(g * sigmoid(g)) on the bf16-rounded g (thinker_moe.py:44-47)
    return bf16r(g * (1.0f / (1.0f + expf(-g))));
}

template <int MODE, bool BF16>
__global__ void __launch_bounds__(MOE_THREADS, 1)
    k_moe_gemm(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb, const MoeGemmArgs a) {
    // instruction descriptor: D f32, A/B bf16 (1) or f16 (0), K-major, N=256, M=128
    constexpr uint32_t IDESC = (1u << 4) | ((BF16 ? 1u : 0u) << 7) | ((BF16 ? 1u : 0u) << 10) |
                               (uint32_t(MOE_BN >> 3) << 17) | (uint32_t(MOE_BM >> 4) << 24);
    extern __shared__ __align__(1024) unsigned char moe_smem[];
    unsigned char *base = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(moe_smem) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(base + MOE_STAGES * MOE_STAGE_BYTES);
    uint64_t *empty = full + MOE_STAGES;
    uint64_t *acc_full = empty + MOE_STAGES;
    uint64_t *acc_empty = acc_full + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + 2);
    __shared__ int failed;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kt = (a.K + MOE_BK - 1) / MOE_BK;
    const int64_t tiles = int64_t(*a.num_tiles) * a.n_tiles;  // written by k_moe_plan earlier on the stream

    if (threadIdx.x == 0) {
        failed = 0;
        for (int s = 0; s < MOE_STAGES; ++s) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(acc_full + b, 1);
            mbar_init(acc_empty + b, MOE_EPI_WARPS);
        }
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                     "r"(512u)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // tile = m-tile (list entry) * n_tiles + n-tile: n fastest, so CTAs working at the
    // same time share the A rows of an expert and stream that expert's weight tiles
    auto coords = [&](int64_t tile, int &e, int &r0, int &r1, int &nt) {
        const int mt = int(tile / a.n_tiles);
        nt = int(tile % a.n_tiles);
        e = a.tiles[3 * mt];
        r0 = a.tiles[3 * mt + 1];
        r1 = a.tiles[3 * mt + 2];
    };

    if (warp == 0) {
        if (lane == 0) {
            int64_t it = 0;
            for (int64_t tile = blockIdx.x; tile < tiles && !failed; tile += gridDim.x) {
                int e, r0, r1, nt;
                coords(tile, e, r0, r1, nt);
                for (int i = 0; i < kt; ++i, ++it) {
                    const int s = int(it % MOE_STAGES);
                    if (!mbar_wait_bounded(empty + s, uint32_t(((it / MOE_STAGES) & 1) ^ 1))) {
                        atomicOr(&failed, 1);
                        break;
                    }
                    unsigned char *sa = base + s * MOE_STAGE_BYTES;
                    mbar_expect_tx(full + s, MOE_STAGE_BYTES);
                    tma_load_2d(sa, &ta, i * MOE_BK, r0, full + s);
                    tma_load_2d(sa + MOE_A_BYTES, &tb, i * MOE_BK, e * a.w_rows + nt * MOE_BN, full + s);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            int64_t it = 0, local = 0;
            for (int64_t tile = blockIdx.x; tile < tiles && !failed; tile += gridDim.x, ++local) {
                const int buf = int(local & 1);
                if (!mbar_wait_bounded(acc_empty + buf, uint32_t(((local >> 1) & 1) ^ 1))) {
                    atomicOr(&failed, 1);
                    break;
                }
                tc_fence_after();
                const uint32_t acc = tmem + uint32_t(buf * MOE_BN);
                for (int i = 0; i < kt; ++i, ++it) {
                    const int s = int(it % MOE_STAGES);
                    if (!mbar_wait_bounded(full + s, uint32_t((it / MOE_STAGES) & 1))) {
                        atomicOr(&failed, 1);
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = smem_addr(base + s * MOE_STAGE_BYTES);
                    const uint64_t da = sw128_desc(sa), db = sw128_desc(sa + MOE_A_BYTES);
#pragma unroll
                    for (int kk = 0; kk < MOE_BK / 16; ++kk)
                        umma_f16(acc, da + uint64_t(2 * kk), db + uint64_t(2 * kk), IDESC, (i | kk) != 0);
                    umma_commit(empty + s);
                }
                umma_commit(acc_full + buf);
            }
        }
    } else {
        const int q = warp & 3;            // TMEM lane quarter this warp may read
        const int cg = (warp - 2) / 4;     // its quarter of the tile's columns
        int64_t local = 0;
        for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++local) {
            const int buf = int(local & 1);
            if (!mbar_wait_bounded(acc_full + buf, uint32_t((local >> 1) & 1))) {
                atomicOr(&failed, 1);
                break;
            }
            tc_fence_after();
            int e, r0, r1, nt;
            coords(tile, e, r0, r1, nt);
            const int row = r0 + 32 * q + lane;
            const uint32_t tb0 = tmem + (uint32_t(32 * q) << 16) + uint32_t(buf * MOE_BN);
            if (MODE == MOE_SWIGLU) {
                // columns [0,128) gate, [128,256) up of output columns nt*128 + [0,128):
                // this warp's block c = cg of each
                for (int c = cg; c < cg + 1; ++c) {
                    uint32_t g[32], u[32];
                    tmem_ld32(tb0 + uint32_t(c * 32), g);
                    tmem_ld32(tb0 + uint32_t(128 + c * 32), u);
                    if (row < r1) {
                        float mid[32];
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            const float gv = bf16r(__uint_as_float(g[j]));
                            const float uv = bf16r(__uint_as_float(u[j]));
                            mid[j] = bf16r(silu_bf16(gv) * uv);
                        }
                        const int64_t col = int64_t(nt) * 128 + c * 32;
                        if (!a.q8) {  // 16-byte stores: 4 per row chunk
                            uint4 *dst = reinterpret_cast<uint4 *>(static_cast<__nv_bfloat16 *>(a.mid) +
                                                                   int64_t(row) * a.I + col);
#pragma unroll
                            for (int j = 0; j < 32; j += 8) {
                                uint4 v;
                                __nv_bfloat162 h[4];
#pragma unroll
                                for (int u = 0; u < 4; ++u) h[u] = __floats2bfloat162_rn(mid[j + 2 * u], mid[j + 2 * u + 1]);
                                memcpy(&v, h, 16);
                                dst[j / 8] = v;
                            }
                        } else {
                            // this thread's 32 values are one Q8_0 block of the row
                            float amax = 0.0f;
#pragma unroll
                            for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(mid[j]));
                            const float d = __fdiv_rn(amax, 127.0f);
                            float id;
                            if (a.rounding == 2) id = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
                            else id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
                            const float dh = __half2float(__float2half_rn(d));
                            uint4 *dst = reinterpret_cast<uint4 *>(static_cast<__half *>(a.mid) + int64_t(row) * a.I + col);
#pragma unroll
                            for (int j = 0; j < 32; j += 8) {
                                __half hv[8];
#pragma unroll
                                for (int u = 0; u < 8; ++u) {
                                    const float sv = __fmul_rn(mid[j + u], id);
                                    const int qv = a.rounding == 0 ? int(roundf(sv)) : __float2int_rn(sv);
                                    hv[u] = __float2half_rn(__fmul_rn(float(qv), dh));
                                }
                                uint4 v;
                                memcpy(&v, hv, 16);
                                dst[j / 8] = v;
                            }
                        }
                    }
                }
            } else {
                const float w = row < r1 ? a.topk_w[a.perm[row]] : 0.0f;
                for (int c = 2 * cg; c < 2 * cg + 2; ++c) {   // this warp's two 32-column blocks
                    uint32_t r[32];
                    tmem_ld32(tb0 + uint32_t(c * 32), r);
                    if (row < r1) {  // 16-byte stores: 4 per row chunk
                        uint4 *dst = reinterpret_cast<uint4 *>(a.y + int64_t(row) * (int64_t(a.n_tiles) * MOE_BN) +
                                                               int64_t(nt) * MOE_BN + c * 32);
#pragma unroll
                        for (int j = 0; j < 32; j += 8) {
                            __nv_bfloat162 h[4];
#pragma unroll
                            for (int u = 0; u < 4; ++u)
                                h[u] = __floats2bfloat162_rn(__uint_as_float(r[j + 2 * u]) * w,
                                                             __uint_as_float(r[j + 2 * u + 1]) * w);
                            uint4 v;
                            memcpy(&v, h, 16);
                            dst[j / 8] = v;
                        }
                    }
                }
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
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512u) : "memory");
    }
}

// ------------------------------------------------------------------ weight preparation
// w1 rows interleaved per 256-row tile: tile j = gate rows [128j, 128j+128)
// then up rows [I + 128j, ...); values fp16(q*d) (Q8_0) or the bf16 input.
__global__ void k_moe_prep_w1(const void *__restrict__ src, int q8, int E, int I, int H, void *__restrict__ dst) {
    const int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;  // element of dst [E][2I][H]
    if (i >= int64_t(E) * 2 * I * H) return;
    const int64_t k = i % H, r = (i / H) % (2 * I), e = i / (int64_t(H) * 2 * I);
    const int64_t tile = r / 256, within = r % 256;
    const int64_t srow = within < 128 ? tile * 128 + within : I + tile * 128 + (within - 128);
    const int64_t s_elem = (e * 2 * I + srow) * H + k;
    if (!q8) {
        static_cast<__nv_bfloat16 *>(dst)[i] = static_cast<const __nv_bfloat16 *>(src)[s_elem];
        return;
    }
    const uint8_t *blk = static_cast<const uint8_t *>(src) + ((e * 2 * I + srow) * (H / QK) + k / QK) * Q8_BYTES;
    const float d = __half2float(__ushort_as_half(uint16_t(blk[0]) | uint16_t(uint16_t(blk[1]) << 8)));
    static_cast<__half *>(dst)[i] = __float2half_rn(__fmul_rn(float(int8_t(blk[2 + k % QK])), d));
}

__global__ void k_moe_prep_w2(const void *__restrict__ src, int q8, int64_t count, int K, void *__restrict__ dst) {
    const int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;  // element of [E*H][I]
    if (i >= count) return;
    if (!q8) {
        static_cast<__nv_bfloat16 *>(dst)[i] = static_cast<const __nv_bfloat16 *>(src)[i];
        return;
    }
    const int64_t row = i / K, k = i % K;
    const uint8_t *blk = static_cast<const uint8_t *>(src) + (row * (K / QK) + k / QK) * Q8_BYTES;
    const float d = __half2float(__ushort_as_half(uint16_t(blk[0]) | uint16_t(uint16_t(blk[1]) << 8)));
    static_cast<__half *>(dst)[i] = __float2half_rn(__fmul_rn(float(int8_t(blk[2 + k % QK])), d));
}

// 2-D 16-bit tensor map (bf16 or fp16) over [rows][k], box 64 x box_rows, 128B swizzle
static PFN_cuTensorMapEncodeTiled_v12000 moe_encode() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        cuda_check(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q), "tensor map lookup");
        require(p && q == cudaDriverEntryPointSuccess, "cuTensorMapEncodeTiled is unavailable");
        fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

static void make_map16(CUtensorMap *map, const void *ptr, int64_t rows, int64_t k, int box_rows, bool bf16) {
    require(uintptr_t(ptr) % 16 == 0 && (k * 2) % 16 == 0, "MoE operand must be 16-byte aligned");
    const cuuint64_t dims[2] = {cuuint64_t(k), cuuint64_t(rows)};
    const cuuint64_t strides[1] = {cuuint64_t(k * 2)};
    const cuuint32_t box[2] = {cuuint32_t(MOE_BK), cuuint32_t(box_rows)};
    const cuuint32_t es[2] = {1, 1};
    const CUresult r = moe_encode()(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                                    const_cast<void *>(ptr), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    require(r == CUDA_SUCCESS, "MoE tensor map encoding failed");
}

struct Moe {
    int q8 = 0, E = 0, I = 0, H = 0, topk = 0, max_tokens = 0, max_tiles = 0;
    void *w1 = nullptr, *w2 = nullptr;   // prepared 16-bit weights
    void *xp = nullptr, *mid = nullptr;  // permuted activations / intermediate
    __half *xs = nullptr;                // Q8_0 experts: the tokens' staged rows, before the permutation
    __nv_bfloat16 *y = nullptr;          // per-pair down outputs
    int *ibuf = nullptr;                 // counts, offsets, cursor, tiles, num_tiles, perm, inv
    int *status = nullptr;
    MoePlan plan{};
    CUtensorMap map_w1{}, map_w2{}, map_x{}, map_mid{};
    std::atomic_flag busy = ATOMIC_FLAG_INIT;
    ~Moe() {
        for (void *p : {w1, w2, xp, mid, (void *)xs, (void *)y, (void *)ibuf, (void *)status})
            if (p) cudaFree(p);
    }
};

static int moe_sms() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

template <int MODE, bool BF16>
static void launch_moe_gemm(const CUtensorMap &ta, const CUtensorMap &tb, const MoeGemmArgs &a, int max_tiles,
                            cudaStream_t s) {
    auto kernel = k_moe_gemm<MODE, BF16>;
    static bool configured = false;
    if (!configured) {
        cuda_check(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(MOE_SMEM)),
                   "MoE GEMM shared memory");
        configured = true;
    }
    const int64_t upper = int64_t(max_tiles) * a.n_tiles;
    const unsigned grid = unsigned(upper < moe_sms() ? upper : moe_sms());
    kernel<<<grid, MOE_THREADS, MOE_SMEM, s>>>(ta, tb, a);
}

}  // namespace mb

using namespace mb;

extern "C" {

int mstar_b200_moe_route(const void *x, int64_t tokens, int64_t hidden, const void *router_weight, int32_t experts,
                         int32_t top_k, int32_t renormalize, float *logits, float *topk_weights, int32_t *topk_ids,
                         void *stream, char *error, size_t error_size) {
    try {
        require(x && router_weight && logits && topk_weights && topk_ids, "missing router operand");
        require(tokens >= 1 && hidden >= 1 && experts >= 1 && experts <= 256, "router geometry: 1..256 experts");
        require(top_k >= 1 && top_k <= MOE_MAX_TOPK && top_k <= experts, "top_k outside 1..8");
        check_device(x, "router input");
        check_device(router_weight, "router weight");
        check_device(topk_weights, "top-k weights");
        check_device(topk_ids, "top-k ids");
        require(hidden % 8 == 0 && uintptr_t(x) % 16 == 0 && uintptr_t(router_weight) % 16 == 0,
                "router rows must be 16-byte aligned");
        const size_t smem = size_t(ROUTER_TOKENS) * hidden * 2;
        require(smem <= 200 * 1024, "router token tile exceeds shared memory");
        static bool configured = false;
        if (!configured) {
            cuda_check(cudaFuncSetAttribute(k_router_logits<8, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            200 * 1024),
                       "router shared memory");
            cuda_check(cudaFuncSetAttribute(k_router_logits<8, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            200 * 1024),
                       "router shared memory");
            configured = true;
        }
        check_device(logits, "router logits");
        cudaStream_t s = as_stream(stream);
        const int epw = tokens < 512 ? 1 : 4;   // experts per warp (8 warps per CTA)
        const dim3 grid(unsigned(ceil_div(tokens, ROUTER_TOKENS)), unsigned(ceil_div(experts, 8 * epw)));
        auto logits_kernel = epw == 1 ? k_router_logits<8, 1> : k_router_logits<8, 4>;
        logits_kernel<<<grid, 256, smem, s>>>(static_cast<const __nv_bfloat16 *>(x),
                                                     static_cast<const __nv_bfloat16 *>(router_weight), int(tokens),
                                                     int(hidden), experts, logits);
        k_router_topk<<<unsigned(ceil_div(tokens, 8)), 256, 0, s>>>(logits, int(tokens), experts, top_k, renormalize,
                                                                   topk_weights, topk_ids);
        cuda_check(cudaGetLastError(), "router launch");
        return 0;
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return -1;
    }
}

void *mstar_b200_moe_create(int32_t format, const void *w1, uint64_t w1_bytes, const void *w2, uint64_t w2_bytes,
                            int32_t experts, int32_t intermediate, int32_t hidden, int32_t top_k, int32_t max_tokens,
                            char *error, size_t error_size) {
    std::unique_ptr<Moe> m;
    try {
        require(mstar_b200_capability() == 1, "sm_100a device capability is unavailable");
        require(format == MSTAR_B200_Q8_0 || format == MSTAR_B200_BF16, "MoE weights are Q8_0 or BF16");
        require(experts >= 1 && experts <= 1024 && intermediate % 128 == 0 && intermediate > 0 && hidden % 256 == 0 &&
                    hidden > 0 && top_k >= 1 && top_k <= MOE_MAX_TOPK && max_tokens >= 1,
                "MoE geometry: I multiple of 128, H multiple of 256, 1 <= top_k <= 8");
        m.reset(new Moe);
        m->q8 = format == MSTAR_B200_Q8_0;
        m->E = experts;
        m->I = intermediate;
        m->H = hidden;
        m->topk = top_k;
        m->max_tokens = max_tokens;
        const int64_t E = experts, I = intermediate, H = hidden, P = int64_t(max_tokens) * top_k;
        const uint64_t w1_expect = m->q8 ? uint64_t(E * 2 * I * (H / QK) * Q8_BYTES) : uint64_t(E * 2 * I * H * 2);
        const uint64_t w2_expect = m->q8 ? uint64_t(E * H * (I / QK) * Q8_BYTES) : uint64_t(E * H * I * 2);
        check_range({w1, w1_bytes}, w1_expect, 2, "expert w1");
        check_range({w2, w2_bytes}, w2_expect, 2, "expert w2");
        check_device(w1, "expert w1");
        check_device(w2, "expert w2");
        m->max_tiles = int(P / MOE_BM + E + 1);
        cuda_check(cudaMalloc(&m->w1, size_t(E * 2 * I * H * 2)), "w1 allocation");
        cuda_check(cudaMalloc(&m->w2, size_t(E * H * I * 2)), "w2 allocation");
        cuda_check(cudaMalloc(&m->xp, size_t((P + MOE_BM) * H * 2)), "permuted activations");
        cuda_check(cudaMalloc(&m->mid, size_t((P + MOE_BM) * I * 2)), "intermediate");
        if (m->q8)
            cuda_check(cudaMalloc(reinterpret_cast<void **>(&m->xs), size_t(int64_t(max_tokens) * H * 2)),
                       "staged token rows");
        cuda_check(cudaMalloc(reinterpret_cast<void **>(&m->y), size_t(P * H * 2)), "expert outputs");
        const int64_t ints = 3 * E + 3 * int64_t(m->max_tiles) + 1 + 2 * P + 1;
        cuda_check(cudaMalloc(reinterpret_cast<void **>(&m->ibuf), size_t(ints * 4)), "plan buffers");
        cuda_check(cudaMalloc(reinterpret_cast<void **>(&m->status), 4), "status");
        cuda_check(cudaMemset(m->status, 0, 4), "status reset");
        cuda_check(cudaMemset(m->xp, 0, size_t((P + MOE_BM) * H * 2)), "activation reset");
        cuda_check(cudaMemset(m->mid, 0, size_t((P + MOE_BM) * I * 2)), "intermediate reset");
        int *p = m->ibuf;
        m->plan.counts = p;
        m->plan.offsets = p + E;
        m->plan.cursor = p + 2 * E;
        m->plan.tiles = p + 3 * E;
        m->plan.num_tiles = p + 3 * E + 3 * m->max_tiles;
        m->plan.perm = m->plan.num_tiles + 1;
        m->plan.inv = m->plan.perm + P;
        m->plan.valid = m->plan.inv + P;
        cuda_check(cudaMemset(m->ibuf, 0, size_t(ints * 4)), "plan reset");
        const int64_t n1 = E * 2 * I * H, n2 = E * H * I;
        k_moe_prep_w1<<<unsigned(ceil_div(n1, 256)), 256>>>(w1, m->q8, int(E), int(I), int(H), m->w1);
        k_moe_prep_w2<<<unsigned(ceil_div(n2, 256)), 256>>>(w2, m->q8, n2, int(I), m->w2);
        cuda_check(cudaGetLastError(), "weight preparation");
        cuda_check(cudaDeviceSynchronize(), "weight preparation");
        const bool bf16 = !m->q8;
        make_map16(&m->map_w1, m->w1, E * 2 * I, H, MOE_BN, bf16);
        make_map16(&m->map_w2, m->w2, E * H, I, MOE_BN, bf16);
        make_map16(&m->map_x, m->xp, P + MOE_BM, H, MOE_BM, bf16);
        make_map16(&m->map_mid, m->mid, P + MOE_BM, I, MOE_BM, bf16);
        return m.release();
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return nullptr;
    }
}

}  // extern "C"

namespace mb {

// Routing plan, permuted activations and both grouped GEMMs of one call: expert
// rows land in y at their permuted positions (y rows [0, pairs with a held
// expert)); plan.inv maps each (token, slot) pair to its row, or -1.
static void moe_experts(Moe &m, const void *x, int64_t tokens, const float *topk_weights, const int32_t *topk_ids,
                        int e0, int e_total, __nv_bfloat16 *y, int32_t *status, int32_t rounding, bool vec,
                        cudaStream_t s) {
    const int P = int(tokens) * m.topk;
    cuda_check(cudaMemsetAsync(status, 0, 4, s), "status reset");
    cuda_check(cudaMemsetAsync(m.plan.counts, 0, size_t(m.E) * 4, s), "count reset");
    k_moe_count<<<unsigned(ceil_div(P, 256)), 256, 0, s>>>(topk_ids, P, m.E, e0, e_total, m.plan.counts, status);
    k_moe_plan<<<1, 256, 0, s>>>(m.plan, m.E, m.max_tiles);
    k_moe_scatter<<<unsigned(ceil_div(P, 256)), 256, 0, s>>>(topk_ids, P, m.E, e0, e_total, m.plan);
    if (vec && m.q8) {
        // each token's Q8_0 staging once (not once per routed pair), then a 16-byte row copy
        launch_stage_rows_bf16(rounding, x, tokens, m.H, m.xs, nullptr, s);
        k_moe_gather_vec<<<unsigned(P), 256, 0, s>>>(m.xs, m.plan.perm, m.plan.valid, P, m.H, m.topk, m.xp);
    } else if (vec)
        k_moe_gather_vec<<<unsigned(P), 256, 0, s>>>(x, m.plan.perm, m.plan.valid, P, m.H, m.topk, m.xp);
    else
        k_moe_gather<<<unsigned(P), 256, 0, s>>>(static_cast<const __nv_bfloat16 *>(x), m.plan.perm, m.plan.valid,
                                                 P, m.H, m.topk, m.q8, rounding, m.xp);
    MoeGemmArgs g{};
    g.tiles = m.plan.tiles;
    g.num_tiles = m.plan.num_tiles;
    g.status = status;
    g.q8 = m.q8;
    g.rounding = rounding;
    g.perm = m.plan.perm;
    g.topk_w = topk_weights;
    // gate/up: N = 2I rows per expert, output I columns of mid
    g.n_tiles = 2 * m.I / MOE_BN;
    g.w_rows = 2 * m.I;
    g.K = m.H;
    g.mid = m.mid;
    g.I = m.I;
    if (m.q8) launch_moe_gemm<MOE_SWIGLU, false>(m.map_x, m.map_w1, g, m.max_tiles, s);
    else launch_moe_gemm<MOE_SWIGLU, true>(m.map_x, m.map_w1, g, m.max_tiles, s);
    // down: N = H rows per expert, K = I
    g.n_tiles = m.H / MOE_BN;
    g.w_rows = m.H;
    g.K = m.I;
    g.y = y;
    if (m.q8) launch_moe_gemm<MOE_DOWN, false>(m.map_mid, m.map_w2, g, m.max_tiles, s);
    else launch_moe_gemm<MOE_DOWN, true>(m.map_mid, m.map_w2, g, m.max_tiles, s);
}

// out_inv[i] = inv[i] + row_base for a held pair, -1 otherwise
__global__ void k_moe_inv_out(const int *__restrict__ inv, int P, int64_t row_base, int32_t *__restrict__ out_inv) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= P) return;
    const int r = inv[i];
    out_inv[i] = r < 0 ? -1 : int32_t(row_base + r);
}

}  // namespace mb

extern "C" {

int mstar_b200_moe_run(void *handle, const void *x, int64_t tokens, const float *topk_weights,
                       const int32_t *topk_ids, void *out, int32_t *status, int32_t rounding, void *stream,
                       char *error, size_t error_size) {
    try {
        require(handle, "missing MoE handle");
        auto &m = *static_cast<Moe *>(handle);
        require(!m.busy.test_and_set(std::memory_order_acquire), "MoE handle is busy");
        struct Release {
            std::atomic_flag &f;
            ~Release() { f.clear(std::memory_order_release); }
        } release{m.busy};
        require(tokens >= 1 && tokens <= m.max_tokens, "token count outside the prepared capacity");
        require(rounding >= 0 && rounding <= 2, "unknown Q8_0 activation rounding");
        require(x && topk_weights && topk_ids && out && status, "missing MoE operand");
        const uint64_t xb = uint64_t(tokens) * m.H * 2;
        require(disjoint({x, xb}, {out, xb}), "MoE output overlaps its input");
        for (const void *p : {x, (const void *)topk_weights, (const void *)topk_ids, (const void *)out,
                              (const void *)status})
            check_device(p, "MoE operand");
        cudaStream_t s = as_stream(stream);
        const bool vec = uintptr_t(x) % 16 == 0 && uintptr_t(out) % 16 == 0 && m.H % 128 == 0;
        moe_experts(m, x, tokens, topk_weights, topk_ids, 0, m.E, m.y, status, rounding, vec, s);
        if (vec)
            k_moe_combine_vec<<<unsigned(tokens), 256, 0, s>>>(m.y, m.plan.inv, int(tokens), m.H, m.topk,
                                                               static_cast<__nv_bfloat16 *>(out));
        else
            k_moe_combine<<<unsigned(tokens), 256, 0, s>>>(m.y, m.plan.inv, int(tokens), m.H, m.topk,
                                                           static_cast<__nv_bfloat16 *>(out));
        cuda_check(cudaGetLastError(), "MoE launch");
        return 0;
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return -1;
    }
}

int mstar_b200_moe_run_experts(void *handle, const void *x, int64_t tokens, const float *topk_weights,
                               const int32_t *topk_ids, int32_t expert0, int32_t experts_total, void *y,
                               int64_t y_rows, int64_t row_base, int32_t *inv, int32_t *status, int32_t rounding,
                               void *stream, char *error, size_t error_size) {
    try {
        require(handle, "missing MoE handle");
        auto &m = *static_cast<Moe *>(handle);
        require(!m.busy.test_and_set(std::memory_order_acquire), "MoE handle is busy");
        struct Release {
            std::atomic_flag &f;
            ~Release() { f.clear(std::memory_order_release); }
        } release{m.busy};
        require(tokens >= 1 && tokens <= m.max_tokens, "token count outside the prepared capacity");
        require(rounding >= 0 && rounding <= 2, "unknown Q8_0 activation rounding");
        require(expert0 >= 0 && experts_total >= m.E && int64_t(expert0) + m.E <= experts_total,
                "the held experts must lie inside [0, experts_total)");
        require(x && topk_weights && topk_ids && y && inv && status, "missing MoE operand");
        const int64_t P = tokens * m.topk;
        require(row_base >= 0 && y_rows >= row_base + P && y_rows <= (int64_t(1) << 31) - 1,
                "expert output rows outside the given buffer");
        require(uintptr_t(y) % 16 == 0 && uintptr_t(x) % 16 == 0, "x and y must be 16-byte aligned");
        const uint64_t xb = uint64_t(tokens) * m.H * 2;
        require(disjoint({x, xb}, {y, uint64_t(y_rows) * m.H * 2}), "expert outputs overlap the input");
        for (const void *p : {x, (const void *)topk_weights, (const void *)topk_ids, (const void *)y,
                              (const void *)inv, (const void *)status})
            check_device(p, "MoE operand");
        cudaStream_t s = as_stream(stream);
        const bool vec = m.H % 128 == 0;
        moe_experts(m, x, tokens, topk_weights, topk_ids, expert0, experts_total,
                    static_cast<__nv_bfloat16 *>(y) + row_base * m.H, status, rounding, vec, s);
        k_moe_inv_out<<<unsigned(ceil_div(P, 256)), 256, 0, s>>>(m.plan.inv, int(P), row_base, inv);
        cuda_check(cudaGetLastError(), "MoE launch");
        return 0;
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return -1;
    }
}

int mstar_b200_moe_combine(const void *y, int64_t y_rows, const int32_t *rows, int64_t tokens, int32_t top_k,
                           int64_t hidden, void *out, void *stream, char *error, size_t error_size) {
    try {
        require(y && rows && out, "missing combine operand");
        require(tokens >= 1 && tokens <= (int64_t(1) << 24) && top_k >= 1 && top_k <= MOE_MAX_TOPK && hidden >= 1 &&
                    hidden <= 65536 && y_rows >= 0 && y_rows <= (int64_t(1) << 31),
                "invalid combine geometry");
        check_device(y, "expert outputs");
        check_device(rows, "slot rows");
        check_device(out, "combined output");
        cudaStream_t s = as_stream(stream);
        if (uintptr_t(y) % 16 == 0 && uintptr_t(out) % 16 == 0 && hidden % 8 == 0)
            k_moe_combine_rows_vec<<<unsigned(tokens), 256, 0, s>>>(static_cast<const __nv_bfloat16 *>(y), y_rows,
                                                                    rows, int(tokens), int(hidden), top_k,
                                                                    static_cast<__nv_bfloat16 *>(out));
        else
            k_moe_combine_rows<<<unsigned(tokens), 256, 0, s>>>(static_cast<const __nv_bfloat16 *>(y), y_rows, rows,
                                                                int(tokens), int(hidden), top_k,
                                                                static_cast<__nv_bfloat16 *>(out));
        cuda_check(cudaGetLastError(), "combine launch");
        return 0;
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return -1;
    }
}

int mstar_b200_moe_dispatch(const void *x, int64_t tokens, int64_t hidden, const float *topk_weights,
                            const int32_t *topk_ids, int32_t top_k, int32_t experts, int32_t ranks, int64_t *meta,
                            void *rows, int32_t *pairs, int32_t *inverse, void *stream, char *error,
                            size_t error_size) {
    try {
        require(tokens >= 0 && tokens <= (int64_t(1) << 24) && top_k >= 1 && top_k <= MOE_MAX_TOPK &&
                    hidden >= 1 && hidden <= 65536,
                "invalid dispatch geometry");
        require(ranks >= 1 && ranks <= EP_MAX_RANKS && experts >= ranks && experts % ranks == 0,
                "experts must divide evenly over 1..32 ranks");
        require(meta, "missing dispatch meta");
        check_device(meta, "dispatch meta");
        cudaStream_t s = as_stream(stream);
        const int P = int(tokens) * top_k;
        if (P > 0) {
            require(x && topk_weights && topk_ids && rows && pairs && inverse, "missing dispatch operand");
            for (const void *q : {x, (const void *)topk_weights, (const void *)topk_ids, (const void *)rows,
                                  (const void *)pairs, (const void *)inverse})
                check_device(q, "dispatch operand");
            const uint64_t xb = uint64_t(tokens) * hidden * 2, rb = uint64_t(P) * hidden * 2;
            require(disjoint({x, xb}, {rows, rb}), "dispatch rows overlap x");
        }
        k_ep_plan<<<1, EP_THREADS, 0, s>>>(topk_ids, topk_weights, P, experts / ranks, experts, ranks, meta, pairs,
                                            inverse);
        if (P > 0) {
            const int vec = uintptr_t(x) % 16 == 0 && uintptr_t(rows) % 16 == 0 && hidden % 8 == 0;
            k_ep_rows<<<unsigned(P), 256, 0, s>>>(static_cast<const __nv_bfloat16 *>(x), inverse, P, int(hidden),
                                                  top_k, vec, static_cast<__nv_bfloat16 *>(rows));
        }
        cuda_check(cudaGetLastError(), "dispatch launch");
        return 0;
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return -1;
    }
}

int mstar_b200_moe_close(void *handle, char *error, size_t error_size) {
    try {
        if (handle) {
            auto *m = static_cast<Moe *>(handle);
            require(!m->busy.test_and_set(std::memory_order_acquire), "cannot close a busy MoE handle");
            cudaDeviceSynchronize();
            delete m;
        }
        return 0;
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return -1;
    }
}

}  // extern "C"
