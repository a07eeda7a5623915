// One Whisper decoder greedy step as ONE persistent kernel (cooperative launch,
// one CTA per SM): embedding, four layers of (LayerNorm + Q8_0 quantization,
// fused QKV GEMV, causal self attention with the K/V append, out_proj +
// residual, LayerNorm, cross-query GEMV, split-key cross attention and merge,
// out_proj + residual, LayerNorm, fc1 + GELU, fc2 + residual), the final
// LayerNorm and the Q4_0 / Q8_0 vocab readout with suppression and the
// first-index argmax (backends/cpu_ggml/decoder.cpp:489-600, 683-696).
//
// Phases are separated by a grid barrier (a counter and a generation word in
// global memory; every wait is bounded and a timeout sets status bit value 32)
// instead of kernel boundaries, so the step is one launch instead of ~60. The
// arithmetic of every phase is the one of the multi-kernel path, element for
// element (the same fragment quantization, the same block-ordered fp32 folds,
// the same attention tiles), so both paths produce identical logits.
#include <cmath>
#include <memory>
#include <vector>

#include "../../include/mstar_b200.h"
#include "attend.cuh"
#include "gemv_dev.cuh"
#include "linear_handle.cuh"
#include "quant.cuh"

namespace mb {

constexpr int STEP_THREADS = 256, STEP_WARPS = STEP_THREADS / 32;
constexpr int STEP_MAX_LAYERS = 8;
constexpr long long STEP_SPIN_LIMIT = 1ll << 24;  // polls of 64 ns before a barrier gives up (about 1 s)

struct StepLinear {
    const uint4 *wq;
    const __half2 *ws;
    const float *bias;
    int64_t groups, nb, nb_pad, n;
    int q4;
};

enum { L_QKV = 0, L_OUT, L_CQ, L_COUT, L_FC1, L_FC2 };

struct StepLayer {
    StepLinear lin[6];
    const float *ln[6];  // ln1 w, b; ln2 w, b; ln3 w, b
    __half *self_k, *self_v, *cross_k, *cross_v;
};

struct StepArgs {
    int B, L, d, heads, ffn, target, source, shared, mtiles, rounding;
    float eps, scale;
    const float *tok, *pos;
    int64_t vocab, npos;
    StepLayer layer[STEP_MAX_LAYERS];
    StepLinear head;
    const float *lnf_w, *lnf_b;
    const int64_t *suppressed;
    int64_t nsup;
    const int64_t *tokens, *positions, *cross_len;
    float *logits;
    int64_t *next;
    float *x, *qkv, *att, *cq, *h;
    uint32_t *xf;
    float *xs;
    int *xsum;
    float *part;
    unsigned long long *keys;  // [32] argmax keys, zero between steps
    unsigned int *bar;         // [2] arrivals, generation
    int *status;
    long long spin_limit;      // polls of a grid barrier before it gives up
    const uint16_t *gelu;
};

// ------------------------------------------------------------------ barrier
// Grid barrier: an arrival counter and a generation word in global memory
// (bar[0], bar[1]); the last CTA to arrive resets the counter and advances the
// generation, the others watch it. Every wait is bounded; a timeout sets status
// bit value 32. (One arrival slot per CTA watched by CTA 0 measured slower:
// about 4.5 us against 3 us per barrier.)
__device__ __forceinline__ void grid_barrier(unsigned int *bar, unsigned int &gen, int *status, long long limit) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned int g = gen;
        if (atomicAdd(bar, 1u) == gridDim.x - 1) {
            atomicExch(bar, 0u);
            __threadfence();
            atomicAdd(bar + 1, 1u);
        } else {
            long long n = 0;
            unsigned int v;
            for (;;) {
                asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(bar + 1) : "memory");
                if (v != g) break;
                if (++n > limit) {
                    atomicOr(status, 32);
                    break;
                }
                __nanosleep(64);
            }
        }
        __threadfence();
        gen = g + 1;
    }
    __syncthreads();
}

// Self-test of the barrier's timeout: a grid of two CTAs where CTA 1 leaves
// without arriving, so CTA 0's wait runs out after `limit` polls and sets
// status bit value 32 (bar: two zeroed words).
__global__ void k_grid_barrier_selftest(unsigned int *bar, int *status, long long limit) {
    if (blockIdx.x != 0) return;
    unsigned int gen = 0;
    grid_barrier(bar, gen, status, limit);
}

void launch_grid_barrier_selftest(unsigned int *bar, int *status, long long limit, cudaStream_t s) {
    k_grid_barrier_selftest<<<2, 32, 0, s>>>(bar, status, limit);
}

// ------------------------------------------------------------------ activations -> A fragments
// frag_block (quant.cuh) writes one 32-element block of a token.

// LayerNorm statistics of one token row, in k_quantize_frag's block order
// exactly (virtual threads v = 32 w + lane of a 128 / 256-thread block, a warp
// reduction per virtual warp, then the warps' partials in order).
__device__ __forceinline__ void ln_stats(const float *xr, int64_t K, float eps, float &mean, float &rstd) {
    const int lane = threadIdx.x & 31;
    const int vwarps = K >= 1024 ? 8 : 4, vthreads = 32 * vwarps;
    float sum = 0.0f;
    for (int w = 0; w < vwarps; ++w) {
        float s = 0.0f;
        for (int64_t i = 32 * w + lane; i < K; i += vthreads) s += xr[i];
#pragma unroll
        for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        sum += s;
    }
    mean = sum / float(K);
    float var = 0.0f;
    for (int w = 0; w < vwarps; ++w) {
        float s = 0.0f;
        for (int64_t i = 32 * w + lane; i < K; i += vthreads) {
            const float y = xr[i] - mean;
            s = fmaf(y, y, s);
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        var += s;
    }
    rstd = 1.0f / sqrtf(var / float(K) + eps);
}

// Quantize the live token rows (and zero the padding tokens) of x [B][K] for the
// linear that consumes them (its padded block count nb_pad): one warp per
// (token, block) task over the whole grid; with a LayerNorm every task
// recomputes its token's statistics (the same values for every block).
template <int MODE>
__device__ void phase_quant(const StepArgs &a, const float *x, int64_t K, const float *lnw, const float *lnb,
                            int64_t nb_pad) {
    const int lane = threadIdx.x & 31;
    const int64_t W = int64_t(gridDim.x) * STEP_WARPS;
    const int mpad = a.mtiles * 16;
    const int64_t nb = K / QK;
    for (int64_t task = int64_t(blockIdx.x) * STEP_WARPS + (threadIdx.x >> 5); task < mpad * nb_pad; task += W) {
        const int token = int(task / nb_pad);
        const int64_t b = task % nb_pad;
        const bool live = token < a.B && b < nb;
        const float *xr = x + int64_t(token) * K;
        float v = 0.0f;
        if (live) {
            v = xr[b * QK + lane];
            if (lnw) {
                float mean, rstd;
                ln_stats(xr, K, a.eps, mean, rstd);
                const int64_t i = b * QK + lane;
                v = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v, mean), rstd), __ldg(lnw + i)), __ldg(lnb + i));
            }
        }
        frag_block<MODE>(v, live, b, token, a.mtiles, a.xf, a.xs, a.xsum, a.status);
    }
}

// ------------------------------------------------------------------ GEMV phases
struct StepSmem {
    uint4 *xf;
    float *xs;
    int *xsum;
    float4 *terms;
    unsigned long long *best;
};

template <int MT>
__device__ __forceinline__ void stage(const StepArgs &a, int64_t nb_pad, const StepSmem &s) {
    constexpr int MPAD = MT * 16;
    const int64_t nf = nb_pad * MT * 32;
    for (int64_t i = threadIdx.x; i < nf; i += blockDim.x) s.xf[i] = reinterpret_cast<const uint4 *>(a.xf)[i];
    for (int64_t i = threadIdx.x; i < nb_pad * MPAD; i += blockDim.x) {
        s.xs[i] = a.xs[i];
        s.xsum[i] = a.xsum[i];
    }
    __syncthreads();
}

struct Epi {
    float *out;
    int64_t ldo;
    const float *residual;  // [m][ldo] or null
    bool gelu;
};

__device__ __forceinline__ float epilogue(const StepArgs &a, const StepLinear &L, const Epi &e, int m, int64_t n,
                                          float v) {
    if (L.bias) v = __fadd_rn(v, __ldg(L.bias + n));
    if (e.gelu) v = gelu_ggml(v, a.gelu);
    if (e.residual) v = __fadd_rn(e.residual[m * e.ldo + n], v);
    e.out[m * e.ldo + n] = v;
    return v;
}

// Weights of this CTA's first row group for this warp's chunk range, loaded
// before the barrier that precedes the phase (they do not depend on it).
constexpr int PRE_CHUNKS = 3;  // chunks per warp: K <= 3 * 8 * 2 * 32 = 1536 for Q8_0
struct Pre {
    uint4 w[PRE_CHUNKS];
    __half2 sc[PRE_CHUNKS][2];
};

__device__ __forceinline__ void prefetch_gemv(const StepLinear &L, Pre &p) {
    constexpr int BPC = 2;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, t = lane & 3;
    const int64_t G = blockIdx.x;
    if (G >= L.groups) return;
    const int nb_pad = int(L.nb_pad), chunks = nb_pad / BPC, cpw = (chunks + STEP_WARPS - 1) / STEP_WARPS;
    const int c0 = warp * cpw, c1 = min(c0 + cpw, chunks);
#pragma unroll
    for (int i = 0; i < PRE_CHUNKS; ++i) {
        const int c = c0 + i;
        if (c < c1) {
            p.w[i] = ldg_stream(L.wq + (G * chunks + c) * 32 + lane);
#pragma unroll
            for (int j = 0; j < BPC; ++j) p.sc[i][j] = __ldg(L.ws + G * int64_t(nb_pad) * 4 + t + (c * BPC + j) * 4);
        }
    }
}

// Split-K GEMV (Q8_0 weights) over the row groups assigned to this CTA: the 8
// warps share a group's chunks; the per-block terms are folded in block order
// in shared memory (k_gemv's split path). `pre` holds the first group's weights.
template <int MT>
__device__ void phase_gemv(const StepArgs &a, const StepLinear &L, const Epi &e, const StepSmem &s, const Pre &pre) {
    constexpr bool Q4 = false;
    constexpr int BPC = 2;
    constexpr int MPAD = MT * 16;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, t = lane & 3;
    const int nb_pad = int(L.nb_pad), nb = int(L.nb), m_live = a.B;
    const int chunks = nb_pad / BPC, cpw = (chunks + STEP_WARPS - 1) / STEP_WARPS;
    if (int64_t(blockIdx.x) >= L.groups) return;  // no group for this CTA: nothing to stage
    stage<MT>(a, nb_pad, s);
    bool hi_live[MT];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) hi_live[mt] = mt * 16 + 8 < m_live;
    for (int64_t G = blockIdx.x; G < L.groups; G += gridDim.x) {
        const int c0 = warp * cpw, c1 = min(c0 + cpw, chunks);
#pragma unroll
        for (int i = 0; i < PRE_CHUNKS; ++i) {
            const int c = c0 + i;
            if (c >= c1) break;
            uint4 w;
            __half2 sc[BPC];
            if (G == blockIdx.x) {
                w = pre.w[i];
                sc[0] = pre.sc[i][0];
                sc[1] = pre.sc[i][1];
            } else {
                w = ldg_stream(L.wq + (G * chunks + c) * 32 + lane);
#pragma unroll
                for (int j = 0; j < BPC; ++j) sc[j] = __ldg(L.ws + G * int64_t(nb_pad) * 4 + t + (c * BPC + j) * 4);
            }
#pragma unroll
            for (int j = 0; j < BPC; ++j) {
                const int b = c * BPC + j;
                const uint32_t b0 = word(w, 2 * j), b1 = word(w, 2 * j + 1);
                const float2 dw = __half22float2(sc[j]);
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    int d[4];
                    mma_q<Q4>(d, s.xf[(b * MT + mt) * 32 + lane], b0, b1, s.xsum + b * MPAD + mt * 16 + g);
                    const float dx0 = s.xs[b * MPAD + mt * 16 + g], dx1 = s.xs[b * MPAD + mt * 16 + g + 8];
                    float2 lo_t, hi_t = make_float2(0.0f, 0.0f);
                    block_terms<Q4>(d, dw, dx0, dx1, hi_live[mt], lo_t, hi_t);
                    s.terms[(b * MT + mt) * 32 + lane] = make_float4(lo_t.x, lo_t.y, hi_t.x, hi_t.y);
                }
            }
        }
        __syncthreads();
        for (int o = threadIdx.x; o < MT * 128; o += blockDim.x) {
            const int mt = o / 128, ln = (o / 4) % 32, i = o % 4;
            const int m = mt * 16 + (ln >> 2) + 8 * (i >> 1);
            const int64_t n = G * 8 + 2 * (ln & 3) + (i & 1);
            if (m >= m_live || n >= L.n) continue;
            const float *tg = reinterpret_cast<const float *>(s.terms) + (mt * 32 + ln) * 4 + i;
            float v = 0.0f;
            for (int b = 0; b < nb; ++b) v = __fadd_rn(v, tg[b * MT * 128]);
            epilogue(a, L, e, m, n, v);
        }
        __syncthreads();
    }
}

// Vocab readout: one warp per row group (the whole K in registers, folded in
// block order), the next group's weights loaded while this one computes;
// suppression; argmax keys per token reduced per CTA and then across CTAs with
// 64-bit atomics. `first` holds the warp's first group, loaded before the barrier.
constexpr int RO_CHUNKS = 6;  // chunks per group: K <= 384 (Q8_0) / 768 (Q4_0)
struct RoPre {
    uint4 w[RO_CHUNKS];
};

template <bool Q4>
__device__ __forceinline__ void load_group(const StepLinear &L, int64_t G, RoPre &p) {
    constexpr int BPC = Q4 ? 4 : 2;
    const int lane = threadIdx.x & 31;
    const int chunks = int(L.nb_pad) / BPC;
    if (G >= L.groups) return;
#pragma unroll
    for (int c = 0; c < RO_CHUNKS; ++c)
        if (c < chunks) p.w[c] = ldg_stream(L.wq + (G * chunks + c) * 32 + lane);
}

template <int MT, bool Q4>
__device__ void phase_readout(const StepArgs &a, const StepSmem &s, RoPre first) {
    constexpr int BPC = Q4 ? 4 : 2;
    constexpr int MPAD = MT * 16;
    const StepLinear &L = a.head;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, t = lane & 3;
    const int nb_pad = int(L.nb_pad), m_live = a.B;
    const int chunks = nb_pad / BPC;
    stage<MT>(a, nb_pad, s);
    if (threadIdx.x < MPAD) s.best[threadIdx.x] = 0ull;
    __syncthreads();
    bool hi_live[MT];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) hi_live[mt] = mt * 16 + 8 < m_live;
    const int64_t W = int64_t(gridDim.x) * STEP_WARPS;
    RoPre cur = first;
    for (int64_t G = int64_t(blockIdx.x) * STEP_WARPS + warp; G < L.groups; G += W) {
        RoPre nxt;
        load_group<Q4>(L, G + W, nxt);
        float2 acc[MT][2];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) acc[mt][0] = acc[mt][1] = make_float2(0.0f, 0.0f);
#pragma unroll
        for (int c = 0; c < RO_CHUNKS; ++c) {
            if (c >= chunks) break;
#pragma unroll
            for (int j = 0; j < BPC; ++j) {
                const int b = c * BPC + j;
                const float2 dw = __half22float2(__ldg(L.ws + G * int64_t(nb_pad) * 4 + t + b * 4));
                uint32_t b0, b1;
                if (Q4) unpack_q4(word(cur.w[c], j), b0, b1);
                else {
                    b0 = word(cur.w[c], 2 * j);
                    b1 = word(cur.w[c], 2 * j + 1);
                }
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    int d[4];
                    mma_q<Q4>(d, s.xf[(b * MT + mt) * 32 + lane], b0, b1, s.xsum + b * MPAD + mt * 16 + g);
                    const float dx0 = s.xs[b * MPAD + mt * 16 + g], dx1 = s.xs[b * MPAD + mt * 16 + g + 8];
                    float2 lo_t, hi_t = make_float2(0.0f, 0.0f);
                    block_terms<Q4>(d, dw, dx0, dx1, hi_live[mt], lo_t, hi_t);
                    acc[mt][0].x = __fadd_rn(acc[mt][0].x, lo_t.x);
                    acc[mt][0].y = __fadd_rn(acc[mt][0].y, lo_t.y);
                    if (hi_live[mt]) {
                        acc[mt][1].x = __fadd_rn(acc[mt][1].x, hi_t.x);
                        acc[mt][1].y = __fadd_rn(acc[mt][1].y, hi_t.y);
                    }
                }
            }
        }
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                const int m = mt * 16 + g + 8 * hh;
                unsigned long long best = 0ull;
                if (m < m_live) {
#pragma unroll
                    for (int cc = 0; cc < 2; ++cc) {
                        const int64_t n = G * 8 + 2 * t + cc;
                        if (n < L.n) {
                            float v = cc ? acc[mt][hh].y : acc[mt][hh].x;
                            if (L.bias) v = __fadd_rn(v, __ldg(L.bias + n));
                            for (int64_t i = 0; i < a.nsup; ++i)
                                if (__ldg(a.suppressed + i) == n) v = -INFINITY;
                            if (a.logits) a.logits[m * L.n + n] = v;
                            const unsigned long long key = argmax_key(v, uint32_t(n));
                            best = key > best ? key : best;
                        }
                    }
                }
                if (mt * 16 + 8 * hh < m_live) reduce_best(best, s.best + m, t);
            }
        cur = nxt;
    }
    __syncthreads();
    if (threadIdx.x < m_live && s.best[threadIdx.x]) atomicMax(a.keys + threadIdx.x, s.best[threadIdx.x]);
}

// ------------------------------------------------------------------ the step
template <int MT, bool HEAD_Q4, int MODE>
__global__ void __launch_bounds__(STEP_THREADS, 1) k_decode_step(const StepArgs *__restrict__ args) {
    extern __shared__ __align__(16) unsigned char step_smem[];
    const StepArgs &a = *args;
    unsigned int gen = 0;
    if (threadIdx.x == 0) gen = *reinterpret_cast<volatile unsigned int *>(a.bar + 1);
    const int d = a.d;
    // shared-memory carve-up for the GEMV phases (the attention phases reuse the same bytes)
    StepSmem s;
    {
        const int64_t nbp_max = (a.ffn / QK + 3) / 4 * 4;
        unsigned char *p = step_smem;
        s.xf = reinterpret_cast<uint4 *>(p);
        p += nbp_max * MT * 32 * 16;
        s.terms = reinterpret_cast<float4 *>(p);
        p += nbp_max * MT * 32 * 16;
        s.xs = reinterpret_cast<float *>(p);
        p += nbp_max * MT * 16 * 4;
        s.xsum = reinterpret_cast<int *>(p);
        p += nbp_max * MT * 16 * 4;
        s.best = reinterpret_cast<unsigned long long *>(p);
    }
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    Pre pre;

    // embedding (decoder.cpp:513-518): x[b] = tok[id] + pos[p]
    for (int64_t e = int64_t(blockIdx.x) * blockDim.x + tid; e < int64_t(a.B) * d; e += int64_t(gridDim.x) * blockDim.x) {
        const int64_t b = e / d, i = e % d;
        const int64_t id = a.tokens[b], p = a.positions[b];
        if (id < 0 || id >= a.vocab || p < 0 || p >= a.npos) {
            if (i == 0) atomicOr(a.status, 4);
            a.x[e] = 0.0f;
            continue;
        }
        a.x[e] = __fadd_rn(a.tok[id * d + i], a.pos[p * d + i]);
    }
    grid_barrier(a.bar, gen, a.status, a.spin_limit);

    for (int li = 0; li < a.L; ++li) {
        const StepLayer &Ly = a.layer[li];
        // self attention block
        phase_quant<MODE>(a, a.x, d, Ly.ln[0], Ly.ln[1], Ly.lin[L_QKV].nb_pad);
        prefetch_gemv(Ly.lin[L_QKV], pre);
        grid_barrier(a.bar, gen, a.status, a.spin_limit);
        phase_gemv<MT>(a, Ly.lin[L_QKV], Epi{a.qkv, 3 * d, nullptr, false}, s, pre);
        grid_barrier(a.bar, gen, a.status, a.spin_limit);
        {
            AttArgs at{};
            at.q = a.qkv;
            at.q_stride = 3 * d;
            at.knew = a.qkv + d;
            at.vnew = a.qkv + 2 * d;
            at.kv_stride = 3 * d;
            at.kc = Ly.self_k;
            at.vc = Ly.self_v;
            at.capacity = a.target;
            at.heads = a.heads;
            at.nq = 1;
            at.batch = a.B;
            at.shared = 0;
            at.splits = 1;
            at.rows = 1;
            at.tiles_per_split = int(ceil_div(a.target, TILE_KEYS));
            at.begin = a.positions;
            at.out = a.att;
            at.out_stride = d;
            at.scale = a.scale;
            at.status = a.status;
            for (int task = blockIdx.x; task < a.B * a.heads; task += gridDim.x) {
                attend_task<true>(at, task, step_smem);
                __syncthreads();
                const int b = task / a.heads, hh = task % a.heads;
                if (warp < 2) {
                    const int64_t blk = 2 * hh + warp;
                    frag_block<MODE>(a.att[int64_t(b) * d + blk * QK + lane], true, blk, b, a.mtiles, a.xf, a.xs,
                                     a.xsum, a.status);
                }
                __syncthreads();
            }
        }
        prefetch_gemv(Ly.lin[L_OUT], pre);
        grid_barrier(a.bar, gen, a.status, a.spin_limit);
        phase_gemv<MT>(a, Ly.lin[L_OUT], Epi{a.x, d, a.x, false}, s, pre);
        grid_barrier(a.bar, gen, a.status, a.spin_limit);
        // cross attention block
        phase_quant<MODE>(a, a.x, d, Ly.ln[2], Ly.ln[3], Ly.lin[L_CQ].nb_pad);
        prefetch_gemv(Ly.lin[L_CQ], pre);
        grid_barrier(a.bar, gen, a.status, a.spin_limit);
        phase_gemv<MT>(a, Ly.lin[L_CQ], Epi{a.cq, d, nullptr, false}, s, pre);
        grid_barrier(a.bar, gen, a.status, a.spin_limit);
        {
            AttArgs at{};
            at.q = a.cq;
            at.q_stride = d;
            at.kc = Ly.cross_k;
            at.vc = Ly.cross_v;
            at.capacity = a.source;
            at.heads = a.heads;
            at.nq = 1;
            at.batch = a.B;
            at.shared = a.shared;
            const int tiles = int(ceil_div(a.source, TILE_KEYS));
            at.splits = a.shared ? shared_splits(tiles) : 1;
            at.rows = a.shared ? a.B : 1;
            at.tiles_per_split = int(ceil_div(tiles, at.splits));
            at.kv_len = a.cross_len;
            at.out = a.att;
            at.out_stride = d;
            at.scale = a.scale;
            at.status = a.status;
            at.partial = a.part;
            const int groups = a.shared ? 1 : a.B;
            for (int task = blockIdx.x; task < groups * a.heads * at.splits; task += gridDim.x) {
                attend_task<false>(at, task, step_smem);
                __syncthreads();
                if (!a.shared) {  // one CTA saw every key: quantize the row's two blocks now
                    const int b = task / a.heads, hh = task % a.heads;
                    if (warp < 2) {
                        const int64_t blk = 2 * hh + warp;
                        frag_block<MODE>(a.att[int64_t(b) * d + blk * QK + lane], true, blk, b, a.mtiles, a.xf,
                                         a.xs, a.xsum, a.status);
                    }
                    __syncthreads();
                }
            }
            if (a.shared) {
                grid_barrier(a.bar, gen, a.status, a.spin_limit);
                // merge of the key splits and the Q8_0 quantization of the two blocks, one warp per (head, row)
                const int64_t W = int64_t(gridDim.x) * STEP_WARPS;
                for (int64_t task = int64_t(blockIdx.x) * STEP_WARPS + warp; task < int64_t(a.B) * a.heads; task += W) {
                    const int hh = int(task / a.B), b = int(task % a.B);
                    const float *base = at.partial + int64_t(hh) * at.splits * a.B * (HEAD_DIM + 2) +
                                        int64_t(b) * (HEAD_DIM + 2);
                    const int64_t step = int64_t(a.B) * (HEAD_DIM + 2);
                    float M = -INFINITY;
                    for (int sp = 0; sp < at.splits; ++sp) M = fmaxf(M, base[sp * step + HEAD_DIM]);
                    float o0 = 0.0f, o1 = 0.0f, l = 0.0f;
                    if (M != -INFINITY) {
                        for (int sp = 0; sp < at.splits; ++sp) {
                            const float *pr = base + sp * step;
                            const float m = pr[HEAD_DIM];
                            const float w = m == -INFINITY ? 0.0f : __expf(m - M);
                            o0 = fmaf(w, pr[lane], o0);
                            o1 = fmaf(w, pr[lane + 32], o1);
                            l = fmaf(w, pr[HEAD_DIM + 1], l);
                        }
                    }
                    const float v0 = l > 0.0f ? o0 / l : 0.0f, v1 = l > 0.0f ? o1 / l : 0.0f;
                    a.att[int64_t(b) * d + hh * HEAD_DIM + lane] = v0;
                    a.att[int64_t(b) * d + hh * HEAD_DIM + lane + 32] = v1;
                    frag_block<MODE>(v0, true, 2 * hh, b, a.mtiles, a.xf, a.xs, a.xsum, a.status);
                    frag_block<MODE>(v1, true, 2 * hh + 1, b, a.mtiles, a.xf, a.xs, a.xsum, a.status);
                }
            }
        }
        prefetch_gemv(Ly.lin[L_COUT], pre);
        grid_barrier(a.bar, gen, a.status, a.spin_limit);
        phase_gemv<MT>(a, Ly.lin[L_COUT], Epi{a.x, d, a.x, false}, s, pre);
        grid_barrier(a.bar, gen, a.status, a.spin_limit);
        // feed-forward block
        phase_quant<MODE>(a, a.x, d, Ly.ln[4], Ly.ln[5], Ly.lin[L_FC1].nb_pad);
        prefetch_gemv(Ly.lin[L_FC1], pre);
        grid_barrier(a.bar, gen, a.status, a.spin_limit);
        phase_gemv<MT>(a, Ly.lin[L_FC1], Epi{a.h, a.ffn, nullptr, true}, s, pre);
        grid_barrier(a.bar, gen, a.status, a.spin_limit);
        phase_quant<MODE>(a, a.h, a.ffn, nullptr, nullptr, Ly.lin[L_FC2].nb_pad);
        prefetch_gemv(Ly.lin[L_FC2], pre);
        grid_barrier(a.bar, gen, a.status, a.spin_limit);
        phase_gemv<MT>(a, Ly.lin[L_FC2], Epi{a.x, d, a.x, false}, s, pre);
        grid_barrier(a.bar, gen, a.status, a.spin_limit);
    }
    // final LayerNorm + readout + argmax
    phase_quant<MODE>(a, a.x, d, a.lnf_w, a.lnf_b, a.head.nb_pad);
    RoPre first;
    load_group<HEAD_Q4>(a.head, int64_t(blockIdx.x) * STEP_WARPS + warp, first);
    grid_barrier(a.bar, gen, a.status, a.spin_limit);
    phase_readout<MT, HEAD_Q4>(a, s, first);
    grid_barrier(a.bar, gen, a.status, a.spin_limit);
    if (blockIdx.x == 0 && tid < a.B) {
        const unsigned long long k = atomicExch(a.keys + tid, 0ull);
        a.next[tid] = int64_t(0xFFFFFFFFu - uint32_t(k & 0xFFFFFFFFull));
    }
}

// ------------------------------------------------------------------ host side
static size_t step_smem_bytes(int64_t ffn, int mt) {
    const int64_t nbp_max = (ffn / QK + 3) / 4 * 4;
    const size_t gemv = size_t(nbp_max) * mt * 32 * 16 * 2 + size_t(nbp_max) * mt * 16 * 4 * 2 + 32 * 8;
    const size_t att = att_smem_bytes(mt * 16);  // attention over up to mt * 16 shared rows
    return gemv > att ? gemv : att;
}

struct DecodeStep {
    StepArgs host{};
    StepArgs *dev = nullptr;
    std::vector<void *> owned;  // scratch buffers
    size_t smem = 0;
    int grid = 0;
    ~DecodeStep() {
        if (dev) cudaFree(dev);
        for (void *p : owned) cudaFree(p);
    }
    template <class T>
    T *alloc(size_t count, const char *what) {
        void *p = nullptr;
        cuda_check(cudaMalloc(&p, count * sizeof(T) > 0 ? count * sizeof(T) : 16), what);
        owned.push_back(p);
        cuda_check(cudaMemset(p, 0, count * sizeof(T) > 0 ? count * sizeof(T) : 16), what);
        return static_cast<T *>(p);
    }
};

static StepLinear describe(void *handle, int64_t rows, int64_t width, const char *what) {
    require(handle, what);
    const auto &h = *static_cast<Linear *>(handle);
    require(h.rows == rows && h.width == width && h.gemv_ok, what);
    StepLinear L{};
    L.wq = h.wq;
    L.ws = reinterpret_cast<const __half2 *>(h.ws);
    L.bias = h.bias;
    L.groups = h.groups;
    L.nb = h.nb;
    L.nb_pad = h.nb_pad;
    L.n = h.rows;
    L.q4 = h.q4;
    return L;
}

template <int MT, bool Q4, int MODE>
static void launch_step(const DecodeStep &st, cudaStream_t s) {
    auto kernel = k_decode_step<MT, Q4, MODE>;
    static bool configured = false;
    if (!configured) {
        cuda_check(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(200 * 1024)),
                   "decode-step shared-memory attribute");
        configured = true;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(unsigned(st.grid));
    cfg.blockDim = dim3(STEP_THREADS);
    cfg.dynamicSmemBytes = st.smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cuda_check(cudaLaunchKernelEx(&cfg, kernel, const_cast<const StepArgs *>(st.dev)), "decode-step launch");
}

template <int MT, bool Q4>
static void launch_step_mode(const DecodeStep &st, cudaStream_t s) {
    if (st.host.rounding == 0) launch_step<MT, Q4, 0>(st, s);
    else if (st.host.rounding == 2) launch_step<MT, Q4, 2>(st, s);
    else launch_step<MT, Q4, 1>(st, s);
}

}  // namespace mb

using namespace mb;

extern "C" {

void *mstar_b200_decode_step_create(const mstar_b200_decode_step_config *c, char *error, size_t error_size) {
    try {
        require(c, "missing decode-step configuration");
        require(c->batch >= 1 && c->batch <= 32, "decode-step batch is 1..32 sequences");
        require(c->layers >= 1 && c->layers <= STEP_MAX_LAYERS, "1..8 decoder layers");
        require(c->heads >= 1 && c->width == c->heads * HEAD_DIM && c->width % QK == 0 && c->width <= 1536,
                "width must be heads x 64 and at most 1536");
        require(c->ffn % QK == 0 && c->ffn >= c->width && c->ffn <= 4096, "invalid FFN width");
        require(c->target >= 1 && c->target <= 4096 && c->source >= 1 && c->source <= 4096, "invalid capacities");
        require(c->rounding >= 0 && c->rounding <= 2, "unknown Q8_0 activation rounding");
        require(c->token_table && c->position_table && c->tokens && c->positions && c->next_token && c->status &&
                    c->cross_length && c->final_norm_weight && c->final_norm_bias,
                "missing decode-step operand");
        require(!c->suppressed_count || c->suppressed, "suppression list missing");
        auto st = std::make_unique<DecodeStep>();
        StepArgs &a = st->host;
        a.B = c->batch;
        a.L = c->layers;
        a.d = c->width;
        a.heads = c->heads;
        a.ffn = c->ffn;
        a.target = c->target;
        a.source = c->source;
        a.shared = c->shared_cross ? 1 : 0;
        a.mtiles = c->batch <= 16 ? 1 : 2;
        a.rounding = c->rounding;
        a.spin_limit = wait_limits().grid_barrier > 0 ? wait_limits().grid_barrier : STEP_SPIN_LIMIT;
        a.eps = c->eps;
        a.scale = 1.0f / sqrtf(float(HEAD_DIM));
        a.tok = c->token_table;
        a.pos = c->position_table;
        a.vocab = c->vocab;
        a.npos = c->positions_count;
        const int64_t d = c->width, f = c->ffn;
        for (int i = 0; i < c->layers; ++i) {
            StepLayer &Ly = a.layer[i];
            Ly.lin[L_QKV] = describe(c->linears[i][0], 3 * d, d, "QKV handle must be [3 width, width]");
            Ly.lin[L_OUT] = describe(c->linears[i][1], d, d, "out handle must be [width, width]");
            Ly.lin[L_CQ] = describe(c->linears[i][2], d, d, "cross-query handle must be [width, width]");
            Ly.lin[L_COUT] = describe(c->linears[i][3], d, d, "cross-out handle must be [width, width]");
            Ly.lin[L_FC1] = describe(c->linears[i][4], f, d, "fc1 handle must be [ffn, width]");
            Ly.lin[L_FC2] = describe(c->linears[i][5], d, f, "fc2 handle must be [width, ffn]");
            for (int k = 0; k < 6; ++k) {
                require(c->norms[i][k] && uintptr_t(c->norms[i][k]) % 16 == 0, "LayerNorm vectors (16-byte aligned)");
                require(!Ly.lin[k].q4, "body linears are Q8_0");
                Ly.ln[k] = c->norms[i][k];
            }
            require(c->self_k[i] && c->self_v[i] && c->cross_k[i] && c->cross_v[i], "missing KV planes");
            Ly.self_k = static_cast<__half *>(c->self_k[i]);
            Ly.self_v = static_cast<__half *>(c->self_v[i]);
            Ly.cross_k = static_cast<__half *>(c->cross_k[i]);
            Ly.cross_v = static_cast<__half *>(c->cross_v[i]);
        }
        a.head = describe(c->head, c->vocab, d, "readout handle must be [vocab, width]");
        require(a.head.nb_pad <= RO_CHUNKS * (a.head.q4 ? 4 : 2), "readout width too large for the step kernel");
        for (int i = 0; i < c->layers; ++i)
            for (int k = 0; k < 6; ++k)
                require(ceil_div(a.layer[i].lin[k].nb_pad / 2, STEP_WARPS) <= PRE_CHUNKS,
                        "linear width too large for the step kernel");
        a.lnf_w = c->final_norm_weight;
        a.lnf_b = c->final_norm_bias;
        a.suppressed = c->suppressed;
        a.nsup = int64_t(c->suppressed_count);
        a.tokens = c->tokens;
        a.positions = c->positions;
        a.cross_len = c->cross_length;
        a.logits = c->logits;
        a.next = c->next_token;
        a.status = c->status;
        a.gelu = gelu_table();
        const int64_t B = c->batch, mpad = 16 * a.mtiles;
        a.x = st->alloc<float>(size_t(B * d), "decode-step x");
        a.qkv = st->alloc<float>(size_t(B * 3 * d), "decode-step qkv");
        a.att = st->alloc<float>(size_t(B * d), "decode-step attention");
        a.cq = st->alloc<float>(size_t(B * d), "decode-step cross query");
        a.h = st->alloc<float>(size_t(B * f), "decode-step hidden");
        const int64_t nbp_max = (f / QK + 3) / 4 * 4;
        a.xf = st->alloc<uint32_t>(size_t(nbp_max * a.mtiles * 32 * 4), "decode-step fragments");
        a.xs = st->alloc<float>(size_t(nbp_max * mpad), "decode-step scales");
        a.xsum = st->alloc<int>(size_t(nbp_max * mpad), "decode-step quant sums");
        const int tiles = int(ceil_div(c->source, TILE_KEYS));
        const int splits = shared_splits(tiles);
        a.part = st->alloc<float>(size_t(c->heads) * splits * B * (HEAD_DIM + 2), "decode-step partials");
        a.keys = st->alloc<unsigned long long>(32, "decode-step argmax keys");
        a.bar = st->alloc<unsigned int>(2, "decode-step barrier");
        cuda_check(cudaMalloc(&st->dev, sizeof(StepArgs)), "decode-step arguments");
        cuda_check(cudaMemcpy(st->dev, &a, sizeof(StepArgs), cudaMemcpyHostToDevice), "decode-step arguments");
        st->smem = step_smem_bytes(f, a.mtiles);
        require(st->smem <= 200 * 1024, "decode-step shared memory exceeds 200 KB");
        int dev = 0, sms = 0;
        cuda_check(cudaGetDevice(&dev), "device");
        cuda_check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "SM count");
        st->grid = sms;  // one persistent CTA per SM (cooperative launch checks co-residency)
        cuda_check(cudaDeviceSynchronize(), "decode-step preparation");
        return st.release();
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return nullptr;
    }
}

int mstar_b200_decode_step_run(void *step, void *stream, char *error, size_t error_size) {
    try {
        require(step, "missing decode-step handle");
        const auto &st = *static_cast<DecodeStep *>(step);
        cudaStream_t s = as_stream(stream);
        const bool q4 = st.host.head.q4;
        if (st.host.mtiles == 1) {
            if (q4) launch_step_mode<1, true>(st, s);
            else launch_step_mode<1, false>(st, s);
        } else {
            if (q4) launch_step_mode<2, true>(st, s);
            else launch_step_mode<2, false>(st, s);
        }
        return 0;
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return -1;
    }
}

int mstar_b200_decode_step_close(void *step, char *error, size_t error_size) {
    try {
        if (step) {
            cuda_check(cudaDeviceSynchronize(), "decode-step close");
            delete static_cast<DecodeStep *>(step);
        }
        return 0;
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return -1;
    }
}

}  // extern "C"
