// Decode-shape block-quantized linear (M <= 32 tokens), HBM-streaming.
//
// Each CTA (8 warps) owns 8/wpg row groups of 8 rows; the wpg warps of a group
// split its K chunks. Per warp-step every lane issues one 16-byte streaming
// load (2 Q8_0 or 4 Q4_0 blocks of its rows); mma.m16n8k32 s8 gives the exact
// int32 block dots; the per-block fp32 terms are formed with ggml's generic
// roundings (ggml-cpu/quants.c:451-480 Q8_0: sumi*(dw*dx); quants.c:225-258
// Q4_0: sumi*dw*dx) and folded into the output strictly in block order — in
// registers when one warp owns the whole row, through shared memory when K is
// split — so results are bit-identical to the reference's generic vec_dot.
//
// Prologue: the first weight chunks are requested before the kernel waits
// (griddepcontrol.wait) for the quantize kernel launched just before it, so
// the HBM stream overlaps that kernel; then the CTA stages the call's
// activation fragments and scales from L2 into shared memory.
//
// Epilogue: bias, ggml GELU (fp16-table tanh form) or erf GELU, residual add;
// for the vocab readout also suppression and the first-index / NaN-first
// argmax (decoder.cpp:686-696), reduced per warp, per CTA, then across CTAs
// through 64-bit atomics; the last CTA to finish writes the tokens and resets
// the shared state for the next call.
#include "quant.cuh"

namespace mb {

constexpr int GEMV_THREADS = 256;  // upper bound; a CTA is 8 warps (wpg == 1) or wpg warps
constexpr int GEMV_WARPS = GEMV_THREADS / 32;
constexpr int CHUNKS_IN_FLIGHT = 4;

struct GemvSmem {
    uint4 *xf;
    float *xs;
    float *terms;
    float *stats;
    unsigned long long *best;
};

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Copy this call's activation fragments and scales (written by the quantize
// kernel that precedes this launch) into shared memory.
template <int MT>
__device__ __forceinline__ void stage_activations(const GemvArgs &a, GemvSmem &s) {
    constexpr int MPAD = MT * 16;
    const int64_t nf = a.nb_pad * MT * 32;
    for (int64_t i = threadIdx.x; i < nf; i += blockDim.x) s.xf[i] = a.xf[i];
    const int64_t ns = a.nb_pad * MPAD / 4;
    for (int64_t i = threadIdx.x; i < ns; i += blockDim.x)
        reinterpret_cast<float4 *>(s.xs)[i] = reinterpret_cast<const float4 *>(a.xs)[i];
    __syncthreads();
}

// Epilogue of one output element; returns the value stored (readout: after suppression).
template <bool READOUT>
__device__ __forceinline__ float finish(const GemvArgs &a, int m, int64_t n, float v) {
    if (a.flags & 1) v = __fadd_rn(v, __ldg(a.bias + n));
    if (a.flags & 2) v = gelu_ggml(v);
    else if (a.flags & 8) v = gelu_erf(v);
    if (a.flags & 4) v = __fadd_rn(a.residual[m * a.ldo + n], v);
    if (READOUT) {
        for (int64_t i = 0; i < a.suppressed_count; ++i)
            if (__ldg(a.suppressed + i) == n) v = -INFINITY;
    }
    a.out[m * a.ldo + n] = v;
    return v;
}

// Per-block fp32 terms of one m16n8 tile: rows g (c0, c1) and g+8 (c2, c3)
// with ggml's generic rounding order (see the file comment).
template <bool Q4>
__device__ __forceinline__ void block_terms(const int (&d)[4], float2 dw, float dx0, float dx1, bool hi,
                                            float2 &lo_t, float2 &hi_t) {
    const float2 i01 = i2f2(d[0], d[1]);
    if (Q4) lo_t = mul2(mul2(i01, dw), make_float2(dx0, dx0));
    else lo_t = mul2(i01, mul2(dw, make_float2(dx0, dx0)));
    if (hi) {
        const float2 i23 = i2f2(d[2], d[3]);
        if (Q4) hi_t = mul2(mul2(i23, dw), make_float2(dx1, dx1));
        else hi_t = mul2(i23, mul2(dw, make_float2(dx1, dx1)));
    }
}

template <int MT, bool Q4, bool READOUT, bool SUMS, bool SPLIT>
__global__ void __launch_bounds__(GEMV_THREADS) k_gemv(const GemvArgs a) {
    constexpr int BPC = Q4 ? 4 : 2;  // blocks per 16-byte chunk
    constexpr int MPAD = MT * 16;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, t = lane & 3;
    const int wpg = SPLIT ? a.wpg : 1, gpc = SPLIT ? 1 : GEMV_WARPS;
    const int gi = warp / wpg, ks = warp % wpg;
    const int nb_pad = int(a.nb_pad), nb = int(a.nb), m_live = int(a.m);
    const int chunks = nb_pad / BPC;
    const int cpw = (chunks + wpg - 1) / wpg;
    const int c_begin = ks * cpw < chunks ? ks * cpw : chunks;
    const int c_end = c_begin + cpw < chunks ? c_begin + cpw : chunks;
    const int64_t G = int64_t(blockIdx.x) * gpc + gi;
    const bool active = G < a.groups;

    GemvSmem s;
    s.xf = reinterpret_cast<uint4 *>(smem_raw);
    s.xs = reinterpret_cast<float *>(s.xf + nb_pad * MT * 32);
    s.stats = s.xs + nb_pad * MPAD;
    s.best = reinterpret_cast<unsigned long long *>(s.stats + 2 * MPAD);
    s.terms = reinterpret_cast<float *>(s.best + MPAD);
    if (READOUT && threadIdx.x < MPAD) s.best[threadIdx.x] = 0ull;

    const uint4 *wp = a.wq + (active ? G : 0) * int64_t(chunks) * 32 + lane;
    const __half2 *sp = a.ws + (active ? G : 0) * int64_t(nb_pad) * 4 + t;

    uint4 w[CHUNKS_IN_FLIGHT];
    __half2 sc[CHUNKS_IN_FLIGHT][BPC];
    auto fetch = [&](int c0) {
#pragma unroll
        for (int u = 0; u < CHUNKS_IN_FLIGHT; ++u)
            if (active && c0 + u < c_end) {
                w[u] = ldg_stream(wp + (c0 + u) * 32);
#pragma unroll
                for (int j = 0; j < BPC; ++j) sc[u][j] = __ldg(sp + ((c0 + u) * BPC + j) * 4);
            }
    };
    fetch(c_begin);  // immutable weights: requested before waiting on the producer of x
    pdl_wait();
    stage_activations<MT>(a, s);

    bool hi_live[MT];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) hi_live[mt] = mt * 16 + 8 < m_live;
    float2 acc[MT][2];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) acc[mt][0] = acc[mt][1] = make_float2(0.0f, 0.0f);
    float4 *terms = reinterpret_cast<float4 *>(s.terms);

    for (int c0 = c_begin; active && c0 < c_end; c0 += CHUNKS_IN_FLIGHT) {
#pragma unroll
        for (int u = 0; u < CHUNKS_IN_FLIGHT; ++u) {
            if (c0 + u >= c_end) break;
#pragma unroll
            for (int j = 0; j < BPC; ++j) {
                const int b = (c0 + u) * BPC + j;
                uint32_t b0, b1;
                if (Q4) unpack_q4(word(w[u], j), b0, b1);
                else {
                    b0 = word(w[u], 2 * j);
                    b1 = word(w[u], 2 * j + 1);
                }
                const float2 dw = __half22float2(sc[u][j]);
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    int d[4];
                    mma_s8(d, s.xf[(b * MT + mt) * 32 + lane], b0, b1);
                    if (SUMS) {
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const int m = mt * 16 + g + 8 * (i >> 1);
                            const int64_t n = G * 8 + 2 * t + (i & 1);
                            if (m < m_live && n < a.n && b < nb) a.sums[(m * a.n + n) * nb + b] = d[i];
                        }
                        continue;
                    }
                    const float dx0 = s.xs[b * MPAD + mt * 16 + g], dx1 = s.xs[b * MPAD + mt * 16 + g + 8];
                    float2 lo_t, hi_t = make_float2(0.0f, 0.0f);
                    block_terms<Q4>(d, dw, dx0, dx1, hi_live[mt], lo_t, hi_t);
                    if (SPLIT) {
                        terms[(b * MT + mt) * 32 + lane] = make_float4(lo_t.x, lo_t.y, hi_t.x, hi_t.y);
                    } else {
                        acc[mt][0].x = __fadd_rn(acc[mt][0].x, lo_t.x);
                        acc[mt][0].y = __fadd_rn(acc[mt][0].y, lo_t.y);
                        if (hi_live[mt]) {
                            acc[mt][1].x = __fadd_rn(acc[mt][1].x, hi_t.x);
                            acc[mt][1].y = __fadd_rn(acc[mt][1].y, hi_t.y);
                        }
                    }
                }
            }
        }
        fetch(c0 + CHUNKS_IN_FLIGHT);
    }
    if (SUMS) return;

    if (!SPLIT) {
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int m = mt * 16 + g + 8 * h;
                unsigned long long best = 0ull;
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    const int64_t n = G * 8 + 2 * t + c;
                    if (active && m < m_live && n < a.n) {
                        const float2 pair = acc[mt][h];
                        const float v = finish<READOUT>(a, m, n, c ? pair.y : pair.x);
                        if (READOUT) {
                            const unsigned long long key = argmax_key(v, uint32_t(n));
                            best = key > best ? key : best;
                        }
                    }
                }
                if (READOUT) {  // lanes 4g..4g+3 share token m: reduce, then one shared atomic
#pragma unroll
                    for (int o = 1; o <= 2; o <<= 1) {
                        const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
                        best = other > best ? other : best;
                    }
                    if (t == 0 && best) atomicMax(s.best + m, best);
                }
            }
    } else {
        __syncthreads();
        // in-order fold of the per-block terms: one thread per output element
        for (int o = threadIdx.x; o < MT * 128; o += blockDim.x) {
            const int mt = o / 128, ln = (o / 4) % 32, i = o % 4;
            const int m = mt * 16 + (ln >> 2) + 8 * (i >> 1);
            const int64_t n = G * 8 + 2 * (ln & 3) + (i & 1);
            if (!active || m >= m_live || n >= a.n) continue;
            const float *tg = s.terms + (mt * 32 + ln) * 4 + i;
            float v = 0.0f;
            for (int b = 0; b < nb; ++b) v = __fadd_rn(v, tg[b * MT * 128]);
            v = finish<READOUT>(a, m, n, v);
            if (READOUT) atomicMax(s.best + m, argmax_key(v, uint32_t(n)));
        }
    }

    if (READOUT) {
        __shared__ bool last;
        __syncthreads();
        if (threadIdx.x < m_live && s.best[threadIdx.x]) atomicMax(a.keys + threadIdx.x, s.best[threadIdx.x]);
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) last = atomicAdd(a.done, 1u) == gridDim.x - 1;
        __syncthreads();
        if (last) {
            __threadfence();
            if (threadIdx.x < m_live) {
                const unsigned long long k = atomicExch(a.keys + threadIdx.x, 0ull);
                a.token[threadIdx.x] = int64_t(0xFFFFFFFFu - uint32_t(k & 0xFFFFFFFFull));
            }
            if (threadIdx.x == 0) *a.done = 0u;
        }
    }
}

static int sm_count() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

size_t gemv_smem_bytes(int64_t nb_pad, int mt, int wpg) {
    size_t bytes = size_t(nb_pad) * mt * 512 + size_t(nb_pad) * mt * 16 * 4 + 2 * mt * 16 * 4 + mt * 16 * 8;
    if (wpg > 1) bytes += size_t(nb_pad) * mt * 512;  // one group per CTA when K is split
    return bytes;
}

constexpr size_t SMEM_LIMIT = 200 * 1024;
size_t gemv_smem_bytes(int64_t nb_pad, int mt, int wpg);

int choose_wpg(const GemvArgs &a, int q4, int mt) {
    const int64_t chunks = a.nb_pad / (q4 ? 4 : 2);
    const int64_t target = int64_t(sm_count()) * 24;  // warps wanted in flight
    int wpg = 1;
    while (wpg < GEMV_WARPS && a.groups * wpg < target && chunks >= 2 * wpg &&
           gemv_smem_bytes(a.nb_pad, mt, 2 * wpg) <= SMEM_LIMIT)
        wpg *= 2;
    if (a.wpg_override > 0) wpg = a.wpg_override;
    return wpg;
}

template <int MT, bool Q4, bool READOUT, bool SUMS, bool SPLIT>
static void launch_one(GemvArgs a, cudaStream_t s) {
    const size_t smem = gemv_smem_bytes(a.nb_pad, MT, a.wpg);
    auto kernel = k_gemv<MT, Q4, READOUT, SUMS, SPLIT>;
    static size_t configured = 0;
    if (smem > 48 * 1024 && smem > configured) {
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(SMEM_LIMIT + 8192));
        configured = SMEM_LIMIT;
    }
    const int gpc = a.wpg == 1 ? GEMV_WARPS : 1;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(unsigned(ceil_div(a.groups, gpc)));
    cfg.blockDim = dim3(unsigned(32 * a.wpg * gpc));
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kernel, a);
}

template <int MT, bool Q4>
static void launch_variant(GemvArgs a, cudaStream_t s) {
    a.wpg = a.sums ? 1 : choose_wpg(a, Q4, MT);
    if (a.sums) launch_one<MT, Q4, false, true, false>(a, s);
    else if (a.keys) {
        if (a.wpg > 1) launch_one<MT, Q4, true, false, true>(a, s);
        else launch_one<MT, Q4, true, false, false>(a, s);
    } else {
        if (a.wpg > 1) launch_one<MT, Q4, false, false, true>(a, s);
        else launch_one<MT, Q4, false, false, false>(a, s);
    }
}

bool gemv_supported(int64_t nb_pad) { return gemv_smem_bytes(nb_pad, 2, 1) <= SMEM_LIMIT; }

void launch_gemv(int q4, const GemvArgs &a, cudaStream_t s) {
    const int mt = a.m <= 16 ? 1 : 2;
    if (q4) {
        if (mt == 1) launch_variant<1, true>(a, s);
        else launch_variant<2, true>(a, s);
    } else {
        if (mt == 1) launch_variant<1, false>(a, s);
        else launch_variant<2, false>(a, s);
    }
}

}  // namespace mb
