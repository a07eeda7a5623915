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
#include "gemv_dev.cuh"
#include "quant.cuh"

namespace mb {

constexpr int GEMV_THREADS = 256;  // upper bound; a CTA is 8 warps (wpg == 1) or wpg warps
constexpr int GEMV_WARPS = GEMV_THREADS / 32;
constexpr int CHUNKS_IN_FLIGHT = 4;

struct GemvSmem {
    uint4 *xf;
    float *xs;
    int *xsum;
    float *terms;
    float *stats;
    unsigned long long *best;
};


// Copy this call's activation fragments and scales (written by the quantize
// kernel that precedes this launch) into shared memory. Asynchronous 16-byte
// copies, so every thread has all of its copies in flight at once: a plain
// load-then-store loop keeps one per thread, which made the copy (160 KB per
// CTA at K = 4096 and 32 queries) most of a wide-row GEMV's time.
template <int MT>
__device__ __forceinline__ void stage_activations(const GemvArgs &a, GemvSmem &s) {
    constexpr int MPAD = MT * 16;
    const int64_t nf = a.nb_pad * MT * 32;
    for (int64_t i = threadIdx.x; i < nf; i += blockDim.x) cp_async16(s.xf + i, a.xf + i, 16);
    const int64_t ns = a.nb_pad * MPAD / 4;
    for (int64_t i = threadIdx.x; i < ns; i += blockDim.x) {
        cp_async16(reinterpret_cast<float4 *>(s.xs) + i, reinterpret_cast<const float4 *>(a.xs) + i, 16);
        cp_async16(reinterpret_cast<int4 *>(s.xsum) + i, reinterpret_cast<const int4 *>(a.xsum) + i, 16);
    }
    cp_async_wait_all();
    __syncthreads();
}

// Epilogue of one output element; returns the value stored (readout: after suppression).
template <bool READOUT>
__device__ __forceinline__ float finish(const GemvArgs &a, int m, int64_t n, float v) {
    if (a.flags & 1) v = __fadd_rn(v, __ldg(a.bias + n));
    if (a.flags & 2) v = gelu_ggml(v, a.gelu);
    else if (a.flags & 8) v = gelu_erf(v);
    if (a.flags & 4) v = __fadd_rn(a.residual[m * a.ldo + n], v);
    if (READOUT) {
        for (int64_t i = 0; i < a.suppressed_count; ++i)
            if (__ldg(a.suppressed + i) == n) v = -INFINITY;
    }
    a.out[m * a.ldo + n] = v;
    return v;
}

// GX: the activation fragments, scales and quant sums are read where the quantize kernel
// left them (L2) instead of being staged in shared memory, which then holds only the
// split path's per-block terms: the split-K form for wide rows (K >= 2048 at 32 queries,
// where staging 80-160 KB per CTA allowed one CTA per SM or did not fit next to the
// terms at all).
template <int MT, bool Q4, bool READOUT, bool SUMS, bool SPLIT, bool GX = false>
__global__ void __launch_bounds__(GEMV_THREADS) k_gemv(const GemvArgs a) {
    constexpr int BPC = Q4 ? 4 : 2;  // blocks per 16-byte chunk
    constexpr int MPAD = MT * 16;
    constexpr int RING = CHUNKS_IN_FLIGHT;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, t = lane & 3;
    const int nb_pad = int(a.nb_pad), nb = int(a.nb), m_live = int(a.m);
    const int chunks = nb_pad / BPC;

    // Work of this warp as a flat sequence of (group, chunk) steps:
    //   split:   one group per CTA, this warp's contiguous chunk range of it;
    //   streamed: groups G0, G0 + stride, ... (all chunks of each), so the
    //            ring of loads runs ahead across group boundaries.
    int64_t G0, gstride;
    int c_begin, c_len, ngroups;
    if (SPLIT) {
        const int wpg = a.wpg, cpw = (chunks + wpg - 1) / wpg;
        G0 = blockIdx.x;
        gstride = 1;
        c_begin = warp * cpw < chunks ? warp * cpw : chunks;
        c_len = (c_begin + cpw < chunks ? c_begin + cpw : chunks) - c_begin;
        // a warp left without chunks (chunks not a multiple of cpw) loads nothing
        ngroups = G0 < a.groups && c_len > 0 ? 1 : 0;
    } else {
        G0 = int64_t(blockIdx.x) * GEMV_WARPS + warp;
        gstride = int64_t(gridDim.x) * GEMV_WARPS;
        c_begin = 0;
        c_len = chunks;
        ngroups = G0 < a.groups ? int((a.groups - G0 + gstride - 1) / gstride) : 0;
    }
    const int total = ngroups * c_len;

    GemvSmem s;
    if (GX) {
        s.xf = const_cast<uint4 *>(a.xf);
        s.xs = const_cast<float *>(a.xs);
        s.xsum = const_cast<int *>(a.xsum);
        s.stats = reinterpret_cast<float *>(smem_raw);
    } else {
        s.xf = reinterpret_cast<uint4 *>(smem_raw);
        s.xs = reinterpret_cast<float *>(s.xf + nb_pad * MT * 32);
        s.xsum = reinterpret_cast<int *>(s.xs + nb_pad * MPAD);
        s.stats = reinterpret_cast<float *>(s.xsum + nb_pad * MPAD);
    }
    s.best = reinterpret_cast<unsigned long long *>(s.stats + 2 * MPAD);
    s.terms = reinterpret_cast<float *>(s.best + MPAD);
    if (READOUT && threadIdx.x < MPAD) s.best[threadIdx.x] = 0ull;

    uint4 w[RING];
    __half2 sc[RING][BPC];
    int ld_gi = 0, ld_c = 0;  // load cursor: group index (in this warp's sequence) and chunk
    auto load_next = [&](int u) {
        if (ld_gi < ngroups) {
            const int64_t G = G0 + ld_gi * gstride;
            const int c = c_begin + ld_c;
            w[u] = ldg_stream(a.wq + (G * chunks + c) * 32 + lane);
            const __half2 *sp = a.ws + G * int64_t(nb_pad) * 4 + t + c * BPC * 4;
#pragma unroll
            for (int j = 0; j < BPC; ++j) sc[u][j] = __ldg(sp + j * 4);
            if (++ld_c == c_len) {
                ld_c = 0;
                ++ld_gi;
            }
        }
    };
#pragma unroll
    for (int u = 0; u < RING; ++u) load_next(u);  // immutable weights: before waiting on x's producer
    pdl_wait();
    pdl_trigger();  // the next kernel may launch now; it waits for this grid before reading
    if (GX) __syncthreads();   // the readout's shared maxima are initialised before use
    else stage_activations<MT>(a, s);

    bool hi_live[MT];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) hi_live[mt] = mt * 16 + 8 < m_live;
    float2 acc[MT][2];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) acc[mt][0] = acc[mt][1] = make_float2(0.0f, 0.0f);
    float4 *terms = reinterpret_cast<float4 *>(s.terms);
    int cu_gi = 0, cu_c = 0;  // compute cursor

    for (int s0 = 0; s0 < total; s0 += RING) {
#pragma unroll
        for (int u = 0; u < RING; ++u) {
            if (s0 + u >= total) break;
            const int64_t G = G0 + cu_gi * gstride;
            const int c = c_begin + cu_c;
#pragma unroll
            for (int j = 0; j < BPC; ++j) {
                const int b = c * BPC + j;
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
                    mma_q<Q4>(d, s.xf[(b * MT + mt) * 32 + lane], b0, b1, s.xsum + b * MPAD + mt * 16 + g);
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
                        // scalar adds: a packed add after a packed multiply may be contracted
                        acc[mt][0].x = __fadd_rn(acc[mt][0].x, lo_t.x);
                        acc[mt][0].y = __fadd_rn(acc[mt][0].y, lo_t.y);
                        if (hi_live[mt]) {
                            acc[mt][1].x = __fadd_rn(acc[mt][1].x, hi_t.x);
                            acc[mt][1].y = __fadd_rn(acc[mt][1].y, hi_t.y);
                        }
                    }
                }
            }
            load_next(u);  // refill this ring slot
            if (++cu_c == c_len) {
                cu_c = 0;
                ++cu_gi;
                if (!SPLIT && !SUMS) {  // group complete: epilogue, reset
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            const int m = mt * 16 + g + 8 * h;
                            unsigned long long best = 0ull;
                            if (m < m_live) {
#pragma unroll
                                for (int cc = 0; cc < 2; ++cc) {
                                    const int64_t n = G * 8 + 2 * t + cc;
                                    if (n < a.n) {
                                        const float v = finish<READOUT>(a, m, n, cc ? acc[mt][h].y : acc[mt][h].x);
                                        if (READOUT) {
                                            const unsigned long long key = argmax_key(v, uint32_t(n));
                                            best = key > best ? key : best;
                                        }
                                    }
                                }
                            }
                            if (READOUT && mt * 16 + 8 * h < m_live) reduce_best(best, s.best + m, t);
                            acc[mt][h] = make_float2(0.0f, 0.0f);
                        }
                }
            }
        }
    }
    if (SUMS) return;

    if (SPLIT) {
        __syncthreads();
        // in-order fold of the per-block terms: one thread per output element
        const int64_t G = G0;
        for (int o = threadIdx.x; o < MT * 128; o += blockDim.x) {
            const int mt = o / 128, ln = (o / 4) % 32, i = o % 4;
            const int m = mt * 16 + (ln >> 2) + 8 * (i >> 1);
            const int64_t n = G * 8 + 2 * (ln & 3) + (i & 1);
            if (G >= a.groups || m >= m_live || n >= a.n) continue;
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

// Streamed GEMV (unsplit K, many row groups): each warp owns a contiguous run
// of row groups and walks their chunks in order. Lane 0 keeps STREAM_RING
// chunks in flight with 1-D TMA bulk copies (weights 512 B + scales 16*BPC B
// per chunk) into the warp's shared-memory ring, each slot tracked by an
// mbarrier; the in-flight bytes therefore cost no registers. Every wait is
// bounded: on timeout the warp sets status bit 1 (value 2), drains its copies
// (again bounded) and leaves the loop.
constexpr int STREAM_RING = 8;

template <int MT, bool Q4, bool READOUT>
__global__ void __launch_bounds__(GEMV_THREADS) k_gemv_stream(const GemvArgs a) {
    constexpr int BPC = Q4 ? 4 : 2;
    constexpr int MPAD = MT * 16;
    constexpr int SC_BYTES = 16 * BPC;
    constexpr int R = STREAM_RING;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, t = lane & 3;
    const int nb_pad = int(a.nb_pad), m_live = int(a.m);
    const int chunks = nb_pad / BPC;

    GemvSmem s;
    s.xf = reinterpret_cast<uint4 *>(smem_raw);
    s.xs = reinterpret_cast<float *>(s.xf + nb_pad * MT * 32);
    s.xsum = reinterpret_cast<int *>(s.xs + nb_pad * MPAD);
    s.stats = reinterpret_cast<float *>(s.xsum + nb_pad * MPAD);
    s.best = reinterpret_cast<unsigned long long *>(s.stats + 2 * MPAD);
    unsigned char *ring = reinterpret_cast<unsigned char *>(s.best + MPAD) + warp * (R * (512 + SC_BYTES + 8));
    uint4 *wslot = reinterpret_cast<uint4 *>(ring);                     // [R][32] uint4
    __half2 *sslot = reinterpret_cast<__half2 *>(ring + R * 512);      // [R][BPC*4] half2
    uint64_t *bar = reinterpret_cast<uint64_t *>(ring + R * (512 + SC_BYTES));
    if (READOUT && threadIdx.x < MPAD) s.best[threadIdx.x] = 0ull;

    // contiguous group range of this warp
    const int64_t W = int64_t(gridDim.x) * GEMV_WARPS, wid = int64_t(blockIdx.x) * GEMV_WARPS + warp;
    const int64_t base = a.groups / W, rem = a.groups % W;
    const int64_t g_begin = wid * base + (wid < rem ? wid : rem);
    const int64_t ngroups = base + (wid < rem ? 1 : 0);
    const int64_t steps = ngroups * chunks;

    if (lane == 0) {
        for (int u = 0; u < R; ++u) mbar_init(bar + u, 1);
        fence_mbar_init();
    }
    __syncwarp();
    int64_t ld_g = g_begin;
    int ld_c = 0;
    auto issue = [&](int u) {  // lane 0 only
        mbar_expect_tx(bar + u, 512 + SC_BYTES);
        bulk_g2s(wslot + u * 32, a.wq + (ld_g * chunks + ld_c) * 32, 512, bar + u);
        bulk_g2s(sslot + u * BPC * 4, a.ws + (ld_g * nb_pad + ld_c * BPC) * 4, SC_BYTES, bar + u);
        if (++ld_c == chunks) {
            ld_c = 0;
            ++ld_g;
        }
    };
    if (lane == 0)
        for (int u = 0; u < R && u < steps; ++u) issue(u);  // immutable weights: before waiting on x
    pdl_wait();
    pdl_trigger();  // the next kernel may launch now; it waits for this grid before reading
    stage_activations<MT>(a, s);

    bool hi_live[MT];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) hi_live[mt] = mt * 16 + 8 < m_live;
    float2 acc[MT][2];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) acc[mt][0] = acc[mt][1] = make_float2(0.0f, 0.0f);
    int64_t G = g_begin;
    int c = 0;
    int64_t st = 0;
    bool failed = false;
    for (; st < steps; ++st) {
        const int u = int(st % R);
        const uint32_t parity = uint32_t((st / R) & 1);
        if (!mbar_wait_bounded(bar + u, parity)) {
            failed = true;
            break;
        }
        const uint4 wv = wslot[u * 32 + lane];
        __half2 sc[BPC];
#pragma unroll
        for (int j = 0; j < BPC; ++j) sc[j] = sslot[u * BPC * 4 + j * 4 + t];
        __syncwarp();
        if (lane == 0 && st + R < steps) {
            fence_proxy_async();
            issue(u);
        }
#pragma unroll
        for (int j = 0; j < BPC; ++j) {
            const int b = c * BPC + j;
            uint32_t b0, b1;
            if (Q4) unpack_q4(word(wv, j), b0, b1);
            else {
                b0 = word(wv, 2 * j);
                b1 = word(wv, 2 * j + 1);
            }
            const float2 dw = __half22float2(sc[j]);
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                int d[4];
                mma_q<Q4>(d, s.xf[(b * MT + mt) * 32 + lane], b0, b1, s.xsum + b * MPAD + mt * 16 + g);
                const float dx0 = s.xs[b * MPAD + mt * 16 + g], dx1 = s.xs[b * MPAD + mt * 16 + g + 8];
                float2 lo_t, hi_t = make_float2(0.0f, 0.0f);
                block_terms<Q4>(d, dw, dx0, dx1, hi_live[mt], lo_t, hi_t);
                // scalar adds: a packed add after a packed multiply may be contracted
                acc[mt][0].x = __fadd_rn(acc[mt][0].x, lo_t.x);
                acc[mt][0].y = __fadd_rn(acc[mt][0].y, lo_t.y);
                if (hi_live[mt]) {
                    acc[mt][1].x = __fadd_rn(acc[mt][1].x, hi_t.x);
                    acc[mt][1].y = __fadd_rn(acc[mt][1].y, hi_t.y);
                }
            }
        }
        if (++c == chunks) {  // group complete: epilogue, reset
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int m = mt * 16 + g + 8 * h;
                    unsigned long long best = 0ull;
                    if (m < m_live) {
#pragma unroll
                        for (int cc = 0; cc < 2; ++cc) {
                            const int64_t n = G * 8 + 2 * t + cc;
                            if (n < a.n) {
                                const float v = finish<READOUT>(a, m, n, cc ? acc[mt][h].y : acc[mt][h].x);
                                if (READOUT) {
                                    const unsigned long long key = argmax_key(v, uint32_t(n));
                                    best = key > best ? key : best;
                                }
                            }
                        }
                    }
                    if (READOUT && mt * 16 + 8 * h < m_live) reduce_best(best, s.best + m, t);
                    acc[mt][h] = make_float2(0.0f, 0.0f);
                }
            c = 0;
            ++G;
        }
    }
    if (failed) {  // report, then drain this warp's copies still in flight (bounded)
        if (lane == 0 && a.status) atomicOr(a.status, 2);
        for (int64_t q = st; q < steps && q < st + R; ++q) mbar_wait_bounded(bar + int(q % R), uint32_t((q / R) & 1));
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

size_t stream_smem_bytes(int64_t nb_pad, int mt, int q4) {
    const size_t act = size_t(nb_pad) * mt * 512 + 2 * size_t(nb_pad) * mt * 16 * 4 + 2 * mt * 16 * 4 + mt * 16 * 8;
    return act + size_t(GEMV_WARPS) * STREAM_RING * (512 + 16 * (q4 ? 4 : 2) + 8);
}

static int sm_count();
size_t stream_smem_bytes(int64_t nb_pad, int mt, int q4);

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

size_t gemv_smem_bytes(int64_t nb_pad, int mt, int wpg, bool gx = false) {
    size_t bytes = 2 * mt * 16 * 4 + mt * 16 * 8;
    if (!gx) bytes += size_t(nb_pad) * mt * 512 + 2 * size_t(nb_pad) * mt * 16 * 4;   // staged activations
    if (wpg > 1) bytes += size_t(nb_pad) * mt * 512;  // one group per CTA when K is split
    return bytes;
}

constexpr size_t SMEM_LIMIT = 200 * 1024;
size_t gemv_smem_bytes(int64_t nb_pad, int mt, int wpg, bool gx);
constexpr int64_t GX_MIN_BLOCKS = 64;   // K >= 2048: the split form reads the activations from L2

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

template <int MT, bool Q4, bool READOUT, bool SUMS, bool SPLIT, bool GX = false>
static void launch_one(GemvArgs a, cudaStream_t s) {
    const size_t smem = gemv_smem_bytes(a.nb_pad, MT, a.wpg, GX);
    auto kernel = k_gemv<MT, Q4, READOUT, SUMS, SPLIT, GX>;
    static size_t configured = 0;
    if (smem > 48 * 1024 && smem > configured) {
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(SMEM_LIMIT + 8192));
        configured = SMEM_LIMIT;
    }
    // split: one CTA per group; streamed: a few CTAs per SM, warps loop over groups
    int64_t grid = a.wpg == 1 ? ceil_div(a.groups, GEMV_WARPS) : a.groups;
    if (a.wpg == 1) {
        const int64_t cap = int64_t(sm_count()) * a.ctas_per_sm;
        grid = grid < cap ? grid : cap;
    }
    const int gpc = a.wpg == 1 ? GEMV_WARPS : 1;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(unsigned(grid));
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
static void launch_stream(const GemvArgs &a, cudaStream_t s) {
    const size_t smem = stream_smem_bytes(a.nb_pad, MT, Q4);
    auto kernel = a.keys ? k_gemv_stream<MT, Q4, true> : k_gemv_stream<MT, Q4, false>;
    static bool configured[2] = {false, false};
    if (!configured[a.keys ? 1 : 0]) {
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(SMEM_LIMIT + 8192));
        configured[a.keys ? 1 : 0] = true;
    }
    int64_t grid = ceil_div(a.groups, GEMV_WARPS);
    const int64_t cap = int64_t(sm_count()) * a.ctas_per_sm;
    grid = grid < cap ? grid : cap;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(unsigned(grid));
    cfg.blockDim = dim3(GEMV_THREADS);
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
    if (a.ctas_per_sm <= 0) a.ctas_per_sm = 4;
    if (!a.sums && a.wpg_override == 0 && a.nb_pad >= GX_MIN_BLOCKS &&
        gemv_smem_bytes(a.nb_pad, MT, 2, true) <= SMEM_LIMIT) {
        // wide rows: split K over the warps of one row group per CTA, activations from L2
        const int64_t chunks = a.nb_pad / (Q4 ? 4 : 2);
        const int64_t target = int64_t(sm_count()) * 24;
        a.wpg = 2;
        while (a.wpg < GEMV_WARPS && a.groups * a.wpg < target && chunks >= 2 * a.wpg) a.wpg *= 2;
        if (a.keys) launch_one<MT, Q4, true, false, true, true>(a, s);
        else launch_one<MT, Q4, false, false, true, true>(a, s);
        return;
    }
    a.wpg = a.sums ? 1 : choose_wpg(a, Q4, MT);
    if (!a.sums && a.wpg == 1 && stream_smem_bytes(a.nb_pad, MT, Q4) <= SMEM_LIMIT) {
        launch_stream<MT, Q4>(a, s);
        return;
    }
    if (a.sums) launch_one<MT, Q4, false, true, false>(a, s);
    else if (a.keys) {
        if (a.wpg > 1) launch_one<MT, Q4, true, false, true>(a, s);
        else launch_one<MT, Q4, true, false, false>(a, s);
    } else {
        if (a.wpg > 1) launch_one<MT, Q4, false, false, true>(a, s);
        else launch_one<MT, Q4, false, false, false>(a, s);
    }
}

bool gemv_supported(int64_t nb_pad) { return gemv_smem_bytes(nb_pad, 2, 1, false) <= SMEM_LIMIT; }

// Split-K GEMV over Q8_0 weights whose CTA owns FRAG_GROUPS = 4 row groups: 32
// consecutive outputs, one Q8_0 block of the next linear's input. After the
// block-order fold and the epilogue (bias, GELU, residual; the values stored
// to `out`), every query row's 32 outputs are quantized into the next linear's
// activation fragments (frag_block: the quantization launch_quantize_frag would
// apply to `out`), so that linear needs no quantize launch (the decoder's fc1
// feeding fc2). Warp w takes group w / wpg and the w % wpg-th part of its chunks.
constexpr int FRAG_GROUPS = 4;

template <int MT, int MODE>
__global__ void __launch_bounds__(FRAG_GROUPS * GEMV_THREADS / 2, 1) k_gemv_frag(const GemvArgs a, const Q8Frags f) {
    constexpr int BPC = 2;  // Q8_0 blocks per 16-byte chunk
    constexpr int MPAD = MT * 16;
    constexpr int RING = CHUNKS_IN_FLIGHT;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, t = lane & 3;
    const int nb_pad = int(a.nb_pad), nb = int(a.nb), m_live = int(a.m), wpg = a.wpg;
    const int chunks = nb_pad / BPC;
    const int gi = warp / wpg, wp = warp % wpg;
    const int64_t G = int64_t(blockIdx.x) * FRAG_GROUPS + gi;
    const int cpw = (chunks + wpg - 1) / wpg;
    const int c_begin = wp * cpw < chunks ? wp * cpw : chunks;
    const int c_len = (c_begin + cpw < chunks ? c_begin + cpw : chunks) - c_begin;
    const int total = G < a.groups ? c_len : 0;

    GemvSmem s;
    s.xf = reinterpret_cast<uint4 *>(smem_raw);
    s.xs = reinterpret_cast<float *>(s.xf + nb_pad * MT * 32);
    s.xsum = reinterpret_cast<int *>(s.xs + nb_pad * MPAD);
    float *tile = reinterpret_cast<float *>(s.xsum + nb_pad * MPAD);  // [MPAD][32] epilogue outputs
    float4 *terms = reinterpret_cast<float4 *>(tile + MPAD * 32) + size_t(gi) * nb_pad * MT * 32;

    uint4 w[RING];
    __half2 sc[RING][BPC];
    int ld = 0;
    auto load_next = [&](int u) {
        if (ld < total) {
            const int c = c_begin + ld;
            w[u] = ldg_stream(a.wq + (G * chunks + c) * 32 + lane);
            const __half2 *sp = a.ws + G * int64_t(nb_pad) * 4 + t + c * BPC * 4;
#pragma unroll
            for (int j = 0; j < BPC; ++j) sc[u][j] = __ldg(sp + j * 4);
            ++ld;
        }
    };
#pragma unroll
    for (int u = 0; u < RING; ++u) load_next(u);  // immutable weights: before waiting on x's producer
    pdl_wait();
    pdl_trigger();
    stage_activations<MT>(a, s);

    bool hi_live[MT];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) hi_live[mt] = mt * 16 + 8 < m_live;
    for (int s0 = 0; s0 < total; s0 += RING) {
#pragma unroll
        for (int u = 0; u < RING; ++u) {
            if (s0 + u >= total) break;
            const int c = c_begin + s0 + u;
#pragma unroll
            for (int j = 0; j < BPC; ++j) {
                const int b = c * BPC + j;
                const uint32_t b0 = word(w[u], 2 * j), b1 = word(w[u], 2 * j + 1);
                const float2 dw = __half22float2(sc[u][j]);
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    int d[4];
                    mma_q<false>(d, s.xf[(b * MT + mt) * 32 + lane], b0, b1, s.xsum + b * MPAD + mt * 16 + (lane >> 2));
                    const float dx0 = s.xs[b * MPAD + mt * 16 + (lane >> 2)], dx1 = s.xs[b * MPAD + mt * 16 + (lane >> 2) + 8];
                    float2 lo_t, hi_t = make_float2(0.0f, 0.0f);
                    block_terms<false>(d, dw, dx0, dx1, hi_live[mt], lo_t, hi_t);
                    terms[(b * MT + mt) * 32 + lane] = make_float4(lo_t.x, lo_t.y, hi_t.x, hi_t.y);
                }
            }
            load_next(u);
        }
    }
    __syncthreads();
    // in-order fold of the per-block terms, epilogue, stores: one thread per output element
    for (int o = threadIdx.x; o < FRAG_GROUPS * MT * 128; o += blockDim.x) {
        const int g2 = o / (MT * 128), rem = o % (MT * 128);
        const int mt = rem / 128, ln = (rem / 4) % 32, i = rem % 4;
        const int m = mt * 16 + (ln >> 2) + 8 * (i >> 1);
        const int col = g2 * 8 + 2 * (ln & 3) + (i & 1);
        const int64_t n = int64_t(blockIdx.x) * 32 + col;
        float v = 0.0f;
        if (m < m_live && n < a.n) {
            const float *tg = reinterpret_cast<const float *>(reinterpret_cast<float4 *>(tile + MPAD * 32) +
                                                              size_t(g2) * nb_pad * MT * 32) +
                              (mt * 32 + ln) * 4 + i;
            for (int b = 0; b < nb; ++b) v = __fadd_rn(v, tg[b * MT * 128]);
            v = finish<false>(a, m, n, v);
        }
        tile[m * 32 + col] = v;
    }
    __syncthreads();
    const int nwarps = blockDim.x >> 5;
    for (int q = warp; q < MPAD; q += nwarps)  // lane = column of the block
        frag_block<MODE>(tile[q * 32 + lane], q < m_live, blockIdx.x, q, MT, f.xf, f.xs, f.xsum, a.status);
}

template <int MT, int MODE>
static void launch_frag_mode(const GemvArgs &a, const Q8Frags &f, cudaStream_t s) {
    const size_t smem = size_t(a.nb_pad) * MT * 512 + 2 * size_t(a.nb_pad) * MT * 16 * 4 + MT * 16 * 32 * 4 +
                        size_t(FRAG_GROUPS) * a.nb_pad * MT * 512;
    auto kernel = k_gemv_frag<MT, MODE>;
    static bool configured = false;
    if (!configured) {
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(SMEM_LIMIT + 8192));
        configured = true;
    }
    launch_pdl(kernel, dim3(unsigned(a.n / 32)), dim3(unsigned(FRAG_GROUPS * a.wpg * 32)), smem, s, a, f);
}

size_t gemv_frag_smem_bytes(int64_t nb_pad, int mt) {
    return size_t(nb_pad) * mt * 512 + 2 * size_t(nb_pad) * mt * 16 * 4 + mt * 16 * 32 * 4 +
           size_t(FRAG_GROUPS) * nb_pad * mt * 512;
}

// Q8_0 weights, n a multiple of 32, m <= 32 (f.mpad = 16 for m <= 16, else 32).
void launch_gemv_frag(GemvArgs a, const Q8Frags &f, cudaStream_t s) {
    const int mt = a.m <= 16 ? 1 : 2;
    const int64_t chunks = a.nb_pad / 2;
    a.wpg = int(chunks / 2 < 4 ? (chunks / 2 > 0 ? chunks / 2 : 1) : 4);  // about two chunks per warp
    if (mt == 1) {
        if (f.mode == 0) launch_frag_mode<1, 0>(a, f, s);
        else if (f.mode == 2) launch_frag_mode<1, 2>(a, f, s);
        else launch_frag_mode<1, 1>(a, f, s);
    } else {
        if (f.mode == 0) launch_frag_mode<2, 0>(a, f, s);
        else if (f.mode == 2) launch_frag_mode<2, 2>(a, f, s);
        else launch_frag_mode<2, 1>(a, f, s);
    }
}

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
