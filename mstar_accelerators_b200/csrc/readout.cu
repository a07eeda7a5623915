// Greedy vocab readout on a 16-row tile layout (decoder.cpp:686-696 over the
// ggml_mul_mat of the tied Q4_0 / Q8_0 readout).
//
// The decode GEMV (gemv.cu) puts the <= 32 queries on the MMA's M side and 8
// weight rows on N. For the readout, a long, thin stream of weight rows, this
// kernel turns that around: 16 vocabulary rows are the A operand of
// mma.m16n8k32 and the queries the B operand (8 per n-tile), and the weights
// are repacked once into a tile layout so that one bulk copy moves a whole
// tile chunk (all 16 rows' fragments and scales for up to RO_SLOT bytes of
// blocks) into a warp's shared-memory ring.
//
// Per 16 x 8 x 32 block product the fp32 work is three packed f32x2
// operations per pair (ptxas fuses a packed multiply into a packed add that
// follows it, so each term is formed by an fma with a +0 addend, which equals
// the rounded product up to the sign of a zero; a running sum that starts at
// +0 never holds -0, so that sign never reaches a result):
//   * the MMA accumulator starts at the bit pattern of 1.5 * 2^23, so the
//     int32 result read as fp32 is 12582912 + sumi exactly (|sumi| < 2^22);
//   * Q4_0 nibbles are unpacked as 16 * (n - 8) (signed), so no -8 * sum(x)
//     correction is needed; the first rescale is one fma
//       RN((12582912 + 16 sumi) * dw/16 - 786432 * dw) = RN(sumi * dw)
//     (dw/16 and 786432 * dw are exact, the fma rounds once), then * dx;
//   * Q8_0: (value - 12582912) * RN(dw * dx), the generic order;
//   * the per-query sums are folded strictly in block order.
// Results are bit-identical to the reference's generic vec_dot
// (ggml-cpu/quants.c:225-258 Q4_0, :451-480 Q8_0).
//
// Prologue: every CTA quantizes the <= 32 query rows itself (after the
// optional LayerNorm), in the order of the stand-alone quantize kernel, into
// shared memory while its first weight chunks are in flight, so a readout is
// one launch.
//
// Epilogue: suppression (a per-CTA bitmask over the CTA's rows), logits
// stores, a running first-index / NaN-first maximum per (lane, query), then
// per-warp, per-CTA and cross-CTA 64-bit key reductions; the last CTA writes
// the tokens and the call's status and resets the shared state.
#include "../../include/mstar_b200.h"
#include "linear_handle.cuh"
#include "quant.cuh"

namespace mb {

constexpr int RO_SLOT = 4096;      // bytes of one ring slot (one chunk of a tile)
constexpr int RO_MAX_WARPS = 16;
constexpr size_t RO_SMEM_LIMIT = 220 * 1024;
constexpr uint32_t RO_MAGIC = 0x4B400000u;  // 1.5 * 2^23
constexpr int64_t RO_SELF_QUANT_BLOCKS = 32;  // rows up to 1024 wide are quantized inside the kernel

__host__ __device__ constexpr int ro_block_bytes(bool q4) { return q4 ? 288 : 544; }  // 16 rows of one block
__host__ __device__ constexpr int ro_quant_bytes(bool q4) { return q4 ? 256 : 512; }

// ---------------------------------------------------------------- repack
// Tile T, block b occupies ro_block_bytes at (T * nb + b): first the quants
// as each lane's A fragment (Q4_0: uint2 {row g bytes 4t..4t+3, row g+8 bytes
// 4t..4t+3}; Q8_0: uint4 {row g k 4t.., row g+8 k 4t.., row g k 16+4t..,
// row g+8 k 16+4t..}), then the fp16 scales as half2 (row g, row g+8) per g.
// Rows past the end are zero.
template <bool Q4>
__global__ void k_readout_repack(const uint8_t *__restrict__ blocks, uint8_t *__restrict__ wt, int64_t rows,
                                 int64_t nb, int64_t tiles) {
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= tiles * nb * 32) return;
    const int lane = int(i & 31), g = lane >> 2, t = lane & 3;
    const int64_t b = (i >> 5) % nb, tile = (i >> 5) / nb;
    constexpr int BB = Q4 ? Q4_BYTES : Q8_BYTES;
    uint8_t *dst = wt + (tile * nb + b) * ro_block_bytes(Q4);
    const int64_t r0 = tile * 16 + g, r1 = r0 + 8;
    auto qbyte = [&](int64_t r, int j) -> uint32_t {
        return r < rows ? blocks[(r * nb + b) * BB + 2 + j] : 0u;
    };
    auto word = [&](int64_t r, int j0) -> uint32_t {
        return qbyte(r, j0) | (qbyte(r, j0 + 1) << 8) | (qbyte(r, j0 + 2) << 16) | (qbyte(r, j0 + 3) << 24);
    };
    if (Q4) {
        uint2 v;
        v.x = word(r0, 4 * t);
        v.y = word(r1, 4 * t);
        reinterpret_cast<uint2 *>(dst)[lane] = v;
    } else {
        uint4 v;
        v.x = word(r0, 4 * t);
        v.y = word(r1, 4 * t);
        v.z = word(r0, 16 + 4 * t);
        v.w = word(r1, 16 + 4 * t);
        reinterpret_cast<uint4 *>(dst)[lane] = v;
    }
    if (t == 0) {
        auto scale = [&](int64_t r) -> uint32_t {
            if (r >= rows) return 0u;
            const uint8_t *p = blocks + (r * nb + b) * BB;
            return uint32_t(p[0]) | (uint32_t(p[1]) << 8);
        };
        reinterpret_cast<uint32_t *>(dst + ro_quant_bytes(Q4))[g] = scale(r0) | (scale(r1) << 16);
    }
}

// ---------------------------------------------------------------- kernel
struct ReadoutArgs {
    const uint8_t *wt;      // tile layout
    int64_t tiles, nb, rows;
    int cb;                 // blocks per chunk (cb * block bytes <= RO_SLOT)
    int ring;               // slots per warp
    int sup_words;          // words of the per-CTA suppression bitmask
    const float *x;         // [m][ldx] fp32 query rows
    const uint4 *pre_xf;    // non-null: queries already quantized by launch_quantize_frag ([nb_pad][mt][32] fragments,
    const float *pre_xs;    //           [nb_pad][mpad] scales), copied instead of quantized here
    int64_t ldx, m;
    const float *ln_w, *ln_b;  // optional LayerNorm applied before quantization
    float eps;
    int mode;               // Q8_0 activation rounding (0 ref, 1 arm, 2 x86)
    float *out;             // [m][ldo]
    int64_t ldo;
    const float *bias;      // [rows] or null (added before the residual, as the GEMV epilogue)
    const float *residual;  // [m][ldo] or null
    unsigned long long *keys;  // [32] running per-query maxima, zero between calls; null: logits only
    unsigned int *done;        // CTA completion counter, zero between calls
    int *flags;                // status bits of the call in flight, zero between calls
    int64_t *token;
    const int64_t *suppressed;
    int64_t nsup;
    int *status;            // written once, by the last CTA
};

__device__ __forceinline__ void mma_magic(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(RO_MAGIC));
}

__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
    float2 r;
    asm("{.reg .b64 ra, rb, rc, rd; mov.b64 ra, {%2,%3}; mov.b64 rb, {%4,%5}; mov.b64 rc, {%6,%7}; "
        "fma.rn.f32x2 rd, ra, rb, rc; mov.b64 {%0,%1}, rd;}"
        : "=f"(r.x), "=f"(r.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return r;
}

// (12582912 + i) as fp32 bits -> pair
__device__ __forceinline__ float2 biased(int a, int b) { return make_float2(__int_as_float(a), __int_as_float(b)); }

// running first-index / NaN-first maximum over increasing row indexes
__device__ __forceinline__ void running_max(float &bv, uint32_t &bn, float v, uint32_t n) {
    const bool take = v > bv || (v != v && bv == bv);
    bv = take ? v : bv;
    bn = take ? n : bn;
}

// LayerNorm statistics of one row in launch_quantize_frag's reduction order
// (virtual warps v of its 128 / 256-thread block, a warp reduction each, then
// the partials in order), so the quantized queries are the ones the decode
// GEMV path sees. Lane l holds elements 32 k + l; element 32 k + l belongs to
// virtual warp k mod (threads / 32), so each virtual warp's per-thread sum is
// this lane's sum over those k in increasing order. KC > 0: a compile-time
// width whose row is loaded into registers at once.
template <int KC>
__device__ __forceinline__ void row_stats(const float *xr, int64_t K, float eps, float &mean, float &rstd) {
    const int lane = threadIdx.x & 31;
    const int vwarps = K >= 1024 ? 8 : 4;
    float sum = 0.0f, var = 0.0f;
    if (KC) {
        constexpr int NK = KC / 32 > 0 ? KC / 32 : 1;
        constexpr int VW = KC >= 1024 ? 8 : 4;
        float v[NK];
#pragma unroll
        for (int k = 0; k < NK; ++k) v[k] = xr[32 * k + lane];
#pragma unroll
        for (int w = 0; w < VW; ++w) {
            float s = 0.0f;
#pragma unroll
            for (int k = w; k < NK; k += VW) s += v[k];
#pragma unroll
            for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            sum += s;
        }
        mean = sum / float(KC ? KC : 1);
#pragma unroll
        for (int w = 0; w < VW; ++w) {
            float s = 0.0f;
#pragma unroll
            for (int k = w; k < NK; k += VW) {
                const float y = v[k] - mean;
                s = fmaf(y, y, s);
            }
#pragma unroll
            for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            var += s;
        }
        rstd = 1.0f / sqrtf(var / float(KC ? KC : 1) + eps);
        return;
    }
    const int vthreads = 32 * vwarps;
    for (int w = 0; w < vwarps; ++w) {
        float s = 0.0f;
        for (int64_t i = 32 * w + lane; i < K; i += vthreads) s += xr[i];
#pragma unroll
        for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        sum += s;
    }
    mean = sum / float(K);
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

// Quantize the queries into shared-memory B fragments and fp32 scales (the
// k_quantize_frag result: quantize_row_q8_0 with the selected rounding, after
// the optional LayerNorm); rows >= m are zero. The LayerNorm statistics take
// one warp per row (row_stats). The blocks go four at a time to a warp: one
// coalesced 16-byte load per lane, the block maximum over its 8 lanes, and
// each lane's four quants are exactly one word of the fragment layout. A warp
// issues the loads of RO_QBATCH = 8 such tasks before it uses any of them; the
// 32 block scales of the batch are divided one per lane. Scales are stored per
// lane t of the B fragments: [block][t][n-tile][2] (queries 8 nt + 2 t + c).
constexpr int RO_QBATCH = 8;
static_assert(RO_QBATCH * 4 == 32, "one lane per block of a batch");

template <int MT, int KC>
__device__ __forceinline__ void stage_queries(const ReadoutArgs &a, int nb, uint4 *s_xf, float *s_xs,
                                              float2 *s_stats, int warps) {
    constexpr int MPAD = MT * 16;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t K = int64_t(nb) * QK;
    if (a.ln_w) {
        for (int q = warp; q < a.m; q += warps) {
            float mean, rstd;
            row_stats<KC>(a.x + int64_t(q) * a.ldx, K, a.eps, mean, rstd);
            if (lane == 0) s_stats[q] = make_float2(mean, rstd);
        }
        __syncthreads();
    }
    uint32_t *xw = reinterpret_cast<uint32_t *>(s_xf);
    const int nchunk = (nb + 3) / 4, ntask = MPAD * nchunk, j = lane & 7;
    // each phase runs over the whole batch, so the batch's shuffle and division
    // chains overlap instead of following one another
    for (int t0 = warp; t0 < ntask; t0 += RO_QBATCH * warps) {
        float4 v[RO_QBATCH];
        int qk[RO_QBATCH], bk[RO_QBATCH];
        bool live[RO_QBATCH];
#pragma unroll
        for (int k = 0; k < RO_QBATCH; ++k) {
            const int task = t0 + k * warps;
            qk[k] = task / nchunk;
            bk[k] = (task % nchunk) * 4 + (lane >> 3);
            live[k] = task < ntask && qk[k] < a.m && bk[k] < nb;
            v[k] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (live[k])
                v[k] = *reinterpret_cast<const float4 *>(a.x + int64_t(qk[k]) * a.ldx + int64_t(bk[k]) * QK + 4 * j);
        }
        float amax[RO_QBATCH];
        bool finite = true;
#pragma unroll
        for (int k = 0; k < RO_QBATCH; ++k) {
            if (live[k]) {
                if (a.ln_w) {
                    const int64_t e = int64_t(bk[k]) * QK + 4 * j;
                    const float2 ms = s_stats[qk[k]];
                    const float4 w = __ldg(reinterpret_cast<const float4 *>(a.ln_w + e));
                    const float4 c = __ldg(reinterpret_cast<const float4 *>(a.ln_b + e));
                    auto nf = [&](float x, float ww, float bb) {
                        return __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(x, ms.x), ms.y), ww), bb);
                    };
                    v[k] = make_float4(nf(v[k].x, w.x, c.x), nf(v[k].y, w.y, c.y), nf(v[k].z, w.z, c.z),
                                       nf(v[k].w, w.w, c.w));
                }
                finite = finite && isfinite(v[k].x) && isfinite(v[k].y) && isfinite(v[k].z) && isfinite(v[k].w);
            }
            amax[k] = fmaxf(fmaxf(fabsf(v[k].x), fabsf(v[k].y)), fmaxf(fabsf(v[k].z), fabsf(v[k].w)));
        }
        if (!finite && blockIdx.x == 0) atomicOr(a.flags, 1);
#pragma unroll
        for (int o = 1; o < 8; o <<= 1)
#pragma unroll
            for (int k = 0; k < RO_QBATCH; ++k) amax[k] = fmaxf(amax[k], __shfl_xor_sync(0xffffffffu, amax[k], o));
        // the batch holds 8 x 4 blocks: lane L divides for block (task L / 4, sub-block L % 4)
        // once, instead of every lane of the warp dividing for its own block
        float my_amax = 0.0f;
#pragma unroll
        for (int k = 0; k < RO_QBATCH; ++k) {
            const float m = __shfl_sync(0xffffffffu, amax[k], 8 * (lane & 3));
            if ((lane >> 2) == k) my_amax = m;
        }
        const float my_d = __fdiv_rn(my_amax, 127.0f);
        float my_id;
        if (a.mode == 2) my_id = my_amax != 0.0f ? __fdiv_rn(127.0f, my_amax) : 0.0f;
        else my_id = my_d != 0.0f ? __fdiv_rn(1.0f, my_d) : 0.0f;
        {  // the block scale, stored by the lane that divided for it
            const int k = lane >> 2, task = t0 + k * warps;
            const int q = task / nchunk, b = (task % nchunk) * 4 + (lane & 3);
            if (task < ntask && b < nb)
                s_xs[b * MPAD + ((q & 7) >> 1) * (MPAD / 4) + (q >> 3) * 2 + (q & 1)] =
                    __half2float(__float2half_rn(my_d));
        }
        float id[RO_QBATCH];
#pragma unroll
        for (int k = 0; k < RO_QBATCH; ++k) id[k] = __shfl_sync(0xffffffffu, my_id, 4 * k + (lane >> 3));
#pragma unroll
        for (int k = 0; k < RO_QBATCH; ++k) {
            const int task = t0 + k * warps;
            const int q = qk[k], b = bk[k];
            if (task >= ntask || b >= nb) continue;  // lanes past the last block of the row hold nothing
            auto quant = [&](float x) -> uint32_t {
                const float sv = __fmul_rn(x, id[k]);
                return uint32_t(a.mode == 0 ? int(roundf(sv)) : __float2int_rn(sv)) & 0xffu;
            };
            const uint32_t word =
                quant(v[k].x) | (quant(v[k].y) << 8) | (quant(v[k].z) << 16) | (quant(v[k].w) << 24);
            // word j holds elements 4j..4j+3: fragment lane 4g + (j & 3), register hi + 2 * (j >> 2)
            const int mt = q / 16, r = q % 16, g = r & 7, hi = r >> 3;
            xw[((b * MT + mt) * 32 + 4 * g + (j & 3)) * 4 + hi + 2 * (j >> 2)] = word;
        }
    }
}

template <int NT, bool Q4, int NBC>
__global__ void __launch_bounds__(RO_MAX_WARPS * 32, 1) k_readout(const ReadoutArgs a) {
    constexpr int MT = (NT + 1) / 2;
    constexpr int MPAD = MT * 16;
    constexpr int BB = ro_block_bytes(Q4);
    constexpr int QB = ro_quant_bytes(Q4);
    // NBC > 0: the block count is a compile-time constant (every loop below unrolls)
    constexpr int CBC = NBC ? (NBC < RO_SLOT / BB ? NBC : RO_SLOT / BB) : 1;
    constexpr int CPTC = NBC ? (NBC + CBC - 1) / CBC : 1;
    extern __shared__ __align__(128) unsigned char smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, t = lane & 3;
    const int warps = blockDim.x >> 5, R = a.ring;
    const int nb = NBC ? NBC : int(a.nb), cb = NBC ? CBC : a.cb, cpt = NBC ? CPTC : (nb + cb - 1) / cb;

    // shared memory: rings, barriers, query fragments and scales, per-warp keys, suppression bits
    unsigned char *ring = smem + size_t(warp) * R * RO_SLOT;
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem + size_t(warps) * R * RO_SLOT) + warp * R;
    uint4 *s_xf = reinterpret_cast<uint4 *>(smem + size_t(warps) * R * (RO_SLOT + 8));
    float *s_xs = reinterpret_cast<float *>(s_xf + nb * MT * 32);
    unsigned long long *s_keys = reinterpret_cast<unsigned long long *>(s_xs + nb * MPAD);  // [warps][32]
    float2 *s_stats = reinterpret_cast<float2 *>(s_keys + warps * 32);                      // [32]
    uint32_t *s_sup = reinterpret_cast<uint32_t *>(s_stats + 32);

    // tiles: a balanced contiguous range per CTA, dealt round-robin to its warps
    // (rows stay increasing per lane, which the running maximum relies on)
    const int64_t cta_t0 = a.tiles * blockIdx.x / gridDim.x, cta_t1 = a.tiles * (blockIdx.x + 1) / gridDim.x;
    const int64_t cta_row0 = cta_t0 * 16, cta_row1 = cta_t1 * 16;
    const int64_t ntiles = cta_t1 - cta_t0 > warp ? (cta_t1 - cta_t0 - warp + warps - 1) / warps : 0;
    const int64_t steps = ntiles * cpt;
    auto tile_of = [&](int64_t i) { return cta_t0 + warp + i * warps; };

    if (lane == 0) {
        for (int u = 0; u < R; ++u) mbar_init(bar + u, 1);
        fence_mbar_init();
    }
    __syncwarp();
    auto issue = [&](int64_t s, int u) {  // lane 0 only
        const int64_t tile = tile_of(s / cpt);
        const int b0 = int(s % cpt) * cb;
        const int nblk = nb - b0 < cb ? nb - b0 : cb;
        const uint32_t bytes = uint32_t(nblk * BB);
        mbar_expect_tx(bar + u, bytes);
        bulk_g2s(ring + u * RO_SLOT, a.wt + (tile * nb + b0) * BB, bytes, bar + u);
    };
    if (lane == 0)
        for (int u = 0; u < R && u < steps; ++u) issue(u, u);  // immutable weights: before waiting on x

    for (int i = threadIdx.x; i < a.sup_words; i += blockDim.x) s_sup[i] = 0u;
    pdl_wait();
    pdl_trigger();  // the next kernel may launch now; it waits for this grid before reading
    if (a.pre_xf) {  // wide rows: one quantization for the whole grid, each CTA copies the 8-bit fragments
        // (asynchronous 16-byte copies: all of a thread's copies in flight at once)
        for (int i = threadIdx.x; i < nb * MT * 32; i += blockDim.x) cp_async16(s_xf + i, a.pre_xf + i, 16);
        for (int i = threadIdx.x; i < nb * MPAD; i += blockDim.x) {
            const int b = i / MPAD, q = i % MPAD;
            s_xs[b * MPAD + ((q & 7) >> 1) * (MPAD / 4) + (q >> 3) * 2 + (q & 1)] = a.pre_xs[i];
        }
        cp_async_wait_all();
    } else {
        stage_queries<MT, NBC * QK>(a, nb, s_xf, s_xs, s_stats, warps);
    }
    __syncthreads();  // bitmask zeroed before it is set
    for (int64_t i = threadIdx.x; i < a.nsup; i += blockDim.x) {
        const int64_t n = a.suppressed[i];
        if (n >= cta_row0 && n < cta_row1) {
            const int64_t o = n - cta_row0;
            atomicOr(s_sup + (o >> 5), 1u << (o & 31));
        }
    }
    __syncthreads();

    float bv[NT][2];
    uint32_t bn[NT][2];
    {
        const int64_t r = tile_of(0) * 16 + g;  // this lane's first row (its later rows are larger)
        const uint32_t n0 = ntiles > 0 && r < a.rows ? uint32_t(r) : 0xFFFFFFFFu;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) bv[nt][0] = bv[nt][1] = -INFINITY, bn[nt][0] = bn[nt][1] = n0;
    }
    const bool all_queries = a.m == 8 * NT;
    const bool argmax = a.keys != nullptr;

    int64_t st = 0;
    bool failed = false;
    for (int64_t i = 0; i < ntiles && !failed; ++i) {
        const int64_t tile = tile_of(i);
        float2 acc[NT][2];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = make_float2(0.0f, 0.0f);
        // one block of the tile: 16 rows x 8 * NT queries x 32
        auto block = [&](const unsigned char *blk, int b) {
            uint32_t a0, a1, a2, a3;
            if (Q4) {
                const uint2 w = reinterpret_cast<const uint2 *>(blk)[lane];
                a0 = ((w.x << 4) ^ 0x80808080u) & 0xF0F0F0F0u;  // row g, k 4t..: 16 * (low nibble - 8)
                a2 = (w.x ^ 0x80808080u) & 0xF0F0F0F0u;         // row g, k 16+4t..: high nibbles
                a1 = ((w.y << 4) ^ 0x80808080u) & 0xF0F0F0F0u;  // row g+8
                a3 = (w.y ^ 0x80808080u) & 0xF0F0F0F0u;
            } else {
                const uint4 w = reinterpret_cast<const uint4 *>(blk)[lane];
                a0 = w.x;
                a1 = w.y;
                a2 = w.z;
                a3 = w.w;
            }
            const __half2 hw = reinterpret_cast<const __half2 *>(blk + QB)[g];  // rows g, g+8
            // per row, as broadcast pairs: Q4 dw/16 and -786432 * dw; Q8 dw
            float2 s0 = __half22float2(__low2half2(hw));
            float2 s1 = __half22float2(__high2half2(hw));
            float2 c0, c1;
            if (Q4) {
                s0 = mul2(s0, make_float2(0.0625f, 0.0625f));
                s1 = mul2(s1, make_float2(0.0625f, 0.0625f));
                c0 = mul2(s0, make_float2(-12582912.0f, -12582912.0f));
                c1 = mul2(s1, make_float2(-12582912.0f, -12582912.0f));
            }
            // this lane's query scales of the block: pairs (8 nt + 2 t, +1) for every n-tile
            float2 dxs[NT];
            if (NT == 1) {
                dxs[0] = *reinterpret_cast<const float2 *>(s_xs + b * MPAD + t * (MPAD / 4));
            } else {
                const float4 *xs4 = reinterpret_cast<const float4 *>(s_xs + b * MPAD + t * (MPAD / 4));
#pragma unroll
                for (int i = 0; i < NT / 2; ++i) {
                    const float4 f = xs4[i];
                    dxs[2 * i] = make_float2(f.x, f.y);
                    dxs[2 * i + 1] = make_float2(f.z, f.w);
                }
            }
            const float2 zero = make_float2(0.0f, 0.0f);
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                const uint4 xf = s_xf[(b * MT + mt) * 32 + lane];
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int nt = 2 * mt + h;
                    if (nt >= NT) break;
                    int d[4];
                    mma_magic(d, a0, a1, a2, a3, h ? xf.y : xf.x, h ? xf.w : xf.z);
                    const float2 dx = dxs[nt];
                    // each term is an fma with a +0 addend (exactly the product here, since a
                    // running sum never holds -0): ptxas would fuse a packed multiply into the
                    // packed add that follows it, an fma it cannot fuse
                    float2 lo, hi;
                    if (Q4) {
                        lo = fma2(fma2(biased(d[0], d[1]), s0, c0), dx, zero);
                        hi = fma2(fma2(biased(d[2], d[3]), s1, c1), dx, zero);
                    } else {
                        const float2 unbias = make_float2(-12582912.0f, -12582912.0f);  // exact
                        lo = fma2(add2(biased(d[0], d[1]), unbias), mul2(s0, dx), zero);
                        hi = fma2(add2(biased(d[2], d[3]), unbias), mul2(s1, dx), zero);
                    }
                    acc[nt][0] = add2(acc[nt][0], lo);
                    acc[nt][1] = add2(acc[nt][1], hi);
                }
            }
        };
#pragma unroll
        for (int c = 0; c < (NBC ? CPTC : cpt); ++c, ++st) {
            const int u = int(st % R);
            if (!mbar_wait_bounded(bar + u, uint32_t((st / R) & 1))) {
                failed = true;
                break;
            }
            const unsigned char *slot = ring + u * RO_SLOT;
            if (NBC) {
#pragma unroll
                for (int j = 0; j < CBC; ++j)
                    if (c * CBC + j < NBC) block(slot + j * BB, c * CBC + j);
            } else {
                const int b0 = c * cb, nblk = nb - b0 < cb ? nb - b0 : cb;
#pragma unroll 2
                for (int j = 0; j < nblk; ++j) block(slot + j * BB, b0 + j);
            }
            __syncwarp();  // every lane has read the slot before it is refilled
            if (lane == 0 && st + R < steps) {
                fence_proxy_async();
                issue(st + R, u);
            }
        }
        if (failed) break;
        // epilogue of the tile: rows n0 (g) and n1 (g + 8)
        const int64_t n0 = tile * 16 + g, n1 = n0 + 8;
        bool z0 = false, z1 = false;
        if (a.nsup) {
            auto suppressed = [&](int64_t n) {
                const int64_t o = n - cta_row0;
                return n < a.rows && ((s_sup[o >> 5] >> (o & 31)) & 1u);
            };
            z0 = suppressed(n0);
            z1 = suppressed(n1);
        }
        float *o0 = a.out + n0, *o1 = a.out + n1;
        if (!argmax) {  // plain linear: bias, then residual (the GEMV epilogue order)
            const float b0 = a.bias && n0 < a.rows ? a.bias[n0] : 0.0f, b1 = a.bias && n1 < a.rows ? a.bias[n1] : 0.0f;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int cc = 0; cc < 2; ++cc) {
                    const int64_t q = 8 * nt + 2 * t + cc;
                    if (q >= a.m) continue;
                    float v0 = cc ? acc[nt][0].y : acc[nt][0].x, v1 = cc ? acc[nt][1].y : acc[nt][1].x;
                    if (a.bias) {
                        v0 = __fadd_rn(v0, b0);
                        v1 = __fadd_rn(v1, b1);
                    }
                    if (n0 < a.rows) {
                        if (a.residual) v0 = __fadd_rn(a.residual[q * a.ldo + n0], v0);
                        o0[q * a.ldo] = v0;
                    }
                    if (n1 < a.rows) {
                        if (a.residual) v1 = __fadd_rn(a.residual[q * a.ldo + n1], v1);
                        o1[q * a.ldo] = v1;
                    }
                }
        } else if (all_queries && (tile + 1) * 16 <= a.rows) {  // full tile, every query live: no predicates
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int cc = 0; cc < 2; ++cc) {
                    const int64_t q = 8 * nt + 2 * t + cc;
                    const float v0 = z0 ? -INFINITY : (cc ? acc[nt][0].y : acc[nt][0].x);
                    const float v1 = z1 ? -INFINITY : (cc ? acc[nt][1].y : acc[nt][1].x);
                    o0[q * a.ldo] = v0;
                    o1[q * a.ldo] = v1;
                    running_max(bv[nt][cc], bn[nt][cc], v0, uint32_t(n0));
                    running_max(bv[nt][cc], bn[nt][cc], v1, uint32_t(n1));
                }
        } else {
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int cc = 0; cc < 2; ++cc) {
                    const int64_t q = 8 * nt + 2 * t + cc;
                    if (q >= a.m) continue;
                    const float v0 = z0 ? -INFINITY : (cc ? acc[nt][0].y : acc[nt][0].x);
                    const float v1 = z1 ? -INFINITY : (cc ? acc[nt][1].y : acc[nt][1].x);
                    if (n0 < a.rows) {
                        o0[q * a.ldo] = v0;
                        running_max(bv[nt][cc], bn[nt][cc], v0, uint32_t(n0));
                    }
                    if (n1 < a.rows) {
                        o1[q * a.ldo] = v1;
                        running_max(bv[nt][cc], bn[nt][cc], v1, uint32_t(n1));
                    }
                }
        }
    }
    if (failed) {  // report, then drain this warp's copies still in flight (bounded)
        if (lane == 0) atomicOr(a.flags, 2);
        for (int64_t q = st; q < steps && q < st + R; ++q) mbar_wait_bounded(bar + int(q % R), uint32_t((q / R) & 1));
    }

    // keys: per warp over the 8 lanes sharing t, per CTA over the warps (in
    // shared memory), across CTAs with one 64-bit atomic max per query
    if (argmax) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
            unsigned long long key = bn[nt][cc] < uint32_t(a.rows) ? argmax_key(bv[nt][cc], bn[nt][cc]) : 0ull;
#pragma unroll
            for (int o = 4; o < 32; o <<= 1) {
                const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
                key = other > key ? other : key;
            }
            if (g == 0) s_keys[warp * 32 + 8 * nt + 2 * t + cc] = key;
        }
    }
    __shared__ bool last;
    __syncthreads();
    if (argmax && threadIdx.x < a.m) {
        unsigned long long best = 0ull;
        for (int w = 0; w < warps; ++w) {
            const unsigned long long k = s_keys[w * 32 + threadIdx.x];
            best = k > best ? k : best;
        }
        if (best) atomicMax(a.keys + threadIdx.x, best);
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(a.done, 1u) == gridDim.x - 1;
    __syncthreads();
    if (last) {
        __threadfence();
        if (argmax && threadIdx.x < a.m) {
            const unsigned long long k = atomicExch(a.keys + threadIdx.x, 0ull);
            a.token[threadIdx.x] = int64_t(0xFFFFFFFFu - uint32_t(k & 0xFFFFFFFFull));
        }
        if (threadIdx.x == 0) {
            *a.status = atomicExch(a.flags, 0);
            *a.done = 0u;
        }
    }
}

// ---------------------------------------------------------------- host
static int ro_sm_count() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

struct ReadoutPlan {
    int warps = 0, ring = 0, cb = 0, sup_words = 0, grid = 0;
    size_t smem = 0;
};

// Launch shape: one CTA per SM; the most warps and ring slots whose shared
// memory fits, preferring warps.
static ReadoutPlan plan_readout(int64_t tiles, int64_t nb, int q4, int mt) {
    ReadoutPlan p;
    const int bb = ro_block_bytes(q4);
    p.cb = int(nb < RO_SLOT / bb ? nb : RO_SLOT / bb);
    p.grid = int(tiles < ro_sm_count() ? tiles : ro_sm_count());
    const size_t act = size_t(nb) * mt * 512 + size_t(nb) * mt * 16 * 4;
    const int64_t cta_tiles = (tiles + p.grid - 1) / p.grid;
    const int words = int((cta_tiles * 16 + 31) / 32) + 1;
    const int shapes[][2] = {{16, 3}, {16, 2}, {8, 4}, {8, 3}, {8, 2}, {4, 2}};
    for (const auto &sh : shapes) {
        const size_t bytes =
            size_t(sh[0]) * sh[1] * (RO_SLOT + 8) + act + size_t(sh[0]) * 32 * 8 + 32 * 8 + size_t(words) * 4;
        if (bytes <= RO_SMEM_LIMIT) {
            p.warps = sh[0];
            p.ring = sh[1];
            p.sup_words = words;
            p.smem = bytes;
            return p;
        }
    }
    return p;  // warps == 0: does not fit
}

bool readout_tiles_fit(int64_t rows, int64_t nb, int q4) {
    return plan_readout(ceil_div(rows, 16), nb, q4, 2).warps > 0;
}

void launch_readout_repack(int q4, const uint8_t *blocks, uint8_t *wt, int64_t rows, int64_t nb, cudaStream_t s) {
    const int64_t tiles = ceil_div(rows, 16);
    const int64_t threads = tiles * nb * 32;
    const unsigned grid = unsigned(ceil_div(threads, 256));
    if (q4) k_readout_repack<true><<<grid, 256, 0, s>>>(blocks, wt, rows, nb, tiles);
    else k_readout_repack<false><<<grid, 256, 0, s>>>(blocks, wt, rows, nb, tiles);
}

template <int NT, bool Q4, int NBC>
static void launch_nbc(const ReadoutArgs &a, const ReadoutPlan &p, cudaStream_t s) {
    auto kernel = k_readout<NT, Q4, NBC>;
    static bool configured = false;
    if (!configured) {
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(RO_SMEM_LIMIT));
        configured = true;
    }
    launch_pdl(kernel, dim3(unsigned(p.grid)), dim3(unsigned(p.warps * 32)), p.smem, s, a);
}

// Specialised block counts: 12 (K = 384, Whisper tiny); anything else runs the generic loop.
template <int NT, bool Q4>
static void launch_nt(const ReadoutArgs &a, const ReadoutPlan &p, cudaStream_t s) {
    if (a.nb == 12) launch_nbc<NT, Q4, 12>(a, p, s);
    else launch_nbc<NT, Q4, 0>(a, p, s);
}

// One readout launch over the handle's tile layout: quantization (after the
// optional LayerNorm), the block products, suppression, logits, argmax and
// status, for 1..32 query rows.
void launch_readout(const Linear &h, const float *x, int64_t ldx, int64_t m, const float *ln_w,
                    const float *ln_b, float eps, int mode, float *logits, int64_t *token, int *status,
                    const int64_t *suppressed, int64_t nsup, cudaStream_t s, int64_t ldo, const float *bias,
                    const float *residual) {
    const int nt = m <= 8 ? 1 : m <= 16 ? 2 : 4;
    const int mt = (nt + 1) / 2;
    const ReadoutPlan p = plan_readout(h.tiles, h.nb, h.q4, mt);
    require(p.warps > 0, "readout tile plan does not fit in shared memory");
    ReadoutArgs a{};
    a.wt = h.wt;
    a.tiles = h.tiles;
    a.nb = h.nb;
    a.rows = h.rows;
    a.cb = p.cb;
    a.ring = p.ring;
    a.sup_words = p.sup_words;
    a.x = x;
    a.ldx = ldx;
    a.m = m;
    if (h.nb > RO_SELF_QUANT_BLOCKS) {  // every CTA quantizing wide rows would re-read them from L2 148 times
        launch_quantize_frag(mode, x, ldx, m, h.width, mt * 16, h.nb_pad, ln_w, ln_b, eps, h.xf, h.xs, h.xsum,
                             h.ro_flags, s);
        a.pre_xf = reinterpret_cast<const uint4 *>(h.xf);
        a.pre_xs = h.xs;
    }
    a.ln_w = ln_w;
    a.ln_b = ln_b;
    a.eps = eps;
    a.mode = mode;
    a.out = logits;
    a.ldo = ldo > 0 ? ldo : h.rows;
    a.bias = bias;
    a.residual = residual;
    a.keys = token ? h.keys : nullptr;
    a.done = h.done;
    a.flags = h.ro_flags;
    a.token = token;
    a.suppressed = suppressed;
    a.nsup = nsup;
    a.status = status;
    if (h.q4) {
        if (nt == 1) launch_nt<1, true>(a, p, s);
        else if (nt == 2) launch_nt<2, true>(a, p, s);
        else launch_nt<4, true>(a, p, s);
    } else {
        if (nt == 1) launch_nt<1, false>(a, p, s);
        else if (nt == 2) launch_nt<2, false>(a, p, s);
        else launch_nt<4, false>(a, p, s);
    }
}

}  // namespace mb
