#pragma once
// Decode / prefill attention over fp16 K/V planes as device functions, shared
// by the attention kernels (decoder.cu) and the persistent decode-step kernel
// (step.cu).
#include "quant.cuh"

namespace mb {

constexpr int HEAD_DIM = 64;
constexpr int MAX_Q = 4;
constexpr int TILE_KEYS = 64;        // keys per shared-memory tile
constexpr int ATT_THREADS = 128;      // CTA size for up to 4 row tiles
constexpr int ATT_MAX_THREADS = 256;  // one warp per 16-row tile up to 128 rows
constexpr int ATT_MAX_ROWS = 128;    // query rows one CTA attends (all B*NQ rows when the planes are shared)
constexpr int SHARED_SPLITS = 16;    // key splits per head over shared planes at most (one thread-block cluster per head)
constexpr int ATT_PRE = 4;           // key tiles a CTA loads into shared memory at once

// Key splits of one head over shared planes: at most SHARED_SPLITS, each with the same
// number of 64-key tiles (a 1500-position source: 24 tiles as 12 splits of 2), so that no
// CTA of the head's cluster is left without keys.
__host__ __device__ inline int shared_splits(int tiles) {
    const int per = (tiles + SHARED_SPLITS - 1) / SHARED_SPLITS;
    return (tiles + per - 1) / per;
}

struct AttArgs {
    const float *q;
    int64_t q_stride;
    const float *knew, *vnew;
    int64_t kv_stride;
    __half *kc, *vc;
    int64_t capacity;
    int heads, nq, batch, shared, splits, rows;  // rows per CTA: shared ? batch * nq : nq
    int tiles_per_split;
    const int64_t *begin, *kv_len;
    float *out;
    int64_t out_stride;
    float scale;
    int *status;
    float *partial;  // splits > 1: [groups * heads][splits][rows][HEAD_DIM + 2] (O, max, sum)
    Q8Frags frags;   // xf != null: also write the output rows as the next linear's Q8_0 fragments
};

// Q8_0 fragments of one output row of a head from the attention epilogue: lane
// (g, t4) of the row's 4-lane group holds dims 8 j + 2 t4 + c, so block kb
// (dims 32 kb ..) is j = 4 kb + jj with element 8 jj + 2 t4 + c. The block
// maximum and quant sum take the 4 lanes; fragment word w = 2 jj + t4 / 2
// (elements 4 w .. 4 w + 3) joins the bytes of lanes t4 and t4 + 1.
template <int MODE>
__device__ __forceinline__ void frag_head_row(const Q8Frags &f, const float (&v)[8][2], int64_t token, int h,
                                              int t4, unsigned group, int *status) {
    const int64_t mtiles = f.mpad / 16, mt = token / 16;
    const int r = int(token % 16), gq = r & 7, hi = r >> 3;
#pragma unroll
    for (int kb = 0; kb < 2; ++kb) {
        const int64_t b = 2 * h + kb;
        float amax = 0.0f;
        bool finite = true;
#pragma unroll
        for (int jj = 0; jj < 4; ++jj)
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                amax = fmaxf(amax, fabsf(v[4 * kb + jj][c]));
                finite = finite && isfinite(v[4 * kb + jj][c]);
            }
        if (!finite) atomicOr(status, 1);
#pragma unroll
        for (int o = 1; o <= 2; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(group, amax, o));
        const float d = __fdiv_rn(amax, 127.0f);
        float id;
        if (MODE == 2) id = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
        else id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        int qsum = 0;
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
            int qv[2];
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                const float sv = __fmul_rn(v[4 * kb + jj][c], id);
                qv[c] = MODE == 0 ? int(roundf(sv)) : __float2int_rn(sv);
                qsum += qv[c];
            }
            const uint32_t hw = (uint32_t(qv[0]) & 0xffu) | ((uint32_t(qv[1]) & 0xffu) << 8);
            const uint32_t other = __shfl_xor_sync(group, hw, 1);
            if ((t4 & 1) == 0) {
                const int w = 2 * jj + (t4 >> 1);
                f.xf[((b * mtiles + mt) * 32 + 4 * gq + (w & 3)) * 4 + hi + 2 * (w >> 2)] = hw | (other << 16);
            }
        }
#pragma unroll
        for (int o = 1; o <= 2; o <<= 1) qsum += __shfl_xor_sync(group, qsum, o);
        if (t4 == 0) {
            f.xs[b * f.mpad + token] = __half2float(__float2half_rn(d));
            f.xsum[b * f.mpad + token] = qsum;
        }
    }
}

// D += A(16x16 f16, row) * B(16x8 f16, col), fp32 accumulate.
__device__ __forceinline__ void mma_f16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) { return half2_bits(__floats2half2_rn(lo, hi)); }

constexpr int ATT_LD = HEAD_DIM + 8;  // fp16 row stride of the shared tiles (72 halves: conflict-free fragment loads)

// Warps per 16-row tile of attend_task ("tile lanes", key tiles processed side
// by side): a function of the row count only, so every caller (its own block
// size permitting mtiles * lanes warps) computes the same bits.
__host__ __device__ constexpr int att_tile_lanes(int rows) {
    return (rows + 15) / 16 <= 2 ? 4 : (rows + 15) / 16 <= 4 ? 2 : 1;
}
__host__ __device__ constexpr int att_threads(int rows) { return 32 * ((rows + 15) / 16) * att_tile_lanes(rows); }

// Shared memory of attend_task for `rows` query rows: fp16 Q hi / lo, ATT_PRE K
// tiles and V tiles, the per-row key limits (the tile buffers hold the lanes'
// states for the final merge).
__host__ __device__ constexpr size_t att_smem_bytes(int rows) {
    return (2 * size_t((rows + 15) / 16 * 16) + 2 * size_t(ATT_PRE) * TILE_KEYS) * ATT_LD * 2 +
           size_t((rows + 15) / 16 * 16) * 4;
}

// Decode / prefill attention over the fp16 K/V planes, flash-attention style
// on the tensor cores (mma.sync m16n8k16, fp16 operands, fp32 accumulation).
// CTA (group g, head h, split s) walks its key tiles of 64: S = Q K^T, online
// softmax in registers, O += P V. K and V are exact fp16 (the planes); Q and P
// are fp32 values carried as fp16 pairs hi + lo (two MMAs each), so scores and
// sums keep about 22 bits, like the fp32 attention they replace. With shared planes
// one group holds every sequence's query rows (r = b*nq + i) so the cross
// attention of the whole batch reuses each K/V tile, and the keys are split
// across SHARED_SPLITS CTAs per head (flash-decoding) whose partial results
// k_attend_merge combines; otherwise group g is sequence b with its nq rows.
// Row (b, i) sees keys [0, len), len = causal ? begin_b + i + 1 : kv_len_b; the
// CTA whose tile holds the new positions begin_b .. begin_b + nq - 1 first
// writes their K/V rows to the planes (fp16, ggml_set_rows,
// decoder.cpp:566-567). Warp w owns the 16-row tile w (the CTA has
// max(4, row tiles) warps).
//
// A CTA loads up to ATT_PRE of its key tiles at once (one round of loads for
// the group), then runs the tiles' math in order. With part_dst (splits > 1)
// the split's partial rows go to that shared-memory array instead of the
// global partial buffer.
template <bool CAUSAL>
__device__ __forceinline__ void attend_task(const AttArgs &a, int task, unsigned char *att_smem,
                                            float *part_dst = nullptr) {
    const int R = a.rows, mtiles = (R + 15) / 16;
    __half *qs = reinterpret_cast<__half *>(att_smem);            // [mtiles*16][72] fp16(q)
    __half *ql = qs + mtiles * 16 * ATT_LD;                       // [mtiles*16][72] fp16(q - fp16(q))
    __half *ks0 = ql + mtiles * 16 * ATT_LD;                      // [ATT_PRE][64 keys][72]
    __half *vs0 = ks0 + ATT_PRE * TILE_KEYS * ATT_LD;             // [ATT_PRE][64 keys][72]
    int *lim = reinterpret_cast<int *>(vs0 + ATT_PRE * TILE_KEYS * ATT_LD);  // [mtiles*16]
    __shared__ int maxlim;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t4 = lane & 3;
    const int split = task % a.splits, gh = task / a.splits;
    const int h = gh % a.heads, grp = gh / a.heads;
    const int width = a.heads * HEAD_DIM;
    const int64_t seq = a.shared ? 0 : grp;
    __half *kp = a.kc + seq * a.capacity * width + h * HEAD_DIM;
    __half *vp = a.vc + seq * a.capacity * width + h * HEAD_DIM;
    auto row_seq = [&](int r) { return a.shared ? r / a.nq : grp; };
    auto row_q = [&](int r) { return a.shared ? int64_t(r) : int64_t(grp) * a.nq + r; };  // global query row

    if (tid == 0) maxlim = 0;
    __syncthreads();
    for (int r = tid; r < mtiles * 16; r += blockDim.x) {
        int64_t len = 0;
        if (r < R) {
            const int b = row_seq(r), i = r % a.nq;
            bool ok;
            if (CAUSAL) {
                const int64_t b0 = a.begin[b];
                ok = b0 >= 0 && b0 + a.nq <= a.capacity;
                len = b0 + i + 1;
            } else {
                len = a.kv_len[b];
                ok = len >= 1 && len <= a.capacity;
            }
            if (!ok) {
                len = 0;
                if (split == 0) atomicOr(a.status, 8);
            }
        }
        lim[r] = int(len);
        atomicMax(&maxlim, int(len));
    }
    for (int e = tid; e < mtiles * 16 * (HEAD_DIM / 2); e += blockDim.x) {
        const int r = e / (HEAD_DIM / 2), d2 = (e % (HEAD_DIM / 2)) * 2;
        float2 v = make_float2(0.0f, 0.0f);
        if (r < R) v = *reinterpret_cast<const float2 *>(a.q + row_q(r) * a.q_stride + h * HEAD_DIM + d2);
        const __half2 hi = __floats2half2_rn(v.x, v.y);
        const float2 back = __half22float2(hi);
        *reinterpret_cast<__half2 *>(qs + r * ATT_LD + d2) = hi;
        *reinterpret_cast<__half2 *>(ql + r * ATT_LD + d2) = __floats2half2_rn(v.x - back.x, v.y - back.y);
    }
    __syncthreads();

    // this warp's 16-row tile mt and tile lane tl: the warps of a row tile take the key tiles of a
    // group in turn (tile gi goes to lane gi mod TL), each with its own O [16 x 64] (8 n-tiles x 4)
    // and running max / sum of rows g, g+8; the lanes' states are merged in lane order at the end
    const int TL = att_tile_lanes(R);
    const int mt = warp % mtiles, tl = warp / mtiles;
    const bool active = tl < TL;
    float o[8][4];
    float mrun[2] = {-INFINITY, -INFINITY}, lrun[2] = {0.0f, 0.0f};
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
    const int64_t t_begin = int64_t(split) * a.tiles_per_split;
    int64_t t_end = t_begin + a.tiles_per_split;
    if (t_end * TILE_KEYS > maxlim) t_end = (int64_t(maxlim) + TILE_KEYS - 1) / TILE_KEYS;  // tiles past every row
    for (int64_t tg = t_begin; tg < t_end; tg += ATT_PRE) {
      const int ng = int(t_end - tg < ATT_PRE ? t_end - tg : ATT_PRE);
      // K and V tiles [key][dim] of the group, fp16, by 16-byte asynchronous copies all in flight at
      // once; keys past every row's length are zero-filled (never stale plane bytes); the new
      // rows of a causal step come from knew / vnew and are written to the planes as well
      for (int e = tid; e < ng * TILE_KEYS * HEAD_DIM / 8; e += blockDim.x) {
            const int gi = e / (TILE_KEYS * HEAD_DIM / 8), ee = e % (TILE_KEYS * HEAD_DIM / 8);
            const int jj = ee / (HEAD_DIM / 8), d8 = (ee % (HEAD_DIM / 8)) * 8;
            const int64_t j = (tg + gi) * TILE_KEYS + jj;
            __half *ks = ks0 + gi * TILE_KEYS * ATT_LD + jj * ATT_LD + d8;
            __half *vs = vs0 + gi * TILE_KEYS * ATT_LD + jj * ATT_LD + d8;
            const bool live = j < maxlim;
            const int64_t b0 = CAUSAL && a.knew ? a.begin[grp] : -1;
            if (live && CAUSAL && a.knew && b0 >= 0 && j >= b0 && j < b0 + a.nq && b0 + a.nq <= a.capacity) {
                const int64_t src = (int64_t(grp) * a.nq + (j - b0)) * a.kv_stride + h * HEAD_DIM + d8;
                __half kh[8], vh[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    kh[u] = __float2half_rn(a.knew[src + u]);
                    vh[u] = __float2half_rn(a.vnew[src + u]);
                }
                uint4 kr, vr;
                memcpy(&kr, kh, 16);
                memcpy(&vr, vh, 16);
                *reinterpret_cast<uint4 *>(kp + j * width + d8) = kr;
                *reinterpret_cast<uint4 *>(vp + j * width + d8) = vr;
                *reinterpret_cast<uint4 *>(ks) = kr;
                *reinterpret_cast<uint4 *>(vs) = vr;
            } else {
                const int64_t jr = live ? j : 0;  // a valid row address; nothing is read when not live
                cp_async16(ks, kp + jr * width + d8, live ? 16 : 0);
                cp_async16(vs, vp + jr * width + d8, live ? 16 : 0);
            }
      }
      cp_async_wait_all();
      __syncthreads();
      for (int gi = tl; gi < ng; gi += TL) {
        const int64_t c0 = (tg + gi) * TILE_KEYS;
        const __half *ks = ks0 + gi * TILE_KEYS * ATT_LD, *vs = vs0 + gi * TILE_KEYS * ATT_LD;
        if (active) {
            const int r0 = mt * 16 + g, r1 = r0 + 8;
            // S = Q K^T over the 64 dims (4 k-steps) for the 8 key n-tiles
            float sc[8][4];
#pragma unroll
            for (int j = 0; j < 8; ++j) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.0f;
#pragma unroll
            for (int kk = 0; kk < HEAD_DIM / 16; ++kk) {
                uint32_t af[4], al[4];
                const int o0 = r0 * ATT_LD + kk * 16 + 2 * t4, o1 = r1 * ATT_LD + kk * 16 + 2 * t4;
                af[0] = *reinterpret_cast<const uint32_t *>(qs + o0);
                af[1] = *reinterpret_cast<const uint32_t *>(qs + o1);
                af[2] = *reinterpret_cast<const uint32_t *>(qs + o0 + 8);
                af[3] = *reinterpret_cast<const uint32_t *>(qs + o1 + 8);
                al[0] = *reinterpret_cast<const uint32_t *>(ql + o0);
                al[1] = *reinterpret_cast<const uint32_t *>(ql + o1);
                al[2] = *reinterpret_cast<const uint32_t *>(ql + o0 + 8);
                al[3] = *reinterpret_cast<const uint32_t *>(ql + o1 + 8);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const __half *kb = ks + (8 * j + g) * ATT_LD + kk * 16 + 2 * t4;
                    const uint32_t b0 = *reinterpret_cast<const uint32_t *>(kb), b1 = *reinterpret_cast<const uint32_t *>(kb + 8);
                    mma_f16(sc[j], af, b0, b1);
                    mma_f16(sc[j], al, b0, b1);
                }
            }
            // scale, mask, online softmax of rows r0 (c0, c1) and r1 (c2, c3)
            const int l0 = lim[r0], l1 = lim[r1];
            float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int64_t key = c0 + 8 * j + 2 * t4;
                sc[j][0] = key < l0 ? sc[j][0] * a.scale : -INFINITY;
                sc[j][1] = key + 1 < l0 ? sc[j][1] * a.scale : -INFINITY;
                sc[j][2] = key < l1 ? sc[j][2] * a.scale : -INFINITY;
                sc[j][3] = key + 1 < l1 ? sc[j][3] * a.scale : -INFINITY;
                mx0 = fmaxf(mx0, fmaxf(sc[j][0], sc[j][1]));
                mx1 = fmaxf(mx1, fmaxf(sc[j][2], sc[j][3]));
            }
#pragma unroll
            for (int off = 1; off <= 2; off <<= 1) {
                mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
                mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
            }
            const float mn0 = fmaxf(mrun[0], mx0), mn1 = fmaxf(mrun[1], mx1);
            const float al0 = mn0 == -INFINITY || mrun[0] == -INFINITY ? 0.0f : __expf(mrun[0] - mn0);
            const float al1 = mn1 == -INFINITY || mrun[1] == -INFINITY ? 0.0f : __expf(mrun[1] - mn1);
            float sum0 = 0.0f, sum1 = 0.0f;
            uint32_t pf[8][2], pl[8][2];  // P = fp16 pairs + fp16 remainders: rows r0 / r1, key n-tile j
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float p0 = mn0 == -INFINITY ? 0.0f : __expf(sc[j][0] - mn0);
                const float p1 = mn0 == -INFINITY ? 0.0f : __expf(sc[j][1] - mn0);
                const float p2 = mn1 == -INFINITY ? 0.0f : __expf(sc[j][2] - mn1);
                const float p3 = mn1 == -INFINITY ? 0.0f : __expf(sc[j][3] - mn1);
                sum0 += p0 + p1;
                sum1 += p2 + p3;
                const __half2 h01 = __floats2half2_rn(p0, p1), h23 = __floats2half2_rn(p2, p3);
                const float2 b01 = __half22float2(h01), b23 = __half22float2(h23);
                pf[j][0] = half2_bits(h01);
                pf[j][1] = half2_bits(h23);
                pl[j][0] = pack_half2(p0 - b01.x, p1 - b01.y);
                pl[j][1] = pack_half2(p2 - b23.x, p3 - b23.y);
            }
#pragma unroll
            for (int off = 1; off <= 2; off <<= 1) {
                sum0 += __shfl_xor_sync(0xffffffffu, sum0, off);
                sum1 += __shfl_xor_sync(0xffffffffu, sum1, off);
            }
            lrun[0] = fmaf(lrun[0], al0, sum0);
            lrun[1] = fmaf(lrun[1], al1, sum1);
            mrun[0] = mn0;
            mrun[1] = mn1;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                o[j][0] *= al0;
                o[j][1] *= al0;
                o[j][2] *= al1;
                o[j][3] *= al1;
            }
            // O += P V: k-steps of 16 keys (P fragments from the score n-tiles 2ks, 2ks+1)
#pragma unroll
            for (int kk = 0; kk < TILE_KEYS / 16; ++kk) {
                const uint32_t af[4] = {pf[2 * kk][0], pf[2 * kk][1], pf[2 * kk + 1][0], pf[2 * kk + 1][1]};
                const uint32_t al[4] = {pl[2 * kk][0], pl[2 * kk][1], pl[2 * kk + 1][0], pl[2 * kk + 1][1]};
                // B fragments of V (16 keys x 8 dims) for n-tiles 2 jp and 2 jp + 1, transposed from
                // the row-major tile: thread 8 m + r addresses key 16 kk + r + 8 (m & 1), dims 8 (2 jp + m / 2)
#pragma unroll
                for (int jp = 0; jp < 4; ++jp) {
                    uint32_t vb[4];
                    ldmatrix_x4_trans(vb, vs + (kk * 16 + (lane & 7) + 8 * ((lane >> 3) & 1)) * ATT_LD +
                                              8 * (2 * jp + (lane >> 4)));
                    mma_f16(o[2 * jp], af, vb[0], vb[1]);
                    mma_f16(o[2 * jp], al, vb[0], vb[1]);
                    mma_f16(o[2 * jp + 1], af, vb[2], vb[3]);
                    mma_f16(o[2 * jp + 1], al, vb[2], vb[3]);
                }
            }
        }
      }
      __syncthreads();
    }
    const int used = int(t_end - t_begin < TL ? (t_end > t_begin ? t_end - t_begin : 0) : TL);  // lanes that saw a tile
    if (used > 1) {  // lanes 1.. leave their states in the (now free) tile buffers; lane 0 merges them in order
        float *st = reinterpret_cast<float *>(ks0);  // [mtiles][TL - 1][16 rows][HEAD_DIM + 2]
        if (active && tl > 0 && tl < used) {
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                if (mt * 16 + g + 8 * half >= R) continue;  // only live rows are merged
                float *row = st + ((mt * (TL - 1) + tl - 1) * 16 + g + 8 * half) * (HEAD_DIM + 2);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    row[8 * j + 2 * t4] = o[j][2 * half];
                    row[8 * j + 2 * t4 + 1] = o[j][2 * half + 1];
                }
                if (t4 == 0) {
                    row[HEAD_DIM] = mrun[half];
                    row[HEAD_DIM + 1] = lrun[half];
                }
            }
        }
        __syncthreads();
        if (active && tl == 0) {
            for (int l2 = 1; l2 < used; ++l2) {
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    if (mt * 16 + g + 8 * half >= R) continue;
                    const float *row = st + ((mt * (TL - 1) + l2 - 1) * 16 + g + 8 * half) * (HEAD_DIM + 2);
                    const float mb = row[HEAD_DIM], lb = row[HEAD_DIM + 1];
                    const float M = fmaxf(mrun[half], mb);
                    const float wa = M == -INFINITY || mrun[half] == -INFINITY ? 0.0f : __expf(mrun[half] - M);
                    const float wb = M == -INFINITY || mb == -INFINITY ? 0.0f : __expf(mb - M);
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        o[j][2 * half] = fmaf(row[8 * j + 2 * t4], wb, o[j][2 * half] * wa);
                        o[j][2 * half + 1] = fmaf(row[8 * j + 2 * t4 + 1], wb, o[j][2 * half + 1] * wa);
                    }
                    lrun[half] = fmaf(lb, wb, lrun[half] * wa);
                    mrun[half] = M;
                }
            }
        }
    }
    if (active && tl == 0) {
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            const int r = mt * 16 + g + 8 * half;
            if (r >= R) continue;
            if (a.splits == 1) {  // one CTA saw every key: normalise and write the row
                const float l = lrun[half], inv = l > 0.0f ? 1.0f / l : 0.0f;
                float *dst = a.out + row_q(r) * a.out_stride + h * HEAD_DIM + 2 * t4;
                float v[8][2];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    v[j][0] = o[j][2 * half] * inv;
                    v[j][1] = o[j][2 * half + 1] * inv;
                    *reinterpret_cast<float2 *>(dst + 8 * j) = make_float2(v[j][0], v[j][1]);
                }
                if (a.frags.xf) {  // the row's 4 lanes are live together
                    const unsigned group = 0xFu << (lane & ~3);
                    if (a.frags.mode == 0) frag_head_row<0>(a.frags, v, row_q(r), h, t4, group, a.status);
                    else if (a.frags.mode == 2) frag_head_row<2>(a.frags, v, row_q(r), h, t4, group, a.status);
                    else frag_head_row<1>(a.frags, v, row_q(r), h, t4, group, a.status);
                }
            } else {
                float *part = part_dst ? part_dst + int64_t(r) * (HEAD_DIM + 2)
                                       : a.partial + ((int64_t(gh) * a.splits + split) * R + r) * (HEAD_DIM + 2);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    part[8 * j + 2 * t4] = o[j][2 * half];
                    part[8 * j + 2 * t4 + 1] = o[j][2 * half + 1];
                }
                if (t4 == 0) {
                    part[HEAD_DIM] = mrun[half];
                    part[HEAD_DIM + 1] = lrun[half];
                }
            }
        }
    }
}

// Merge of the key splits of (group, head, row) `task`: thread dd < 64 takes one dim.
__device__ __forceinline__ void merge_task(const AttArgs &a, int task, int dd) {
    const int R = a.rows;
    const int r = task % R, gh = task / R;
    const int h = gh % a.heads, grp = gh / a.heads;
    const float *base = a.partial + int64_t(gh) * a.splits * R * (HEAD_DIM + 2) + int64_t(r) * (HEAD_DIM + 2);
    const int64_t step = int64_t(R) * (HEAD_DIM + 2);
    float M = -INFINITY;
    for (int sp = 0; sp < a.splits; ++sp) M = fmaxf(M, base[sp * step + HEAD_DIM]);
    float o = 0.0f, l = 0.0f;
    if (M != -INFINITY) {
#pragma unroll 4
        for (int sp = 0; sp < a.splits; ++sp) {
            const float m = base[sp * step + HEAD_DIM];
            const float w = m == -INFINITY ? 0.0f : __expf(m - M);
            o = fmaf(w, base[sp * step + dd], o);
            l = fmaf(w, base[sp * step + HEAD_DIM + 1], l);
        }
    }
    const int64_t qrow = a.shared ? int64_t(r) : int64_t(grp) * a.nq + r;
    const float v = l > 0.0f ? o / l : 0.0f;
    a.out[qrow * a.out_stride + h * HEAD_DIM + dd] = v;
    if (a.frags.xf) {  // warp dd / 32 holds block 2 h + dd / 32 of the row
        const Q8Frags &f = a.frags;
        const int64_t b = 2 * h + dd / 32;
        const int mtiles = int(f.mpad / 16);
        if (f.mode == 0) frag_block<0>(v, true, b, int(qrow), mtiles, f.xf, f.xs, f.xsum, a.status);
        else if (f.mode == 2) frag_block<2>(v, true, b, int(qrow), mtiles, f.xf, f.xs, f.xsum, a.status);
        else frag_block<1>(v, true, b, int(qrow), mtiles, f.xf, f.xs, f.xsum, a.status);
    }
}


}  // namespace mb
