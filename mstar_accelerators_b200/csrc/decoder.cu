// Non-linear pieces of the Whisper decoder step that sit between the
// block-quantized linears: token + position embedding (ggml_get_rows + add,
// backends/cpu_ggml/decoder.cpp:513-518) and attention over the fp16 KV planes
// (ggml_flash_attn_ext with scale 1/sqrt(head_dim), decoder.cpp:504-511), with
// the new self-attention K/V rows appended first (ggml_set_rows,
// decoder.cpp:566-567). Attention math is fp32 (scores, split softmax, weighted
// sums); K/V are stored fp16 like the reference's F16 plain storage.
#include "../../include/mstar_b200.h"
#include "quant.cuh"

namespace mb {

// x[r] = tok[ids[r]] * scale + pos[positions[r]]  (rows r < n, width d)
__global__ void k_embed(const float *__restrict__ tok, const float *__restrict__ pos, const int64_t *__restrict__ ids,
                        const int64_t *__restrict__ positions, float scale, float *__restrict__ x, int64_t n,
                        int64_t d, int64_t vocab, int64_t npos, int *__restrict__ status) {
    pdl_wait();
    pdl_trigger();
    const int64_t r = blockIdx.x;
    if (r >= n) return;
    const int64_t id = ids[r], p = positions[r];
    if (id < 0 || id >= vocab || p < 0 || p >= npos) {
        if (threadIdx.x == 0) atomicOr(status, 4);
        for (int64_t i = threadIdx.x; i < d; i += blockDim.x) x[r * d + i] = 0.0f;
        return;
    }
    for (int64_t i = threadIdx.x; i < d; i += blockDim.x) {
        float v = tok[id * d + i];
        if (scale != 1.0f) v = __fmul_rn(v, scale);
        x[r * d + i] = __fadd_rn(v, pos[p * d + i]);
    }
}

constexpr int HEAD_DIM = 64;
constexpr int MAX_Q = 4;
constexpr int TILE_KEYS = 64;        // keys per shared-memory tile
constexpr int ATT_THREADS = 128;      // CTA size for up to 4 row tiles
constexpr int ATT_MAX_THREADS = 256;  // one warp per 16-row tile up to 128 rows
constexpr int ATT_MAX_ROWS = 128;    // query rows one CTA attends (all B*NQ rows when the planes are shared)
constexpr int SHARED_SPLITS = 24;    // key splits per head over shared planes (6 heads -> 144 CTAs)

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
};

// D += A(16x16 f16, row) * B(16x8 f16, col), fp32 accumulate.
__device__ __forceinline__ void mma_f16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) { return half2_bits(__floats2half2_rn(lo, hi)); }

constexpr int ATT_LD = HEAD_DIM + 8;  // fp16 row stride of the shared tiles (72 halves: conflict-free fragment loads)

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
template <bool CAUSAL>
__global__ void __launch_bounds__(ATT_MAX_THREADS) k_attend_tiles(const AttArgs a) {
    extern __shared__ __align__(16) unsigned char att_smem[];
    const int R = a.rows, mtiles = (R + 15) / 16;
    __half *qs = reinterpret_cast<__half *>(att_smem);            // [mtiles*16][72] fp16(q)
    __half *ql = qs + mtiles * 16 * ATT_LD;                       // [mtiles*16][72] fp16(q - fp16(q))
    __half *ks = ql + mtiles * 16 * ATT_LD;                       // [64 keys][72]
    __half *vt = ks + TILE_KEYS * ATT_LD;                         // [64 dims][72] (V transposed)
    int *lim = reinterpret_cast<int *>(vt + HEAD_DIM * ATT_LD);   // [mtiles*16]
    __shared__ int maxlim;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t4 = lane & 3;
    const int split = blockIdx.x % a.splits, gh = blockIdx.x / a.splits;
    const int h = gh % a.heads, grp = gh / a.heads;
    const int width = a.heads * HEAD_DIM;
    const int64_t seq = a.shared ? 0 : grp;
    __half *kp = a.kc + seq * a.capacity * width + h * HEAD_DIM;
    __half *vp = a.vc + seq * a.capacity * width + h * HEAD_DIM;
    auto row_seq = [&](int r) { return a.shared ? r / a.nq : grp; };
    auto row_q = [&](int r) { return a.shared ? int64_t(r) : int64_t(grp) * a.nq + r; };  // global query row

    pdl_wait();  // q, begin / kv_len and the planes come from the kernels before this one
    pdl_trigger();
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

    // this warp's 16-row tile: O [16 x 64] (8 n-tiles x 4), running max / sum of rows g, g+8
    const int mt = warp;
    float o[8][4];
    float mrun[2] = {-INFINITY, -INFINITY}, lrun[2] = {0.0f, 0.0f};
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
    const int64_t t_begin = int64_t(split) * a.tiles_per_split;
    for (int64_t t = t_begin; t < t_begin + a.tiles_per_split && t * TILE_KEYS < maxlim; ++t) {
        const int64_t c0 = t * TILE_KEYS;
        // K tile [key][dim] and transposed V tile [dim][key], fp16; new rows from knew/vnew
        for (int e = tid; e < TILE_KEYS * HEAD_DIM / 8; e += blockDim.x) {
            const int jj = e / (HEAD_DIM / 8), d8 = (e % (HEAD_DIM / 8)) * 8;
            const int64_t j = c0 + jj;
            uint4 kr = make_uint4(0u, 0u, 0u, 0u), vr = kr;
            if (j < maxlim) {  // keys past every row's length stay zero (never stale plane bytes)
                const int64_t b0 = CAUSAL && a.knew ? a.begin[grp] : -1;
                if (CAUSAL && a.knew && b0 >= 0 && j >= b0 && j < b0 + a.nq && b0 + a.nq <= a.capacity) {
                    const int64_t src = (int64_t(grp) * a.nq + (j - b0)) * a.kv_stride + h * HEAD_DIM + d8;
                    __half kh[8], vh[8];
#pragma unroll
                    for (int u = 0; u < 8; ++u) {
                        kh[u] = __float2half_rn(a.knew[src + u]);
                        vh[u] = __float2half_rn(a.vnew[src + u]);
                    }
                    memcpy(&kr, kh, 16);
                    memcpy(&vr, vh, 16);
                    *reinterpret_cast<uint4 *>(kp + j * width + d8) = kr;
                    *reinterpret_cast<uint4 *>(vp + j * width + d8) = vr;
                } else {
                    kr = *reinterpret_cast<const uint4 *>(kp + j * width + d8);
                    vr = *reinterpret_cast<const uint4 *>(vp + j * width + d8);
                }
            }
            *reinterpret_cast<uint4 *>(ks + jj * ATT_LD + d8) = kr;
            const __half *vh = reinterpret_cast<const __half *>(&vr);
#pragma unroll
            for (int u = 0; u < 8; ++u) vt[(d8 + u) * ATT_LD + jj] = vh[u];
        }
        __syncthreads();
        if (mt < mtiles) {
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
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const __half *vb = vt + (8 * j + g) * ATT_LD + kk * 16 + 2 * t4;
                    const uint32_t b0 = *reinterpret_cast<const uint32_t *>(vb), b1 = *reinterpret_cast<const uint32_t *>(vb + 8);
                    mma_f16(o[j], af, b0, b1);
                    mma_f16(o[j], al, b0, b1);
                }
            }
        }
        __syncthreads();
    }
    if (mt < mtiles) {
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            const int r = mt * 16 + g + 8 * half;
            if (r >= R) continue;
            if (a.splits == 1) {  // one CTA saw every key: normalise and write the row
                const float l = lrun[half], inv = l > 0.0f ? 1.0f / l : 0.0f;
                float *dst = a.out + row_q(r) * a.out_stride + h * HEAD_DIM + 2 * t4;
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    *reinterpret_cast<float2 *>(dst + 8 * j) =
                        make_float2(o[j][2 * half] * inv, o[j][2 * half + 1] * inv);
            } else {
                float *part = a.partial + ((int64_t(gh) * a.splits + split) * R + r) * (HEAD_DIM + 2);
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

// Merge of the key splits: one CTA per (group, head, row), one thread per dim.
__global__ void __launch_bounds__(HEAD_DIM) k_attend_merge(const AttArgs a) {
    pdl_wait();
    pdl_trigger();
    const int R = a.rows;
    const int r = blockIdx.x % R, gh = blockIdx.x / R;
    const int h = gh % a.heads, grp = gh / a.heads;
    const int dd = threadIdx.x;
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
    a.out[qrow * a.out_stride + h * HEAD_DIM + dd] = l > 0.0f ? o / l : 0.0f;
}

static size_t tiles_smem_bytes(int rows) {
    const size_t padded = size_t(rows + 15) / 16 * 16;
    return (2 * padded + TILE_KEYS + HEAD_DIM) * ATT_LD * 2 + padded * 4;
}

struct SplitPlan {
    int groups, rows, splits, tiles_per_split;
    uint64_t partial_bytes;
};

static SplitPlan split_plan(int heads, int batch, int queries, int64_t capacity, int shared) {
    SplitPlan p{};
    p.groups = shared ? 1 : batch;
    p.rows = shared ? batch * queries : queries;
    const int tiles = int(ceil_div(capacity, TILE_KEYS));
    p.splits = shared ? (tiles < SHARED_SPLITS ? tiles : SHARED_SPLITS) : 1;
    p.tiles_per_split = int(ceil_div(tiles, p.splits));
    p.partial_bytes = p.splits > 1 ? uint64_t(p.groups) * heads * p.splits * p.rows * (HEAD_DIM + 2) * 4 : 0;
    return p;
}

// K/V planes from projected rows: kc/vc[seq][r][:] = fp16(src[r][k_off / v_off + :]) + bias
__global__ void k_fill_kv(const float *__restrict__ src, int64_t src_stride, int64_t k_off, int64_t v_off,
                          const float *__restrict__ kbias, const float *__restrict__ vbias, __half *__restrict__ kc,
                          __half *__restrict__ vc, int64_t rows, int64_t width) {
    const int64_t r = blockIdx.x;
    if (r >= rows) return;
    for (int64_t i = threadIdx.x; i < width; i += blockDim.x) {
        float kv = src[r * src_stride + k_off + i], vv = src[r * src_stride + v_off + i];
        if (kbias) kv = __fadd_rn(kv, kbias[i]);
        if (vbias) vv = __fadd_rn(vv, vbias[i]);
        kc[r * width + i] = __float2half_rn(kv);
        vc[r * width + i] = __float2half_rn(vv);
    }
}

}  // namespace mb

using namespace mb;

extern "C" {

int mstar_b200_embed(const float *token_table, int64_t vocab, const float *position_table, int64_t positions_count,
                     int64_t width, const int64_t *ids, const int64_t *positions, int64_t rows, float scale,
                     float *x, int32_t *status, void *stream, char *error, size_t error_size) {
    try {
        require(token_table && position_table && ids && positions && x && status, "missing embedding operand");
        require(rows > 0 && width > 0 && vocab > 0 && positions_count > 0, "invalid embedding shape");
        cudaStream_t s = as_stream(stream);
        launch_pdl(k_embed, dim3(unsigned(rows)), dim3(128), 0, s, token_table, position_table, ids, positions, scale,
                   x, rows, width, vocab, positions_count, status);
        cuda_check(cudaGetLastError(), "embedding launch");
        return 0;
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return -1;
    }
}

uint64_t mstar_b200_attend_workspace(int32_t heads, int32_t batch, int32_t queries, int64_t capacity,
                                     int32_t shared) {
    if (heads < 1 || batch < 1 || queries < 1 || queries > MAX_Q || capacity < 1 || capacity > 4096) return 0;
    const SplitPlan p = split_plan(heads, batch, queries, capacity, shared);
    if (p.rows > ATT_MAX_ROWS) return 0;
    return p.partial_bytes > 0 ? p.partial_bytes : 256;
}

int mstar_b200_attend(const float *q, int64_t q_stride, const float *k_new, const float *v_new, int64_t kv_stride,
                      void *k_plane, void *v_plane, int64_t capacity, int32_t heads, int32_t head_dim,
                      int32_t batch, int32_t queries, const int64_t *begin, const int64_t *kv_length, int32_t causal,
                      int32_t shared, float *out, int64_t out_stride, float scale, int32_t *status, void *workspace,
                      uint64_t workspace_bytes, void *stream, char *error, size_t error_size) {
    try {
        require(head_dim == HEAD_DIM, "attention head_dim must be 64");
        require(queries >= 1 && queries <= MAX_Q && batch >= 1 && heads >= 1, "invalid attention geometry");
        require(capacity >= 1 && capacity <= 4096, "attention capacity outside 1..4096");
        require(q && k_plane && v_plane && out && status && workspace, "missing attention operand");
        require(causal ? (begin != nullptr) : (kv_length != nullptr), "attention lengths missing");
        require(!k_new == !v_new, "new K and V rows must be given together");
        require(!(k_new && (shared || !causal)), "new K/V rows are appended only to causal per-sequence planes");
        require(uintptr_t(k_plane) % 16 == 0 && uintptr_t(v_plane) % 16 == 0, "KV planes must be 16-byte aligned");
        const SplitPlan p = split_plan(heads, batch, queries, capacity, shared);
        require(p.rows <= ATT_MAX_ROWS, "more than 128 query rows share one K/V plane");
        require(workspace_bytes == (p.partial_bytes > 0 ? p.partial_bytes : 256) && uintptr_t(workspace) % 256 == 0,
                "attention workspace must be mstar_b200_attend_workspace() bytes, 256-byte aligned");
        check_device(workspace, "attention workspace");
        const size_t smem = tiles_smem_bytes(p.rows);
        static bool configured = false;
        if (!configured) {
            cuda_check(cudaFuncSetAttribute(k_attend_tiles<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            int(tiles_smem_bytes(ATT_MAX_ROWS))),
                       "attention shared-memory attribute");
            cuda_check(cudaFuncSetAttribute(k_attend_tiles<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            int(tiles_smem_bytes(ATT_MAX_ROWS))),
                       "attention shared-memory attribute");
            configured = true;
        }
        AttArgs a{};
        a.q = q;
        a.q_stride = q_stride;
        a.knew = k_new;
        a.vnew = v_new;
        a.kv_stride = kv_stride;
        a.kc = static_cast<__half *>(k_plane);
        a.vc = static_cast<__half *>(v_plane);
        a.capacity = capacity;
        a.heads = heads;
        a.nq = queries;
        a.batch = batch;
        a.shared = shared;
        a.splits = p.splits;
        a.rows = p.rows;
        a.tiles_per_split = p.tiles_per_split;
        a.begin = begin;
        a.kv_len = kv_length;
        a.out = out;
        a.out_stride = out_stride;
        a.scale = scale;
        a.status = status;
        a.partial = static_cast<float *>(workspace);
        cudaStream_t s = as_stream(stream);
        const unsigned grid = unsigned(p.groups * heads * p.splits);
        const int threads = 32 * (p.rows > 64 ? (p.rows + 15) / 16 : 4);
        if (causal) launch_pdl(k_attend_tiles<true>, dim3(grid), dim3(threads), smem, s, a);
        else launch_pdl(k_attend_tiles<false>, dim3(grid), dim3(threads), smem, s, a);
        if (p.splits > 1) launch_pdl(k_attend_merge, dim3(unsigned(p.groups * heads * p.rows)), dim3(HEAD_DIM), 0, s, a);
        cuda_check(cudaGetLastError(), "attention launch");
        return 0;
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return -1;
    }
}

int mstar_b200_fill_kv(const float *projected, int64_t stride, int64_t k_offset, int64_t v_offset,
                       const float *k_bias, const float *v_bias, void *k_plane, void *v_plane, int64_t rows,
                       int64_t width, void *stream, char *error, size_t error_size) {
    try {
        require(projected && k_plane && v_plane && rows > 0 && width > 0, "invalid KV fill");
        cudaStream_t s = as_stream(stream);
        k_fill_kv<<<unsigned(rows), 128, 0, s>>>(projected, stride, k_offset, v_offset, k_bias, v_bias,
                                                 static_cast<__half *>(k_plane), static_cast<__half *>(v_plane), rows,
                                                 width);
        cuda_check(cudaGetLastError(), "KV fill launch");
        return 0;
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return -1;
    }
}

}  // extern "C"
