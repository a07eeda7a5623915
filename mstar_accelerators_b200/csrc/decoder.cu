// Non-linear pieces of the Whisper decoder step that sit between the
// block-quantized linears: token + position embedding (ggml_get_rows + add,
// backends/cpu_ggml/decoder.cpp:513-518) and attention over the fp16 KV planes
// (ggml_flash_attn_ext with scale 1/sqrt(head_dim), decoder.cpp:504-511), with
// the new self-attention K/V rows appended first (ggml_set_rows,
// decoder.cpp:566-567). Attention math is fp32 (scores, split softmax, weighted
// sums); K/V are stored fp16 like the reference's F16 plain storage.
#include <cooperative_groups.h>

#include "../../include/mstar_b200.h"
#include "attend.cuh"
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

template <bool CAUSAL>
__global__ void __launch_bounds__(ATT_MAX_THREADS) k_attend_tiles(const AttArgs a) {
    extern __shared__ __align__(16) unsigned char att_smem[];
    pdl_wait();  // q, begin / kv_len and the planes come from the kernels before this one
    pdl_trigger();
    attend_task<CAUSAL>(a, blockIdx.x, att_smem);
}

__global__ void __launch_bounds__(HEAD_DIM) k_attend_merge(const AttArgs a) {
    pdl_wait();
    pdl_trigger();
    merge_task(a, blockIdx.x, threadIdx.x);
}

// Attention over shared planes with the key splits of a head as one thread-block
// cluster (cluster rank = split): every CTA keeps its partial rows (O, max,
// sum) in shared memory; after a cluster barrier CTA k merges rows
// k * R / splits .. through distributed shared memory, in split order exactly
// as k_attend_merge, writes them (and their Q8_0 fragments when asked) and
// waits at a second barrier so that no partial is read after its CTA exits.
__global__ void __launch_bounds__(ATT_MAX_THREADS) k_attend_cluster(const AttArgs a) {
    namespace cg = cooperative_groups;
    extern __shared__ __align__(16) unsigned char att_smem[];
    cg::cluster_group cluster = cg::this_cluster();
    float *part = reinterpret_cast<float *>(att_smem + att_smem_bytes(a.rows));  // [rows][HEAD_DIM + 2]
    pdl_wait();
    pdl_trigger();
    attend_task<false>(a, blockIdx.x, att_smem, part);
    cluster.sync();
    const int R = a.rows, S = a.splits, k = int(cluster.block_rank());
    const int h = int(blockIdx.x) / S % a.heads;
    const int per = (R + S - 1) / S, r0 = k * per, r1 = r0 + per < R ? r0 + per : R;
    const int lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
    for (int pair = int(threadIdx.x >> 5); pair < (r1 - r0) * 2; pair += nwarps) {  // (row, 32-dim block) per warp
        const int r = r0 + pair / 2, dd = (pair % 2) * 32 + lane;
        float M = -INFINITY;
        for (int sp = 0; sp < S; ++sp) M = fmaxf(M, cluster.map_shared_rank(part, sp)[r * (HEAD_DIM + 2) + HEAD_DIM]);
        float o = 0.0f, l = 0.0f;
        if (M != -INFINITY) {
#pragma unroll 4
            for (int sp = 0; sp < S; ++sp) {
                const float *pr = cluster.map_shared_rank(part, sp) + r * (HEAD_DIM + 2);
                const float m = pr[HEAD_DIM];
                const float w = m == -INFINITY ? 0.0f : __expf(m - M);
                o = fmaf(w, pr[dd], o);
                l = fmaf(w, pr[HEAD_DIM + 1], l);
            }
        }
        const float v = l > 0.0f ? o / l : 0.0f;
        a.out[int64_t(r) * a.out_stride + h * HEAD_DIM + dd] = v;
        if (a.frags.xf) {
            const Q8Frags &f = a.frags;
            const int64_t b = 2 * h + dd / 32;
            const int mtiles = int(f.mpad / 16);
            if (f.mode == 0) frag_block<0>(v, true, b, r, mtiles, f.xf, f.xs, f.xsum, a.status);
            else if (f.mode == 2) frag_block<2>(v, true, b, r, mtiles, f.xf, f.xs, f.xsum, a.status);
            else frag_block<1>(v, true, b, r, mtiles, f.xf, f.xs, f.xsum, a.status);
        }
    }
    cluster.sync();
}

static size_t tiles_smem_bytes(int rows) { return att_smem_bytes(rows); }

struct SplitPlan {
    int groups, rows, splits, tiles_per_split;
    uint64_t partial_bytes;
};

static SplitPlan split_plan(int heads, int batch, int queries, int64_t capacity, int shared) {
    SplitPlan p{};
    p.groups = shared ? 1 : batch;
    p.rows = shared ? batch * queries : queries;
    const int tiles = int(ceil_div(capacity, TILE_KEYS));
    p.splits = shared ? shared_splits(tiles) : 1;
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

int mstar_b200_attend_q8(const float *q, int64_t q_stride, const float *k_new, const float *v_new, int64_t kv_stride,
                         void *k_plane, void *v_plane, int64_t capacity, int32_t heads, int32_t head_dim,
                         int32_t batch, int32_t queries, const int64_t *begin, const int64_t *kv_length,
                         int32_t causal, int32_t shared, float *out, int64_t out_stride, float scale, int32_t *status,
                         void *workspace, uint64_t workspace_bytes, const mstar_b200_q8_frags *frags, void *stream,
                         char *error, size_t error_size) {
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
        const size_t cluster_smem = smem + size_t(p.rows) * (HEAD_DIM + 2) * 4;
        static bool configured = false;
        if (!configured) {
            cuda_check(cudaFuncSetAttribute(k_attend_cluster, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            int(tiles_smem_bytes(ATT_MAX_ROWS) + ATT_MAX_ROWS * (HEAD_DIM + 2) * 4)),
                       "attention shared-memory attribute");
            // clusters of more than 8 CTAs (up to SHARED_SPLITS key splits of a head)
            cuda_check(cudaFuncSetAttribute(k_attend_cluster, cudaFuncAttributeNonPortableClusterSizeAllowed, 1),
                       "attention cluster size attribute");
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
        if (frags) {
            const int64_t rows = int64_t(batch) * queries;
            require(frags->fragments && frags->scales && frags->sums, "missing fragment buffers");
            require(rows <= frags->rows && (frags->rows == 16 || frags->rows == 32), "fragment rows too few");
            require(frags->blocks >= int64_t(heads) * HEAD_DIM / QK, "fragment blocks fewer than the output width");
            require(frags->rounding >= 0 && frags->rounding <= 2, "unknown Q8_0 activation rounding");
            check_device(frags->fragments, "fragment buffer");
            a.frags.xf = static_cast<uint32_t *>(frags->fragments);
            a.frags.xs = frags->scales;
            a.frags.xsum = frags->sums;
            a.frags.nb_pad = frags->blocks;
            a.frags.mpad = frags->rows;
            a.frags.mode = frags->rounding;
        }
        cudaStream_t s = as_stream(stream);
        const unsigned grid = unsigned(p.groups * heads * p.splits);
        const int threads = att_threads(p.rows);
        if (p.splits > 1 && !causal) {  // one cluster of p.splits CTAs per (group, head); merge inside
            cudaLaunchConfig_t cfg{};
            cfg.gridDim = dim3(grid);
            cfg.blockDim = dim3(unsigned(threads));
            cfg.dynamicSmemBytes = cluster_smem;
            cfg.stream = s;
            cudaLaunchAttribute attr[2];
            attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            attr[0].val.programmaticStreamSerializationAllowed = 1;
            attr[1].id = cudaLaunchAttributeClusterDimension;
            attr[1].val.clusterDim.x = unsigned(p.splits);
            attr[1].val.clusterDim.y = 1;
            attr[1].val.clusterDim.z = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 2;
            cuda_check(cudaLaunchKernelEx(&cfg, k_attend_cluster, a), "attention cluster launch");
        } else {
            if (causal) launch_pdl(k_attend_tiles<true>, dim3(grid), dim3(threads), smem, s, a);
            else launch_pdl(k_attend_tiles<false>, dim3(grid), dim3(threads), smem, s, a);
            if (p.splits > 1)
                launch_pdl(k_attend_merge, dim3(unsigned(p.groups * heads * p.rows)), dim3(HEAD_DIM), 0, s, a);
        }
        cuda_check(cudaGetLastError(), "attention launch");
        return 0;
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return -1;
    }
}

int mstar_b200_attend(const float *q, int64_t q_stride, const float *k_new, const float *v_new, int64_t kv_stride,
                      void *k_plane, void *v_plane, int64_t capacity, int32_t heads, int32_t head_dim,
                      int32_t batch, int32_t queries, const int64_t *begin, const int64_t *kv_length, int32_t causal,
                      int32_t shared, float *out, int64_t out_stride, float scale, int32_t *status, void *workspace,
                      uint64_t workspace_bytes, void *stream, char *error, size_t error_size) {
    return mstar_b200_attend_q8(q, q_stride, k_new, v_new, kv_stride, k_plane, v_plane, capacity, heads, head_dim,
                                batch, queries, begin, kv_length, causal, shared, out, out_stride, scale, status,
                                workspace, workspace_bytes, nullptr, stream, error, error_size);
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
