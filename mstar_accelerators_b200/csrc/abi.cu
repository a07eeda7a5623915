// extern "C" boundary of libmstar_b200 (declarations and reference citations
// in include/mstar_b200.h). Host-side validation happens before any launch;
// nothing here throws across the C boundary.
#include <atomic>
#include <cerrno>
#include <cmath>
#include <memory>
#include <vector>

#include "../../include/mstar_b200.h"
#include "gemm.cuh"
#include "linear_handle.cuh"
#include "quant.cuh"

namespace mb {

__global__ void k_probe() {}

template <class T>
T *device_alloc(size_t count, const char *what) {
    void *p = nullptr;
    cuda_check(cudaMalloc(&p, count * sizeof(T) ? count * sizeof(T) : 16), what);
    return static_cast<T *>(p);
}

constexpr int64_t CHUNK = 32;             // tokens per GEMV launch
constexpr int64_t GEMM_MIN_QUERIES = 64;  // larger calls use the tcgen05 GEMM once it is prepared

// Quantize one chunk of <= 32 queries, then describe the GEMV over it.
GemvArgs stage(Linear &h, const float *x, int64_t ldx, int64_t m, int rounding, const float *ln_w,
               const float *ln_b, float ln_eps, int *status, cudaStream_t s) {
    const int64_t mpad = m <= 16 ? 16 : 32;
    launch_quantize_frag(rounding, x, ldx, m, h.width, mpad, h.nb_pad, ln_w, ln_b, ln_eps, h.xf, h.xs, h.xsum, status,
                         s);
    GemvArgs a{};
    a.status = status;
    a.wq = h.wq;
    a.ws = reinterpret_cast<const __half2 *>(h.ws);
    a.xf = reinterpret_cast<const uint4 *>(h.xf);
    a.xs = h.xs;
    a.xsum = h.xsum;
    a.groups = h.groups;
    a.nb_pad = h.nb_pad;
    a.nb = h.nb;
    a.n = h.rows;
    a.m = m;
    return a;
}

void check_rounding(int r) { require(r >= 0 && r <= 2, "unknown Q8_0 activation rounding"); }

// readout.cu
bool readout_tiles_fit(int64_t rows, int64_t nb, int q4);
void launch_readout_repack(int q4, const uint8_t *blocks, uint8_t *wt, int64_t rows, int64_t nb, cudaStream_t s);
void launch_readout(const Linear &h, const float *x, int64_t ldx, int64_t m, const float *ln_w,
                    const float *ln_b, float eps, int mode, float *logits, int64_t *token, int *status,
                    const int64_t *suppressed, int64_t nsup, cudaStream_t s, int64_t ldo = 0,
                    const float *bias = nullptr, const float *residual = nullptr);

}  // namespace mb

using namespace mb;

namespace mb {
WaitLimits &wait_limits() {
    static WaitLimits limits;
    return limits;
}
void launch_grid_barrier_selftest(unsigned int *bar, int *status, long long limit, cudaStream_t s);

// An mbarrier that nothing arrives at: mbar_wait_bounded (the wait every TMA /
// MMA pipeline here uses) must give up after `limit` polls and report status
// bit value 2, leaving the context usable.
__global__ void k_mbarrier_selftest(int *status, uint32_t limit) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0 && !mbar_wait_bounded(&bar, 0, limit)) atomicOr(status, 2);
}
}  // namespace mb

extern "C" {

int mstar_b200_abi(void) { return 1; }

int mstar_b200_capability(void) {
    int dev = 0, major = 0, minor = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) { cudaGetLastError(); return 0; }
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    if (major != 10 || minor != 0) return 0;
    cudaFuncAttributes attr{};
    if (cudaFuncGetAttributes(&attr, k_probe) != cudaSuccess) { cudaGetLastError(); return 0; }
    return 1;
}

int mstar_b200_pack(int format, const float *input, uint64_t input_bytes, void *output, uint64_t output_bytes,
                    int64_t rows, int64_t width, int preround, int fused, void *stream, char *error,
                    size_t error_size) {
    int *flags = nullptr;
    try {
        require(format == MSTAR_B200_Q8_0 || format == MSTAR_B200_Q4_0, "unsupported block format");
        require(rows > 0 && rows <= (int64_t(1) << 31) && width > 0 && width <= 65536 && width % QK == 0,
                "invalid packing shape");
        const int q4 = format == MSTAR_B200_Q4_0;
        const uint64_t count = uint64_t(rows) * uint64_t(width);
        check_range({input, input_bytes}, count * 4, alignof(float), "packing input");
        check_range({output, output_bytes}, uint64_t(rows) * (width / QK) * (q4 ? Q4_BYTES : Q8_BYTES), 2,
                    "packing output");
        require(disjoint({input, input_bytes}, {output, output_bytes}), "packing input/output overlap");
        check_device(input, "packing input");
        check_device(output, "packing output");
        cudaStream_t s = as_stream(stream);
        cuda_check(cudaMallocAsync(reinterpret_cast<void **>(&flags), sizeof(int), s), "flag allocation");
        cuda_check(cudaMemsetAsync(flags, 0, sizeof(int), s), "flag reset");
        launch_pack(input, static_cast<uint8_t *>(output), rows, width, q4, preround, fused, flags, s);
        cuda_check(cudaGetLastError(), "pack launch");
        int host = 0;
        cuda_check(cudaMemcpyAsync(&host, flags, sizeof(int), cudaMemcpyDeviceToHost, s), "flag read");
        cuda_check(cudaFreeAsync(flags, s), "flag free");
        flags = nullptr;
        cuda_check(cudaStreamSynchronize(s), "pack");
        require(!(host & 1), "nonfinite weight");
        require(!(host & 2), "weight overflows F16");
        return 0;
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return -1;
    }
}

int mstar_b200_q8_quantize(const float *x, void *packed, size_t bytes, int64_t rows, int64_t k, int rounding,
                           void *stream) {
    if (!mstar_b200_capability()) return ENOTSUP;
    if (!x || !packed || rows <= 0 || k <= 0 || k % QK || rounding < 0 || rounding > 2 || uintptr_t(packed) % 2 ||
        bytes != size_t(rows) * size_t(k / QK) * Q8_BYTES)
        return EINVAL;
    int *status = nullptr;
    cudaStream_t s = as_stream(stream);
    if (cudaMallocAsync(reinterpret_cast<void **>(&status), sizeof(int), s) != cudaSuccess) return ENOMEM;
    cudaMemsetAsync(status, 0, sizeof(int), s);
    // quantize rows in groups of 16 "tokens" through the same kernel
    launch_quantize_rows(rounding, x, k, rows, k, static_cast<uint8_t *>(packed), status, s);
    int host = 0;
    cudaMemcpyAsync(&host, status, sizeof(int), cudaMemcpyDeviceToHost, s);
    cudaFreeAsync(status, s);
    if (cudaStreamSynchronize(s) != cudaSuccess) return EIO;
    return host ? EDOM : 0;
}

void *mstar_b200_linear_create(int format, const void *blocks, uint64_t bytes, int64_t rows, int64_t width,
                               const float *bias, char *error, size_t error_size) {
    std::unique_ptr<Linear> h;
    try {
        require(mstar_b200_capability() == 1, "sm_100a device capability is unavailable");
        require(format == MSTAR_B200_Q8_0 || format == MSTAR_B200_Q4_0, "unsupported block format");
        require(rows > 0 && rows <= (int64_t(1) << 31) && width > 0 && width <= 65536 && width % QK == 0,
                "invalid linear shape");
        h.reset(new Linear);
        h->q4 = format == MSTAR_B200_Q4_0;
        h->rows = rows;
        h->width = width;
        h->nb = width / QK;
        h->nb_pad = h->q4 ? ceil_div(h->nb, 4) * 4 : ceil_div(h->nb, 2) * 2;
        h->groups = ceil_div(rows, 8);
        check_range({blocks, bytes}, uint64_t(rows) * h->nb * (h->q4 ? Q4_BYTES : Q8_BYTES), 1, "linear weights");
        h->gemv_ok = gemv_supported(h->nb_pad);
        h->gelu = gelu_table();
        h->xf = device_alloc<uint32_t>(size_t(h->nb_pad * 2 * 32 * 4), "activation fragments");
        h->xs = device_alloc<float>(size_t(h->nb_pad * 32), "activation scales");
        h->xsum = device_alloc<int>(size_t(h->nb_pad * 32), "activation block sums");
        check_device(blocks, "linear weights");
        const int64_t chunks = h->nb_pad / (h->q4 ? 4 : 2);
        h->wq = device_alloc<uint4>(size_t(h->groups * chunks * 32), "weight allocation");
        h->ws = device_alloc<__half>(size_t(h->groups * h->nb_pad * 8), "scale allocation");
        h->status = device_alloc<int>(1, "status scratch");
        h->keys = device_alloc<unsigned long long>(32, "argmax scratch");
        h->done = device_alloc<unsigned int>(1, "argmax counter");
        cudaStream_t s = nullptr;
        cuda_check(cudaMemset(h->keys, 0, 32 * sizeof(unsigned long long)), "argmax reset");
        cuda_check(cudaMemset(h->done, 0, sizeof(unsigned int)), "counter reset");
        cuda_check(cudaMemset(h->status, 0, sizeof(int)), "status reset");
        if (bias) {
            check_device(bias, "bias");
            h->bias = device_alloc<float>(size_t(rows), "bias allocation");
            cuda_check(cudaMemcpy(h->bias, bias, size_t(rows) * 4, cudaMemcpyDeviceToDevice), "bias copy");
        }
        launch_repack(h->q4, static_cast<const uint8_t *>(blocks), h->wq, h->ws, rows, h->nb, h->nb_pad,
                      h->groups, s);
        cuda_check(cudaGetLastError(), "repack launch");
        cuda_check(cudaDeviceSynchronize(), "repack");
        return h.release();
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return nullptr;
    }
}

static void validate_run(Linear &h, const float *x, int64_t x_stride, int64_t queries, const float *out,
                         int64_t out_stride) {
    require(queries >= 1 && queries <= (int64_t(1) << 31), "invalid query count");
    require(x_stride >= h.width && out_stride >= h.rows, "invalid row stride");
    require(uintptr_t(x) % 16 == 0 && x_stride % 4 == 0, "activation rows must be 16-byte aligned");
    const uint64_t xb = uint64_t((queries - 1) * x_stride + h.width) * 4;
    const uint64_t ob = uint64_t((queries - 1) * out_stride + h.rows) * 4;
    check_range({x, xb}, xb, 4, "activations");
    check_range({out, ob}, ob, 4, "output");
    require(disjoint({x, xb}, {out, ob}), "output overlaps activations");
    check_device(x, "activations");
    check_device(out, "output");
}

static void validate_norm(Linear &h, const float *ln_weight, const float *ln_bias, float ln_eps) {
    if (!ln_weight) {
        require(!ln_bias, "LayerNorm bias given without its weight");
        return;
    }
    require(ln_bias && std::isfinite(ln_eps) && ln_eps >= 0.0f, "invalid LayerNorm parameters");
    check_device(ln_weight, "LayerNorm weight");
    check_device(ln_bias, "LayerNorm bias");
}

int mstar_b200_linear_run(void *handle, const float *x, int64_t x_stride, int64_t queries, float *out,
                          int64_t out_stride, const float *residual, int flags, const float *ln_weight,
                          const float *ln_bias, float ln_eps, int rounding, void *stream, char *error,
                          size_t error_size) {
    try {
        require(handle, "missing linear handle");
        auto &h = *static_cast<Linear *>(handle);
        Busy busy(h.busy);
        check_rounding(rounding);
        require((flags & ~15) == 0 && !((flags & 2) && (flags & 8)), "invalid epilogue flags");
        require(!(flags & 1) || h.bias, "bias epilogue without a prepared bias");
        validate_run(h, x, x_stride, queries, out, out_stride);
        validate_norm(h, ln_weight, ln_bias, ln_eps);
        if (flags & 4) {
            const uint64_t rb = uint64_t((queries - 1) * out_stride + h.rows) * 4;
            check_range({residual, rb}, rb, 4, "residual");
            require(residual == out || disjoint({residual, rb}, {out, rb}), "residual partially overlaps output");
            check_device(residual, "residual");
        } else require(!residual, "residual given without its epilogue flag");
        cudaStream_t s = as_stream(stream);
        if (h.w16 && !ln_weight && queries >= GEMM_MIN_QUERIES && queries <= h.gemm_rows) {
            // the activation side of the GEMM: Q8_0 blocks staged as fp16(q * d); a warp per row
            // with 16-byte loads where the rows allow it (the same bytes as a warp per block)
            if (uintptr_t(x) % 16 == 0 && x_stride % 4 == 0)
                launch_stage_rows(rounding, x, 0, x_stride, queries, h.width, nullptr, nullptr, 0.0f, h.x16, h.width,
                                  h.status, s);
            else launch_dequant_act(rounding, x, x_stride, queries, h.width, h.x16, h.status, s);
            CUtensorMap xmap;
            make_fp16_map(&xmap, h.x16, queries, h.width, GEMM_TILE_M);
            GemmArgs g{};
            g.M = queries;
            g.N = h.rows;
            g.K = h.width;
            g.out = out;
            g.ldo = out_stride;
            g.bias = h.bias;
            g.residual = (flags & 4) ? residual : nullptr;
            g.ldr = out_stride;
            g.flags = flags;
            g.gelu = h.gelu;
            g.out_mode = GEMM_OUT_F32;
            g.rounding = rounding;
            g.status = h.status;
            launch_gemm(xmap, h.wmap, h.wmap_pair, g, s);
            cuda_check(cudaGetLastError(), "GEMM launch");
            return 0;
        }
        require(h.gemv_ok, "width beyond 4096 needs the prepared GEMM and at least 64 queries without LayerNorm");
        const bool tiles = h.wt && !h.wpg_override && !(flags & (2 | 8)) &&
                           (!ln_weight || (uintptr_t(ln_weight) % 16 == 0 && uintptr_t(ln_bias) % 16 == 0));
        for (int64_t m0 = 0; m0 < queries; m0 += CHUNK) {
            const int64_t mc = queries - m0 < CHUNK ? queries - m0 : CHUNK;
            if (tiles) {  // the tile GEMV (prepare_readout): query quantization inside, one launch per chunk
                launch_readout(h, x + m0 * x_stride, x_stride, mc, ln_weight, ln_bias, ln_eps, rounding,
                               out + m0 * out_stride, nullptr, h.status, nullptr, 0, s, out_stride,
                               (flags & 1) ? h.bias : nullptr, (flags & 4) ? residual + m0 * out_stride : nullptr);
                continue;
            }
            const int64_t m = queries - m0 < CHUNK ? queries - m0 : CHUNK;
            GemvArgs a = stage(h, x + m0 * x_stride, x_stride, m, rounding, ln_weight, ln_bias, ln_eps, h.status, s);
            a.out = out + m0 * out_stride;
            a.ldo = out_stride;
            a.bias = h.bias;
            a.residual = (flags & 4) ? residual + m0 * out_stride : nullptr;
            a.flags = flags;
            a.gelu = h.gelu;
            a.wpg_override = h.wpg_override;
            launch_gemv(h.q4, a, s);
        }
        cuda_check(cudaGetLastError(), "linear launch");
        return 0;
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return -1;
    }
}

int mstar_b200_linear_run_q8out(void *handle, const float *x, int64_t x_stride, int64_t queries, float *out,
                                int64_t out_stride, const float *residual, int flags, const float *ln_weight,
                                const float *ln_bias, float ln_eps, int rounding, const mstar_b200_q8_frags *next,
                                void *stream, char *error, size_t error_size) {
    try {
        require(handle && next, "missing linear handle or fragment descriptor");
        auto &h = *static_cast<Linear *>(handle);
        Busy busy(h.busy);
        check_rounding(rounding);
        require(!h.q4, "fragment output needs Q8_0 weights");
        require(queries >= 1 && queries <= CHUNK, "fragment output takes 1..32 queries");
        require(h.gemv_ok && h.rows % 32 == 0, "fragment output needs whole 32-output blocks");
        require((flags & ~15) == 0 && !((flags & 2) && (flags & 8)), "invalid epilogue flags");
        require(!(flags & 1) || h.bias, "bias epilogue without a prepared bias");
        validate_run(h, x, x_stride, queries, out, out_stride);
        validate_norm(h, ln_weight, ln_bias, ln_eps);
        if (flags & 4) {
            const uint64_t rb = uint64_t((queries - 1) * out_stride + h.rows) * 4;
            check_range({residual, rb}, rb, 4, "residual");
            require(residual == out || disjoint({residual, rb}, {out, rb}), "residual partially overlaps output");
            check_device(residual, "residual");
        } else require(!residual, "residual given without its epilogue flag");
        require(next->fragments && next->scales && next->sums, "missing fragment buffers");
        require(next->rows == (queries <= 16 ? 16 : 32), "fragment rows differ from the query count");
        require(next->blocks >= h.rows / QK, "fragment blocks fewer than the output width");
        require(next->rounding >= 0 && next->rounding <= 2, "unknown Q8_0 activation rounding");
        require(gemv_frag_smem_bytes(h.nb_pad, queries <= 16 ? 1 : 2) <= 200 * 1024, "input too wide");
        check_device(next->fragments, "fragment buffer");
        cudaStream_t s = as_stream(stream);
        GemvArgs a = stage(h, x, x_stride, queries, rounding, ln_weight, ln_bias, ln_eps, h.status, s);
        a.out = out;
        a.ldo = out_stride;
        a.bias = h.bias;
        a.residual = (flags & 4) ? residual : nullptr;
        a.flags = flags;
        a.gelu = h.gelu;
        Q8Frags f{};
        f.xf = static_cast<uint32_t *>(next->fragments);
        f.xs = next->scales;
        f.xsum = next->sums;
        f.nb_pad = next->blocks;
        f.mpad = next->rows;
        f.mode = next->rounding;
        launch_gemv_frag(a, f, s);
        cuda_check(cudaGetLastError(), "fragment-output GEMV launch");
        return 0;
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return -1;
    }
}

int mstar_b200_linear_frags(void *handle, int64_t queries, int32_t rounding, mstar_b200_q8_frags *frags,
                            char *error, size_t error_size) {
    try {
        require(handle && frags, "missing linear handle or fragment descriptor");
        auto &h = *static_cast<Linear *>(handle);
        check_rounding(rounding);
        require(queries >= 1 && queries <= CHUNK, "fragment staging takes 1..32 queries");
        require(h.gemv_ok, "fragment staging needs a width of at most 4096");
        frags->fragments = h.xf;
        frags->scales = h.xs;
        frags->sums = h.xsum;
        frags->blocks = h.nb_pad;
        frags->rows = queries <= 16 ? 16 : 32;
        frags->rounding = rounding;
        return 0;
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return -1;
    }
}

int mstar_b200_linear_run_frags(void *handle, int64_t queries, float *out, int64_t out_stride, const float *residual,
                                int flags, void *stream, char *error, size_t error_size) {
    try {
        require(handle, "missing linear handle");
        auto &h = *static_cast<Linear *>(handle);
        Busy busy(h.busy);
        require(queries >= 1 && queries <= CHUNK, "fragment GEMV takes 1..32 queries");
        require(h.gemv_ok, "fragment GEMV needs a width of at most 4096");
        require((flags & ~15) == 0 && !((flags & 2) && (flags & 8)), "invalid epilogue flags");
        require(!(flags & 1) || h.bias, "bias epilogue without a prepared bias");
        require(out_stride >= h.rows, "invalid row stride");
        const uint64_t ob = uint64_t((queries - 1) * out_stride + h.rows) * 4;
        check_range({out, ob}, ob, 4, "output");
        check_device(out, "output");
        if (flags & 4) {
            check_range({residual, ob}, ob, 4, "residual");
            require(residual == out || disjoint({residual, ob}, {out, ob}), "residual partially overlaps output");
            check_device(residual, "residual");
        } else require(!residual, "residual given without its epilogue flag");
        GemvArgs a{};
        a.status = h.status;
        a.wq = h.wq;
        a.ws = reinterpret_cast<const __half2 *>(h.ws);
        a.xf = reinterpret_cast<const uint4 *>(h.xf);
        a.xs = h.xs;
        a.xsum = h.xsum;
        a.groups = h.groups;
        a.nb_pad = h.nb_pad;
        a.nb = h.nb;
        a.n = h.rows;
        a.m = queries;
        a.out = out;
        a.ldo = out_stride;
        a.bias = h.bias;
        a.residual = (flags & 4) ? residual : nullptr;
        a.flags = flags;
        a.gelu = h.gelu;
        a.wpg_override = h.wpg_override;
        launch_gemv(h.q4, a, as_stream(stream));
        cuda_check(cudaGetLastError(), "fragment GEMV launch");
        return 0;
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return -1;
    }
}

int mstar_b200_linear_block_sums(void *handle, const float *x, int64_t queries, int32_t *sums,
                                 uint64_t sums_bytes, int rounding, void *stream, char *error, size_t error_size) {
    try {
        require(handle, "missing linear handle");
        auto &h = *static_cast<Linear *>(handle);
        Busy busy(h.busy);
        check_rounding(rounding);
        require(queries >= 1 && queries <= CHUNK, "block sums take 1..32 queries");
        require(h.gemv_ok, "block sums need a width of at most 4096");
        const uint64_t xb = uint64_t(queries * h.width) * 4;
        check_range({x, xb}, xb, 16, "activations");
        check_range({sums, sums_bytes}, uint64_t(queries) * h.rows * h.nb * 4, 4, "block sums");
        check_device(x, "activations");
        check_device(sums, "block sums");
        cudaStream_t s = as_stream(stream);
        GemvArgs a = stage(h, x, h.width, queries, rounding, nullptr, nullptr, 0.0f, h.status, s);
        a.sums = sums;
        launch_gemv(h.q4, a, s);
        cuda_check(cudaGetLastError(), "block sums launch");
        return 0;
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return -1;
    }
}

int mstar_b200_linear_readout(void *handle, const float *x, int64_t x_stride, int64_t queries, float *logits,
                              int64_t *token, int32_t *status, const int64_t *suppressed,
                              uint64_t suppressed_count, const float *ln_weight, const float *ln_bias, float ln_eps,
                              int rounding, void *stream, char *error, size_t error_size) {
    try {
        require(handle, "missing linear handle");
        auto &h = *static_cast<Linear *>(handle);
        Busy busy(h.busy);
        check_rounding(rounding);
        require(queries >= 1 && queries <= CHUNK, "readout takes 1..32 queries");
        require(h.gemv_ok, "readout needs a width of at most 4096");
        validate_run(h, x, x_stride, queries, logits, h.rows);
        validate_norm(h, ln_weight, ln_bias, ln_eps);
        const uint64_t lb = uint64_t(queries * h.rows) * 4;
        check_range({token, uint64_t(queries) * 8}, uint64_t(queries) * 8, 8, "token");
        check_range({status, 4}, 4, 4, "status");
        require(suppressed_count <= uint64_t(h.rows), "suppression count exceeds vocabulary");
        if (suppressed_count) {
            check_range({suppressed, suppressed_count * 8}, suppressed_count * 8, 8, "suppression list");
            check_device(suppressed, "suppression list");
        } else require(!suppressed, "empty suppression list given a pointer");
        require(disjoint({logits, lb}, {token, uint64_t(queries) * 8}) && disjoint({logits, lb}, {status, 4}) &&
                    disjoint({token, uint64_t(queries) * 8}, {status, 4}),
                "readout outputs overlap");
        check_device(token, "token");
        check_device(status, "status");
        cudaStream_t s = as_stream(stream);
        if (h.wt && !h.wpg_override) {  // one launch: it writes the status itself
            require(!ln_weight || (uintptr_t(ln_weight) % 16 == 0 && uintptr_t(ln_bias) % 16 == 0),
                    "LayerNorm vectors must be 16-byte aligned");
            launch_readout(h, x, x_stride, queries, ln_weight, ln_bias, ln_eps, rounding, logits, token, status,
                           suppressed, int64_t(suppressed_count), s);
            cuda_check(cudaGetLastError(), "readout launch");
            return 0;
        }
        cuda_check(cudaMemsetAsync(status, 0, 4, s), "status reset");
        GemvArgs a = stage(h, x, x_stride, queries, rounding, ln_weight, ln_bias, ln_eps, status, s);
        a.out = logits;
        a.ldo = h.rows;
        a.keys = h.keys;
        a.done = h.done;
        a.token = token;
        a.suppressed = suppressed;
        a.suppressed_count = int64_t(suppressed_count);
        a.wpg_override = h.wpg_override;
        launch_gemv(h.q4, a, s);
        cuda_check(cudaGetLastError(), "readout launch");
        return 0;
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return -1;
    }
}

int mstar_b200_q8_readout(void *handle, const float *x, float *out, int64_t *token, int32_t *status,
                          const int64_t *suppressed, size_t suppressed_count, void *stream) {
    if (!mstar_b200_capability()) return ENOTSUP;
    if (!handle || !x || !out || !token || !status || (suppressed_count && !suppressed)) return EINVAL;
    auto &h = *static_cast<Linear *>(handle);
    if (h.q4 || h.width > 4096) return EINVAL;
    char e[256];
    if (uintptr_t(x) % 16) return EINVAL;
    return mstar_b200_linear_readout(handle, x, h.width, 1, out, token, status, suppressed, suppressed_count,
                                     nullptr, nullptr, 0.0f, MSTAR_B200_Q8_ARM, stream, e, sizeof(e))
               ? EINVAL
               : 0;
}

int mstar_b200_linear_prepare_readout(void *handle, const void *blocks, uint64_t bytes, char *error,
                                      size_t error_size) {
    try {
        require(handle, "missing linear handle");
        auto &h = *static_cast<Linear *>(handle);
        Busy busy(h.busy);
        check_range({blocks, bytes}, uint64_t(h.rows) * h.nb * (h.q4 ? Q4_BYTES : Q8_BYTES), 1, "linear weights");
        check_device(blocks, "linear weights");
        require(readout_tiles_fit(h.rows, h.nb, h.q4), "readout width too large for the tile kernel");
        if (!h.wt) {
            cuda_check(cudaDeviceSynchronize(), "readout preparation");
            const int64_t tiles = ceil_div(h.rows, 16);
            h.wt = device_alloc<uint8_t>(size_t(tiles * h.nb * (h.q4 ? 288 : 544)), "readout tiles");
            h.ro_flags = device_alloc<int>(1, "readout status bits");
            cuda_check(cudaMemset(h.ro_flags, 0, sizeof(int)), "readout status reset");
            launch_readout_repack(h.q4, static_cast<const uint8_t *>(blocks), h.wt, h.rows, h.nb, nullptr);
            cuda_check(cudaGetLastError(), "readout repack");
            cuda_check(cudaDeviceSynchronize(), "readout preparation");
            h.tiles = tiles;
        }
        return 0;
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return -1;
    }
}

int mstar_b200_linear_prepare_gemm(void *handle, const void *blocks, uint64_t bytes, int64_t max_queries,
                                   char *error, size_t error_size) {
    try {
        require(handle, "missing linear handle");
        auto &h = *static_cast<Linear *>(handle);
        Busy busy(h.busy);
        require(max_queries >= GEMM_MIN_QUERIES && max_queries <= (int64_t(1) << 31), "invalid GEMM query capacity");
        check_range({blocks, bytes}, uint64_t(h.rows) * h.nb * (h.q4 ? Q4_BYTES : Q8_BYTES), 1, "linear weights");
        check_device(blocks, "linear weights");
        cuda_check(cudaDeviceSynchronize(), "GEMM preparation");
        if (!h.w16) {
            h.w16 = device_alloc<__half>(size_t(h.rows * h.width), "fp16 GEMM weights");
            launch_dequant_weights(static_cast<const uint8_t *>(blocks), h.w16, h.rows, h.nb, h.q4, nullptr);
            cuda_check(cudaGetLastError(), "weight dequantization");
            make_fp16_map(&h.wmap, h.w16, h.rows, h.width, GEMM_TILE_N);
            make_fp16_map(&h.wmap_pair, h.w16, h.rows, h.width, GEMM_PAIR_TILE_N);
        }
        if (max_queries > h.gemm_rows) {
            if (h.x16) cudaFree(h.x16);
            h.x16 = nullptr;
            h.x16 = device_alloc<__half>(size_t(max_queries * h.width), "fp16 GEMM activations");
            h.gemm_rows = max_queries;
        }
        cuda_check(cudaDeviceSynchronize(), "GEMM preparation");
        return 0;
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return -1;
    }
}

int mstar_b200_linear_gemm(void *handle, const void *staged, uint64_t staged_bytes, int64_t rows, void *out,
                           uint64_t out_bytes, int64_t out_stride, int32_t out_format, const float *residual,
                           uint64_t residual_bytes, int64_t residual_stride, int64_t residual_period,
                           int64_t segment_rows, int64_t out_segment_rows, int32_t flags, int32_t rounding,
                           int32_t *status, void *stream, char *error, size_t error_size) {
    try {
        require(handle, "missing linear handle");
        auto &h = *static_cast<Linear *>(handle);
        Busy busy(h.busy);
        require(h.w16, "linear_gemm needs prepare_gemm first");
        check_rounding(rounding);
        require((flags & ~15) == 0 && !((flags & 2) && (flags & 8)), "invalid epilogue flags");
        require(!(flags & 1) || h.bias, "bias epilogue without a prepared bias");
        require(out_format == MSTAR_B200_OUT_F32 || out_format == MSTAR_B200_OUT_F16 ||
                    out_format == MSTAR_B200_OUT_STAGED,
                "unknown output format");
        require(out_format != MSTAR_B200_OUT_STAGED || h.rows % QK == 0, "staged output needs a multiple of 32 rows");
        require(rows >= 1 && rows <= (int64_t(1) << 31), "invalid row count");
        require(out_stride >= h.rows, "invalid output stride");
        require(segment_rows >= 0 && (segment_rows == 0) == (out_segment_rows == 0) &&
                    (segment_rows == 0 || out_segment_rows >= segment_rows),
                "invalid output segments");
        require(status, "missing status word");
        const uint64_t sb = uint64_t(rows) * h.width * 2;
        check_range({staged, staged_bytes}, sb, 16, "staged operand");
        // output rows span up to the last segment's padded extent
        const int64_t last = segment_rows ? ((rows - 1) / segment_rows) * out_segment_rows + (rows - 1) % segment_rows
                                          : rows - 1;
        const int64_t out_rows = segment_rows ? ceil_div(rows, segment_rows) * out_segment_rows : rows;
        require(last < out_rows, "output segment arithmetic");
        const uint64_t esz = out_format == MSTAR_B200_OUT_F32 ? 4 : 2;
        const uint64_t ob = uint64_t((out_rows - 1) * out_stride + h.rows) * esz;
        check_range({out, out_bytes}, ob, esz == 4 ? 4 : 2, "output");
        require(disjoint({staged, sb}, {out, ob}), "output overlaps the staged operand");
        if (flags & 4) {
            require(residual_stride >= h.rows && residual_period >= 0, "invalid residual layout");
            const int64_t res_rows = residual_period ? (residual_period < rows ? residual_period : rows) : rows;
            const uint64_t rb = uint64_t((res_rows - 1) * residual_stride + h.rows) * 4;
            check_range({residual, residual_bytes}, rb, 4, "residual");
            const bool same = static_cast<const void *>(residual) == out && out_format == MSTAR_B200_OUT_F32 &&
                              residual_stride == out_stride && !residual_period && !segment_rows;
            require(same || disjoint({residual, rb}, {out, ob}), "residual partially overlaps output");
            check_device(residual, "residual");
        } else require(!residual && !residual_period, "residual given without its epilogue flag");
        check_device(staged, "staged operand");
        check_device(out, "output");
        check_device(status, "status word");
        cudaStream_t s = as_stream(stream);
        CUtensorMap xmap;
        make_fp16_map(&xmap, staged, rows, h.width, GEMM_TILE_M);
        GemmArgs g{};
        g.M = rows;
        g.N = h.rows;
        g.K = h.width;
        g.out = out;
        g.ldo = out_stride;
        g.bias = h.bias;
        g.residual = (flags & 4) ? residual : nullptr;
        g.ldr = residual_stride;
        g.res_period = residual_period;
        g.seg_rows = segment_rows;
        g.out_seg_rows = out_segment_rows;
        g.flags = flags;
        g.gelu = h.gelu;
        g.out_mode = out_format == MSTAR_B200_OUT_F32 ? GEMM_OUT_F32
                     : out_format == MSTAR_B200_OUT_F16 ? GEMM_OUT_F16 : GEMM_OUT_Q8;
        g.rounding = rounding;
        g.status = status;
        launch_gemm(xmap, h.wmap, h.wmap_pair, g, s);
        cuda_check(cudaGetLastError(), "GEMM launch");
        return 0;
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return -1;
    }
}

int mstar_b200_linear_gemm_push(void *handle, const void *staged, uint64_t staged_bytes, int64_t rows,
                                float *const *recv_ptrs, int32_t *const *flag_ptrs, int32_t world, int32_t rank,
                                int64_t owner_rows, int32_t *status, void *stream, char *error, size_t error_size) {
    try {
        require(handle, "missing linear handle");
        auto &h = *static_cast<Linear *>(handle);
        Busy busy(h.busy);
        require(h.w16, "linear_gemm_push needs prepare_gemm first");
        require(world >= 1 && world <= 8 && rank >= 0 && rank < world, "invalid rank / world");
        require(rows > GEMM_TILE_M && rows <= (int64_t(1) << 31), "pushed partial products need more than 128 rows");
        require(h.rows % QK == 0, "pushed partial products need a multiple of 32 output columns");
        require(owner_rows > 0 && owner_rows % 32 == 0, "owner rows must be a positive multiple of 32");
        require(owner_rows * world >= rows, "the owners' row ranges must cover every row");
        require(recv_ptrs && flag_ptrs && status, "missing push operand");
        const uint64_t sb = uint64_t(rows) * h.width * 2;
        check_range({staged, staged_bytes}, sb, 16, "staged operand");
        check_device(staged, "staged operand");
        check_device(status, "status word");
        CUtensorMap xmap;
        make_fp16_map(&xmap, staged, rows, h.width, GEMM_TILE_M);
        GemmArgs g{};
        g.M = rows;
        g.N = h.rows;
        g.K = h.width;
        g.ldo = h.rows;
        g.out_mode = GEMM_OUT_PUSH;
        g.status = status;
        g.push_out = recv_ptrs;
        g.push_flags = flag_ptrs;
        g.push_rows = owner_rows;
        g.push_rank = rank;
        launch_gemm(xmap, h.wmap, h.wmap_pair, g, as_stream(stream));
        cuda_check(cudaGetLastError(), "GEMM launch");
        return 0;
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return -1;
    }
}

int mstar_b200_linear_set_split(void *handle, int warps, char *error, size_t error_size) {
    try {
        require(handle, "missing linear handle");
        auto &h = *static_cast<Linear *>(handle);
        Busy busy(h.busy);
        require(warps == 0 || warps == 1 || warps == 2 || warps == 4 || warps == 8, "split must be 0, 1, 2, 4 or 8");
        h.wpg_override = warps;
        return 0;
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return -1;
    }
}

int mstar_b200_linear_close(void *handle, char *error, size_t error_size) {
    try {
        if (handle) {
            auto *h = static_cast<Linear *>(handle);
            require(!h->busy.test_and_set(std::memory_order_acquire), "cannot close a busy linear handle");
            cudaDeviceSynchronize();
            delete h;
        }
        return 0;
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return -1;
    }
}

int mstar_b200_set_wait_limits(int64_t tp_barrier_polls, int64_t grid_barrier_polls, char *error,
                               size_t error_size) {
    try {
        require(tp_barrier_polls >= 0 && grid_barrier_polls >= 0, "wait limits must not be negative");
        wait_limits().tp_barrier = tp_barrier_polls;
        wait_limits().grid_barrier = grid_barrier_polls;
        return 0;
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return -1;
    }
}

int mstar_b200_wait_selftest(int32_t kind, int64_t limit, uint32_t *words, int32_t *status, void *stream,
                             char *error, size_t error_size) {
    try {
        require(mstar_b200_capability() == 1, "sm_100a device capability is unavailable");
        require(limit > 0 && limit <= (int64_t(1) << 30), "selftest wait limit out of range");
        require(status != nullptr, "status word missing");
        check_device(status, "status word");
        cudaStream_t s = as_stream(stream);
        if (kind == MSTAR_B200_WAIT_MBARRIER) {
            k_mbarrier_selftest<<<1, 32, 0, s>>>(status, uint32_t(limit));
        } else if (kind == MSTAR_B200_WAIT_GRID_BARRIER) {
            require(words != nullptr, "barrier words missing");
            check_device(words, "barrier words");
            cuda_check(cudaMemsetAsync(words, 0, 2 * sizeof(uint32_t), s), "barrier words");
            launch_grid_barrier_selftest(words, status, limit, s);
        } else {
            require(false, "unknown wait kind");
        }
        cuda_check(cudaGetLastError(), "wait selftest launch");
        return 0;
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return -1;
    }
}

}  // extern "C"
