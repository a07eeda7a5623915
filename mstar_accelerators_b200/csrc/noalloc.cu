// Q8_0 greedy readout that allocates no device memory.
//
// Some callers cannot allocate: a serving runtime that owns all device memory
// and hands kernels only the buffers it planned up front, or a latency-bound
// caller (a streaming decoder step) that must not pay for cudaMalloc and the
// synchronisation it can cause. mstar_b200_linear_create allocates (the B200
// weight layout and per-handle scratch), so those callers use this entry point
// instead: it reads the caller's canonical ggml Q8_0 bytes directly and keeps
// its scratch (quantized activations, the argmax state) in one file-scope
// device array of fixed size, so a call needs nothing but the caller's inputs
// and outputs.
//
// The array is sizeof(NoAllocScratch), about 81 KB, per device, loaded with this
// library's device code and held by every GPU that loads the library until
// the process exits. Every call shares it: calls whose work overlaps on the
// GPU (different streams without ordering between them) race on it. Each call
// clears the fields that must start at zero.
//
// Host code cannot use the array's name as a device address (in host code the
// symbol is a host-side stand-in). The first call on each device, with that
// device current, resolves the address with cudaGetSymbolAddress and caches
// it; make that first call before capturing any stream.
//
// The math is the same as the handle-based readout (per-block int32 dots with
// mma.m16n8k32, fp32 fold in ggml's generic block order, suppression,
// first-index / NaN-first argmax), so its results are bit-identical to
// mstar_b200_q8_readout on a handle made from the same bytes.
#include <cerrno>
#include <mutex>

#include "../../include/mstar_b200.h"
#include "quant.cuh"

namespace mb {

constexpr int64_t NOALLOC_MAX_WIDTH = 4096;  // K limit (q8cpu_readout's own limit, readout.c:36)
constexpr int64_t NOALLOC_MAX_BLOCKS = NOALLOC_MAX_WIDTH / QK;
constexpr int NOALLOC_MAX_DEVICES = 64;

struct NoAllocScratch {
    uint4 xf[NOALLOC_MAX_BLOCKS * 32];     // A fragments of one 16-row tile (one query + 15 zero rows)
    float xs[NOALLOC_MAX_BLOCKS * 16];     // activation scales, [block][row]
    int xsum[NOALLOC_MAX_BLOCKS * 16];     // activation quant sums (written by the quantizer)
    unsigned long long key;                // running argmax key: zero at the start of a call
    unsigned int done;                     // finished-CTA counter: zero at the start of a call
    unsigned int pad;
};

static __device__ __align__(256) NoAllocScratch g_noalloc_scratch;

// This device's copy of the array and its SM count, resolved once per device
// under one lock (the first call on a device does it; make that call before any
// stream capture).
struct NoAllocDevice {
    NoAllocScratch *scratch = nullptr;
    int sms = 0;
};

static bool noalloc_device(int device, NoAllocDevice &out) {
    static std::mutex lock;
    static NoAllocDevice known[NOALLOC_MAX_DEVICES] = {};
    if (device < 0 || device >= NOALLOC_MAX_DEVICES) return false;
    std::lock_guard<std::mutex> guard(lock);
    NoAllocDevice &d = known[device];
    if (!d.scratch) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess) {
            cudaGetLastError();
            return false;
        }
        int sms = 0;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || sms <= 0) {
            cudaGetLastError();
            sms = 148;
        }
        d.sms = sms;
        d.scratch = static_cast<NoAllocScratch *>(p);
    }
    out = d;
    return true;
}

__device__ __forceinline__ float block_scale(const uint8_t *block) {
    return __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short *>(block)));
}

// One warp per 8-row group, reading canonical 34-byte blocks (2-byte aligned
// 16-bit loads). Query 0 is row g == 0 of the m16 tile, so lanes 0..3 own its
// eight outputs.
__global__ void __launch_bounds__(256) k_readout_canonical(const uint8_t *__restrict__ blocks, int64_t rows, int nb,
                                                           NoAllocScratch *__restrict__ s, float *__restrict__ out,
                                                           int64_t *__restrict__ token,
                                                           const int64_t *__restrict__ suppressed, int64_t nsup) {
    __shared__ unsigned long long cta_best;
    __shared__ bool last;
    if (threadIdx.x == 0) cta_best = 0ull;
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, t = lane & 3;
    const int64_t groups = (rows + 7) / 8;
    unsigned long long best = 0ull;
    for (int64_t G = int64_t(blockIdx.x) * 8 + warp; G < groups; G += int64_t(gridDim.x) * 8) {
        const int64_t row = G * 8 + g, c0 = G * 8 + 2 * t, c1 = c0 + 1;
        float acc0 = 0.0f, acc1 = 0.0f;
        for (int b = 0; b < nb; ++b) {
            uint32_t b0 = 0, b1 = 0;
            if (row < rows) {
                const unsigned short *q = reinterpret_cast<const unsigned short *>(blocks + (row * nb + b) * Q8_BYTES + 2);
                b0 = uint32_t(q[2 * t]) | (uint32_t(q[2 * t + 1]) << 16);
                b1 = uint32_t(q[8 + 2 * t]) | (uint32_t(q[8 + 2 * t + 1]) << 16);
            }
            int d[4];
            mma_s8(d, s->xf[b * 32 + lane], b0, b1);
            const float dx = s->xs[b * 16 + g];
            const float dw0 = c0 < rows ? block_scale(blocks + (c0 * nb + b) * Q8_BYTES) : 0.0f;
            const float dw1 = c1 < rows ? block_scale(blocks + (c1 * nb + b) * Q8_BYTES) : 0.0f;
            acc0 = __fadd_rn(acc0, __fmul_rn(__int2float_rn(d[0]), __fmul_rn(dw0, dx)));
            acc1 = __fadd_rn(acc1, __fmul_rn(__int2float_rn(d[1]), __fmul_rn(dw1, dx)));
        }
        if (g == 0) {
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                const int64_t n = c ? c1 : c0;
                if (n >= rows) continue;
                float v = c ? acc1 : acc0;
                for (int64_t i = 0; i < nsup; ++i)
                    if (suppressed[i] == n) v = -INFINITY;
                out[n] = v;
                const unsigned long long k = argmax_key(v, uint32_t(n));
                best = k > best ? k : best;
            }
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
    }
    if (lane == 0 && best) atomicMax(&cta_best, best);
    __syncthreads();
    if (threadIdx.x == 0) {
        if (cta_best) atomicMax(&s->key, cta_best);
        __threadfence();
        last = atomicAdd(&s->done, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (last && threadIdx.x == 0) {
        __threadfence();
        const unsigned long long k = atomicExch(&s->key, 0ull);
        *token = int64_t(0xFFFFFFFFu - uint32_t(k & 0xFFFFFFFFull));
        s->done = 0u;
    }
}

}  // namespace mb

using namespace mb;

extern "C" {

int mstar_b200_q8_readout_noalloc(const void *blocks, size_t bytes, int64_t rows, int64_t k, const float *x,
                                  float *out, int64_t *token, int32_t *status, const int64_t *suppressed,
                                  size_t suppressed_count, void *stream) {
    if (!mstar_b200_capability()) return ENOTSUP;
    if (!blocks || !x || !out || !token || !status || (suppressed_count && !suppressed)) return EINVAL;
    if (rows <= 0 || rows > (int64_t(1) << 31) || k <= 0 || k % QK) return EINVAL;
    if (k > NOALLOC_MAX_WIDTH) return E2BIG;  // the static scratch holds at most 4096-wide activations
    if (suppressed_count > size_t(rows)) return EINVAL;
    const size_t row_bytes = size_t(k / QK) * Q8_BYTES;
    if (size_t(rows) > SIZE_MAX / row_bytes || bytes != size_t(rows) * row_bytes) return EINVAL;
    if (uintptr_t(blocks) % 2 || uintptr_t(x) % 16 || uintptr_t(out) % 4 || uintptr_t(token) % 8 ||
        uintptr_t(status) % 4)
        return EINVAL;
    int device = -1;
    if (cudaGetDevice(&device) != cudaSuccess) {
        cudaGetLastError();
        return EIO;
    }
    NoAllocDevice dev;
    if (!noalloc_device(device, dev)) return EIO;
    NoAllocScratch *s = dev.scratch;
    cudaStream_t st = as_stream(stream);
    const int64_t nb = k / QK, nb_pad = (nb + 1) / 2 * 2;
    // the argmax state and the caller's status start at zero
    if (cudaMemsetAsync(&s->key, 0, sizeof(s->key) + sizeof(s->done), st) != cudaSuccess ||
        cudaMemsetAsync(status, 0, sizeof(int32_t), st) != cudaSuccess) {
        cudaGetLastError();
        return EIO;
    }
    launch_quantize_frag(MSTAR_B200_Q8_ARM, x, k, 1, k, 16, nb_pad, nullptr, nullptr, 0.0f,
                         reinterpret_cast<uint32_t *>(s->xf), s->xs, s->xsum, status, st);
    const int64_t groups = (rows + 7) / 8;
    int64_t grid = (groups + 7) / 8;
    if (grid > int64_t(dev.sms) * 8) grid = int64_t(dev.sms) * 8;
    k_readout_canonical<<<unsigned(grid), 256, 0, st>>>(static_cast<const uint8_t *>(blocks), rows, int(nb), s, out,
                                                        token, suppressed, int64_t(suppressed_count));
    if (cudaGetLastError() != cudaSuccess) return EIO;
    return 0;
}

}  // extern "C"
