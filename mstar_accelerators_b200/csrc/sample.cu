// Positive-temperature categorical sampling of readout logits: the reference's
// philox4x32-10-gumbel23-v1 operation (backends/pi/docs/categorical.md), a
// stateless Philox4x32-10 draw per (row, vocabulary entry) turned into Gumbel
// noise, and the lowest index of the highest perturbed score:
//   key = (seed lo, seed hi), counter = (offset lo, offset hi, j, 0);
//   u = ((word0 >> 9) + 0.5) * 2^-23 (exact, strictly inside (0, 1));
//   score_j = centered_j / T - log(-log(u_j)), centered_j = 0 for a row maximum,
//   else fp32(logit_j - max) / T, every step rounded to fp32 (the two logarithms
//   evaluated in double and rounded, as the reference's scalar oracle does, so
//   draws agree with it token for token);
//   -1 for a row with a NaN, no finite-or-+inf entry, or a temperature that is not
//   positive and finite; with +inf logits only the +inf entries compete (equally).
// Three launches: per-row maximum and validity; scores over vocabulary chunks
// (many CTAs per row) folded into one 64-bit key per row with atomicMax
// (ordered score bits, then the complement of the index, so ties go to the
// lower index); tokens from the keys. The row's position in the batch never
// enters the draw. Scratch: 16 bytes per row, in the caller's workspace.
#include <cmath>

#include "../../include/mstar_b200.h"
#include "common.cuh"

namespace mb {

constexpr int CAT_THREADS = 256;
constexpr int64_t CAT_CHUNK = int64_t(CAT_THREADS) * 8;  // vocabulary entries per sampling CTA

struct CatRow {
    float max;
    int bad;
    unsigned long long key;
};

__device__ __forceinline__ uint32_t philox_word0(uint64_t seed, uint64_t offset, uint32_t j) {
    uint32_t c0 = uint32_t(offset), c1 = uint32_t(offset >> 32), c2 = j, c3 = 0;
    uint32_t k0 = uint32_t(seed), k1 = uint32_t(seed >> 32);
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        const uint32_t hi0 = __umulhi(0xD2511F53u, c0), lo0 = 0xD2511F53u * c0;
        const uint32_t hi1 = __umulhi(0xCD9E8D57u, c2), lo1 = 0xCD9E8D57u * c2;
        c0 = hi1 ^ c1 ^ k0;
        c1 = lo1;
        c2 = hi0 ^ c3 ^ k1;
        c3 = lo0;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    return c0;
}

__device__ __forceinline__ unsigned long long score_key(float s, uint32_t j) {
    const uint32_t b = __float_as_uint(s == 0.0f ? 0.0f : s);
    const uint32_t o = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return (static_cast<unsigned long long>(o) << 32) | (0xFFFFFFFFu - j);
}

__global__ void __launch_bounds__(CAT_THREADS) k_cat_rowmax(const float *__restrict__ logits, int64_t ld, int64_t vocab,
                                                            const float *__restrict__ temps, CatRow *__restrict__ ws) {
    const int64_t r = blockIdx.x;
    const float *x = logits + r * ld;
    float m = -INFINITY;
    int nan = 0;
    for (int64_t j = threadIdx.x; j < vocab; j += CAT_THREADS) {
        const float v = x[j];
        nan |= v != v;
        m = fmaxf(m, v);
    }
    __shared__ float sm[CAT_THREADS / 32];
    __shared__ int sn[CAT_THREADS / 32];
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        nan |= __shfl_xor_sync(0xffffffffu, nan, o);
    }
    if ((threadIdx.x & 31) == 0) {
        sm[threadIdx.x >> 5] = m;
        sn[threadIdx.x >> 5] = nan;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < CAT_THREADS / 32; ++w) {
            m = fmaxf(m, sm[w]);
            nan |= sn[w];
        }
        const float t = temps[r];
        ws[r].max = m;
        ws[r].bad = nan || m == -INFINITY || !(t > 0.0f) || !isfinite(t);
        ws[r].key = 0ull;
    }
}

__global__ void __launch_bounds__(CAT_THREADS) k_cat_sample(const float *__restrict__ logits, int64_t ld, int64_t vocab,
                                                            const int64_t *__restrict__ seeds,
                                                            const int64_t *__restrict__ offsets,
                                                            const float *__restrict__ temps, CatRow *__restrict__ ws) {
    const int64_t r = blockIdx.y;
    if (ws[r].bad) return;
    const float m = ws[r].max, t = temps[r];
    const uint64_t seed = uint64_t(seeds[r]), offset = uint64_t(offsets[r]);
    const float *x = logits + r * ld;
    const int64_t j0 = int64_t(blockIdx.x) * CAT_CHUNK, j1 = j0 + CAT_CHUNK < vocab ? j0 + CAT_CHUNK : vocab;
    unsigned long long best = 0ull;
    for (int64_t j = j0 + threadIdx.x; j < j1; j += CAT_THREADS) {
        const float v = x[j];
        if (v == -INFINITY || (m == INFINITY && v != m)) continue;
        const float centered = v == m ? 0.0f : __fdiv_rn(__fsub_rn(v, m), t);
        const uint32_t w = philox_word0(seed, offset, uint32_t(j));
        const float u = __fmul_rn(__fadd_rn(float(w >> 9), 0.5f), 0x1p-23f);
        const float inner = float(log(double(u)));
        const float noise = float(log(double(-inner)));
        const unsigned long long k = score_key(__fsub_rn(centered, noise), uint32_t(j));
        best = k > best ? k : best;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
    }
    if ((threadIdx.x & 31) == 0 && best) atomicMax(&ws[r].key, best);
}

__global__ void k_cat_finish(const CatRow *__restrict__ ws, int64_t rows, int64_t *__restrict__ tokens) {
    const int64_t r = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    const unsigned long long k = ws[r].key;
    tokens[r] = (ws[r].bad || !k) ? -1 : int64_t(0xFFFFFFFFu - uint32_t(k & 0xFFFFFFFFull));
}

}  // namespace mb

using namespace mb;

extern "C" {

uint64_t mstar_b200_categorical_workspace(int64_t rows) { return rows > 0 ? uint64_t(rows) * sizeof(CatRow) : 0; }

int mstar_b200_categorical(const float *logits, int64_t rows, int64_t vocab, int64_t ld, const int64_t *seeds,
                           const int64_t *offsets, const float *temperatures, int64_t *tokens, void *workspace,
                           uint64_t workspace_bytes, void *stream, char *error, size_t error_size) {
    try {
        require(rows >= 1 && rows <= 65535, "rows must be 1..65535");
        require(vocab >= 1 && vocab <= 0x7FFFFFFF && ld >= vocab, "invalid vocabulary extent");
        require(logits && seeds && offsets && temperatures && tokens && workspace, "missing sampling operand");
        require(workspace_bytes >= uint64_t(rows) * sizeof(CatRow), "sampling workspace too small");
        require(uintptr_t(workspace) % 16 == 0 && uintptr_t(tokens) % 8 == 0 && uintptr_t(seeds) % 8 == 0 &&
                    uintptr_t(offsets) % 8 == 0 && uintptr_t(logits) % 4 == 0 && uintptr_t(temperatures) % 4 == 0,
                "sampling operands are misaligned");
        for (const void *p : {static_cast<const void *>(logits), static_cast<const void *>(seeds),
                              static_cast<const void *>(offsets), static_cast<const void *>(temperatures),
                              static_cast<const void *>(tokens), static_cast<const void *>(workspace)})
            check_device(p, "sampling operand");
        cudaStream_t s = as_stream(stream);
        auto *ws = static_cast<CatRow *>(workspace);
        k_cat_rowmax<<<unsigned(rows), CAT_THREADS, 0, s>>>(logits, ld, vocab, temperatures, ws);
        const dim3 grid(unsigned(ceil_div(vocab, CAT_CHUNK)), unsigned(rows));
        k_cat_sample<<<grid, CAT_THREADS, 0, s>>>(logits, ld, vocab, seeds, offsets, temperatures, ws);
        k_cat_finish<<<unsigned(ceil_div(rows, 256)), 256, 0, s>>>(ws, rows, tokens);
        cuda_check(cudaGetLastError(), "sampling launch");
        return 0;
    } catch (const std::exception &e) {
        message(error, error_size, e.what());
        return -1;
    }
}

}  // extern "C"
