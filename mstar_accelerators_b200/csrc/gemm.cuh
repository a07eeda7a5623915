#pragma once
#include <cuda.h>

#include "quant.cuh"

namespace mb {

struct GemmArgs {
    int64_t M, N, K;
    float *out;             // [M][ldo]
    int64_t ldo;
    const float *bias;      // [N] or null
    const float *residual;  // [M][ldo] or null (may alias out)
    int flags;              // MSTAR_B200_BIAS / GELU / RESIDUAL / GELU_ERF
    int *status;            // bit value 2: a bounded pipeline wait timed out
};

void make_fp16_map(CUtensorMap *map, const void *ptr, int64_t rows, int64_t k, int box_rows);
void launch_dequant_weights(const uint8_t *blocks, __half *out, int64_t rows, int64_t nb, int q4, cudaStream_t s);
void launch_dequant_act(int mode, const float *x, int64_t ldx, int64_t m, int64_t k, __half *out, int *status,
                        cudaStream_t s);
void launch_gemm(const CUtensorMap &ta, const CUtensorMap &tb, const GemmArgs &a, cudaStream_t s);

constexpr int GEMM_TILE_M = 128, GEMM_TILE_N = 256;

}  // namespace mb
