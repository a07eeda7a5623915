#pragma once
#include <cuda.h>

#include "quant.cuh"

namespace mb {

struct GemmArgs {
    int64_t M, N, K;
    void *out;              // [rows][ldo]: fp32, or fp16 for the fp16 / Q8_0-staging output modes
    int64_t ldo;
    const float *bias;      // [N] or null
    const float *residual;  // [rows][ldr] fp32 or null (may alias an fp32 out)
    int64_t ldr;
    int64_t res_period;     // > 0: residual row = row % res_period (a table shared by every segment)
    int64_t seg_rows;       // > 0: output row = (row / seg_rows) * out_seg_rows + row % seg_rows
    int64_t out_seg_rows;
    int flags;              // MSTAR_B200_BIAS / GELU / RESIDUAL / GELU_ERF
    const uint16_t *gelu;   // ggml GELU table (gelu_table()), copied to shared memory with the GELU flag
    int out_mode;           // GEMM_OUT_F32 / GEMM_OUT_F16 / GEMM_OUT_Q8
    int rounding;           // Q8_0 rounding of GEMM_OUT_Q8
    int *status;            // bit value 2: a bounded pipeline wait timed out; 1: nonfinite Q8_0 input
    // GEMM_OUT_PUSH (row-parallel partial products delivered to their owners):
    float *const *push_out; // [world] device pointers: each rank's receive buffer [world][push_rows][N] fp32
    int *const *push_flags; // [world] device pointers: each rank's arrival counters, one per 32 owned rows
    int64_t push_rows;      // rows per owner (a multiple of 32); row r belongs to owner r / push_rows
    int push_rank;          // this rank: the slot its partials land in at every owner
};

// Output modes: fp32 rows; fp16 rows; or each 32-column block Q8_0-quantized
// (ggml quantize_row_q8_0, selected rounding) and stored as fp16(q * d), the
// staged A operand of the next GEMM; or (PUSH) the fp32 partial product stored
// straight into the owning rank's receive slot over NVLink, followed by an
// arrival on the owner's counter of those rows.
constexpr int GEMM_OUT_F32 = 0, GEMM_OUT_F16 = 1, GEMM_OUT_Q8 = 2, GEMM_OUT_PUSH = 3;
// Arrivals a 32-row group of an owner receives from one rank per pushed GEMM: one per
// epilogue warp column group (4) and 256-column tile.
__host__ __device__ constexpr int push_arrivals_per_rank(int64_t n) { return int(4 * ((n + 255) / 256)); }

void make_fp16_map(CUtensorMap *map, const void *ptr, int64_t rows, int64_t k, int box_rows);
void launch_dequant_weights(const uint8_t *blocks, __half *out, int64_t rows, int64_t nb, int q4, cudaStream_t s);
void launch_dequant_act(int mode, const float *x, int64_t ldx, int64_t m, int64_t k, __half *out, int *status,
                        cudaStream_t s);
// rows of fp32 or fp16 [-> LayerNorm] -> Q8_0 (selected rounding) -> fp16(q * d) [rows][k]
void launch_stage_rows(int mode, const void *x, int x_f16, int64_t ldx, int64_t rows, int64_t k, const float *ln_w,
                       const float *ln_b, float ln_eps, __half *out, int64_t ldo, int *status, cudaStream_t s);
// contiguous bf16 rows [rows][k] (16-byte aligned, k a multiple of 32) -> Q8_0 (selected
// rounding) -> fp16(q * d) [rows][k]; status (may be null) gets bit value 1 for a nonfinite value
void launch_stage_rows_bf16(int mode, const void *x, int64_t rows, int64_t k, __half *out, int *status,
                            cudaStream_t s);
// 1-D convolution columns (kernel 3, padding 1, dilation 1) -> Q8_0 -> fp16(q * d),
// K = 3 * channels zero-padded to k_padded; row = b * time_out + t, column = c * 3 + tap
void launch_stage_conv(int mode, const float *src, int time_major, int64_t batch, int64_t channels,
                       int64_t time_in, int64_t time_out, int stride, int64_t k_padded, __half *out, int *status,
                       cudaStream_t s);
void launch_layer_norm(const float *x, int64_t ldx, int64_t rows, int64_t k, const float *w, const float *b, float eps,
                       float *out, int64_t ldo, cudaStream_t s);
// tb: weights with 256-row boxes (single-CTA kernel, M <= 128); tb_pair: the same
// weights with 128-row boxes (the CTA-pair kernel used above 128 rows)
void launch_gemm(const CUtensorMap &ta, const CUtensorMap &tb, const CUtensorMap &tb_pair, const GemmArgs &a,
                 cudaStream_t s);

constexpr int GEMM_TILE_M = 128, GEMM_TILE_N = 256, GEMM_PAIR_TILE_N = 128;

}  // namespace mb
