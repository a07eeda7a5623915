/*
 * ORACLE — test infrastructure only.
 *
 * Driver for the reference's own Q8_0/Q4_0 arithmetic, compiled from the
 * vendored ggml sources where they lie (oracle/Makefile builds
 * oracle/_ref/libggml_quant_ref.so from ggml-quants.c, ggml-cpu/quants.c and
 * ggml-cpu/arch/x86/quants.c; none of those sources are copied here).
 *
 * This file supplies (1) the handful of ggml core symbols those three files
 * reference but that live in ggml.c (an fp16 table, type-size queries, abort),
 * written here from scratch, and (2) a row-parallel mul_mat loop standing in
 * for ggml_compute_forward_mul_mat (ggml-cpu.c:1255): quantize each fp32
 * activation row with the vec_dot_type quantizer, then one vec_dot per
 * (row, column). It is the CPU baseline "reference" leg and a second reference
 * for the restatement in oracle/q8_oracle.c.
 */
#include <stdint.h>
#include <stddef.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <omp.h>

/* --- symbols owned by ggml.c in the full library ------------------------- */
uint16_t orc_fp32_to_fp16(float f);   /* from q8_oracle.c, linked in */
float orc_fp16_to_fp32(uint16_t h);

float ggml_table_f32_f16[1 << 16];
float ggml_table_f32_e8m0_half[1 << 8];
float ggml_table_f32_ue4m3[1 << 8];

__attribute__((constructor)) static void init_tables(void) {
    for (int i = 0; i < (1 << 16); ++i) ggml_table_f32_f16[i] = orc_fp16_to_fp32((uint16_t)i);
}

void ggml_abort(const char *file, int line, const char *fmt, ...) {
    fprintf(stderr, "ggml_abort at %s:%d (%s)\n", file, line, fmt);
    abort();
}

/* Only the Q8_0 / Q4_0 paths are driven; other types are never queried. */
size_t ggml_type_size(int type) { (void)type; abort(); }
size_t ggml_row_size(int type, int64_t ne) { (void)type; (void)ne; abort(); }
const char *ggml_type_name(int type) { (void)type; return "?"; }

/* --- the reference kernels (vendored ggml) -------------------------------- */
void quantize_row_q8_0_ref(const float *x, void *y, int64_t k);          /* ggml-quants.c:276 */
void quantize_row_q4_0_ref(const float *x, void *y, int64_t k);          /* ggml-quants.c:113 */
void quantize_row_q8_0(const float *x, void *y, int64_t k);              /* arch/x86/quants.c:302 */
void ggml_vec_dot_q8_0_q8_0(int n, float *s, size_t bs, const void *vx, size_t bx,
                            const void *vy, size_t by, int nrc);        /* arch/x86/quants.c:1372 */
void ggml_vec_dot_q4_0_q8_0(int n, float *s, size_t bs, const void *vx, size_t bx,
                            const void *vy, size_t by, int nrc);        /* arch/x86/quants.c:765 */
void ggml_vec_dot_q8_0_q8_0_generic(int n, float *s, size_t bs, const void *vx, size_t bx,
                                    const void *vy, size_t by, int nrc); /* quants.c:451 */
void ggml_vec_dot_q4_0_q8_0_generic(int n, float *s, size_t bs, const void *vx, size_t bx,
                                    const void *vy, size_t by, int nrc); /* quants.c:225 */

void ref_quantize_q8_0_ref(const float *x, void *y, int64_t k) { quantize_row_q8_0_ref(x, y, k); }
void ref_quantize_q8_0_x86(const float *x, void *y, int64_t k) { quantize_row_q8_0(x, y, k); }
void ref_quantize_q4_0_ref(const float *x, void *y, int64_t k) { quantize_row_q4_0_ref(x, y, k); }

float ref_vec_dot(int q4, int generic, int k, const void *w, const void *xq) {
    float s = 0.0f;
    if (q4) (generic ? ggml_vec_dot_q4_0_q8_0_generic : ggml_vec_dot_q4_0_q8_0)(k, &s, 0, w, 0, xq, 0, 1);
    else (generic ? ggml_vec_dot_q8_0_q8_0_generic : ggml_vec_dot_q8_0_q8_0)(k, &s, 0, w, 0, xq, 0, 1);
    return s;
}

/* out[m][n] = W[n] . quantize_q8_0_x86(x[m]); W ggml row-major blocks.
 * xq_scratch holds m * (k/32) * 34 bytes. threads <= 0 uses every OpenMP thread.
 *
 * Work split in the manner of ggml_compute_forward_mul_mat (ggml-cpu.c:1255,
 * ggml_compute_forward_mul_mat_one_chunk): the (weight row, activation row)
 * plane is cut into 64 x 64 chunks dealt dynamically to the threads, and each
 * chunk is walked in 16 x 16 blocks, one vec_dot per (row, column) pair, so a
 * block's weight rows and quantized activation rows stay in cache. */
void ref_mul_mat(const void *w, int q4, const float *x, float *out, int64_t m, int64_t n,
                 int64_t k, void *xq_scratch, int threads) {
    const int64_t nb = k / 32, xrow = nb * 34, wrow = nb * (q4 ? 18 : 34);
    uint8_t *xq = (uint8_t *)xq_scratch;
    const int nt = threads > 0 ? threads : omp_get_max_threads();
    const uint8_t *wb = (const uint8_t *)w;
    const int64_t CH = 64, BL = 16;
    const int64_t cn = (n + CH - 1) / CH, cm = (m + CH - 1) / CH;
#pragma omp parallel for schedule(static) num_threads(nt)
    for (int64_t i = 0; i < m; ++i) quantize_row_q8_0(x + i * k, xq + i * xrow, k);
#pragma omp parallel for schedule(dynamic, 1) num_threads(nt)
    for (int64_t c = 0; c < cn * cm; ++c) {
        const int64_t r0 = (c % cn) * CH, i0 = (c / cn) * CH;
        const int64_t r1 = r0 + CH < n ? r0 + CH : n, i1 = i0 + CH < m ? i0 + CH : m;
        for (int64_t bi = i0; bi < i1; bi += BL)
            for (int64_t br = r0; br < r1; br += BL)
                for (int64_t i = bi; i < bi + BL && i < i1; ++i)
                    for (int64_t r = br; r < br + BL && r < r1; ++r) {
                        float s = 0.0f;
                        if (q4) ggml_vec_dot_q4_0_q8_0((int)k, &s, 0, wb + r * wrow, 0, xq + i * xrow, 0, 1);
                        else ggml_vec_dot_q8_0_q8_0((int)k, &s, 0, wb + r * wrow, 0, xq + i * xrow, 0, 1);
                        out[i * n + r] = s;
                    }
    }
}
