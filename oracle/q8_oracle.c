/*
 * ORACLE — test infrastructure only.
 *
 * A plain-C restatement of the reference's block-quantized arithmetic for the
 * Q8_0 / Q4_0 linear contractions, used by the tests, the smoke check and the
 * CPU-baseline leg of bench.py to compare against. Nothing in the product path
 * (mstar_accelerators_b200) links or calls this file.
 *
 * Every function names the reference file:line it restates (paths are inside
 * rohanchanani/mstar_accelerators; ggml is vendored at
 * backends/pi/third_party/ggml, llama.cpp revision 1b29621b).
 *
 * Build with -ffp-contract=off: every rounding step below is explicit.
 * Parity is pinned by tests/test_oracle.py against (1) the reference's own
 * known-answer tests (tests/whisper/test_q8_readout.py:13-36,
 * tests/test_cpu_ggml_q4_readout.py:79-91), re-expressed as golden fixtures,
 * and (2) the vendored ggml quantizers/dots compiled from the reference
 * sources into oracle/_ref (see oracle/Makefile).
 */
#include <math.h>
#include <stdint.h>
#include <stddef.h>
#include <string.h>

#define QK 32
#define Q8_BLOCK_BYTES 34
#define Q4_BLOCK_BYTES 18

/* Activation-quantizer rounding variants of quantize_row_q8_0. */
enum {
    ORC_Q8_REF = 0, /* ggml-quants.c:276-297   id = 1/d, roundf (half away from zero) */
    ORC_Q8_ARM = 1, /* ggml-cpu/arch/arm/quants.c:41-75  id = 1/d, vcvtnq (half to even) */
    ORC_Q8_X86 = 2, /* ggml-cpu/arch/x86/quants.c:302-350 id = 127/amax, _MM_ROUND_NEAREST */
};

/* ---------------- IEEE binary16 <-> binary32, round-to-nearest-even --------
 * Written from the IEEE 754 definitions (ggml's GGML_FP32_TO_FP16 is the
 * same rounding: ggml-impl.h uses RNE in software, F16C _cvtss_sh(x, 0) on
 * x86 and the AArch64 FCVT instruction on ARM). */
uint16_t orc_fp32_to_fp16(float f) {
    uint32_t x; memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t absx = x & 0x7fffffffu;
    if (absx >= 0x7f800000u) {              /* inf or nan */
        if (absx > 0x7f800000u) return (uint16_t)(sign | 0x7e00u | ((absx >> 13) & 0x3ffu));
        return (uint16_t)(sign | 0x7c00u);
    }
    if (absx >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* rounds to >= 65520 -> inf */
    if (absx < 0x38800000u) {               /* result is subnormal in fp16 (or zero) */
        if (absx < 0x33000000u) return (uint16_t)sign;          /* < 2^-25 rounds to 0 (tie at 2^-25 -> even 0) */
        uint32_t e = absx >> 23;
        uint32_t mant = (absx & 0x7fffffu) | 0x800000u;
        uint32_t shift = 126u - e;          /* value = mant * 2^(e-150); fp16 subnormal unit 2^-24 */
        /* q = mant >> (shift - 0) ... compute units of 2^-24: mant * 2^(e-150+24) */
        uint32_t s = 150u - 24u - e;        /* right shift amount, >= 1 */
        uint32_t q = mant >> s;
        uint32_t rem = mant & ((1u << s) - 1u);
        uint32_t half = 1u << (s - 1u);
        (void)shift;
        if (rem > half || (rem == half && (q & 1u))) q += 1u;
        return (uint16_t)(sign | q);
    }
    uint32_t e = (absx >> 23) - 127u + 15u;
    uint32_t mant = absx & 0x7fffffu;
    uint32_t q = (e << 10) | (mant >> 13);
    uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q += 1u;  /* carry may bump exponent: correct */
    return (uint16_t)(sign | q);
}

float orc_fp16_to_fp32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu, x;
    if (e == 0) {
        if (m == 0) x = sign;
        else {                                   /* subnormal: normalise */
            int k = 0;
            while (!(m & 0x400u)) { m <<= 1; ++k; }
            m &= 0x3ffu;
            x = sign | ((uint32_t)(127 - 15 + 1 - k) << 23) | (m << 13);
        }
    } else if (e == 31) x = sign | 0x7f800000u | (m << 13);
    else x = sign | ((e - 15u + 127u) << 23) | (m << 13);
    float f; memcpy(&f, &x, 4); return f;
}

/* round-half-to-even of a finite float to int (vcvtnq / _MM_ROUND_NEAREST) */
static int round_even(float v) { return (int)nearbyintf(v); }

/* ---------------- Q8_0 quantizer (activations and weights) ----------------
 * ref: ggml-quants.c:276-297 quantize_row_q8_0_ref
 * arm: ggml-cpu/arch/arm/quants.c:41-75 (Raspberry Pi production path)
 * x86: ggml-cpu/arch/x86/quants.c:302-350
 * Block layout {fp16 d; int8 qs[32]} = 34 bytes, ggml-common.h:251-256. */
void orc_quantize_row_q8_0(const float *x, uint8_t *y, int64_t k, int mode) {
    const int64_t nb = k / QK;
    for (int64_t i = 0; i < nb; ++i) {
        const float *b = x + i * QK;
        uint8_t *o = y + i * Q8_BLOCK_BYTES;
        float amax = 0.0f;
        for (int j = 0; j < QK; ++j) { float a = fabsf(b[j]); amax = amax > a ? amax : a; }
        const float d = amax / 127.0f;
        float id;
        if (mode == ORC_Q8_X86) id = amax != 0.0f ? 127.0f / amax : 0.0f;
        else id = d != 0.0f ? 1.0f / d : 0.0f;
        uint16_t h = orc_fp32_to_fp16(d);
        memcpy(o, &h, 2);
        for (int j = 0; j < QK; ++j) {
            const float v = b[j] * id;
            int q = mode == ORC_Q8_REF ? (int)roundf(v) : round_even(v);
            o[2 + j] = (uint8_t)(int8_t)q;
        }
    }
}

/* ---------------- Q4_0 quantizer --------------------------------------------
 * ggml-quants.c:113-147 quantize_row_q4_0_ref. `fused` selects a single
 * rounding of x*id + 8.5 (what GCC's FMLA contraction produces on the Pi
 * target) versus separate multiply and add roundings
 * (tests/test_cpu_ggml_q4_readout.py:72-88 names both contracts).
 * Layout {fp16 d; uint8 qs[16]}: element j in the low nibble of byte j and
 * element j+16 in the high nibble (ggml-common.h:194-199). */
void orc_quantize_row_q4_0(const float *x, uint8_t *y, int64_t k, int fused) {
    const int64_t nb = k / QK;
    for (int64_t i = 0; i < nb; ++i) {
        const float *b = x + i * QK;
        uint8_t *o = y + i * Q4_BLOCK_BYTES;
        float amax = 0.0f, max = 0.0f;
        for (int j = 0; j < QK; ++j) {
            const float v = b[j];
            if (amax < fabsf(v)) { amax = fabsf(v); max = v; }
        }
        const float d = max / -8.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        uint16_t h = orc_fp32_to_fp16(d);
        memcpy(o, &h, 2);
        for (int j = 0; j < QK / 2; ++j) {
            float t0, t1;
            if (fused) { t0 = fmaf(b[j], id, 8.5f); t1 = fmaf(b[j + 16], id, 8.5f); }
            else {
                volatile float p0 = b[j] * id, p1 = b[j + 16] * id;
                t0 = p0 + 8.5f; t1 = p1 + 8.5f;
            }
            int q0 = (int8_t)t0, q1 = (int8_t)t1;   /* C truncation toward zero */
            if (q0 > 15) q0 = 15;
            if (q1 > 15) q1 = 15;
            o[2 + j] = (uint8_t)(q0 | (q1 << 4));
        }
    }
}

/* ---------------- weight packers --------------------------------------------
 * Native uploads pre-round each logical fp32 weight through fp16 before the
 * canonical quantizer: decoder.cpp:307-316 (Q8 body), decoder.cpp:816-842
 * (Q4 readout; rejects nonfinite input and fp16 overflow). The Python packer
 * pack_q8_0 (implementations/whisper/pi_v3d/q8.py:16-45) does not pre-round.
 * Returns 0, or -1 nonfinite input, -2 fp16 overflow. */
int orc_pack_weights(const float *w, uint8_t *out, int64_t rows, int64_t k,
                     int q4, int preround, int fused) {
    float buf[16384];
    if (k > 16384 || k % QK) return -3;
    const int64_t row_bytes = (k / QK) * (q4 ? Q4_BLOCK_BYTES : Q8_BLOCK_BYTES);
    for (int64_t r = 0; r < rows; ++r) {
        for (int64_t j = 0; j < k; ++j) {
            float v = w[r * k + j];
            if (!isfinite(v)) return -1;
            if (preround) {
                v = orc_fp16_to_fp32(orc_fp32_to_fp16(v));
                if (!isfinite(v)) return -2;
            }
            buf[j] = v;
        }
        if (q4) orc_quantize_row_q4_0(buf, out + r * row_bytes, k, fused);
        else orc_quantize_row_q8_0(buf, out + r * row_bytes, k, ORC_Q8_REF);
    }
    return 0;
}

/* ---------------- block dots -------------------------------------------------
 * Per-block exact int32 sums, and the fp32 accumulation in the generic block
 * order: ggml-cpu/quants.c:451-480 (q8_0 x q8_0: sumf += sumi*(dx*dy)) and
 * ggml-cpu/quants.c:225-258 (q4_0 x q8_0: sumf += sumi*dx*dy, left to right). */
void orc_block_sums_q8_0(const uint8_t *w, const uint8_t *x, int64_t nb, int32_t *sumi) {
    for (int64_t b = 0; b < nb; ++b) {
        const int8_t *wq = (const int8_t *)(w + b * Q8_BLOCK_BYTES + 2);
        const int8_t *xq = (const int8_t *)(x + b * Q8_BLOCK_BYTES + 2);
        int32_t s = 0;
        for (int j = 0; j < QK; ++j) s += (int32_t)wq[j] * (int32_t)xq[j];
        sumi[b] = s;
    }
}

void orc_block_sums_q4_0(const uint8_t *w, const uint8_t *x, int64_t nb, int32_t *sumi) {
    for (int64_t b = 0; b < nb; ++b) {
        const uint8_t *wq = w + b * Q4_BLOCK_BYTES + 2;
        const int8_t *xq = (const int8_t *)(x + b * Q8_BLOCK_BYTES + 2);
        int32_t s0 = 0, s1 = 0;
        for (int j = 0; j < QK / 2; ++j) {
            s0 += ((int32_t)(wq[j] & 0x0f) - 8) * xq[j];
            s1 += ((int32_t)(wq[j] >> 4) - 8) * xq[j + 16];
        }
        sumi[b] = s0 + s1;
    }
}

static float scale_of(const uint8_t *block) { uint16_t h; memcpy(&h, block, 2); return orc_fp16_to_fp32(h); }

float orc_vec_dot_q8_0(const uint8_t *w, const uint8_t *x, int64_t nb) {
    float sumf = 0.0f;
    for (int64_t b = 0; b < nb; ++b) {
        int32_t s; orc_block_sums_q8_0(w + b * Q8_BLOCK_BYTES, x + b * Q8_BLOCK_BYTES, 1, &s);
        const float dd = scale_of(w + b * Q8_BLOCK_BYTES) * scale_of(x + b * Q8_BLOCK_BYTES);
        sumf = sumf + (float)s * dd;
    }
    return sumf;
}

float orc_vec_dot_q4_0(const uint8_t *w, const uint8_t *x, int64_t nb) {
    float sumf = 0.0f;
    for (int64_t b = 0; b < nb; ++b) {
        int32_t s; orc_block_sums_q4_0(w + b * Q4_BLOCK_BYTES, x + b * Q8_BLOCK_BYTES, 1, &s);
        float t = (float)s * scale_of(w + b * Q4_BLOCK_BYTES);
        t = t * scale_of(x + b * Q8_BLOCK_BYTES);
        sumf = sumf + t;
    }
    return sumf;
}

/* ---------------- mul_mat ----------------------------------------------------
 * ggml_compute_forward_mul_mat (ggml-cpu.c:1255): each fp32 activation row is
 * quantized with the vec_dot_type quantizer (Q8_0 for both Q8_0 and Q4_0
 * weights, ggml-cpu.c:240-248, 272-280), then out[m][n] = vec_dot(W[n], xq[m]).
 * W is ggml row-major blocks [N][K/32]; x is [M][K] fp32; out is [M][N]. */
void orc_mul_mat(const uint8_t *w, int q4, const float *x, float *out,
                 int64_t m, int64_t n, int64_t k, int mode, uint8_t *xq_scratch) {
    const int64_t nb = k / QK;
    const int64_t wrow = nb * (q4 ? Q4_BLOCK_BYTES : Q8_BLOCK_BYTES);
    const int64_t CH = 64, cn = (n + CH - 1) / CH, cm = (m + CH - 1) / CH;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < m; ++i)
        orc_quantize_row_q8_0(x + i * k, xq_scratch + i * nb * Q8_BLOCK_BYTES, k, mode);
    /* 64 x 64 (weight row, activation row) chunks so both operands stay in cache;
     * every output is one generic-order dot, so the split never changes a bit */
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t c = 0; c < cn * cm; ++c) {
        const int64_t r0 = (c % cn) * CH, i0 = (c / cn) * CH;
        const int64_t r1 = r0 + CH < n ? r0 + CH : n, i1 = i0 + CH < m ? i0 + CH : m;
        for (int64_t i = i0; i < i1; ++i) {
            const uint8_t *xr = xq_scratch + i * nb * Q8_BLOCK_BYTES;
            for (int64_t r = r0; r < r1; ++r)
                out[i * n + r] = q4 ? orc_vec_dot_q4_0(w + r * wrow, xr, nb) : orc_vec_dot_q8_0(w + r * wrow, xr, nb);
        }
    }
}

/* ---------------- readout ------------------------------------------------------
 * Suppression then first-index argmax where the first NaN wins over any
 * non-NaN: backends/cpu_ggml/decoder.cpp:686-696, backends/cpu_q8/readout.c:47-53. */
int64_t orc_argmax(float *logits, int64_t rows, const int64_t *suppressed, int64_t count) {
    for (int64_t i = 0; i < count; ++i) logits[suppressed[i]] = -INFINITY;
    int64_t best = 0;
    for (int64_t r = 1; r < rows; ++r)
        if ((!isnan(logits[best]) && isnan(logits[r])) || logits[r] > logits[best]) best = r;
    return best;
}

/* ggml stock GELU (tanh form through the fp16 table): ggml-cpu/vec.h:963-969 and
 * :1000-1013, table built at ggml-cpu.c:3889. Input and output are rounded
 * through fp16; |x| >= 10 short-circuits. */
float orc_gelu_ggml(float x) {
    if (x <= -10.0f) return 0.0f;
    if (x >= 10.0f) return x;
    const float h = orc_fp16_to_fp32(orc_fp32_to_fp16(x));
    const float c = 0.79788456080286535587989211986876f, a = 0.044715f;
    const float g = 0.5f * h * (1.0f + tanhf(c * h * (1.0f + a * h * h)));
    return orc_fp16_to_fp32(orc_fp32_to_fp16(g));
}

/* orc_gelu_ggml over n values (ggml_vec_gelu_f32 on a row). */
void orc_gelu_ggml_rows(const float *x, float *y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) y[i] = orc_gelu_ggml(x[i]);
}

/* ---------------- categorical sampling (readout epilogue) ------------------------
 * philox4x32-10-gumbel23-v1 (backends/pi/docs/categorical.md; its scalar test
 * oracle backends/pi/torch/tests/categorical_reference.py:18-64): Philox4x32-10
 * (Random123: ten rounds, multipliers 0xD2511F53 / 0xCD9E8D57, Weyl key steps
 * 0x9E3779B9 / 0xBB67AE85) with key = (seed lo, seed hi), counter = (offset lo,
 * offset hi, token, 0); u = ((word0 >> 9) + 0.5) * 2^-23; score = centered / T -
 * log(-log(u)), each step rounded to fp32 (the logarithms evaluated in double
 * and rounded, as that oracle does), centered = 0 for a row maximum, else
 * fp32(logit - max) / T; the lowest index of the highest score wins. A NaN
 * logit, an all -inf row or a temperature that is not positive and finite give
 * -1; with a +inf logit only the +inf entries compete. */
void orc_philox4x32_10(const uint32_t counter[4], const uint32_t key[2], uint32_t out[4]) {
    uint32_t c0 = counter[0], c1 = counter[1], c2 = counter[2], c3 = counter[3];
    uint32_t k0 = key[0], k1 = key[1];
    for (int r = 0; r < 10; ++r) {
        const uint64_t a = (uint64_t)0xD2511F53u * c0, b = (uint64_t)0xCD9E8D57u * c2;
        const uint32_t n0 = (uint32_t)(b >> 32) ^ c1 ^ k0, n1 = (uint32_t)b;
        const uint32_t n2 = (uint32_t)(a >> 32) ^ c3 ^ k1, n3 = (uint32_t)a;
        c0 = n0; c1 = n1; c2 = n2; c3 = n3;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

static float orc_uniform(uint64_t seed, uint64_t offset, uint32_t token) {
    const uint32_t ctr[4] = {(uint32_t)offset, (uint32_t)(offset >> 32), token, 0};
    const uint32_t key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
    uint32_t w[4];
    orc_philox4x32_10(ctr, key, w);
    return ((float)(w[0] >> 9) + 0.5f) * 0x1p-23f;
}

int64_t orc_categorical_row(const float *logits, int64_t vocab, uint64_t seed, uint64_t offset, float temperature) {
    if (vocab <= 0 || !isfinite(temperature) || !(temperature > 0.0f)) return -1;
    float m = -INFINITY;
    for (int64_t j = 0; j < vocab; ++j) {
        if (isnan(logits[j])) return -1;
        if (logits[j] > m) m = logits[j];
    }
    if (m == -INFINITY) return -1;
    int64_t best = -1;
    float best_score = -INFINITY;
    for (int64_t j = 0; j < vocab; ++j) {
        const float v = logits[j];
        if (v == -INFINITY || (m == INFINITY && v != m)) continue;
        const float centered = v == m ? 0.0f : (float)(v - m) / temperature;
        const float u = orc_uniform(seed, offset, (uint32_t)j);
        const float inner = (float)log((double)u);
        const float noise = (float)log((double)(-inner));
        const float score = centered - noise;
        if (best < 0 || score > best_score) {
            best = j;
            best_score = score;
        }
    }
    return best;
}

void orc_categorical(const float *logits, int64_t rows, int64_t vocab, const int64_t *seeds, const int64_t *offsets,
                     const float *temperatures, int64_t *tokens) {
    for (int64_t r = 0; r < rows; ++r)
        tokens[r] = orc_categorical_row(logits + r * vocab, vocab, (uint64_t)seeds[r], (uint64_t)offsets[r],
                                        temperatures[r]);
}
