/*
 * mstar_b200 — C ABI of the B200 (sm_100a) block-quantized linear kernels.
 *
 * Drop-in boundary for the reference's native Q8_0/Q4_0 contractions
 * (rohanchanani/mstar_accelerators). Every entry point below names the
 * reference interface it replaces. Plain pointers and sizes only; no torch
 * types. Device pointers are CUDA global memory of the current device.
 *
 * Conventions, kept from the reference:
 *  - *_abi() and *_capability() return int 1 when usable
 *    (backends/cpu_ggml/encoder.h:29-31).
 *  - create(...) returns an opaque handle, or NULL with a message in
 *    (error, error_size) (encoder.h:32-37).
 *  - run(...)/close(...) return 0 on success, -1 with a message on error,
 *    and never throw (encoder.cpp:811-834). close rejects a busy handle.
 *  - The two q8cpu mirrors return errno codes (0, EINVAL, EDOM, ENOTSUP)
 *    exactly like backends/cpu_q8/readout.c:21-54.
 * B200 differences: every run takes a cudaStream_t (passed as void *) and is
 * stream-ordered; extents, alignment and disjointness are validated on the
 * host before any launch; borrowed inputs must stay valid until the stream
 * reaches the call's completion. Results that the reference reports through
 * a return code after computing (a nonfinite readout input) are written to a
 * caller-visible device status word instead.
 */
#pragma once
#include <stddef.h>
#include <stdint.h>

#if defined(_WIN32)
#define MSTAR_B200_API __declspec(dllexport)
#else
#define MSTAR_B200_API __attribute__((visibility("default")))
#endif
#ifdef __cplusplus
extern "C" {
#endif

/* Activation quantizer rounding variants of ggml quantize_row_q8_0. */
enum mstar_b200_q8_rounding {
    MSTAR_B200_Q8_REF = 0, /* ggml-quants.c:276-297: id = 1/d, roundf */
    MSTAR_B200_Q8_ARM = 1, /* ggml-cpu/arch/arm/quants.c:41-75: id = 1/d, half-even (default) */
    MSTAR_B200_Q8_X86 = 2, /* ggml-cpu/arch/x86/quants.c:302-350: id = 127/amax, half-even */
};
enum mstar_b200_format { MSTAR_B200_Q8_0 = 8, MSTAR_B200_Q4_0 = 4, MSTAR_B200_BF16 = 16 };
/* Epilogue flags of mstar_b200_linear_run; applied in this order after the
 * block-quantized dot, each as the reference's separate fp32 ggml op. */
enum mstar_b200_epilogue {
    MSTAR_B200_BIAS = 1,      /* ggml_add(mul_mat, bias)              decoder.cpp:498-500 */
    MSTAR_B200_GELU = 2,      /* ggml_gelu, fp16-table tanh form      decoder.cpp:580     */
    MSTAR_B200_RESIDUAL = 4,  /* ggml_add(current, linear)            decoder.cpp:565-581 */
    MSTAR_B200_GELU_ERF = 8,  /* ggml_gelu_erf (F32 graphs)           decoder.cpp:581     */
};
/* Element type of activation rows handed to mstar_b200_stage_rows. */
enum mstar_b200_activation { MSTAR_B200_ACT_F32 = 0, MSTAR_B200_ACT_F16 = 1 };
/* Output form of mstar_b200_linear_gemm. STAGED: every 32-column block is
 * Q8_0-quantized (rounding) and stored as fp16(q * d), i.e. already the staged
 * activation operand of the next GEMM (the handle's row count, i.e. the output
 * width, must then be a multiple of 32). */
enum mstar_b200_output { MSTAR_B200_OUT_F32 = 0, MSTAR_B200_OUT_F16 = 1, MSTAR_B200_OUT_STAGED = 2 };

/* --- library identity (encoder.h:29-31, backends/torch/q8.py:42-77) -------- */
MSTAR_B200_API int mstar_b200_abi(void);
/* 1 iff the current CUDA device is compute capability 10.0 (B200) and this
 * library's sm_100a kernels load on it; 0 otherwise (never a fallback). */
MSTAR_B200_API int mstar_b200_capability(void);

/* --- weight packers ------------------------------------------------------------
 * Logical fp32 [rows][width] (device) -> canonical ggml blocks (device),
 * bit-exact with the reference packers:
 *   Q8_0, preround=1: decoder.cpp:307-316 upload_q8 (fp16 pre-round, then
 *                     quantize_row_q8_0_ref);  preround=0: pi_v3d/q8.py:16-45.
 *   Q4_0:             cpu_decoder_pack_readout_q4, decoder.cpp:816-842
 *                     (fp16 pre-round, quantize_row_q4_0_ref); fused=1 rounds
 *                     x*id+8.5 once (FMA contract), fused=0 twice
 *                     (tests/test_cpu_ggml_q4_readout.py:72-88).
 * Rejects nonfinite input ("nonfinite") and fp16 overflow ("overflows F16")
 * like decoder.cpp:829-833; those checks synchronise the stream. */
MSTAR_B200_API int mstar_b200_pack(int format, const float *input, uint64_t input_bytes,
    void *output, uint64_t output_bytes, int64_t rows, int64_t width, int preround, int fused,
    void *stream, char *error, size_t error_size);

/* --- q8cpu mirrors (backends/cpu_q8/readout.c:21-54) ---------------------------
 * mstar_b200_q8_quantize: fp32 x[rows][k] (device) -> Q8_0 blocks (device) with
 * the selected rounding; EDOM if any input is nonfinite (synchronises). */
MSTAR_B200_API int mstar_b200_q8_quantize(const float *x, void *packed, size_t bytes, int64_t rows,
    int64_t k, int rounding, void *stream);

/* --- prepared block-quantized linear (ggml mul_mat(Q8_0|Q4_0 W, F32 x) + epilogue)
 * Replaces the Q8_0 graph nodes of backends/cpu_ggml/encoder.cpp:467-479,
 * 694-723 and decoder.cpp:498-500, 563-588 and the Q4_0/Q8_0 vocab projection
 * set by cpu_decoder_set_readout_q4/q8 (decoder_readout.h:11-24).
 * create: blocks = canonical ggml bytes [rows][width/32] (device, borrowed only
 * during create; the handle owns its B200 layout copy). bias may be NULL. */
MSTAR_B200_API void *mstar_b200_linear_create(int format, const void *blocks, uint64_t bytes,
    int64_t rows, int64_t width, const float *bias, char *error, size_t error_size);
/* out[m][n] = epilogue(sum_b sumi_b * (d_w * d_x)) for m < queries; x is fp32
 * [queries][width] (device, 16-byte aligned rows of stride x_stride floats),
 * optionally LayerNorm-ed first (ln_weight/ln_bias non-NULL: ggml_norm(eps)
 * then mul and add, decoder.cpp:501-503), then quantized on the fly with
 * `rounding`; residual [queries][rows] (stride out_stride) if flagged (it may
 * alias out exactly). The fp32 accumulation follows ggml's generic block
 * order, so results are bit-identical to ggml_vec_dot_q8_0_q8_0_generic /
 * q4_0_q8_0_generic. Queries beyond 32 run in 32-row chunks. */
MSTAR_B200_API int mstar_b200_linear_run(void *handle, const float *x, int64_t x_stride,
    int64_t queries, float *out, int64_t out_stride, const float *residual, int flags,
    const float *ln_weight, const float *ln_bias, float ln_eps,
    int rounding, void *stream, char *error, size_t error_size);
/* Exact per-block int32 dots sums[m][n][b] of the same kernel path (the parity
 * probe for "bit-exact per-block integer dot products"). queries <= 32. */
MSTAR_B200_API int mstar_b200_linear_block_sums(void *handle, const float *x, int64_t queries,
    int32_t *sums, uint64_t sums_bytes, int rounding, void *stream, char *error, size_t error_size);
/* Greedy vocab readout on the same handle: logits[m][rows] (suppressed rows
 * -inf), then first-index argmax where the first NaN wins
 * (decoder.cpp:686-696, readout.c:47-53) into token[m] (int64). status[0]
 * becomes 1 if any x is nonfinite (decoder.cpp:479-487 rejects such a call).
 * suppressed: device int64 list (may be NULL when count is 0). */
MSTAR_B200_API int mstar_b200_linear_readout(void *handle, const float *x, int64_t x_stride,
    int64_t queries, float *logits, int64_t *token, int32_t *status, const int64_t *suppressed,
    uint64_t suppressed_count, const float *ln_weight, const float *ln_bias, float ln_eps,
    int rounding, void *stream, char *error, size_t error_size);
MSTAR_B200_API int mstar_b200_linear_close(void *handle, char *error, size_t error_size);
/* Q8_0 activation fragments of a handle's decode GEMV (the layout its
 * quantizer writes: fragments [blocks][rows / 16][32][4] words, scales and
 * quant sums [blocks][rows]), for a producer kernel that quantizes its own
 * output straight into them (mstar_b200_attend_q8). */
typedef struct mstar_b200_q8_frags {
    void *fragments;
    float *scales;
    int32_t *sums;
    int64_t blocks;    /* padded block count of the handle's width */
    int64_t rows;      /* 16 or 32 */
    int32_t rounding;  /* MSTAR_B200_Q8_REF / ARM / X86 */
} mstar_b200_q8_frags;
/* Describe the handle's fragment buffers for `queries` (1..32) rows. */
MSTAR_B200_API int mstar_b200_linear_frags(void *handle, int64_t queries, int32_t rounding,
    mstar_b200_q8_frags *frags, char *error, size_t error_size);
/* mstar_b200_linear_run (Q8_0 weights, 1..32 queries, rows a multiple of 32)
 * that also quantizes its outputs into `next` (from mstar_b200_linear_frags of
 * the linear that consumes them, e.g. fc2 after fc1 with GELU,
 * decoder.cpp:580): the bytes mstar_b200_linear_run on `out` would produce, so
 * mstar_b200_linear_run_frags on the next handle needs no quantize launch. */
MSTAR_B200_API int mstar_b200_linear_run_q8out(void *handle, const float *x, int64_t x_stride, int64_t queries,
    float *out, int64_t out_stride, const float *residual, int flags, const float *ln_weight,
    const float *ln_bias, float ln_eps, int rounding, const mstar_b200_q8_frags *next, void *stream,
    char *error, size_t error_size);
/* The decode GEMV (+ bias / GELU / residual epilogue, flags as linear_run) on
 * the fragments a producer wrote for `queries` rows: equal to linear_run on the
 * producer's fp32 output (ggml_mul_mat + the same epilogue). */
MSTAR_B200_API int mstar_b200_linear_run_frags(void *handle, int64_t queries, float *out, int64_t out_stride,
    const float *residual, int flags, void *stream, char *error, size_t error_size);
/* Prepare the vocab-readout tile layout of a handle (16 weight rows per tile,
 * the whole tile's fragments and scales contiguous): later linear_readout
 * calls on the handle use the tile kernel, bit-identical to the GEMV path.
 * Takes the canonical blocks given to create. Synchronises. Replaces nothing
 * in the reference: its readout is the same ggml_mul_mat + argmax
 * (decoder.cpp:686-696). */
MSTAR_B200_API int mstar_b200_linear_prepare_readout(void *handle, const void *blocks, uint64_t bytes,
    char *error, size_t error_size);
/* Prepare the tcgen05 GEMM used by linear_run calls of 64..max_queries rows
 * without a fused LayerNorm (prefill / encoder shapes, the M = 1500 and
 * M = 24000 mul_mat of encoder.cpp:467-479, 694-723): keeps fp16(q*d) of the
 * canonical blocks (the same bytes given to create) and an activation buffer
 * of max_queries rows. Results match ggml's mul_mat to reorder and fp16
 * product-rounding tolerance (the decode GEMV stays bit-exact). Synchronises. */
MSTAR_B200_API int mstar_b200_linear_prepare_gemm(void *handle, const void *blocks, uint64_t bytes,
    int64_t max_queries, char *error, size_t error_size);
/* The prepared GEMM on an operand that is already staged: staged = fp16(q * d)
 * [rows][width] of the Q8_0-quantized activations (from mstar_b200_stage_rows,
 * mstar_b200_stage_conv or a previous call's STAGED output; 16-byte aligned),
 * so a chain of encoder linears (encoder.cpp:692-725) never materialises its
 * fp32 activations. Output element (r, n) goes to out row
 *   o(r) = segment_rows ? (r / segment_rows) * out_segment_rows + r % segment_rows : r
 * (a per-utterance padded plane such as the F16 K/V rows padded to 256 of
 * qkv_scatter, encoder.cpp:202-234, when out_segment_rows > segment_rows), in
 * out_format, after the flagged epilogue (bias, GELU, then + residual row
 * residual_period ? r % residual_period : r, stride residual_stride: the
 * positional table of encoder.cpp:689 repeats per utterance). Pass status
 * (device int32): bit value 1 nonfinite STAGED input, 2 a bounded wait timed out.
 * rows may exceed the capacity given to prepare_gemm (no handle buffer is used). */
MSTAR_B200_API int mstar_b200_linear_gemm(void *handle, const void *staged, uint64_t staged_bytes, int64_t rows,
    void *out, uint64_t out_bytes, int64_t out_stride, int32_t out_format, const float *residual,
    uint64_t residual_bytes, int64_t residual_stride, int64_t residual_period, int64_t segment_rows,
    int64_t out_segment_rows, int32_t flags, int32_t rounding, int32_t *status, void *stream, char *error,
    size_t error_size);
/* Physical policy, set on an idle handle (the role of
 * cpu_decoder_set_cross_threads, decoder.h:44-47): warps that split one
 * 8-row group's K range (1, 2, 4 or 8; 0 restores the automatic choice).
 * Results are identical for every setting. */
MSTAR_B200_API int mstar_b200_linear_set_split(void *handle, int warps, char *error, size_t error_size);

/* q8cpu_readout twin over a prepared Q8_0 handle (readout.c:30-54): quantize
 * x[k] (one row), all rows' dots, suppression, argmax. errno-style result. */
MSTAR_B200_API int mstar_b200_q8_readout(void *handle, const float *x, float *out, int64_t *token,
    int32_t *status, const int64_t *suppressed, size_t suppressed_count, void *stream);

/* --- Qwen3-Omni thinker MoE expert FFN ----------------------------------------------
 * Router (ConsistentBF16Router.forward, qwen3_omni/amd/router_consistency.py:54-62):
 * x bf16 [tokens][hidden], router_weight bf16 [experts][hidden] -> logits rounded
 * to bf16 (written to logits fp32 [tokens][experts]), softmax in fp32, top_k
 * (ties: lower expert index), optional renormalisation (norm_topk_prob) ->
 * topk_weights fp32 / topk_ids int32 [tokens][top_k]. 1..256 experts. */
MSTAR_B200_API int mstar_b200_moe_route(const void *x, int64_t tokens, int64_t hidden,
    const void *router_weight, int32_t experts, int32_t top_k, int32_t renormalize, float *logits,
    float *topk_weights, int32_t *topk_ids, void *stream, char *error, size_t error_size);
/* Expert weights of one MoE layer (the experts_backend of SmallTokenThinkerMoE,
 * thinker_moe.py:104-188; layout preparation.py:13-36): w1 [E][2I][H] (gate rows
 * then up rows), w2 [E][H][I], as bf16 (format BF16) or canonical Q8_0 blocks
 * along the last dimension (format Q8_0, no counterpart in the reference).
 * Borrowed during create only. max_tokens bounds a run's token count. */
MSTAR_B200_API void *mstar_b200_moe_create(int32_t format, const void *w1, uint64_t w1_bytes,
    const void *w2, uint64_t w2_bytes, int32_t experts, int32_t intermediate, int32_t hidden,
    int32_t top_k, int32_t max_tokens, char *error, size_t error_size);
/* out bf16 [tokens][hidden] = sum over slots of bf16(down(bf16 SwiGLU(gate, up)) * w):
 * the bf16 rounding points of gate_up_vector / down_vector_reduce
 * (thinker_moe.py:17-83) and the slot-ordered fp32 sum (:75-81). Q8_0 format:
 * x and mid are Q8_0-quantized (rounding) before each contraction. Status bit
 * value 4: an expert id outside [0, E) (that slot contributes nothing, the
 * skip_invalid behaviour of the reference backends); value 2: a bounded wait
 * timed out. */
MSTAR_B200_API int mstar_b200_moe_run(void *handle, const void *x, int64_t tokens,
    const float *topk_weights, const int32_t *topk_ids, void *out, int32_t *status, int32_t rounding,
    void *stream, char *error, size_t error_size);
MSTAR_B200_API int mstar_b200_moe_close(void *handle, char *error, size_t error_size);
/* moe_run_experts: the experts half of moe_run for a handle holding experts
 * [expert0, expert0 + E) of experts_total (expert parallelism with every rank
 * routing all tokens; thinker_moe.py:17-83 for the held experts): pairs whose id
 * is another rank's expert are skipped, an id outside [0, experts_total) sets
 * status bit value 4. The held pairs' routed down-projection rows
 * bf16(w * down(SwiGLU(gate/up(x)))) land in y (bf16 [y_rows][hidden], 16-byte
 * aligned) at rows row_base + their permuted position, and inv[token * top_k +
 * slot] (int32, tokens * top_k entries) receives that row, or -1 for a pair not
 * held here. No combine: mstar_b200_thinker_combine sums the slots. */
MSTAR_B200_API int mstar_b200_moe_run_experts(void *handle, const void *x, int64_t tokens,
    const float *topk_weights, const int32_t *topk_ids, int32_t expert0, int32_t experts_total, void *y,
    int64_t y_rows, int64_t row_base, int32_t *inv, int32_t *status, int32_t rounding, void *stream,
    char *error, size_t error_size);
/* Slot-ordered combine of expert outputs gathered by the caller (expert
 * parallelism: rows returned by their owners, moe_sum_reduce of
 * thinker_moe.py:75-81): out[t] = bf16(sum_s fp32(y[rows[t*top_k + s]])) in slot
 * order; y bf16 [y_rows][hidden], rows int32 (a row outside [0, y_rows) adds
 * nothing), out bf16 [tokens][hidden]. */
MSTAR_B200_API int mstar_b200_moe_combine(const void *y, int64_t y_rows, const int32_t *rows, int64_t tokens,
    int32_t top_k, int64_t hidden, void *out, void *stream, char *error, size_t error_size);
/* Expert-parallel dispatch plan (the send side of an all_to_all MoE over
 * `ranks` ranks, each owning experts/ranks consecutive experts; the reference
 * runs all experts in one process, thinker_moe.py:104-188, so this has no
 * direct counterpart there). The tokens*top_k (token, slot) pairs are put in
 * send order: grouped by owning rank d = clamp(floor(id / (experts/ranks)), 0,
 * ranks-1), pair order inside a rank. Writes meta int64 [ranks][2] = (pairs for
 * rank d, 1 if any id is outside [0, experts)); rows bf16 [pairs][hidden] =
 * x[pair / top_k] in send order; pairs int32 [pairs][2] = (id - d*(experts/
 * ranks), bits of the fp32 weight) in send order; inverse int32 [pairs] = the
 * send position of each pair (the rows argument of mstar_b200_moe_combine).
 * tokens may be 0 (meta only). No host synchronisation. */
MSTAR_B200_API int mstar_b200_moe_dispatch(const void *x, int64_t tokens, int64_t hidden,
    const float *topk_weights, const int32_t *topk_ids, int32_t top_k, int32_t experts, int32_t ranks,
    int64_t *meta, void *rows, int32_t *pairs, int32_t *inverse, void *stream, char *error, size_t error_size);


/* --- encoder graph staging (backends/cpu_ggml/encoder.cpp:400-754) ------------------
 * stage_rows: rows of x (fp32 or fp16, stride x_stride elements), optionally
 * LayerNorm-ed first (ln_weight/ln_bias: encoder_norm_affine, encoder.cpp:117-142;
 * width <= 1536), Q8_0-quantized per 32 elements (ggml quantize_row_q8_0,
 * `rounding`) and written as fp16(q * d) [rows][width], the staged activation
 * operand of mstar_b200_linear_gemm. staged_bytes = rows * width * 2.
 * status bit value 1: a nonfinite input (quantized as is, like ggml). */
MSTAR_B200_API int mstar_b200_stage_rows(const void *x, int32_t x_format, int64_t x_stride, int64_t rows,
    int64_t width, const float *ln_weight, const float *ln_bias, float ln_eps, void *staged,
    uint64_t staged_bytes, int32_t rounding, int32_t *status, void *stream, char *error, size_t error_size);
/* stage_conv: the columns of convolution_q8 (encoder.cpp:45-52; ggml_im2col with
 * kernel 3, padding 1, dilation 1) of `batch` utterances, source fp32 either
 * channel-major [batch][channels][time_in] (the mel input) or time-major
 * [batch][time_in][channels] (the first convolution's output rows); output row
 * b * time_out + t, column c * 3 + tap, zero columns up to k_padded (3 * channels
 * rounded up to 32, encoder.cpp:551), time_out = (time_in - 1) / stride + 1;
 * staged as in stage_rows. */
MSTAR_B200_API int mstar_b200_stage_conv(const float *source, int32_t time_major, int64_t batch,
    int64_t channels, int64_t time_in, int32_t stride, int64_t k_padded, void *staged, uint64_t staged_bytes,
    int32_t rounding, int32_t *status, void *stream, char *error, size_t error_size);
/* stage_heads: the thinker's prefill attention output (bf16 [seqs][heads][positions]
 * [head_dim] with element strides seq_stride, head_stride, position_stride, head_dim
 * contiguous; the layout scaled_dot_product_attention returns before the transpose in
 * thinker_model.py:106-148) as the output projection's staged operand: row
 * s * positions + t = the heads of position t of sequence s side by side, each 32-value
 * block Q8_0-quantized (rounding) and stored as fp16(q * d), [seqs * positions][heads *
 * head_dim]; the same bytes as mstar_b200_stage_rows on the transposed fp32 rows.
 * head_dim a multiple of 32; the attention output 16-byte aligned, strides multiples of 8. */
MSTAR_B200_API int mstar_b200_stage_heads(const void *attention, int64_t seqs, int64_t heads, int64_t positions,
    int64_t head_dim, int64_t seq_stride, int64_t head_stride, int64_t position_stride, void *staged,
    uint64_t staged_bytes, int32_t rounding, int32_t *status, void *stream, char *error, size_t error_size);
/* layer_norm: fp32 rows -> ggml_norm(eps), mul, add (the final encoder_norm_affine,
 * encoder.cpp:725) -> fp32 out; width <= 1536. */
MSTAR_B200_API int mstar_b200_layer_norm(const float *x, int64_t x_stride, int64_t rows, int64_t width,
    const float *weight, const float *bias, float eps, float *out, int64_t out_stride, void *stream,
    char *error, size_t error_size);

/* --- tensor parallelism over peer memory (accelerations/whisper/cpu_tp2/decoder_all_reduce.py:64-90) ---
 * tp_barrier: the rank's device counter is incremented to g; every rank then
 * stores g into flag_ptrs[p][rank] for all p (system-scope release after a
 * system fence) and waits until my_flags[p] >= g for every p (acquire,
 * bounded: on timeout status bit value 16). flag_ptrs: device array of `world`
 * pointers to each rank's int32[world] flags; flags and counters are zero
 * before the first barrier and every rank calls the barrier equally often
 * (the counter lives on the device, so a captured graph replays correctly).
 * tp_reduce: for this owner's `owned` rows (global rows row0 ..): x = x +
 * (sum over ranks p = 0 .. world-1 of part_ptrs[p][row0 + r] + bias), the
 * partial products read in rank order from every rank's [M][width] fp32
 * partial buffer (peer loads, coalesced), then the bias, then the residual
 * (encoder_bias_residual order, encoder.cpp:146-166), x updated in place; with
 * ln_weight, the new rows are also LayerNorm-ed, Q8_0-quantized (rounding) and
 * stored as fp16(q * d) into every rank's staged operand staged_ptrs[p]
 * ([M][width] fp16, rows row0 ..): the all-gather of the next
 * column-parallel GEMM's input. width <= 1536. Pointer arrays are device
 * arrays of `world` device pointers (peer mappings, e.g. symmetric memory),
 * not checked on the host. */
MSTAR_B200_API int mstar_b200_tp_barrier(int32_t *const *flag_ptrs, int32_t *my_flags, int32_t rank, int32_t world,
    int32_t *counter, int32_t *status, void *stream, char *error, size_t error_size);
MSTAR_B200_API int mstar_b200_tp_reduce(const float *const *part_ptrs, int32_t world, int64_t owned,
    int64_t width, const float *bias, float *x, const float *ln_weight, const float *ln_bias, float ln_eps,
    void *const *staged_ptrs, int64_t row0, int32_t rounding, int32_t *status, void *stream, char *error,
    size_t error_size);
/* tp_reduce_multicast: tp_reduce where the partial buffers and the staged operands
 * are also bound to an NVLink multicast object (NVSwitch NVLS): mc_part and
 * mc_staged are the multicast addresses (16-byte aligned). Each 16 bytes of an
 * owned row's partial sum over all ranks is one multimem.ld_reduce (the switch
 * adds the ranks' partials, in its own fp32 order), and each staged row chunk is
 * one multimem.st that lands in every rank's staged operand. */
MSTAR_B200_API int mstar_b200_tp_reduce_multicast(const float *mc_part, int32_t world, int64_t owned, int64_t width,
    const float *bias, float *x, const float *ln_weight, const float *ln_bias, float ln_eps, void *mc_staged,
    int64_t row0, int32_t rounding, int32_t *status, void *stream, char *error, size_t error_size);
/* linear_gemm_push + tp_reduce_recv: the row-parallel reduction fused into the GEMM
 * epilogue (the same sum as tp_reduce, decoder_all_reduce.py:64-90, with no barrier
 * between the GEMM and the reduction).
 * linear_gemm_push: the prepared linear's product of `rows` (> 128) staged rows, fp32
 * and without bias, delivered by the epilogue straight into the owning rank's receive
 * buffer: row r belongs to owner o = r / owner_rows (owner_rows a multiple of 32,
 * owner_rows * world >= rows) and lands in recv_ptrs[o] at slot `rank`, local row
 * r - o * owner_rows ([world][owner_rows][rows of the linear] fp32, 16-byte aligned).
 * After its stores (system-scope fence) each epilogue warp adds 1 (release) to
 * flag_ptrs[o][(r - o * owner_rows) / 32] for its 32 rows: every 32-row group receives
 * 4 * ceil(N / 256) arrivals from every rank per call. recv_ptrs / flag_ptrs: device
 * arrays of `world` device pointers (peer mappings), not checked on the host.
 * tp_reduce_recv: the owner's side, for its `owned` rows (global rows row0 ..): waits
 * (bounded, status bit value 16) until each 32-row group's counter holds all
 * world * 4 * ceil(width / 256) arrivals, then x = x + (sum over slots p = 0 .. world-1
 * in rank order of recv[p][r] + bias), x updated in place, and with ln_weight the
 * LayerNorm + Q8_0 staging of tp_reduce into every rank's staged operand (staged_ptrs,
 * or the multicast address mc_staged when not null); then clears the counters.
 * counters: this rank's int32[owner_rows / 32 + 1], zero before the first push (the
 * last word is the reduction's own count of finished CTAs). Every rank must pass a
 * barrier (tp_barrier) after this call before any rank pushes into the same receive
 * buffer again. */
MSTAR_B200_API int mstar_b200_linear_gemm_push(void *handle, const void *staged, uint64_t staged_bytes, int64_t rows,
    float *const *recv_ptrs, int32_t *const *flag_ptrs, int32_t world, int32_t rank, int64_t owner_rows,
    int32_t *status, void *stream, char *error, size_t error_size);
MSTAR_B200_API int mstar_b200_tp_reduce_recv(const float *recv, int32_t *counters, int32_t world, int64_t owned,
    int64_t owner_rows, int64_t width, const float *bias, float *x, const float *ln_weight, const float *ln_bias,
    float ln_eps, void *const *staged_ptrs, void *mc_staged, int64_t row0, int32_t rounding, int32_t *status,
    void *stream, char *error, size_t error_size);

/* --- thinker tensor / expert parallelism over peer memory (the thinker layer,
 * implementations/qwen3_omni/amd/thinker_model.py:106-148, with attention
 * column-parallel by heads and the experts spread over the ranks) ---
 * Every rank holds the bf16 residual stream x [T][width] in a peer-visible
 * buffer; x_ptrs / part_ptrs / y_ptrs / inv_ptrs are device arrays of `world`
 * device pointers (peer mappings, e.g. symmetric memory; not checked on the
 * host), rows 16-byte aligned. An owner handles rows row0 .. row0 + owned.
 * thinker_reduce: the row-parallel o_proj reduction: s = sum over ranks p (in
 * rank order, fp32) of part_ptrs[p][row], then x[row] = bf16(x[row] + bf16(s))
 * (torch's bf16 residual add), the new row stored into every rank's x.
 * thinker_combine: the expert-parallel combine (moe_sum_reduce,
 * thinker_moe.py:75-81): for each owned token t, slot s with id = topk_ids[t *
 * top_k + s] in [0, experts_total), rank p = id / experts_per_rank holds the
 * routed row y_ptrs[p][inv_ptrs[p][t * top_k + s]]; the slots are summed in slot
 * order in fp32, rounded to bf16 and added to x[t] as above, the new row stored
 * into every rank's x. A row index at or above y_rows adds nothing and sets
 * status bit value 64. */
MSTAR_B200_API int mstar_b200_thinker_reduce(const float *const *part_ptrs, void *const *x_ptrs, int32_t rank,
    int32_t world, int64_t owned, int64_t width, int64_t row0, void *stream, char *error, size_t error_size);
MSTAR_B200_API int mstar_b200_thinker_combine(const void *const *y_ptrs, const int32_t *const *inv_ptrs,
    int64_t y_rows, const int32_t *topk_ids, int32_t experts_per_rank, int32_t experts_total, int32_t top_k,
    void *const *x_ptrs, int32_t rank, int32_t world, int64_t owned, int64_t hidden, int64_t row0,
    int32_t *status, void *stream, char *error, size_t error_size);

/* --- exact Q8_0 GEMM (ggml_vec_dot_q8_0_q8_0 generic order, ggml-cpu/quants.c:451-480, at
 * prefill row counts; the tcgen05 int8 tensor pipe computes each block's integer dot) ---
 * q8_exact_weights: canonical Q8_0 blocks [rows][width/32] -> int8 quants [rows][width]
 * (weights_i8, rows * width bytes, 16-byte aligned) and fp32 scales [width/32][pad]
 * (scales, pad = q8_exact_pad(rows), rows beyond `rows` zero).
 * q8_exact_activations: fp32 rows [rows][x_stride] -> their Q8_0 quantization (rounding
 * as MSTAR_B200_Q8_*) as int8 quants [rows][width] and fp32 scales [rows][width/32]
 * (each d rounded through fp16, as the block stores it); status bit 1: a nonfinite input.
 * gemm_q8_exact: out[r][n] = sum over blocks b, in order, of float(sumi) * (d_w * d_x)
 * (+ bias[n] after the sum), fp32 [rows][out_stride]; bit-identical to the decode GEMV
 * and to ggml's generic order for every row count. status bit 2: a bounded pipeline
 * wait timed out. Stream-ordered; operands from the two calls above. */
MSTAR_B200_API int64_t mstar_b200_q8_exact_pad(int64_t rows);
MSTAR_B200_API int mstar_b200_q8_exact_weights(const void *blocks, uint64_t bytes, int64_t rows, int64_t width,
    void *weights_i8, float *scales, void *stream, char *error, size_t error_size);
MSTAR_B200_API int mstar_b200_q8_exact_activations(const float *x, int64_t x_stride, int64_t rows, int64_t width,
    int32_t rounding, void *x_i8, float *scales, int32_t *status, void *stream, char *error, size_t error_size);
MSTAR_B200_API int mstar_b200_gemm_q8_exact(const void *x_i8, const float *x_scales, int64_t rows, const void *w_i8,
    const float *w_scales, int64_t out_features, int64_t width, const float *bias, float *out, int64_t out_stride,
    int32_t *status, void *stream, char *error, size_t error_size);

/* --- thinker layer norms (transformers' Qwen3OmniMoeThinkerTextRMSNorm, the input and
 * post-attention norms of the reference's thinker layer, implementations/qwen3_omni/amd/
 * thinker_model.py:106-148) ---
 * rms_norm: for every row of `width` bf16 values (8..4096, a multiple of 8): h = fp32(x),
 * r = rsqrtf(sum(h^2) / width + eps), out = bf16(fp32(weight) * fp32(bf16(h * r))) (bf16
 * [rows][out_stride]); when out_f32 is given the same values are also written as fp32.
 * The sum of squares is a per-lane fp32 sum and a warp butterfly (torch reduces in
 * another order: the mean can differ in the last bit). Operands 16-byte aligned,
 * strides in elements. */
MSTAR_B200_API int mstar_b200_rms_norm(const void *x, int64_t x_stride, int64_t rows, int64_t width,
    const void *weight, float eps, void *out, int64_t out_stride, float *out_f32, int64_t out_f32_stride,
    void *stream, char *error, size_t error_size);
/* residual_add_bf16: out = bf16(fp32(x) + fp32(bf16(v))) for n elements (a multiple of 8):
 * the layer's bf16 residual add of a projection computed in fp32 and rounded to bf16
 * (x + o_proj(att), thinker_model.py:106-148). x, out bf16, v fp32, 16-byte aligned; out
 * may be x. */
MSTAR_B200_API int mstar_b200_residual_add_bf16(const void *x, const float *v, int64_t n, void *out, void *stream,
    char *error, size_t error_size);

/* --- thinker attention prologue (implementations/qwen3_omni/amd/qknorm_rope.py:9-53, the
 * fused QK RMSNorm + prepared MRoPE op; KV write as cp_kernels.py:16-58) ---
 * qknorm_rope: for every token t and head of 128 bf16 values: x = q or k head row,
 * n = bf16((x * (1 / sqrt(sum(x^2) / 128 + eps))) * w) with w the q / k norm weight,
 * y = bf16(bf16(n * cos[t]) + bf16(rotate_half(n) * sin[t])) (products rounded to bf16
 * when round_products, else summed in fp32). q heads are written to out_q [tokens,
 * q_heads, 128]; k heads to k_cache row slots[t] (or t without a slot table), and v
 * heads, when v is given, copied unchanged to v_cache at the same row; a row is
 * cache_slot_stride elements holding kv_heads x 128. A slot outside [0, num_slots)
 * skips the token's k / v and sets status bit value 1. All tensors bf16 on the device;
 * strides in elements; head_dim must be 128. */
MSTAR_B200_API int mstar_b200_qknorm_rope(const void *q, int64_t q_s0, int64_t q_s1, const void *k, int64_t k_s0,
    int64_t k_s1, const void *v, int64_t v_s0, int64_t v_s1, const void *q_weight, const void *k_weight,
    const void *cos, int64_t cos_s0, const void *sin, int64_t sin_s0, int64_t tokens, int32_t q_heads,
    int32_t kv_heads, int32_t head_dim, float eps, int32_t round_products, void *out_q, void *k_cache,
    void *v_cache, int64_t cache_slot_stride, const int64_t *slots, int64_t num_slots, int32_t *status, void *stream,
    char *error, size_t error_size);
/* qknorm_rope_f32: the same op on fp32 q / k / v rows (the QKV projection's fp32 output,
 * 16-byte aligned), each value rounded to bf16 to nearest even as it is read: the result
 * of qknorm_rope on the .to(bfloat16) of those rows (thinker_model.py:106-148), without
 * writing that bf16 copy. Strides in fp32 elements; everything else as qknorm_rope. */
MSTAR_B200_API int mstar_b200_qknorm_rope_f32(const void *q, int64_t q_s0, int64_t q_s1, const void *k, int64_t k_s0,
    int64_t k_s1, const void *v, int64_t v_s0, int64_t v_s1, const void *q_weight, const void *k_weight,
    const void *cos, int64_t cos_s0, const void *sin, int64_t sin_s0, int64_t tokens, int32_t q_heads,
    int32_t kv_heads, int32_t head_dim, float eps, int32_t round_products, void *out_q, void *k_cache,
    void *v_cache, int64_t cache_slot_stride, const int64_t *slots, int64_t num_slots, int32_t *status, void *stream,
    char *error, size_t error_size);

/* --- categorical sampling of readout logits (backends/pi/docs/categorical.md, the
 * Graph.categorical operation; scalar oracle backends/pi/torch/tests/categorical_reference.py) ---
 * philox4x32-10-gumbel23-v1: for row r and vocabulary entry j, Philox4x32-10 with
 * key (seeds[r] lo, hi) and counter (offsets[r] lo, hi, j, 0) gives u = ((word0 >> 9)
 * + 0.5) * 2^-23, and tokens[r] is the lowest j maximizing centered_j / T - log(-log(u_j))
 * (centered_j = 0 at the row maximum, else (logit_j - max) / T, each step an fp32
 * rounding); -1 for a row with a NaN, nothing above -inf, or a temperature that is not
 * positive and finite; +inf logits restrict the draw to themselves. Seeds and offsets
 * are read as full 64-bit words and never written. logits: [rows][ld] fp32 device rows
 * (vocab <= INT32_MAX entries used of each); workspace: categorical_workspace(rows)
 * bytes of device memory (16-byte aligned), overwritten. Stream-ordered. */
MSTAR_B200_API uint64_t mstar_b200_categorical_workspace(int64_t rows);
MSTAR_B200_API int mstar_b200_categorical(const float *logits, int64_t rows, int64_t vocab, int64_t ld,
    const int64_t *seeds, const int64_t *offsets, const float *temperatures, int64_t *tokens, void *workspace,
    uint64_t workspace_bytes, void *stream, char *error, size_t error_size);

/* --- bounded device waits (no reference counterpart: the reference's native
 * backends run on the CPU and never wait on a device flag) ---
 * Every spin or mbarrier wait in this library gives up after a bounded number of
 * polls and reports it in the call's status word instead of hanging the GPU:
 * bit value 2 for an mbarrier of a TMA / MMA pipeline, 16 for tp_barrier, 32 for
 * the persistent decode step's grid barrier.
 * set_wait_limits: process-wide poll limits for tp_barrier (polls of ~100 ns;
 * default 2^26, about 7 s) and for the decode step's grid barrier (polls of
 * ~64 ns; default 2^24, about 1 s; read when a decode-step handle is created);
 * 0 restores a default. Kernels launched afterwards use them.
 * wait_selftest: makes one wait run out on purpose, on the calling stream, with
 * `limit` polls: MSTAR_B200_WAIT_MBARRIER waits on an mbarrier nothing arrives at
 * (status |= 2); MSTAR_B200_WAIT_GRID_BARRIER runs the grid barrier in a grid of
 * two CTAs one of which never arrives (status |= 32; words: 2 device uint32 the
 * call zeroes first). The context stays usable afterwards. */
#define MSTAR_B200_WAIT_MBARRIER 0
#define MSTAR_B200_WAIT_GRID_BARRIER 1
MSTAR_B200_API int mstar_b200_set_wait_limits(int64_t tp_barrier_polls, int64_t grid_barrier_polls, char *error,
    size_t error_size);
MSTAR_B200_API int mstar_b200_wait_selftest(int32_t kind, int64_t limit, uint32_t *words, int32_t *status,
    void *stream, char *error, size_t error_size);

/* --- the whole decoder step as one persistent kernel ------------------------------
 * One greedy decode step of the Whisper decoder graph (decoder.cpp:489-600,
 * 683-696) for `batch` sequences (one new token each) as a single cooperative
 * launch: embedding, every layer (LayerNorm + Q8_0 activations, fused QKV,
 * causal self attention appending K/V at positions[b], out projection +
 * residual, LayerNorm, cross query, cross attention over the cross planes,
 * out projection + residual, LayerNorm, fc1 + GELU, fc2 + residual), final
 * LayerNorm, the readout with suppression and the argmax into next_token.
 * The arithmetic is that of mstar_b200_linear_run / _readout and
 * mstar_b200_attend on the same handles and planes, so logits and tokens are
 * identical to the multi-launch step. Handles: linears[i] = {QKV [3w x w],
 * out [w x w], cross query [w x w], cross out [w x w], fc1 [ffn x w], fc2 [w x ffn]}
 * (Q8_0), head = the readout ([vocab x w], Q4_0 or Q8_0); norms[i] = {ln1 w, b,
 * ln2 w, b, ln3 w, b}. Every pointer is borrowed and must outlive the step
 * handle (close the step before its linear handles); the buffers are fixed at
 * create, so a captured graph replays the step. Bounded barrier waits set
 * status bit value 32. */
typedef struct mstar_b200_decode_step_config {
    int32_t batch, layers, width, heads, ffn, target, source, shared_cross, rounding;
    float eps;
    const float *token_table, *position_table;
    int64_t vocab, positions_count;
    void *linears[8][6];
    const float *norms[8][6];
    void *self_k[8], *self_v[8], *cross_k[8], *cross_v[8];
    void *head;
    const float *final_norm_weight, *final_norm_bias;
    const int64_t *suppressed;
    uint64_t suppressed_count;
    const int64_t *tokens, *positions, *cross_length;
    float *logits;        /* [batch][vocab] or NULL */
    int64_t *next_token;  /* [batch] */
    int32_t *status;
} mstar_b200_decode_step_config;
MSTAR_B200_API void *mstar_b200_decode_step_create(const mstar_b200_decode_step_config *config, char *error,
    size_t error_size);
MSTAR_B200_API int mstar_b200_decode_step_run(void *step, void *stream, char *error, size_t error_size);
MSTAR_B200_API int mstar_b200_decode_step_close(void *step, char *error, size_t error_size);

/* --- readout that allocates nothing ------------------------------------------------
 * No counterpart in the reference. For callers that cannot allocate device
 * memory (a runtime that owns every device buffer and hands out only planned
 * ones, or a latency-bound caller that must not pay for cudaMalloc and the
 * synchronisation it can bring): the q8cpu_readout contract over the caller's
 * canonical ggml Q8_0 bytes (device, 2-byte aligned) with one fp32 query x[k]
 * (16-byte aligned): logits[rows] (suppressed rows -inf), token (first index,
 * first NaN wins), status[0] = 1 if x is nonfinite. Bit-identical to
 * mstar_b200_q8_readout on a handle created from the same bytes.
 * Scratch lives in one fixed device array (about 81 KB per device, held until
 * the process exits) shared by every call: calls that overlap on the GPU race.
 * Limit k <= 4096: a wider k returns E2BIG; other bad arguments EINVAL.
 * The first call on a device resolves the array's address (cudaGetSymbolAddress,
 * that device current); make it before capturing any stream. */
MSTAR_B200_API int mstar_b200_q8_readout_noalloc(const void *blocks, size_t bytes, int64_t rows, int64_t k,
    const float *x, float *logits, int64_t *token, int32_t *status, const int64_t *suppressed,
    size_t suppressed_count, void *stream);

/* --- decoder-step glue around the linears (not block-quantized) ----------------
 * Token + position embedding: x[r] = token_table[ids[r]]*scale +
 * position_table[positions[r]] (ggml_get_rows + ggml_add, decoder.cpp:513-518;
 * cpu_decoder_set_token_inputs, decoder_tokens.h:15-24). Out-of-range ids or
 * positions zero the row and set status bit 2 (value 4). */
MSTAR_B200_API int mstar_b200_embed(const float *token_table, int64_t vocab, const float *position_table,
    int64_t positions_count, int64_t width, const int64_t *ids, const int64_t *positions, int64_t rows,
    float scale, float *x, int32_t *status, void *stream, char *error, size_t error_size);
/* Multi-head attention over fp16 K/V planes [seq][capacity][heads*64]
 * (ggml_flash_attn_ext, scale 1/sqrt(64), decoder.cpp:504-511). When k_new/v_new
 * are given (causal, per-sequence planes), the `queries` new rows of each
 * sequence are first written at positions begin[b].. (ggml_set_rows,
 * decoder.cpp:566-567) and attention is causal up to each query's own
 * position; otherwise every query sees kv_length[b] keys. shared=1: every
 * sequence reads plane 0 (one encoder state for the whole batch), and all
 * batch*queries rows (at most 128) are attended together against each K/V tile,
 * with the keys split across CTAs (flash-decoding) whose partial results are
 * kept in `workspace` and merged by a second kernel. workspace: device,
 * 256-byte aligned, exactly mstar_b200_attend_workspace() bytes for the same
 * geometry; calls sharing a workspace must be stream-ordered.
 * Bad positions/lengths set status bit 3 (value 8) and zero those rows. */
MSTAR_B200_API uint64_t mstar_b200_attend_workspace(int32_t heads, int32_t batch, int32_t queries,
    int64_t capacity, int32_t shared);
MSTAR_B200_API int mstar_b200_attend(const float *q, int64_t q_stride, const float *k_new, const float *v_new,
    int64_t kv_stride, void *k_plane, void *v_plane, int64_t capacity, int32_t heads, int32_t head_dim,
    int32_t batch, int32_t queries, const int64_t *begin, const int64_t *kv_length, int32_t causal,
    int32_t shared, float *out, int64_t out_stride, float scale, int32_t *status, void *workspace,
    uint64_t workspace_bytes, void *stream, char *error, size_t error_size);
/* mstar_b200_attend that also writes the output rows (batch * queries <= 32)
 * as the Q8_0 activation fragments of the linear that consumes them (out_proj
 * after the attention, decoder.cpp:566-580): the quantization equals the one
 * mstar_b200_linear_run performs on `out`, so mstar_b200_linear_run_frags on
 * that handle gives the same bytes as mstar_b200_linear_run(out). frags comes
 * from mstar_b200_linear_frags; NULL makes this mstar_b200_attend. */
MSTAR_B200_API int mstar_b200_attend_q8(const float *q, int64_t q_stride, const float *k_new, const float *v_new,
    int64_t kv_stride, void *k_plane, void *v_plane, int64_t capacity, int32_t heads, int32_t head_dim,
    int32_t batch, int32_t queries, const int64_t *begin, const int64_t *kv_length, int32_t causal,
    int32_t shared, float *out, int64_t out_stride, float scale, int32_t *status, void *workspace,
    uint64_t workspace_bytes, const mstar_b200_q8_frags *frags, void *stream, char *error, size_t error_size);
/* Cross K/V planes from the fused projection of the encoder states
 * (decoder.cpp:247-250, 322-330: one [3072 x 384] Q8_0 matrix for the four
 * layers' k/v; biases added, then stored fp16 like cross_bias_set_rows). */
MSTAR_B200_API int mstar_b200_fill_kv(const float *projected, int64_t stride, int64_t k_offset,
    int64_t v_offset, const float *k_bias, const float *v_bias, void *k_plane, void *v_plane, int64_t rows,
    int64_t width, void *stream, char *error, size_t error_size);

#ifdef __cplusplus
}
#endif
