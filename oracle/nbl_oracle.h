/* CPU oracle for the attention path: plain-C restatement of nibble's scalar attention, RoPE, softmax and
 * fp16 conversion.
 *
 * TEST INFRASTRUCTURE ONLY. The product library (libnibble_cuda.so) never links, loads or calls this code;
 * only tests/, the smoke check and bench.py's CPU-baseline leg use it, as the checker.
 *
 * Every function names the reference function it restates (paths inside the nibble source tree). The
 * restatement keeps the reference's operation order and types so that, built with -ffp-contract=off like
 * the reference's ref_ops.cpp (CMakeLists.txt:72-73), it is bit-identical to it; tests/test_oracle.py checks
 * that against the compiled reference (oracle/_ref) and against the reference's own known-answer cases.
 */
#ifndef NBL_ORACLE_H
#define NBL_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* IEEE binary16 <-> binary32, exact widening and round-to-nearest-even narrowing (src/fp16.h:18, :46). */
float orc_fp16_to_fp32(uint16_t h);
uint16_t orc_fp32_to_fp16(float f);
/* bfloat16 <-> binary32 (not in the reference; used to round the bf16 prefill inputs the same way the GPU
 * sees them). Narrowing is round-to-nearest-even; NaN stays NaN. */
float orc_bf16_to_fp32(uint16_t h);
uint16_t orc_fp32_to_bf16(float f);
void orc_fp16_to_fp32_n(const uint16_t* src, float* dst, int64_t n);
void orc_fp32_to_fp16_n(const float* src, uint16_t* dst, int64_t n);
void orc_bf16_to_fp32_n(const uint16_t* src, float* dst, int64_t n);
void orc_fp32_to_bf16_n(const float* src, uint16_t* dst, int64_t n);

/* Max-subtracted softmax in place with a double-precision sum (src/backend/cpu/ref_ops.cpp:66-77). */
void orc_softmax_inplace(float* x, int64_t n);

/* Rotary embedding in place on x[n, n_heads, head_dim] at positions pos0.. (src/backend/cpu/ref_ops.cpp:166-185;
 * RopeParams src/backend/backend.h:16-20). Angles pos * base^(-2i/head_dim) / freq_factors[i] in double. */
void orc_rope(float* x, int64_t n, int64_t n_heads, int64_t head_dim, int64_t pos0, float freq_base, int neox,
              const float* freq_factors);

/* Causal GQA attention for heads [head_begin, head_end) (src/backend/cpu/ref_ops.cpp:188-214). q,out
 * [n, n_heads, head_dim]; k,v [ctx, n_kv_heads, head_dim]; row t attends keys 0..pos0+t. scratch holds at
 * least pos0+n floats. */
void orc_attention_heads(const float* q, const float* k, const float* v, float* out, int64_t n, int64_t pos0,
                         int64_t n_heads, int64_t n_kv_heads, int64_t head_dim, int64_t head_begin, int64_t head_end,
                         float* scratch);
/* All heads, scratch allocated internally (the shape CpuBackend::attention exposes,
 * src/backend/cpu/cpu_backend.cpp:272-290). Returns 0, or -1 if scratch cannot be allocated. */
int orc_attention(const float* q, const float* k, const float* v, float* out, int64_t n, int64_t pos0,
                  int64_t n_heads, int64_t n_kv_heads, int64_t head_dim);

/* Broadcast bias add over n rows of width `width` (src/backend/cpu/ref_ops.cpp:156-161). */
void orc_add_bias(float* x, const float* bias, int64_t width, int64_t n);

/* Paged-cache helper (no reference counterpart: the reference cache is one flat block per layer,
 * src/model/transformer.cpp:74-90). Widens the first `len` tokens of one sequence from a paged pool laid
 * out [page][2 (K,V)][n_kv_heads][page_size][head_dim] (fp16 or bf16 bits, `bf16` selects) into contiguous
 * fp32 k,v [len, n_kv_heads, head_dim], the layout the reference attention reads. */
void orc_gather_pages(const uint16_t* pool, const int32_t* page_table, int64_t len, int64_t n_kv_heads,
                      int64_t head_dim, int64_t page_size, int bf16, float* k_out, float* v_out);

/* Log-sum-exp merge of n_parts partial attention results (no reference counterpart: the reference never
 * splits a softmax). part_o [n_parts, rows, head_dim] holds each part's normalised output and part_lse
 * [n_parts, rows] its natural-log sum of exp(scores); writes the merged out [rows, head_dim] and, if
 * lse_out is non-null, the merged lse [rows]. Parts with lse = -inf contribute nothing. Double math. */
void orc_lse_merge(const float* part_o, const float* part_lse, int64_t n_parts, int64_t rows, int64_t head_dim,
                   float* out, float* lse_out);

/* The model's other ops (src/backend/backend.h:54-70). dtype: 0 = F32, 1 = F16 (IEEE binary16 bits). */
/* Embedding lookup: out[t, :] = row ids[t] of table [n_rows, ne0], widened (src/backend/cpu/ref_ops.cpp:80-98).
 * Returns 0, or -1 (nothing written past the bad row) when an id is outside [0, n_rows). */
int orc_embed(const void* table, int dtype, int64_t ne0, int64_t n_rows, const int32_t* ids, int64_t n, float* out);
/* y[t, r] = sum_k x[t, k] * w[r, k] accumulated left to right in float, w [ne1, ne0] F32 or F16
 * (src/backend/cpu/ref_ops.cpp:109-136, the float branch of matmul_rows). */
void orc_matmul(const void* w, int dtype, int64_t ne0, int64_t ne1, const float* x, float* y, int64_t n);
/* RMSNorm of n rows of width d with an F32 weight, in double (src/backend/cpu/ref_ops.cpp:138-148). */
void orc_rmsnorm(const float* x, const float* weight, float* y, int64_t n, int64_t d, float eps);
/* x[i] += y[i] (src/backend/cpu/ref_ops.cpp:151-153). */
void orc_add(float* x, const float* y, int64_t count);
/* gate[i] = g / (1 + e^-g) * up[i] in float (src/backend/cpu/ref_ops.cpp:217-222). */
void orc_silu_mul(float* gate, const float* up, int64_t count);

/* Quantized weights (src/quant.h). dtype codes are nibble's DType ids (ggml's): 2 = Q4_0, 6 = Q5_0, 7 = Q5_1,
 * 8 = Q8_0, 12 = Q4_K, 13 = Q5_K, 14 = Q6_K. Weights are the GGUF block bytes, row after row (ne0 a multiple of
 * the block: 32, or 256 for the k-quants). */
/* Activations to Q8_0 blocks (34 bytes: fp16 d, 32 int8), src/quant.cpp:37-51, :250-257: per block d = max|x| /
 * 127 (NaN if the block holds a NaN), q = roundf(x * (1/d)) clamped to [-127, 127]. n % 32 == 0. */
void orc_quantize_q8_0(const float* x, uint8_t* blocks, int64_t n);
/* As orc_quantize_q8_0 into Q8_1 blocks (36 bytes: fp16 d, fp16 s = fp16(sum(q) * d), 32 int8), src/quant.cpp:260. */
void orc_quantize_q8_1(const float* x, uint8_t* blocks, int64_t n);
/* Activations to Q8_K blocks (292 bytes: float d, 256 int8, 16 int16 sums), src/quant.cpp:276. n % 256 == 0. */
void orc_quantize_q8_K(const float* x, uint8_t* blocks, int64_t n);
/* One row of n elements of a quantized tensor to float (src/quant.cpp:158-246). Returns -1 for another dtype. */
int orc_dequantize_row(int dtype, const void* src, float* dst, int64_t n);
/* y[t, r] = dot(weight row r, Q8_0-quantized x row t): per block the integer dot and the reference's float term
 * (Q4_0: sumi * d_w * d_a; Q8_0: sumi * (d_w * d_a); Q5_0: (d_w * d_a) * sumi, src/quant.cpp:310-366), added to
 * the row's sum in block order; Q5_1 against Q8_1 activations and the k-quants against Q8_K ones in the order of
 * src/quant.cpp:117-146, :371-418. Returns -1 for an unsupported dtype. */
int orc_matmul_q(const void* w, int dtype, int64_t ne0, int64_t ne1, const float* x, float* y, int64_t n);
/* The block dot of one weight row (n_blocks blocks of dtype) with activation blocks already in the companion format
 * (Q8_0 for Q4_0/Q5_0/Q8_0, Q8_1 for Q5_1, Q8_K for the k-quants): nibble's dot_*_q8_* (src/quant.cpp:117-146,
 * :310-418). NaN for another dtype. */
float orc_vec_dot(int dtype, const void* w, const void* act, int64_t n_blocks);

#ifdef __cplusplus
}
#endif
#endif
