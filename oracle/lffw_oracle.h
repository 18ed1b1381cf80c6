/*
 * CPU oracle for the FP8 E4M3 quantized-linear path and the fp16 projection
 * plugins.  TEST INFRASTRUCTURE ONLY: tests/, __graft_entry__.smoke() and the
 * cpu_baseline / reference arm of bench.py use it as the checker.  The product
 * library (liblffw_b200.so) never links or calls it.
 *
 * Every routine restates the reference's arithmetic in plain C:
 *   - Q/DQ convention: cpp/src/network_graph.cpp:115-159 and
 *     python/src/listenflow/fastest_whisper/_fp8.py:20-51 (TensorRT's documented
 *     FP8 quantize = saturate(round_to_nearest_even(x / scale))).
 *   - fp16 GELU edges: cpp/src/network_graph.cpp:168-180 and :63-71 (the 2^-1/2
 *     constant is stored as half), cpp/tests/kernel_reference.hpp:20-25.
 *   - fp16 projection plugins: cpp/kernels.cu:10-78, cpp/tests/kernel_reference.hpp:36-50.
 * Halves travel as raw uint16_t bit patterns, E4M3 codes as uint8_t.
 */
#ifndef LFFW_ORACLE_H
#define LFFW_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* IEEE binary16 <-> binary64/32, round to nearest even, overflow to inf. */
double oracle_half_to_double(uint16_t h);
uint16_t oracle_half_from_double(double v);
uint16_t oracle_half_from_float(float v);

/* E4M3 (OCP "e4m3fn": no infinities, S.1111.111 = NaN, max finite 448).
 * Round to nearest even, saturate finite overflow and infinities to +-448,
 * NaN -> S.1111.111, signed zero kept. */
uint8_t oracle_e4m3_from_float(float v);
float oracle_e4m3_to_float(uint8_t code);

/* Array forms of the conversions above. */
void oracle_e4m3_from_floats(const float *v, size_t count, uint8_t *codes);
void oracle_e4m3_to_floats(const uint8_t *codes, size_t count, float *v);
void oracle_halves_from_doubles(const double *v, size_t count, uint16_t *h);
void oracle_gelu_fp16_array(const uint16_t *x, size_t count, uint16_t *y);

/* Q of one fp16 operand with a scalar scale: code = e4m3(fp32(x / scale)). */
void oracle_quantize(const uint16_t *x, size_t count, float scale, uint8_t *codes);
/* Q of a [rows, cols] fp16 matrix with one scale per row (weights; axis = output channel). */
void oracle_quantize_rows(const uint16_t *x, int64_t rows, int64_t cols, const float *scales,
                          uint8_t *codes);
/* max |x| over fp16 values (NaN ignored), returned as float. */
float oracle_amax(const uint16_t *x, size_t count);
/* Per-output-channel weight scale: max|W[n,:]| / 448 in fp32, non-positive -> 1. */
void oracle_weight_scales(const uint16_t *w, int64_t rows, int64_t cols, float *scales);

/* The FP8 Q/DQ linear with fused epilogue:
 *   acc[m,n] = sum_k e4m3(xq[m,k]) * e4m3(wq[n,k])       (exact, float64)
 *   y16      = half(acc * act_scale * w_scale[n])        (matmul output edge)
 *   y16      = half(y16 + bias[n])                        (if bias)
 *   y16      = gelu_fp16_edges(y16)                       (if gelu)
 *   y[m,n]   = y16                                         (if y)
 *   codes    = e4m3(fp32(y16 / next_scale))                (if next_codes)
 * Rows are processed with up to `threads` host threads (<=0: all cores). */
void oracle_fp8_linear(const uint8_t *xq, const uint8_t *wq, int64_t m, int64_t n, int64_t k,
                       float act_scale, const float *w_scale, const uint16_t *bias, int gelu,
                       uint16_t *y, float next_scale, uint8_t *next_codes, int threads);

/* LayerNorm producer (cpp/src/network_graph.cpp:160-166 with the residual add
 * of :285-287): per row of cols fp16 values,
 *   s[i]  = half(x[i] + residual[i])          (fp16 add; s = x when residual is NULL)
 *   mean  = sum(s) / cols, var = sum((s - mean)^2) / cols        (binary64)
 *   y[i]  = half((s[i] - mean) / sqrt(var + eps) * gamma[i] + beta[i])
 *   codes = e4m3(fp32(y[i] / code_scale))      (if codes)
 * TensorRT's normalization runs in fp32 in an unspecified order; this is the
 * exactly rounded value that such an evaluation approximates. */
void oracle_layer_norm(const uint16_t *x, const uint16_t *residual, int64_t rows, int64_t cols,
                       const float *gamma, const float *beta, float eps, uint16_t *sum_out, uint16_t *y,
                       float code_scale, uint8_t *codes);

/* Decoder cross-attention over a cached encoder K/V (cpp/src/network_graph.cpp:235-244
 * `attend`, with the cross-K/V cache of :401-404), per stream s, head h and query row t:
 *   c        = half(head_dim^-0.25)
 *   q'[d]    = half(q[s,t][h*dim + d] * c),  k'[j][d] = half(k[s][h][j][d] * c)
 *   score[j] = half(sum_d q'[d] k'[j][d])                  (fp16 MatMul output, exact sum)
 *   p[j]     = half(exp(score[j] - max) / sum_i exp(score[i] - max))   (fp32 softmax -> half)
 *   out[s,t][h*dim + d] = half(sum_j p[j] v[s][h][j][d])   (fp16 MatMul output, exact sum)
 *   codes    = e4m3(fp32(out / code_scale))                 (if codes)
 * q / out: fp16 [streams * queries, heads * dim] (row s * queries + t); k, v: fp16
 * [streams, heads, keys, dim].  The softmax is evaluated in binary64 and rounded once:
 * the value TensorRT's fp32 softmax approximates. */
void oracle_cross_attention(const uint16_t *q, const uint16_t *k, const uint16_t *v, int streams, int queries,
                            int heads, int dim, int keys, uint16_t *out, float code_scale, uint8_t *codes);

/* Encoder self-attention (cpp/src/network_graph.cpp:235-247 `attention`: `attend` on
 * the layer's own q/k/v projections, no mask), per stream s, head h, query row i:
 * the same fp16 edges as oracle_cross_attention over the stream's `tokens` keys.
 * q, k, v rows: row s * tokens + t, column h * dim + d, row strides q_ld, k_ld, v_ld
 * (elements; e.g. the fused QKV output with q, k, v at column offsets 0, width,
 * 2 * width and stride 3 * width).  out: [streams * tokens, heads * dim]. */
void oracle_self_attention(const uint16_t *q, const uint16_t *k, const uint16_t *v, int64_t q_ld, int64_t k_ld,
                           int64_t v_ld, int streams, int tokens, int heads, int dim, uint16_t *out,
                           float code_scale, uint8_t *codes);

/* fp16(erf(x)) of an fp16 x, erf in binary64, round to nearest even. */
uint16_t oracle_erf_fp16(uint16_t x);
/* GELU on an fp16 value with every graph edge rounded to fp16. */
uint16_t oracle_gelu_fp16(uint16_t x);

/* fp16 projection plugins (single token). */
void oracle_fp16_fc1(const uint16_t *x, const uint16_t *w, const uint16_t *bias, uint16_t *y,
                     int64_t rows, int64_t width);
void oracle_fp16_qkv(const uint16_t *x, const uint16_t *w, const uint16_t *q_bias,
                     const uint16_t *v_bias, uint16_t *y, int64_t width);
/* The same projections with the reference kernel's fp32 summation order
 * (cpp/kernels.cu:27-49) instead of the CPU model's binary64 dot; 0 on success. */
int oracle_fp16_fc1_kernel_order(const uint16_t *x, const uint16_t *w, const uint16_t *bias, uint16_t *y,
                                 int64_t rows, int64_t width);
int oracle_fp16_qkv_kernel_order(const uint16_t *x, const uint16_t *w, const uint16_t *q_bias,
                                 const uint16_t *v_bias, uint16_t *y, int64_t width);
void oracle_fp16_bias(const uint16_t *x, uint16_t bias, uint16_t *y, int64_t count);

int oracle_threads(void);

#ifdef __cplusplus
}
#endif
#endif
