/*
 * CPU oracle (test infrastructure only; see lffw_oracle.h).  Plain C99 +
 * pthreads, IEEE arithmetic only: build without -ffast-math so that float
 * division and double sums round exactly as written.
 */
#include "lffw_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

double oracle_half_to_double(uint16_t h)
{
    int sign = h >> 15, exponent = (h >> 10) & 31, fraction = h & 1023;
    double magnitude;
    if (exponent == 31)
        magnitude = fraction ? NAN : INFINITY;
    else if (exponent == 0)
        magnitude = ldexp((double)fraction, -24);
    else
        magnitude = ldexp((double)(fraction | 1024), exponent - 25);
    return sign ? -magnitude : magnitude;
}

uint16_t oracle_half_from_double(double v)
{
    uint16_t sign = signbit(v) ? 0x8000 : 0;
    if (isnan(v))
        return sign | 0x7e00;
    double a = fabs(v);
    /* 65520 is the midpoint between 65504 (odd significand) and 2^16: ties go up. */
    if (a >= 65520.0)
        return sign | 0x7c00;
    if (a < 0x1p-14) /* subnormal quantum 2^-24; 1024 quanta is the smallest normal */
        return sign | (uint16_t)nearbyint(a * 0x1p24);
    int e;
    frexp(a, &e); /* a = f * 2^e, f in [0.5, 1) */
    int exponent = e - 1;
    double r = nearbyint(ldexp(a, 10 - exponent)); /* in [1024, 2048] */
    if (r == 2048.0) {
        r = 1024.0;
        ++exponent;
    }
    return sign | (uint16_t)((exponent + 15) << 10) | (uint16_t)((int)r - 1024);
}

uint16_t oracle_half_from_float(float v) { return oracle_half_from_double((double)v); }

uint8_t oracle_e4m3_from_float(float v)
{
    uint8_t sign = signbit(v) ? 0x80 : 0;
    if (isnan(v))
        return sign | 0x7f;
    float a = fabsf(v);
    /* Every finite value at or above 448 rounds to 448 or overflows; satfinite
     * clamps both (and infinities) to the largest finite code. */
    if (a >= 448.0f)
        return sign | 0x7e;
    if (a < 0x1p-6f) /* subnormal quantum 2^-9; 8 quanta is the smallest normal */
        return sign | (uint8_t)nearbyintf(a * 0x1p9f);
    int e;
    frexpf(a, &e);
    int exponent = e - 1; /* a in [2^exponent, 2^(exponent+1)), exponent in [-6, 8] */
    float r = nearbyintf(ldexpf(a, 3 - exponent)); /* in [8, 16] */
    if (r == 16.0f) {
        r = 8.0f;
        ++exponent;
    }
    return sign | (uint8_t)((exponent + 7) << 3) | (uint8_t)((int)r - 8);
}

float oracle_e4m3_to_float(uint8_t code)
{
    int sign = code >> 7, exponent = (code >> 3) & 15, mantissa = code & 7;
    float magnitude;
    if (exponent == 15 && mantissa == 7)
        magnitude = NAN;
    else if (exponent == 0)
        magnitude = ldexpf((float)mantissa, -9);
    else
        magnitude = ldexpf((float)(mantissa | 8), exponent - 10);
    return sign ? -magnitude : magnitude;
}

void oracle_e4m3_from_floats(const float *v, size_t count, uint8_t *codes)
{
    for (size_t i = 0; i < count; ++i)
        codes[i] = oracle_e4m3_from_float(v[i]);
}

void oracle_e4m3_to_floats(const uint8_t *codes, size_t count, float *v)
{
    for (size_t i = 0; i < count; ++i)
        v[i] = oracle_e4m3_to_float(codes[i]);
}

void oracle_halves_from_doubles(const double *v, size_t count, uint16_t *h)
{
    for (size_t i = 0; i < count; ++i)
        h[i] = oracle_half_from_double(v[i]);
}

void oracle_gelu_fp16_array(const uint16_t *x, size_t count, uint16_t *y)
{
    for (size_t i = 0; i < count; ++i)
        y[i] = oracle_gelu_fp16(x[i]);
}

static inline float half_to_float(uint16_t h) { return (float)oracle_half_to_double(h); }

static inline uint8_t quantize_one(uint16_t x, float scale)
{
    /* TensorRT Q on a half tensor with an fp32 scale: fp32 quotient, then
     * round-to-nearest-even into E4M3 with saturation. */
    float q = half_to_float(x) / scale;
    return oracle_e4m3_from_float(q);
}

void oracle_quantize(const uint16_t *x, size_t count, float scale, uint8_t *codes)
{
    for (size_t i = 0; i < count; ++i)
        codes[i] = quantize_one(x[i], scale);
}

void oracle_layer_norm(const uint16_t *x, const uint16_t *residual, int64_t rows, int64_t cols,
                       const float *gamma, const float *beta, float eps, uint16_t *sum_out, uint16_t *y,
                       float code_scale, uint8_t *codes)
{
    double *s = (double *)malloc((size_t)cols * sizeof(double));
    if (!s)
        return;
    for (int64_t r = 0; r < rows; ++r) {
        const uint16_t *xr = x + r * cols;
        double mean = 0.0, var = 0.0;
        for (int64_t c = 0; c < cols; ++c) {
            uint16_t h = xr[c];
            if (residual) /* fp16 add: exact sum in binary64, one rounding to fp16 */
                h = oracle_half_from_double(oracle_half_to_double(h) + oracle_half_to_double(residual[r * cols + c]));
            if (sum_out)
                sum_out[r * cols + c] = h;
            s[c] = oracle_half_to_double(h);
            mean += s[c];
        }
        mean /= (double)cols;
        for (int64_t c = 0; c < cols; ++c)
            var += (s[c] - mean) * (s[c] - mean);
        var /= (double)cols;
        const double inv = 1.0 / sqrt(var + (double)eps);
        for (int64_t c = 0; c < cols; ++c) {
            const uint16_t out = oracle_half_from_double((s[c] - mean) * inv * (double)gamma[c] + (double)beta[c]);
            if (y)
                y[r * cols + c] = out;
            if (codes)
                codes[r * cols + c] = quantize_one(out, code_scale);
        }
    }
    free(s);
}

void oracle_cross_attention(const uint16_t *q, const uint16_t *k, const uint16_t *v, int streams, int queries,
                            int heads, int dim, int keys, uint16_t *out, float code_scale, uint8_t *codes)
{
    const uint16_t c = oracle_half_from_float((float)pow((double)dim, -0.25));
    const double cd = oracle_half_to_double(c);
    const int width = heads * dim;
    double *qs = (double *)malloc((size_t)dim * sizeof(double));
    double *score = (double *)malloc((size_t)keys * sizeof(double));
    if (!qs || !score) {
        free(qs);
        free(score);
        return;
    }
    for (int s = 0; s < streams; ++s)
        for (int h = 0; h < heads; ++h) {
            const uint16_t *kh = k + ((size_t)s * heads + h) * (size_t)keys * dim;
            const uint16_t *vh = v + ((size_t)s * heads + h) * (size_t)keys * dim;
            for (int t = 0; t < queries; ++t) {
                const size_t row = (size_t)s * queries + t;
                for (int d = 0; d < dim; ++d)
                    qs[d] = oracle_half_to_double(
                        oracle_half_from_double(oracle_half_to_double(q[row * width + h * dim + d]) * cd));
                double best = -INFINITY;
                for (int j = 0; j < keys; ++j) {
                    double acc = 0.0; /* products of halves are exact in binary64; the sum rounds little */
                    for (int d = 0; d < dim; ++d)
                        acc += qs[d] * oracle_half_to_double(
                                           oracle_half_from_double(oracle_half_to_double(kh[(size_t)j * dim + d]) * cd));
                    score[j] = oracle_half_to_double(oracle_half_from_double(acc));
                    if (score[j] > best)
                        best = score[j];
                }
                double total = 0.0;
                for (int j = 0; j < keys; ++j) {
                    score[j] = exp(score[j] - best);
                    total += score[j];
                }
                for (int j = 0; j < keys; ++j)
                    score[j] = oracle_half_to_double(oracle_half_from_double(score[j] / total));
                for (int d = 0; d < dim; ++d) {
                    double acc = 0.0;
                    for (int j = 0; j < keys; ++j)
                        acc += score[j] * oracle_half_to_double(vh[(size_t)j * dim + d]);
                    const uint16_t o = oracle_half_from_double(acc);
                    out[row * width + h * dim + d] = o;
                    if (codes)
                        codes[row * width + h * dim + d] = quantize_one(o, code_scale);
                }
            }
        }
    free(qs);
    free(score);
}

struct self_attention_job {
    const uint16_t *q, *k, *v;
    int64_t q_ld, k_ld, v_ld;
    int streams, tokens, heads, dim;
    uint16_t *out;
    float code_scale;
    uint8_t *codes;
    int first, step; /* (stream, head) pairs first, first + step, ... */
};

static void *self_attention_pairs(void *arg)
{
    const struct self_attention_job *j = (const struct self_attention_job *)arg;
    const int dim = j->dim, T = j->tokens, width = j->heads * dim;
    const double c = oracle_half_to_double(oracle_half_from_float((float)pow((double)dim, -0.25)));
    double *ks = (double *)malloc((size_t)T * dim * sizeof(double));
    double *qs = (double *)malloc((size_t)dim * sizeof(double));
    double *score = (double *)malloc((size_t)T * sizeof(double));
    if (!ks || !qs || !score)
        goto done;
    for (int pair = j->first; pair < j->streams * j->heads; pair += j->step) {
        const int s = pair / j->heads, h = pair % j->heads;
        for (int t = 0; t < T; ++t)
            for (int d = 0; d < dim; ++d)
                ks[(size_t)t * dim + d] = oracle_half_to_double(oracle_half_from_double(
                    oracle_half_to_double(j->k[((size_t)s * T + t) * j->k_ld + h * dim + d]) * c));
        for (int i = 0; i < T; ++i) {
            for (int d = 0; d < dim; ++d)
                qs[d] = oracle_half_to_double(oracle_half_from_double(
                    oracle_half_to_double(j->q[((size_t)s * T + i) * j->q_ld + h * dim + d]) * c));
            double best = -INFINITY;
            for (int t = 0; t < T; ++t) {
                double acc = 0.0;
                for (int d = 0; d < dim; ++d)
                    acc += qs[d] * ks[(size_t)t * dim + d];
                score[t] = oracle_half_to_double(oracle_half_from_double(acc));
                if (score[t] > best)
                    best = score[t];
            }
            double total = 0.0;
            for (int t = 0; t < T; ++t) {
                score[t] = exp(score[t] - best);
                total += score[t];
            }
            for (int t = 0; t < T; ++t)
                score[t] = oracle_half_to_double(oracle_half_from_double(score[t] / total));
            for (int d = 0; d < dim; ++d) {
                double acc = 0.0;
                for (int t = 0; t < T; ++t)
                    acc += score[t] * oracle_half_to_double(j->v[((size_t)s * T + t) * j->v_ld + h * dim + d]);
                const uint16_t o = oracle_half_from_double(acc);
                const size_t idx = ((size_t)s * T + i) * width + h * dim + d;
                j->out[idx] = o;
                if (j->codes)
                    j->codes[idx] = quantize_one(o, j->code_scale);
            }
        }
    }
done:
    free(ks);
    free(qs);
    free(score);
    return NULL;
}

void oracle_self_attention(const uint16_t *q, const uint16_t *k, const uint16_t *v, int64_t q_ld, int64_t k_ld,
                           int64_t v_ld, int streams, int tokens, int heads, int dim, uint16_t *out,
                           float code_scale, uint8_t *codes)
{
    int threads = oracle_threads();
    if (threads > streams * heads)
        threads = streams * heads;
    if (threads < 1)
        threads = 1;
    if (threads > 256)
        threads = 256;
    struct self_attention_job jobs[256];
    pthread_t handles[256];
    for (int t = 0; t < threads; ++t) {
        jobs[t] = (struct self_attention_job){q, k, v, q_ld, k_ld, v_ld, streams, tokens, heads, dim,
                                              out, code_scale, codes, t, threads};
        if (threads == 1 || pthread_create(&handles[t], NULL, self_attention_pairs, &jobs[t]) != 0) {
            self_attention_pairs(&jobs[t]);
            handles[t] = 0;
        }
    }
    for (int t = 0; t < threads; ++t)
        if (threads > 1 && handles[t])
            pthread_join(handles[t], NULL);
}

void oracle_quantize_rows(const uint16_t *x, int64_t rows, int64_t cols, const float *scales,
                          uint8_t *codes)
{
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t c = 0; c < cols; ++c)
            codes[r * cols + c] = quantize_one(x[r * cols + c], scales[r]);
}

float oracle_amax(const uint16_t *x, size_t count)
{
    float best = 0.0f;
    for (size_t i = 0; i < count; ++i) {
        float v = fabsf(half_to_float(x[i]));
        if (v > best) /* false for NaN */
            best = v;
    }
    return best;
}

void oracle_weight_scales(const uint16_t *w, int64_t rows, int64_t cols, float *scales)
{
    /* cpp/src/network_graph.cpp:140-148: max in fp32, divide by 448.f, 0 -> 1. */
    for (int64_t r = 0; r < rows; ++r) {
        float best = 0.0f;
        for (int64_t c = 0; c < cols; ++c) {
            float v = fabsf(half_to_float(w[r * cols + c]));
            best = best > v ? best : v;
        }
        best /= 448.0f;
        scales[r] = best > 0.0f ? best : 1.0f;
    }
}

static inline double round_half(double v) { return oracle_half_to_double(oracle_half_from_double(v)); }

uint16_t oracle_erf_fp16(uint16_t h)
{
    return oracle_half_from_double(erf(oracle_half_to_double(h)));
}

uint16_t oracle_gelu_fp16(uint16_t h)
{
    double x = oracle_half_to_double(h);
    const double inv_sqrt2 = round_half(1.0 / sqrt(2.0)); /* 0.70703125 */
    double scaled = round_half(x * inv_sqrt2);
    double erf_value = round_half(erf(scaled));
    double left = round_half(x * 0.5);
    double right = round_half(1.0 + erf_value);
    return oracle_half_from_double(left * right);
}

int oracle_threads(void)
{
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int)n : 1;
}

typedef struct {
    const uint8_t *xq, *wq;
    int64_t m, n, k;
    float act_scale;
    const float *w_scale;
    const uint16_t *bias;
    int gelu;
    uint16_t *y;
    float next_scale;
    uint8_t *next_codes;
    const float *table; /* e4m3 code -> value */
    int64_t row_begin, row_end;
} linear_job;

static void *linear_rows(void *argument)
{
    linear_job *job = (linear_job *)argument;
    double *xrow = (double *)malloc(sizeof(double) * (size_t)job->k);
    for (int64_t r = job->row_begin; r < job->row_end; ++r) {
        for (int64_t c = 0; c < job->k; ++c)
            xrow[c] = job->table[job->xq[r * job->k + c]];
        for (int64_t col = 0; col < job->n; ++col) {
            const uint8_t *w = job->wq + col * job->k;
            /* Each E4M3 product has <= 8 significant bits and lies in
             * [2^-18, 2^17.6]; a sum of <= 2^20 of them is exact in binary64. */
            double acc = 0.0;
            /* Exact in any order, so the reduction may be vectorized. */
#pragma omp simd reduction(+ : acc)
            for (int64_t c = 0; c < job->k; ++c)
                acc += xrow[c] * (double)job->table[w[c]];
            double scale = (double)job->act_scale * (double)job->w_scale[col];
            uint16_t y16 = oracle_half_from_double(acc * scale);
            if (job->bias)
                y16 = oracle_half_from_double(oracle_half_to_double(y16) +
                                              oracle_half_to_double(job->bias[col]));
            if (job->gelu)
                y16 = oracle_gelu_fp16(y16);
            if (job->y)
                job->y[r * job->n + col] = y16;
            if (job->next_codes)
                job->next_codes[r * job->n + col] = quantize_one(y16, job->next_scale);
        }
    }
    free(xrow);
    return NULL;
}

void oracle_fp8_linear(const uint8_t *xq, const uint8_t *wq, int64_t m, int64_t n, int64_t k,
                       float act_scale, const float *w_scale, const uint16_t *bias, int gelu,
                       uint16_t *y, float next_scale, uint8_t *next_codes, int threads)
{
    float table[256];
    for (int i = 0; i < 256; ++i) {
        table[i] = oracle_e4m3_to_float((uint8_t)i);
        if (isnan(table[i]))
            table[i] = NAN;
    }
    if (threads <= 0)
        threads = oracle_threads();
    if (threads > m)
        threads = m > 0 ? (int)m : 1;
    if (threads > 256)
        threads = 256;
    pthread_t handles[256];
    linear_job jobs[256];
    int64_t per = (m + threads - 1) / threads;
    int started = 0;
    for (int t = 0; t < threads; ++t) {
        linear_job job = {xq, wq, m, n, k, act_scale, w_scale, bias, gelu, y, next_scale,
                          next_codes, table, t * per, (t + 1) * per < m ? (t + 1) * per : m};
        jobs[t] = job;
        if (job.row_begin >= job.row_end)
            continue;
        if (threads == 1 || pthread_create(&handles[t], NULL, linear_rows, &jobs[t]) != 0) {
            linear_rows(&jobs[t]);
            handles[t] = 0;
            continue;
        }
        ++started;
    }
    for (int t = 0; t < threads; ++t)
        if (jobs[t].row_begin < jobs[t].row_end && handles[t])
            pthread_join(handles[t], NULL);
    (void)started;
}

void oracle_fp16_fc1(const uint16_t *x, const uint16_t *w, const uint16_t *bias, uint16_t *y,
                     int64_t rows, int64_t width)
{
    /* cpp/tests/kernel_reference.hpp:20-25,36-47: double dot, then the fp16 graph edges. */
    for (int64_t r = 0; r < rows; ++r) {
        double dot = 0.0;
        for (int64_t c = 0; c < width; ++c)
            dot += oracle_half_to_double(x[c]) * oracle_half_to_double(w[r * width + c]);
        double value = round_half(round_half(dot) + oracle_half_to_double(bias[r]));
        y[r] = oracle_gelu_fp16(oracle_half_from_double(value));
    }
}

void oracle_fp16_qkv(const uint16_t *x, const uint16_t *w, const uint16_t *q_bias,
                     const uint16_t *v_bias, uint16_t *y, int64_t width)
{
    /* cpp/tests/kernel_reference.hpp:44-46: Q rows get q_bias, K rows none, V rows v_bias. */
    for (int64_t r = 0; r < 3 * width; ++r) {
        double dot = 0.0;
        for (int64_t c = 0; c < width; ++c)
            dot += oracle_half_to_double(x[c]) * oracle_half_to_double(w[r * width + c]);
        double q = r < width ? oracle_half_to_double(q_bias[r]) : 0.0;
        double v = r >= 2 * width ? oracle_half_to_double(v_bias[r - 2 * width]) : 0.0;
        y[r] = oracle_half_from_double(dot + q + v);
    }
}

/* The reference kernel's fp32 sum of x . w (cpp/kernels.cu:27-49).  DEPTH is the
 * power of two >= width (at least 128) and V = DEPTH / 32.  Lane L forms the
 * products of columns (i/4)*128 + 4L + i%4, i < V, with +0 past the width, folds
 * them by halving strides (p[i] += p[i + s], s = V/2 .. 1), and the 32 lane sums
 * are folded as shfl_down with offsets 16 .. 1 leaves them in lane 0.  fp16 x fp16
 * products are exact in binary32, so this order alone decides the roundings. */
static float fp16_dot_kernel_order(const uint16_t *x, const uint16_t *w, int64_t width, float *scratch)
{
    int64_t depth = 128;
    while (depth < width)
        depth *= 2;
    const int64_t v = depth / 32;
    float lanes[32];
    for (int lane = 0; lane < 32; ++lane) {
        for (int64_t i = 0; i < v; ++i) {
            const int64_t col = (i / 4) * 128 + 4 * lane + i % 4;
            scratch[i] = col < width ? (float)oracle_half_to_double(x[col]) * (float)oracle_half_to_double(w[col])
                                     : 0.0f;
        }
        for (int64_t s = v / 2; s > 0; s /= 2)
            for (int64_t i = 0; i < s; ++i)
                scratch[i] = scratch[i] + scratch[i + s];
        lanes[lane] = scratch[0];
    }
    for (int off = 16; off > 0; off /= 2)
        for (int lane = 0; lane < off; ++lane)
            lanes[lane] = lanes[lane] + lanes[lane + off];
    return lanes[0];
}

int oracle_fp16_fc1_kernel_order(const uint16_t *x, const uint16_t *w, const uint16_t *bias, uint16_t *y,
                                 int64_t rows, int64_t width)
{
    float *scratch = malloc(sizeof(float) * (size_t)(width / 16 + 128)); /* >= DEPTH / 32 */
    if (!scratch)
        return -1;
    for (int64_t r = 0; r < rows; ++r) {
        const float dot = fp16_dot_kernel_order(x, w + r * width, width, scratch);
        /* half(half(dot) + bias): the sum of two halves rounded once to fp16 */
        const double value = round_half(round_half((double)dot) + oracle_half_to_double(bias[r]));
        y[r] = oracle_gelu_fp16(oracle_half_from_double(value));
    }
    free(scratch);
    return 0;
}

int oracle_fp16_qkv_kernel_order(const uint16_t *x, const uint16_t *w, const uint16_t *q_bias,
                                 const uint16_t *v_bias, uint16_t *y, int64_t width)
{
    float *scratch = malloc(sizeof(float) * (size_t)(width / 16 + 128)); /* >= DEPTH / 32 */
    if (!scratch)
        return -1;
    for (int64_t r = 0; r < 3 * width; ++r) {
        const float dot = fp16_dot_kernel_order(x, w + r * width, width, scratch);
        const float q = r < width ? (float)oracle_half_to_double(q_bias[r]) : 0.0f;
        const float v = r >= 2 * width ? (float)oracle_half_to_double(v_bias[r - 2 * width]) : 0.0f;
        y[r] = oracle_half_from_double((double)((dot + q) + v));
    }
    free(scratch);
    return 0;
}

void oracle_fp16_bias(const uint16_t *x, uint16_t bias, uint16_t *y, int64_t count)
{
    /* cpp/kernels.cu:10-17 */
    double b = oracle_half_to_double(bias);
    for (int64_t i = 0; i < count; ++i)
        y[i] = oracle_half_from_double(oracle_half_to_double(x[i]) + b);
}
