/*
 * lffw_fp8.h — C ABI of the B200 (sm_100a) FP8 E4M3 quantized-linear library.
 *
 * This is the drop-in boundary for listenflow-fastest-whisper's FP8 Q/DQ linear
 * and its fp16 projection plugins.  Every pointer argument is caller-owned
 * device memory unless stated otherwise; `stream` is a cudaStream_t (NULL = the
 * legacy default stream).  Nothing here allocates device memory except where a
 * comment says so.  No entry point throws; all return an lffw_status.
 *
 * Reference interfaces replaced (paths inside the reference project):
 *   - FP8 linear:     cpp/src/network_graph.cpp:115-159 (graph::qdq + graph::linear),
 *                     python/src/listenflow/fastest_whisper/_fp8.py:20-51
 *   - fused GELU:     cpp/src/network_graph.cpp:168-183 (graph::gelu, graph::fc1)
 *   - fp16 plugins:   cpp/fc1_plugin.cpp:74-106, cpp/qkv_plugin.cpp:74-107,
 *                     cpp/plugin.cpp:70-92 (IPluginV3OneRuntime::enqueue) and the
 *                     kernels they launch, cpp/kernels.cu:10-78
 *   - plugin creators: cpp/fc1_plugin.cpp:125-155, cpp/qkv_plugin.cpp:126-156,
 *                     cpp/plugin.cpp:95-153 (getCreators / createPlugin / fields)
 *   - status codes:   cpp/include/listenflow/whisper_runtime.h:15-23
 */
#ifndef LFFW_FP8_H
#define LFFW_FP8_H
#include <stddef.h>
#include <stdint.h>

#define LFFW_FP8_ABI_MAJOR 1
#define LFFW_FP8_ABI_MINOR 7
#define LFFW_FP8_API __attribute__((visibility("default")))
#if defined(__cplusplus)
#define LFFW_FP8_NOEXCEPT noexcept
extern "C" {
#else
#define LFFW_FP8_NOEXCEPT
#endif

/* Status values keep the numbering of whisper_runtime.h:17-22; 120+ are new. */
typedef int32_t lffw_status;
enum {
    LFFW_SUCCESS = 0,
    LFFW_INVALID_ARGUMENT = 1,
    LFFW_ABI_MISMATCH = 2,
    LFFW_OUT_OF_MEMORY = 3,
    LFFW_INTERNAL_ERROR = 4,
    LFFW_CUDA_ERROR = 6,
    LFFW_UNSUPPORTED_PRECISION = 9, /* device is not sm_100 (FP8 gate) */
    LFFW_DEVICE_TIMEOUT = 120       /* a bounded device-side wait expired */
};

/* Epilogue selection for lffw_fp8_linear. */
enum { LFFW_EPILOGUE_NONE = 0, LFFW_EPILOGUE_GELU = 1 };

/* Weight layouts.  ROW_MAJOR: [n, k] with k contiguous.  SKINNY_TILES: the
 * weight re-laid by lffw_pack_skinny_weights into contiguous 16 KB tiles that
 * the small-m kernels stream sequentially (only for m <= 32). */
enum { LFFW_WEIGHTS_ROW_MAJOR = 0, LFFW_WEIGHTS_SKINNY_TILES = 1 };

/*
 * One FP8 Q/DQ linear (replaces graph::linear in fp8 precision,
 * network_graph.cpp:124-159):
 *   acc[m,n] = sum_k E4M3(x_codes[m,k]) * E4M3(w_codes[n,k])      fp32 accumulate
 *   y16      = half(acc * act_scale * w_scales[n])                  MatMul output edge
 *   y16      = half(y16 + bias[n])                                  if bias
 *   y16      = GELU with fp16 edges (network_graph.cpp:168-180)     if epilogue == GELU
 *   y[m,n]   = y16                                                  if y
 *   next_codes[m,n] = E4M3_rne_sat(fp32(y16 / next_scale))          if next_codes
 * Layouts are row-major with K (resp. N) contiguous: x_codes [m,k], w_codes
 * [n,k] (the reference's [out,in] weight, i.e. before its [1,in,out] transpose),
 * y / next_codes [m,n].  The activation scale is the static `act_scale`, or is
 * read from device memory when `act_scale_ptr` is non-NULL (dynamic amax/448).
 * Requirements: m,n,k >= 1; k % 16 == 0; n % 16 == 0; 16-byte aligned pointers;
 * act_scale (or *act_scale_ptr) finite and > 0; next_scale in [2^-125, 2^125]
 * (a normal float with a normal reciprocal) when next_codes is set.
 * Stream overlap: the linear and quantize kernels use programmatic dependent
 * launch.  Each lets the next launch on its stream start early, and each waits
 * for the previous kernel before it reads activations or writes outputs, but a
 * linear reads its weights (w_codes, w_scales, bias) before that wait.
 * Weights are layer constants, so this is safe unless the kernel just before
 * a linear is an lffw_fp8_quantize or lffw_fp8_linear call that writes those
 * weights.  In that case, put any other stream operation (an event record, a
 * copy) between the two calls.
 */
typedef struct lffw_fp8_linear_args {
    size_t struct_size; /* sizeof(lffw_fp8_linear_args) */
    int64_t m, n, k;
    const uint8_t *x_codes;
    float act_scale;
    const float *act_scale_ptr;
    const uint8_t *w_codes;
    const float *w_scales;
    const uint16_t *bias;
    int32_t epilogue;
    uint16_t *y;
    float next_scale;
    uint8_t *next_codes;
    int32_t w_layout; /* LFFW_WEIGHTS_*; absent (older struct_size) means ROW_MAJOR */
    /* Optional fp16 [m, n] row-major, 16-byte aligned (absent in older struct_size
     * means none): y = half(linear + residual), the graph's fp16 residual add after
     * the linear's bias (cpp/src/network_graph.cpp:285-287), so the LayerNorm that
     * follows reads one tensor instead of two.  Requires y, no GELU, no next_codes,
     * n % 32 == 0 and row-major weights; y may be the residual itself. */
    const uint16_t *residual;
} lffw_fp8_linear_args;

LFFW_FP8_API lffw_status lffw_fp8_linear(const lffw_fp8_linear_args *args,
                                         void *stream) LFFW_FP8_NOEXCEPT;

/* Q of an fp16 activation with one scalar scale (graph::qdq axis 0,
 * network_graph.cpp:115-123): codes[i] = E4M3_rne_sat(fp32(x[i] / scale)).
 * `scale_ptr` (device, may be NULL) overrides `scale`; scales lie in
 * [2^-125, 2^125].  x and codes are 16-byte aligned. */
LFFW_FP8_API lffw_status lffw_fp8_quantize(const uint16_t *x, int64_t count, float scale,
                                           const float *scale_ptr, uint8_t *codes,
                                           void *stream) LFFW_FP8_NOEXCEPT;

/* A chain of dependent small-m linears in one persistent launch (no counterpart in
 * the reference; it runs the decoder step's linears back to back).  Link i may read
 * what earlier links wrote: its activations are loaded only after every row block
 * of link i-1 is written.  Each link is an lffw_fp8_linear call with the same m
 * (<= 32), packed weights (w_layout = LFFW_WEIGHTS_SKINNY_TILES), a static or
 * device act_scale, and y and/or next_codes; results equal lffw_fp8_linear's bit
 * for bit.  lffw_chain_create validates the links and ALLOCATES device memory
 * for their descriptors (freed by lffw_chain_destroy); the pointers in the links
 * are bound at creation.  lffw_chain_run launches once (capturable in a graph);
 * runs of one chain must not overlap on the GPU. */
typedef struct lffw_chain lffw_chain;

LFFW_FP8_API lffw_status lffw_chain_create(const lffw_fp8_linear_args *links, int32_t count,
                                           lffw_chain **chain) LFFW_FP8_NOEXCEPT;
LFFW_FP8_API lffw_status lffw_chain_run(const lffw_chain *chain, void *stream) LFFW_FP8_NOEXCEPT;
LFFW_FP8_API void lffw_chain_destroy(lffw_chain *chain) LFFW_FP8_NOEXCEPT;

/* LayerNorm producer for the linear that follows it (network_graph.cpp:160-166
 * `norm`, with the fp16 residual add of :285-287 before it), per row of `cols`:
 *   s[i]    = half(x[i] + residual[i])   (s = x when residual is NULL)
 *   sum_out = s                          (if sum_out: the new residual stream)
 *   y[i]    = half((s[i] - mean) * rsqrt(var + epsilon) * gamma[i] + beta[i])
 *             (fp32 statistics over the row; population variance)
 *   codes   = E4M3_rne_sat(fp32(y[i] / code_scale))   (if codes)
 * y and/or codes and/or sum_out are written (at least one).  The activation
 * round trip a separate quantize would make (write y, read y) is skipped when
 * y is NULL.  Requirements: rows >= 1; 8 <= cols <= 4096, cols % 8 == 0;
 * 16-byte aligned pointers; gamma/beta fp32 [cols]; epsilon finite and >= 0;
 * code_scale (or *code_scale_ptr, device) in [2^-125, 2^125] when codes is set. */
typedef struct lffw_layer_norm_args {
    size_t struct_size; /* sizeof(lffw_layer_norm_args) */
    int64_t rows, cols;
    const uint16_t *x;
    const uint16_t *residual;
    uint16_t *sum_out;
    const float *gamma;
    const float *beta;
    float epsilon;
    uint16_t *y;
    float code_scale;
    const float *code_scale_ptr;
    uint8_t *codes;
} lffw_layer_norm_args;

LFFW_FP8_API lffw_status lffw_layer_norm(const lffw_layer_norm_args *args, void *stream) LFFW_FP8_NOEXCEPT;

/* Decoder cross-attention over a cached encoder K/V for one layer
 * (network_graph.cpp:235-244 `attend`, cross_keys/cross_values of :401-404), per
 * stream s, head h, query row t (the beams of a stream share its K/V):
 *   c        = half(head_dim^-0.25)
 *   q', k'   = half(q * c), half(k * c)
 *   score[j] = half(q' . k'[j])                        (fp32 accumulate)
 *   p[j]     = half(softmax_fp32(score)[j])            (over all keys)
 *   out[s*queries + t][h*head_dim + d] = half(sum_j p[j] v[j][d])   (fp32 accumulate)
 *   out_codes = E4M3_rne_sat(fp32(out / code_scale))   (if out_codes: out_proj's input)
 * q and out are fp16 [streams*queries, heads*head_dim] (the q_proj output and the
 * out_proj input, merge_heads layout); k and v are fp16 [streams, heads, keys,
 * head_dim].  Requirements: head_dim == 64; 1 <= queries <= 16; 1 <= keys <= 4096;
 * streams, heads >= 1 with streams*heads*keys < 2^31; 16-byte aligned pointers;
 * out and/or out_codes set; code_scale (or *code_scale_ptr) in [2^-125, 2^125]. */
typedef struct lffw_cross_attention_args {
    size_t struct_size; /* sizeof(lffw_cross_attention_args) */
    int32_t streams, queries, heads, head_dim, keys;
    const uint16_t *q;
    const uint16_t *k;
    const uint16_t *v;
    uint16_t *out;
    float code_scale;
    const float *code_scale_ptr;
    uint8_t *out_codes;
} lffw_cross_attention_args;

LFFW_FP8_API lffw_status lffw_cross_attention(const lffw_cross_attention_args *args,
                                              void *stream) LFFW_FP8_NOEXCEPT;

/* Encoder self-attention for one layer (network_graph.cpp:235-247 `attention`: `attend`
 * on the layer's own projections, no mask), with the same fp16 edges as
 * lffw_cross_attention, per stream s over its `tokens` rows.  q, k and v are read in
 * place: element (s * tokens + t, h * head_dim + d) of each lies at row
 * s * tokens + t, column h * head_dim + d, with row strides q_ld, k_ld, v_ld
 * (elements).  For the fused QKV linear output [rows, 3 * width], pass q = y,
 * k = y + width, v = y + 2 * width and all strides 3 * width.  out: fp16
 * [streams * tokens, heads * head_dim] (out_proj's input) and/or its E4M3 codes.
 * Requirements: head_dim == 64; tokens >= 1; streams * tokens < 2^31;
 * streams * heads * ceil(tokens / 128) + 65536 < 2^31; strides
 * >= heads * 64 and multiples of 8; 16-byte aligned pointers; out and/or out_codes
 * set; code_scale (or *code_scale_ptr) in [2^-125, 2^125]. */
typedef struct lffw_self_attention_args {
    size_t struct_size; /* sizeof(lffw_self_attention_args) */
    int32_t streams, tokens, heads, head_dim;
    const uint16_t *q;
    const uint16_t *k;
    const uint16_t *v;
    int64_t q_ld, k_ld, v_ld;
    uint16_t *out;
    float code_scale;
    const float *code_scale_ptr;
    uint8_t *out_codes;
} lffw_self_attention_args;

LFFW_FP8_API lffw_status lffw_self_attention(const lffw_self_attention_args *args,
                                             void *stream) LFFW_FP8_NOEXCEPT;

/* Encoder front end (network_graph.cpp:257-282): the log-mel input cast to fp16,
 * the two kernel-3 convolutions with padding 1 (the first stride 1, the second
 * stride 2), each followed by GELU with fp16 edges, and the positional embedding
 * added after the second.
 *
 * lffw_mel_frames: mel fp32 [streams, mels, frames] -> x fp16 [streams, frames + 2,
 * mels] with x[s][t + 1][c] = half(mel[s][c][t]) and rows 0 and frames + 1 zero: the
 * time-major, zero-padded layout lffw_conv1d_gelu reads.  Requirements: streams,
 * mels, frames >= 1; mels % 8 == 0; 16-byte aligned pointers. */
LFFW_FP8_API lffw_status lffw_mel_frames(const float *mel, int32_t streams, int32_t mels, int32_t frames,
                                         uint16_t *x, void *stream) LFFW_FP8_NOEXCEPT;

/* Convolution weights from the checkpoint's [c_out, c_in, 3] (conv1d weight
 * layout) to the tap-major [c_out, 3, c_in] lffw_conv1d_gelu reads.  Runs once
 * at load time. */
LFFW_FP8_API lffw_status lffw_conv1d_weight_layout(const uint16_t *weight, int32_t c_out, int32_t c_in,
                                                   uint16_t *out, void *stream) LFFW_FP8_NOEXCEPT;

/* One encoder convolution (replaces the addConvolutionNd + gelu pair of
 * network_graph.cpp:259-275, with the positional add of :280-282 when
 * `positions` is set), on fp16 tensor cores, per stream s and output row t
 * (frames_out = frames_in / stride):
 *   acc  = sum_{j<3} sum_ci w[co][j][ci] * x[s][stride * t + j][ci]   (fp32 accumulate;
 *          x row r holds input frame r - 1, so rows 0 and frames_in + 1 are the padding)
 *   z    = half(acc + bias[co])                                      (fp32 add, one rounding)
 *   z    = GELU with fp16 edges
 *   z    = half(z + positions[t][co])                                (if positions)
 *   y[s][y_row0 + t][co] = z                        (y: [streams, y_rows, c_out])
 * With y_rows = frames_out + 2 and y_row0 = 1 the output is itself the padded input
 * of the next convolution; rows 0 and y_rows - 1 are not written (zero them once).
 * Requirements: stride 1 or 2; frames_in >= stride and a multiple of it; c_in % 64
 * == 0; c_out % 32 == 0; y_row0 >= 0 and y_row0 + frames_out <= y_rows; positions
 * fp16 [frames_out, c_out] or NULL; 16-byte aligned pointers. */
typedef struct lffw_conv1d_args {
    size_t struct_size; /* sizeof(lffw_conv1d_args) */
    int32_t streams, frames_in, c_in, c_out, stride;
    const uint16_t *x;
    const uint16_t *weight;    /* [c_out, 3, c_in], lffw_conv1d_weight_layout */
    const uint16_t *bias;      /* [c_out] */
    const uint16_t *positions; /* [frames_out, c_out] or NULL */
    uint16_t *y;
    int32_t y_rows, y_row0;
} lffw_conv1d_args;

LFFW_FP8_API lffw_status lffw_conv1d_gelu(const lffw_conv1d_args *args, void *stream) LFFW_FP8_NOEXCEPT;

/* The cross-attention K/V projections of every decoder layer as one FP8 linear
 * over the final encoder states (network_graph.cpp:296-300 with project_kv of
 * :231-234: k_proj without bias, v_proj with bias, both on the encoder output),
 * with the output stored split by heads, the cross_keys / cross_values layout of
 * lffw_cross_attention:
 *   y16 = the lffw_fp8_linear value of row s * tokens + t, column c (bias optional;
 *         a bias of -0.0 leaves every value, -0 included, unchanged)
 *   y[c / (64 heads)][s][(c / 64) % heads][t][c % 64] = y16
 * y holds y_streams streams per group (y_streams >= streams; 0 means streams), so a
 * batch computed in slices of streams can write its slice of one larger buffer
 * (pass y offset by the slice's first stream).
 * For the decoder's layers stacked as [k_0, v_0, k_1, v_1, ...] (n = 2 * layers *
 * heads * 64), group g = 2 * layer + (0 for keys, 1 for values).  x_codes: E4M3
 * [streams * tokens, k].  Requirements: streams, tokens, heads >= 1; k % 16 == 0;
 * n a multiple of 64 * heads; 16-byte aligned pointers; act_scale (or
 * *act_scale_ptr) finite and > 0. */
typedef struct lffw_fp8_linear_heads_args {
    size_t struct_size; /* sizeof(lffw_fp8_linear_heads_args) */
    int32_t streams, tokens, heads;
    int64_t n, k;
    const uint8_t *x_codes;
    float act_scale;
    const float *act_scale_ptr;
    const uint8_t *w_codes;
    const float *w_scales;
    const uint16_t *bias;
    uint16_t *y;
    int32_t y_streams;
} lffw_fp8_linear_heads_args;

LFFW_FP8_API lffw_status lffw_fp8_linear_heads(const lffw_fp8_linear_heads_args *args,
                                               void *stream) LFFW_FP8_NOEXCEPT;

/* Decoder step pieces (network_graph.cpp:378-416).  `lengths` (device int32 per
 * stream) is the number of keys in the stream's self-attention cache before the
 * step, which is also the position of the step's token; lffw_greedy_select
 * advances it.  Keeping it on the device lets one captured CUDA graph of a step
 * serve every step of a greedy decode.
 *
 * lffw_decoder_embed: x[s] = half(token_table[tokens[s]] + position_table[lengths[s]])
 * (the two gathers and the fp16 add of :380-388).  token_table fp16 [vocab, width],
 * position_table fp16 [positions, width], x fp16 [streams, width].  A token or
 * position outside its table leaves x[s] unwritten and sets decoder error 1
 * (lffw_decoder_error).  Requirements: width % 8 == 0; 16-byte aligned pointers. */
LFFW_FP8_API lffw_status lffw_decoder_embed(const int32_t *tokens, const int32_t *lengths,
                                            const uint16_t *token_table, const uint16_t *position_table,
                                            int32_t streams, int32_t width, int32_t vocab, int32_t positions,
                                            uint16_t *x, void *stream) LFFW_FP8_NOEXCEPT;

/* Decoder self-attention of one layer over its fp16 KV cache (network_graph.cpp:390-399:
 * the cached keys and values concatenated with the step's own, `attend` with the
 * graph's fp16 edges as in lffw_cross_attention; the reference's mask is zero for
 * every cached position, so no mask is taken).  Per stream s and head h:
 *   cache_k[s][h][lengths[s]] = k, cache_v[s][h][lengths[s]] = v   (the step's row of qkv)
 *   out over keys 0 .. lengths[s] of the cache: q' = half(q c), k' = half(k c),
 *   score = half(q'.k'), p = half(softmax_fp32(score)), out = half(sum_j p_j v_j)
 * qkv: fp16 [streams, qkv_ld] holding q | k | v (heads * 64 columns each) of the
 * step's fused QKV linear; cache_k, cache_v: fp16 [streams, heads, capacity, 64];
 * out fp16 and/or out_codes E4M3 [streams, heads * 64].  A length >= capacity sets
 * decoder error 2 and leaves that (stream, head) untouched.  Requirements: head_dim
 * == 64; 1 <= capacity <= 512; qkv_ld >= 3 * heads * 64 and a multiple of 8;
 * 16-byte aligned pointers; code_scale in [2^-125, 2^125] with out_codes. */
typedef struct lffw_decoder_self_attention_args {
    size_t struct_size; /* sizeof(lffw_decoder_self_attention_args) */
    int32_t streams, heads, head_dim, capacity;
    const uint16_t *qkv;
    int64_t qkv_ld;
    uint16_t *cache_k;
    uint16_t *cache_v;
    const int32_t *lengths;
    uint16_t *out;
    float code_scale;
    uint8_t *out_codes;
} lffw_decoder_self_attention_args;

LFFW_FP8_API lffw_status lffw_decoder_self_attention(const lffw_decoder_self_attention_args *args,
                                                     void *stream) LFFW_FP8_NOEXCEPT;

/* Greedy token choice (network_graph.cpp:332-339 select_token): per stream,
 * score[v] = fp32(logits[s][v]) + suppression[s][v] and tokens[s] = the smallest v
 * whose score equals the maximum (vocab when every score is NaN); then, when
 * `lengths` is not NULL, lengths[s] += 1.  logits fp16 [streams, logits_ld],
 * suppression fp32 [streams, suppression_ld] (0 or -inf per token).
 * Requirements: 1 <= vocab <= logits_ld, suppression_ld. */
LFFW_FP8_API lffw_status lffw_greedy_select(const uint16_t *logits, int64_t logits_ld, const float *suppression,
                                            int64_t suppression_ld, int32_t streams, int32_t vocab,
                                            int32_t *tokens, int32_t *lengths, void *stream) LFFW_FP8_NOEXCEPT;

/* Reads and clears the decoder kernels' error word: 0 none, 1 a token or position
 * outside its table, 2 a full cache.  Synchronises with the device. */
LFFW_FP8_API lffw_status lffw_decoder_error(int32_t *code) LFFW_FP8_NOEXCEPT;

/* Q of an fp16 [rows, cols] weight with one scale per row (the per-output-channel
 * weight Q of network_graph.cpp:140-152, axis 2 of the transposed constant). */
LFFW_FP8_API lffw_status lffw_fp8_quantize_rows(const uint16_t *w, int64_t rows, int64_t cols,
                                                const float *scales, uint8_t *codes,
                                                void *stream) LFFW_FP8_NOEXCEPT;

/* Per-output-channel weight scales: max|w[r,:]| / 448 in fp32, non-positive -> 1
 * (network_graph.cpp:140-148, _fp8.py:37-42). */
LFFW_FP8_API lffw_status lffw_fp8_weight_scales(const uint16_t *w, int64_t rows, int64_t cols,
                                                float *scales, void *stream) LFFW_FP8_NOEXCEPT;

/* Dynamic activation scale: *scale = amax(|x|)/448 (0 -> 1), NaN ignored, the
 * calibration rule of python/scripts/calibrate_fp8.py:384-385 applied to one
 * tensor.  `amax_out` (optional, device) receives the maximum itself. */
LFFW_FP8_API lffw_status lffw_fp8_dynamic_scale(const uint16_t *x, int64_t count, float *scale,
                                                float *amax_out, void *stream) LFFW_FP8_NOEXCEPT;

/* fp16 single-token projections of the reference plugins (cpp/kernels.cu:51-78),
 * rebuilt for sm_100a.  x [width], weight [rows, width] (row = output), all fp16.
 *   fc1: y[r] = GELU-fp16-edges(half(half(x.W[r]) + bias[r])), rows = 5120, width = 1280
 *   qkv: y[r] = half((x.W[r] + q_bias[r if r<width]) + v_bias[r-2w if r>=2w]), rows = 3*width */
LFFW_FP8_API lffw_status lffw_fp16_fc1(const uint16_t *x, const uint16_t *weight,
                                       const uint16_t *bias, uint16_t *y, int64_t rows,
                                       int64_t width, void *stream) LFFW_FP8_NOEXCEPT;
LFFW_FP8_API lffw_status lffw_fp16_qkv(const uint16_t *x, const uint16_t *weight,
                                       const uint16_t *q_bias, const uint16_t *v_bias,
                                       uint16_t *y, int64_t width,
                                       void *stream) LFFW_FP8_NOEXCEPT;
/* y[i] = half(x[i] + bias) (cpp/kernels.cu:10-17); 1 <= count <= INT32_MAX. */
LFFW_FP8_API lffw_status lffw_fp16_bias(const uint16_t *x, uint16_t bias_bits, uint16_t *y,
                                        int64_t count, void *stream) LFFW_FP8_NOEXCEPT;

/* fp16 linear for up to 32 rows (the decoder step's fp16 logits MatMul,
 * 1280 -> vocabulary, cpp/src/network_graph.cpp:379-417): y[m,n] =
 * half(sum_k x[m,k] w[n,k] (+ bias[n])), fp32 accumulate on tensor cores.
 * x [m,k] fp16; weight fp16 in `w_layout` (LFFW_WEIGHTS_*); 1 <= m <= 32;
 * k % 8 == 0; bias may be NULL. */
LFFW_FP8_API lffw_status lffw_fp16_linear(const uint16_t *x, const uint16_t *weight, const uint16_t *bias,
                                          uint16_t *y, int64_t m, int64_t n, int64_t k, int32_t w_layout,
                                          void *stream) LFFW_FP8_NOEXCEPT;

/* Size in bytes of a weight [n, k] (elem_bytes 1 = E4M3, 2 = fp16) in the
 * LFFW_WEIGHTS_SKINNY_TILES layout; 0 for invalid arguments. */
LFFW_FP8_API int64_t lffw_skinny_packed_bytes(int64_t n, int64_t k, int32_t elem_bytes) LFFW_FP8_NOEXCEPT;
/* Re-lays a row-major weight into that layout (a build-time step, like
 * TensorRT's weight reformatting); `packed` holds lffw_skinny_packed_bytes. */
LFFW_FP8_API lffw_status lffw_pack_skinny_weights(const void *weight, int64_t n, int64_t k, int32_t elem_bytes,
                                                  void *packed, void *stream) LFFW_FP8_NOEXCEPT;

/* GELU with every graph edge rounded to fp16, elementwise on `count` halves:
 * y = (x*0.5)*(1 + erf(x*fp16(2^-1/2))) (graph::gelu, network_graph.cpp:168-180).
 * The same device code as the fused GEMM epilogue. */
LFFW_FP8_API lffw_status lffw_fp16_gelu(const uint16_t *x, uint16_t *y, int64_t count,
                                        void *stream) LFFW_FP8_NOEXCEPT;

/* Device gate (replaces the sm86/89/120 gates of cpp/src/precision_policy.hpp:4-7,
 * cpp/src/runtime_model.hpp:88-92 and cpp/fc1_plugin.cpp:90-98): SUCCESS only
 * for compute capability 10.0 (B200, sm_100a); UNSUPPORTED_PRECISION otherwise. */
LFFW_FP8_API lffw_status lffw_device_supported(int32_t device) LFFW_FP8_NOEXCEPT;

/* Reads and clears the calling device's sticky error word, which bounded
 * device-side waits set when they give up (LFFW_DEVICE_TIMEOUT).  Synchronizes
 * the device.  `where` (optional) receives the role/site code that gave up. */
LFFW_FP8_API lffw_status lffw_device_error(int32_t *where) LFFW_FP8_NOEXCEPT;

/* Number of this library's kernels launched by this process so far. */
LFFW_FP8_API uint64_t lffw_launch_count(void) LFFW_FP8_NOEXCEPT;

LFFW_FP8_API const char *lffw_status_string(lffw_status status) LFFW_FP8_NOEXCEPT;
LFFW_FP8_API void lffw_version(uint32_t *major, uint32_t *minor) LFFW_FP8_NOEXCEPT;

/* ---- Allocation-free FP8 linear on fp16 activations ------------------------
 * No counterpart in the reference: an addition of this library.
 *
 * The usual way to run a linear on fp16 activations is lffw_fp8_quantize into
 * a codes buffer the caller allocated, then lffw_fp8_linear (or the
 * LffwFp8Linear plugin with a workspace).  Some callers cannot allocate that
 * buffer: a latency-critical streaming thread must not call cudaMalloc, which
 * can synchronize the whole device and block for milliseconds; a plugin host
 * may hand out only the workspace it sized before the run; a process whose
 * device memory is already reserved by another allocator has nothing left to
 * give.  This entry point keeps the E4M3 codes of x in a fixed buffer inside the
 * library instead (LFFW_STATIC_SCRATCH_BYTES per GPU that loads the library,
 * held until the process exits) and allocates nothing itself.
 *
 * Same arithmetic as lffw_fp8_quantize(x, m*k, act_scale) followed by
 * lffw_fp8_linear with the same weights, bias and epilogue, writing fp16 y.
 * Limits: m * k <= LFFW_STATIC_SCRATCH_BYTES, else LFFW_SCRATCH_TOO_SMALL and
 * nothing runs; the other requirements of lffw_fp8_linear apply.
 * The first call on a device looks up the buffer's device address once; make
 * that first call before any stream capture.  Every call on a device shares
 * the one buffer, and each call overwrites the part it reads: calls whose work
 * overlaps on the GPU (different streams without ordering) race on it. */
#define LFFW_STATIC_SCRATCH_BYTES (8u << 20) /* 8 MiB of E4M3 codes */
enum { LFFW_SCRATCH_TOO_SMALL = 121 };
LFFW_FP8_API lffw_status lffw_fp8_linear_half_static(const uint16_t *x, int64_t m, int64_t n, int64_t k,
                                                     float act_scale, const uint8_t *w_codes,
                                                     const float *w_scales, const uint16_t *bias,
                                                     int32_t epilogue, uint16_t *y,
                                                     void *stream) LFFW_FP8_NOEXCEPT;

/* ---- Plugin surface ------------------------------------------------------
 * A C restatement of the reference's TensorRT IPluginV3 creators
 * (namespace "listenflow.fastest_whisper"): LffwFp16Fc1 v"1", LffwFp16Qkv v"2",
 * LffwFp16Bias v"1" with the same field names/types/lengths and the same shape,
 * dtype and format checks, plus the FP8 family LffwFp8Linear v"1".  A TensorRT
 * adapter forwards createPlugin / onShapeChange / getWorkspaceSize / enqueue to
 * these calls one to one.  Enum values equal TensorRT's (DataType,
 * TensorFormat, PluginFieldType, TensorRTPhase). */
enum { LFFW_DT_FLOAT = 0, LFFW_DT_HALF = 1, LFFW_DT_INT8 = 2, LFFW_DT_INT32 = 3, LFFW_DT_FP8 = 6 };
enum { LFFW_FORMAT_LINEAR = 0, LFFW_FORMAT_CHW2 = 1 };
enum {
    LFFW_FIELD_FLOAT16 = 0, LFFW_FIELD_FLOAT32 = 1, LFFW_FIELD_FLOAT64 = 2, LFFW_FIELD_INT8 = 3,
    LFFW_FIELD_INT16 = 4, LFFW_FIELD_INT32 = 5, LFFW_FIELD_CHAR = 6
};
enum { LFFW_PHASE_BUILD = 0, LFFW_PHASE_RUNTIME = 1 };

typedef struct lffw_plugin_field {
    const char *name;
    const void *data;
    int32_t type;   /* LFFW_FIELD_* */
    int32_t length; /* element count */
} lffw_plugin_field;

typedef struct lffw_tensor_desc {
    int32_t nb_dims;
    int64_t dims[8];
    int32_t type;   /* LFFW_DT_* */
    int32_t format; /* LFFW_FORMAT_* */
} lffw_tensor_desc;

typedef struct lffw_plugin lffw_plugin;

/* extern "C" char const tensoracle_bundle_sha256[] of cpp/fc1_plugin.cpp:11,
 * read by dlsym in network_graph.cpp:196-198 and ctypes in _plugins.py:33:
 * here the SHA-256 (hex) of the kernel source this library was built from. */
LFFW_FP8_API extern const char tensoracle_bundle_sha256[65];

LFFW_FP8_API int32_t lffw_plugin_creator_count(void) LFFW_FP8_NOEXCEPT;
/* Creator i: name, version, namespace and its declared fields (getFieldNames). */
LFFW_FP8_API int32_t lffw_plugin_creator(int32_t index, const char **name, const char **version,
                                         const char **plugin_namespace,
                                         const lffw_plugin_field **fields,
                                         int32_t *field_count) LFFW_FP8_NOEXCEPT;
/* createPlugin: NULL when the creator is unknown, the phase is neither BUILD
 * nor RUNTIME, or the fields are not exactly the declared set with a matching
 * bundle_sha256 (fc1_plugin.cpp:32-37, 143-150). */
LFFW_FP8_API lffw_plugin *lffw_plugin_create(const char *name, const char *version,
                                             const char *plugin_namespace,
                                             const lffw_plugin_field *fields, int32_t count,
                                             int32_t phase) LFFW_FP8_NOEXCEPT;
LFFW_FP8_API lffw_plugin *lffw_plugin_clone(const lffw_plugin *plugin) LFFW_FP8_NOEXCEPT;
LFFW_FP8_API void lffw_plugin_destroy(lffw_plugin *plugin) LFFW_FP8_NOEXCEPT;
/* onShapeChange / validate_shape: 0 when the descriptors are accepted, -1 otherwise. */
LFFW_FP8_API int32_t lffw_plugin_validate(const lffw_plugin *plugin,
                                          const lffw_tensor_desc *inputs, int32_t input_count,
                                          const lffw_tensor_desc *output) LFFW_FP8_NOEXCEPT;
/* getWorkspaceSize (bytes).  fp16 plugins: 0.  LffwFp8Linear with a HALF input:
 * the E4M3 codes of that input (rows * k bytes, rounded up to 256). */
LFFW_FP8_API int64_t lffw_plugin_workspace_size(const lffw_plugin *plugin,
                                                const lffw_tensor_desc *inputs,
                                                int32_t input_count) LFFW_FP8_NOEXCEPT;
/* enqueue: 0 on success, -1 on a null pointer, wrong dtype/format/shape, an
 * unsupported device or a launch failure (fc1_plugin.cpp:74-106). */
LFFW_FP8_API int32_t lffw_plugin_enqueue(const lffw_plugin *plugin,
                                         const lffw_tensor_desc *input_desc,
                                         const lffw_tensor_desc *output_desc,
                                         const void *const *inputs, void *const *outputs,
                                         void *workspace, void *stream) LFFW_FP8_NOEXCEPT;

#if defined(__cplusplus)
}
#endif
#endif
