// Host-side launchers of the sm_100a kernels (defined in kernels.cu).  Argument
// validation happens in capi.cpp before any of these is called; they only
// encode tensor maps, pick a kernel variant and launch.
#pragma once
#include <cstdint>
#include <cuda_runtime_api.h>

namespace lffw {

struct LinearLaunch {
    int64_t m, n, k;
    const uint8_t *x_codes;
    float act_scale;
    const float *act_scale_ptr;
    const uint8_t *w_codes;
    const float *w_scales;
    const uint16_t *bias;
    bool gelu;
    uint16_t *y;
    float next_scale;
    uint8_t *next_codes;
    bool w_packed; // w_codes holds skinny-packed tiles (m <= 32 path only)
    const uint16_t *residual = nullptr; // fp16 [m, n] added after the bias (large-m path only)
};

// Encoder convolution (kernel 3, padding 1, stride 1 or 2) on fp16 tensor cores
// with the fp32 bias add, the fp16-edge GELU and an optional fp16 positional add.
// x: [streams, t_in + 2, c_in] time-major, rows 0 and t_in + 1 of each stream
// zero (the padding); w: [c_out, 3, c_in] (tap-major); output row t of stream s
// lands at y[s][y_row0 + t] of [streams, y_rows, c_out].
struct ConvLaunch {
    int streams, t_in, c_in, c_out, stride; // t_out = t_in / stride
    const uint16_t *x, *w, *bias;
    const uint16_t *pos; // [t_out, c_out] or null
    uint16_t *y;
    int y_rows, y_row0;
};
cudaError_t launch_conv_gelu(const ConvLaunch &p, cudaStream_t stream);
// fp32 log-mel [streams, mels, frames] -> fp16 [streams, frames + 2, mels] (zero rows 0, frames + 1).
cudaError_t launch_mel_frames(const float *mel, int streams, int mels, int frames, uint16_t *x,
                              cudaStream_t stream);
// Convolution weights [c_out, c_in, 3] -> [c_out, 3, c_in].
cudaError_t launch_conv_weight_layout(const uint16_t *w, int64_t c_out, int64_t c_in, uint16_t *out,
                                      cudaStream_t stream);
// FP8 linear over codes [streams, tokens, k] whose fp16 output column c of
// token t lands at y[c / (64 heads)][stream][(c / 64) % heads][t][c % 64].
struct HeadsLinearLaunch {
    int streams, tokens, heads;
    int64_t n, k;
    const uint8_t *x_codes;
    float act_scale;
    const float *act_scale_ptr;
    const uint8_t *w_codes;
    const float *w_scales;
    const uint16_t *bias;
    uint16_t *y;
    int y_streams; // streams per group of y (>= streams)
};
cudaError_t launch_fp8_linear_heads(const HeadsLinearLaunch &p, cudaStream_t stream);

// Decoder step: token + position embedding, self-attention over the KV cache
// (appending the step's key and value), greedy selection.  `lengths` (device,
// int32 per stream) is the number of cached keys, also the new token's position.
constexpr int kDecoderMaxCache = 512;
cudaError_t launch_decoder_embed(const int32_t *tokens, const int32_t *lengths, const uint16_t *token_table,
                                 const uint16_t *position_table, int streams, int width, int vocab, int positions,
                                 uint16_t *x, cudaStream_t stream);
struct DecoderAttentionLaunch {
    int streams, heads, capacity;
    const uint16_t *qkv;
    int64_t qkv_ld;
    uint16_t *cache_k, *cache_v;
    const int32_t *lengths;
    uint16_t *out;
    uint8_t *codes;
    float code_scale;
};
cudaError_t launch_decoder_self_attention(const DecoderAttentionLaunch &p, cudaStream_t stream);
cudaError_t launch_greedy_select(const uint16_t *logits, int64_t logits_ld, const float *suppression,
                                 int64_t suppression_ld, int streams, int vocab, int32_t *tokens, int32_t *lengths,
                                 cudaStream_t stream);
// Reads and clears the decoder kernels' error word (1: token or position out of
// its table, 2: cache full); -1 when it cannot be read.
int read_and_clear_decoder_error();

// Largest M served by the small-M (skinny) kernels.
constexpr int64_t kSmallMaxRows = 32;

cudaError_t launch_fp8_gemm(const LinearLaunch &p, cudaStream_t stream);
// m <= 32 on tensor cores (swap-AB, cluster split-K); fp16 weights for the logits.
cudaError_t launch_fp8_skinny(const LinearLaunch &p, cudaStream_t stream);
cudaError_t launch_fp16_skinny(const uint16_t *x, const uint16_t *w, const uint16_t *bias, uint16_t *y, int64_t m,
                               int64_t n, int64_t k, bool packed, cudaStream_t stream);
// Pre-swizzled 16 KB weight tiles for the skinny kernels (size, then the pack).
int64_t skinny_packed_bytes(int64_t n, int64_t row_bytes);
cudaError_t launch_pack_skinny(const void *w, int64_t n, int64_t row_bytes, void *packed, cudaStream_t stream);
// LayerNorm producer: fp16 residual sum, fp16 LN output and/or E4M3 codes.
constexpr int64_t kLayerNormMaxCols = 4096;
struct LayerNormLaunch {
    int64_t rows, cols; // cols % 8 == 0, cols <= 4096
    const uint16_t *x, *residual;
    uint16_t *sum_out;
    const float *gamma, *beta;
    float eps;
    uint16_t *y;
    float code_scale;
    const float *code_scale_ptr;
    uint8_t *codes;
};
cudaError_t launch_layer_norm(const LayerNormLaunch &p, cudaStream_t stream);
// Decoder cross-attention over a cached encoder K/V (head_dim 64).
constexpr int kAttentionMaxQueries = 16;
constexpr int kAttentionMaxKeys = 4096;
constexpr int kAttentionMaxKeysPerCta = 2048; // score rows in shared memory
struct CrossAttentionLaunch {
    int streams, queries, heads, keys;
    const uint16_t *q, *k, *v;
    uint16_t *out;
    float code_scale;
    const float *code_scale_ptr;
    uint8_t *codes;
};
cudaError_t launch_cross_attention(const CrossAttentionLaunch &p, cudaStream_t stream);
// Encoder self-attention (head_dim 64) on q/k/v rows read in place.
struct SelfAttentionLaunch {
    int streams, tokens, heads;
    const uint16_t *q, *k, *v;
    int64_t q_ld, k_ld, v_ld;
    uint16_t *out;
    float code_scale;
    const float *code_scale_ptr;
    uint8_t *codes;
};
cudaError_t launch_self_attention(const SelfAttentionLaunch &p, cudaStream_t stream);
// Persistent chain of small-M linears (packed weights, one m).
struct ChainPlan; // device descriptors, opaque to callers
cudaError_t chain_create(const LinearLaunch *links, int count, ChainPlan **plan);
cudaError_t chain_run(const ChainPlan *plan, cudaStream_t stream);
void chain_destroy(ChainPlan *plan);
cudaError_t launch_quantize(const uint16_t *x, int64_t count, float scale, const float *scale_ptr,
                            uint8_t *codes, cudaStream_t stream);
cudaError_t launch_quantize_rows(const uint16_t *w, int64_t rows, int64_t cols,
                                 const float *scales, uint8_t *codes, cudaStream_t stream);
cudaError_t launch_weight_scales(const uint16_t *w, int64_t rows, int64_t cols, float *scales,
                                 cudaStream_t stream);
cudaError_t launch_dynamic_scale(const uint16_t *x, int64_t count, float *scale, float *amax_out,
                                 cudaStream_t stream);
cudaError_t launch_fp16_fc1(const uint16_t *x, const uint16_t *w, const uint16_t *bias, uint16_t *y,
                            int64_t rows, int64_t width, cudaStream_t stream);
cudaError_t launch_fp16_qkv(const uint16_t *x, const uint16_t *w, const uint16_t *q_bias,
                            const uint16_t *v_bias, uint16_t *y, int64_t width,
                            cudaStream_t stream);
cudaError_t launch_fp16_gelu(const uint16_t *x, uint16_t *y, int64_t count, cudaStream_t stream);
cudaError_t launch_fp16_bias(const uint16_t *x, uint16_t bias, uint16_t *y, int64_t count,
                             cudaStream_t stream);

cudaError_t read_and_clear_device_error(int *site);
uint64_t launch_count();
void count_launch();

} // namespace lffw
