// C ABI of liblffw_b200.so (declared in include/lffw_fp8.h): argument
// validation, the sm_100 device gate, dispatch to the kernel launchers, and a
// C restatement of the reference's TensorRT plugin creators and runtime checks.
#include "lffw_fp8.h"

#include <cuda_runtime_api.h>

#include <cmath>
#include <cstddef>
#include <cstring>
#include <limits>
#include <mutex>
#include <new>
#include <string>
#include <vector>

#include "launch.h"

#ifndef LFFW_BUNDLE_SHA256
#error "build with -DLFFW_BUNDLE_SHA256=\"<sha256 of kernels.cu>\""
#endif

extern "C" LFFW_FP8_API const char tensoracle_bundle_sha256[65] = LFFW_BUNDLE_SHA256;

namespace {

using lffw::LinearLaunch;

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
bool positive_finite(float v) { return std::isfinite(v) && v > 0.0f; }
// A scale whose reciprocal is also a normal float (Q divides by it).
bool valid_scale(float v) { return std::isfinite(v) && v >= 0x1p-125f && v <= 0x1p125f; }

lffw_status from_cuda(cudaError_t err)
{
    if (err == cudaSuccess)
        return LFFW_SUCCESS;
    if (err == cudaErrorMemoryAllocation)
        return LFFW_OUT_OF_MEMORY;
    return LFFW_CUDA_ERROR;
}

// sm_100 (B200) gate, cached per device.
lffw_status device_gate(int device)
{
    static std::mutex lock;
    static std::vector<int> verdict; // 0 unknown, 1 ok, 2 unsupported
    if (device < 0)
        return LFFW_INVALID_ARGUMENT;
    {
        std::lock_guard<std::mutex> guard(lock);
        if (static_cast<size_t>(device) < verdict.size() && verdict[device] != 0)
            return verdict[device] == 1 ? LFFW_SUCCESS : LFFW_UNSUPPORTED_PRECISION;
    }
    int major = 0, minor = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device) != cudaSuccess ||
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device) != cudaSuccess) {
        cudaGetLastError();
        return LFFW_CUDA_ERROR;
    }
    const bool ok = major == 10 && minor == 0;
    std::lock_guard<std::mutex> guard(lock);
    if (verdict.size() <= static_cast<size_t>(device))
        verdict.resize(device + 1, 0);
    verdict[device] = ok ? 1 : 2;
    return ok ? LFFW_SUCCESS : LFFW_UNSUPPORTED_PRECISION;
}

lffw_status current_device_gate()
{
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) {
        cudaGetLastError();
        return LFFW_CUDA_ERROR;
    }
    return device_gate(device);
}

constexpr int64_t kMaxDim = std::numeric_limits<int32_t>::max();

// The layout field exists only in callers built against ABI 1.1+ headers.
int32_t weight_layout(const lffw_fp8_linear_args *a)
{
    return a->struct_size >= offsetof(lffw_fp8_linear_args, w_layout) + sizeof(int32_t) ? a->w_layout
                                                                                         : LFFW_WEIGHTS_ROW_MAJOR;
}

// The residual field exists only in callers built against ABI 1.7+ headers.
const uint16_t *linear_residual(const lffw_fp8_linear_args *a)
{
    return a->struct_size >= offsetof(lffw_fp8_linear_args, residual) + sizeof(a->residual) ? a->residual
                                                                                           : nullptr;
}

lffw_status validate_linear(const lffw_fp8_linear_args *a)
{
    if (a == nullptr)
        return LFFW_INVALID_ARGUMENT;
    if (a->struct_size < offsetof(lffw_fp8_linear_args, w_layout))
        return LFFW_ABI_MISMATCH;
    if (a->m < 1 || a->n < 1 || a->k < 1 || a->m > kMaxDim || a->n > kMaxDim || a->k > kMaxDim)
        return LFFW_INVALID_ARGUMENT;
    if (a->k % 16 != 0 || a->n % 16 != 0)
        return LFFW_INVALID_ARGUMENT;
    if (a->x_codes == nullptr || a->w_codes == nullptr || a->w_scales == nullptr)
        return LFFW_INVALID_ARGUMENT;
    if (a->y == nullptr && a->next_codes == nullptr)
        return LFFW_INVALID_ARGUMENT;
    if (!aligned16(a->x_codes) || !aligned16(a->w_codes) || !aligned16(a->w_scales) ||
        !aligned16(a->bias) || !aligned16(a->y) || !aligned16(a->next_codes) ||
        (reinterpret_cast<uintptr_t>(a->act_scale_ptr) & 3u) != 0)
        return LFFW_INVALID_ARGUMENT;
    if (a->act_scale_ptr == nullptr && !positive_finite(a->act_scale))
        return LFFW_INVALID_ARGUMENT; // network_graph.cpp:137-139
    if (a->next_codes != nullptr && !valid_scale(a->next_scale))
        return LFFW_INVALID_ARGUMENT;
    if (a->epilogue != LFFW_EPILOGUE_NONE && a->epilogue != LFFW_EPILOGUE_GELU)
        return LFFW_INVALID_ARGUMENT;
    const int32_t layout = weight_layout(a);
    if (layout != LFFW_WEIGHTS_ROW_MAJOR && layout != LFFW_WEIGHTS_SKINNY_TILES)
        return LFFW_INVALID_ARGUMENT;
    if (layout == LFFW_WEIGHTS_SKINNY_TILES && a->m > lffw::kSmallMaxRows)
        return LFFW_INVALID_ARGUMENT;
    const uint16_t *residual = linear_residual(a);
    if (residual != nullptr && (a->y == nullptr || a->next_codes != nullptr || a->epilogue != LFFW_EPILOGUE_NONE ||
                                a->n % 32 != 0 || layout != LFFW_WEIGHTS_ROW_MAJOR || !aligned16(residual)))
        return LFFW_INVALID_ARGUMENT;
    return LFFW_SUCCESS;
}

lffw_status run_linear(const lffw_fp8_linear_args *a, cudaStream_t stream)
{
    LinearLaunch L{};
    L.m = a->m;
    L.n = a->n;
    L.k = a->k;
    L.x_codes = a->x_codes;
    L.act_scale = a->act_scale;
    L.act_scale_ptr = a->act_scale_ptr;
    L.w_codes = a->w_codes;
    L.w_scales = a->w_scales;
    L.bias = a->bias;
    L.gelu = a->epilogue == LFFW_EPILOGUE_GELU;
    L.y = a->y;
    L.next_scale = a->next_scale;
    L.next_codes = a->next_codes;
    L.w_packed = weight_layout(a) == LFFW_WEIGHTS_SKINNY_TILES;
    L.residual = linear_residual(a);
    // The residual add rides on the large-m GEMM's epilogue (which serves any m).
    const bool small = a->m <= lffw::kSmallMaxRows && L.residual == nullptr;
    return from_cuda(small ? lffw::launch_fp8_skinny(L, stream) : lffw::launch_fp8_gemm(L, stream));
}

} // namespace

extern "C" {

lffw_status lffw_fp8_linear(const lffw_fp8_linear_args *args, void *stream) noexcept
{
    lffw_status s = validate_linear(args);
    if (s != LFFW_SUCCESS)
        return s;
    if ((s = current_device_gate()) != LFFW_SUCCESS)
        return s;
    return run_linear(args, static_cast<cudaStream_t>(stream));
}

struct lffw_chain {
    lffw::ChainPlan *plan;
};

lffw_status lffw_chain_create(const lffw_fp8_linear_args *links, int32_t count, lffw_chain **chain) noexcept
{
    if (chain == nullptr)
        return LFFW_INVALID_ARGUMENT;
    *chain = nullptr;
    if (links == nullptr || count < 1 || count > (1 << 20))
        return LFFW_INVALID_ARGUMENT;
    std::vector<lffw::LinearLaunch> launches(static_cast<size_t>(count));
    for (int32_t i = 0; i < count; ++i) {
        const lffw_fp8_linear_args *a = &links[i];
        const lffw_status v = validate_linear(a);
        if (v != LFFW_SUCCESS)
            return v;
        if (weight_layout(a) != LFFW_WEIGHTS_SKINNY_TILES || a->m != links[0].m)
            return LFFW_INVALID_ARGUMENT;
        lffw::LinearLaunch &L = launches[i];
        L.m = a->m;
        L.n = a->n;
        L.k = a->k;
        L.x_codes = a->x_codes;
        L.act_scale = a->act_scale;
        L.act_scale_ptr = a->act_scale_ptr;
        L.w_codes = a->w_codes;
        L.w_scales = a->w_scales;
        L.bias = a->bias;
        L.gelu = a->epilogue == LFFW_EPILOGUE_GELU;
        L.y = a->y;
        L.next_scale = a->next_scale;
        L.next_codes = a->next_codes;
        L.w_packed = true;
    }
    lffw_status s = current_device_gate();
    if (s != LFFW_SUCCESS)
        return s;
    auto *handle = new (std::nothrow) lffw_chain{nullptr};
    if (handle == nullptr)
        return LFFW_OUT_OF_MEMORY;
    const cudaError_t err = lffw::chain_create(launches.data(), count, &handle->plan);
    if (err != cudaSuccess) {
        delete handle;
        return err == cudaErrorMemoryAllocation ? LFFW_OUT_OF_MEMORY : LFFW_CUDA_ERROR;
    }
    *chain = handle;
    return LFFW_SUCCESS;
}

lffw_status lffw_chain_run(const lffw_chain *chain, void *stream) noexcept
{
    if (chain == nullptr || chain->plan == nullptr)
        return LFFW_INVALID_ARGUMENT;
    return from_cuda(lffw::chain_run(chain->plan, static_cast<cudaStream_t>(stream)));
}

void lffw_chain_destroy(lffw_chain *chain) noexcept
{
    if (chain == nullptr)
        return;
    lffw::chain_destroy(chain->plan);
    delete chain;
}

lffw_status lffw_fp8_quantize(const uint16_t *x, int64_t count, float scale, const float *scale_ptr,
                              uint8_t *codes, void *stream) noexcept
{
    if (x == nullptr || codes == nullptr || count < 1 || !aligned16(x) || !aligned16(codes))
        return LFFW_INVALID_ARGUMENT;
    if (scale_ptr == nullptr && !valid_scale(scale))
        return LFFW_INVALID_ARGUMENT;
    lffw_status s = current_device_gate();
    if (s != LFFW_SUCCESS)
        return s;
    return from_cuda(lffw::launch_quantize(x, count, scale, scale_ptr, codes,
                                           static_cast<cudaStream_t>(stream)));
}

lffw_status lffw_layer_norm(const lffw_layer_norm_args *a, void *stream) noexcept
{
    if (a == nullptr || a->struct_size < sizeof(lffw_layer_norm_args))
        return a == nullptr ? LFFW_INVALID_ARGUMENT : LFFW_ABI_MISMATCH;
    if (a->rows < 1 || a->rows > kMaxDim || a->cols < 8 || a->cols % 8 != 0 || a->cols > lffw::kLayerNormMaxCols)
        return LFFW_INVALID_ARGUMENT;
    if (a->x == nullptr || a->gamma == nullptr || a->beta == nullptr)
        return LFFW_INVALID_ARGUMENT;
    if (a->y == nullptr && a->codes == nullptr && a->sum_out == nullptr)
        return LFFW_INVALID_ARGUMENT;
    if (!aligned16(a->x) || !aligned16(a->residual) || !aligned16(a->sum_out) || !aligned16(a->gamma) ||
        !aligned16(a->beta) || !aligned16(a->y) || !aligned16(a->codes))
        return LFFW_INVALID_ARGUMENT;
    if (!(a->epsilon >= 0.0f) || !std::isfinite(a->epsilon))
        return LFFW_INVALID_ARGUMENT;
    if (a->codes != nullptr && a->code_scale_ptr == nullptr && !valid_scale(a->code_scale))
        return LFFW_INVALID_ARGUMENT;
    lffw_status s = current_device_gate();
    if (s != LFFW_SUCCESS)
        return s;
    lffw::LayerNormLaunch L{};
    L.rows = a->rows;
    L.cols = a->cols;
    L.x = a->x;
    L.residual = a->residual;
    L.sum_out = a->sum_out;
    L.gamma = a->gamma;
    L.beta = a->beta;
    L.eps = a->epsilon;
    L.y = a->y;
    L.code_scale = a->code_scale;
    L.code_scale_ptr = a->code_scale_ptr;
    L.codes = a->codes;
    return from_cuda(lffw::launch_layer_norm(L, static_cast<cudaStream_t>(stream)));
}

lffw_status lffw_cross_attention(const lffw_cross_attention_args *a, void *stream) noexcept
{
    if (a == nullptr || a->struct_size < sizeof(lffw_cross_attention_args))
        return a == nullptr ? LFFW_INVALID_ARGUMENT : LFFW_ABI_MISMATCH;
    if (a->head_dim != 64 || a->queries < 1 || a->queries > lffw::kAttentionMaxQueries || a->keys < 1 ||
        a->keys > lffw::kAttentionMaxKeys || a->streams < 1 || a->heads < 1)
        return LFFW_INVALID_ARGUMENT;
    if (static_cast<int64_t>(a->streams) * a->heads * a->keys >= (int64_t(1) << 31))
        return LFFW_INVALID_ARGUMENT;
    if (a->q == nullptr || a->k == nullptr || a->v == nullptr || (a->out == nullptr && a->out_codes == nullptr))
        return LFFW_INVALID_ARGUMENT;
    if (!aligned16(a->q) || !aligned16(a->k) || !aligned16(a->v) || !aligned16(a->out) || !aligned16(a->out_codes))
        return LFFW_INVALID_ARGUMENT;
    if (a->out_codes != nullptr && a->code_scale_ptr == nullptr && !valid_scale(a->code_scale))
        return LFFW_INVALID_ARGUMENT;
    lffw_status s = current_device_gate();
    if (s != LFFW_SUCCESS)
        return s;
    lffw::CrossAttentionLaunch L{};
    L.streams = a->streams;
    L.queries = a->queries;
    L.heads = a->heads;
    L.keys = a->keys;
    L.q = a->q;
    L.k = a->k;
    L.v = a->v;
    L.out = a->out;
    L.code_scale = a->code_scale;
    L.code_scale_ptr = a->code_scale_ptr;
    L.codes = a->out_codes;
    return from_cuda(lffw::launch_cross_attention(L, static_cast<cudaStream_t>(stream)));
}

lffw_status lffw_self_attention(const lffw_self_attention_args *a, void *stream) noexcept
{
    if (a == nullptr || a->struct_size < sizeof(lffw_self_attention_args))
        return a == nullptr ? LFFW_INVALID_ARGUMENT : LFFW_ABI_MISMATCH;
    if (a->head_dim != 64 || a->tokens < 1 || a->streams < 1 || a->heads < 1)
        return LFFW_INVALID_ARGUMENT;
    const int64_t width = static_cast<int64_t>(a->heads) * 64;
    if (static_cast<int64_t>(a->streams) * a->tokens >= (int64_t(1) << 31) || width > kMaxDim)
        return LFFW_INVALID_ARGUMENT;
    // The kernel numbers its (stream, head, 128-query block) items with 32-bit
    // integers, and its persistent loops step an item index by the grid size
    // (at most 65535 CTAs): items + 65536 must stay below 2^31.
    if (static_cast<int64_t>(a->streams) * a->heads * ((a->tokens + 127) / 128) + 65536 >= (int64_t(1) << 31))
        return LFFW_INVALID_ARGUMENT;
    for (const int64_t ld : {a->q_ld, a->k_ld, a->v_ld})
        if (ld < width || ld % 8 != 0)
            return LFFW_INVALID_ARGUMENT;
    if (a->q == nullptr || a->k == nullptr || a->v == nullptr || (a->out == nullptr && a->out_codes == nullptr))
        return LFFW_INVALID_ARGUMENT;
    if (!aligned16(a->q) || !aligned16(a->k) || !aligned16(a->v) || !aligned16(a->out) || !aligned16(a->out_codes))
        return LFFW_INVALID_ARGUMENT;
    if (a->out_codes != nullptr && a->code_scale_ptr == nullptr && !valid_scale(a->code_scale))
        return LFFW_INVALID_ARGUMENT;
    lffw_status s = current_device_gate();
    if (s != LFFW_SUCCESS)
        return s;
    lffw::SelfAttentionLaunch L{};
    L.streams = a->streams;
    L.tokens = a->tokens;
    L.heads = a->heads;
    L.q = a->q;
    L.k = a->k;
    L.v = a->v;
    L.q_ld = a->q_ld;
    L.k_ld = a->k_ld;
    L.v_ld = a->v_ld;
    L.out = a->out;
    L.code_scale = a->code_scale;
    L.code_scale_ptr = a->code_scale_ptr;
    L.codes = a->out_codes;
    return from_cuda(lffw::launch_self_attention(L, static_cast<cudaStream_t>(stream)));
}

lffw_status lffw_mel_frames(const float *mel, int32_t streams, int32_t mels, int32_t frames, uint16_t *x,
                            void *stream) noexcept
{
    if (mel == nullptr || x == nullptr || streams < 1 || mels < 8 || mels % 8 != 0 || frames < 1 ||
        streams > 65535 || !aligned16(mel) || !aligned16(x))
        return LFFW_INVALID_ARGUMENT;
    if (static_cast<int64_t>(streams) * mels * (static_cast<int64_t>(frames) + 2) >= (int64_t(1) << 40))
        return LFFW_INVALID_ARGUMENT;
    lffw_status s = current_device_gate();
    if (s != LFFW_SUCCESS)
        return s;
    return from_cuda(lffw::launch_mel_frames(mel, streams, mels, frames, x, static_cast<cudaStream_t>(stream)));
}

lffw_status lffw_conv1d_weight_layout(const uint16_t *weight, int32_t c_out, int32_t c_in, uint16_t *out,
                                      void *stream) noexcept
{
    if (weight == nullptr || out == nullptr || c_out < 1 || c_in < 1 || weight == out)
        return LFFW_INVALID_ARGUMENT;
    lffw_status s = current_device_gate();
    if (s != LFFW_SUCCESS)
        return s;
    return from_cuda(lffw::launch_conv_weight_layout(weight, c_out, c_in, out, static_cast<cudaStream_t>(stream)));
}

lffw_status lffw_conv1d_gelu(const lffw_conv1d_args *a, void *stream) noexcept
{
    if (a == nullptr || a->struct_size < sizeof(lffw_conv1d_args))
        return a == nullptr ? LFFW_INVALID_ARGUMENT : LFFW_ABI_MISMATCH;
    if (a->stride != 1 && a->stride != 2)
        return LFFW_INVALID_ARGUMENT;
    if (a->streams < 1 || a->frames_in < a->stride || a->frames_in % a->stride != 0 || a->c_in < 64 ||
        a->c_in % 64 != 0 || a->c_out < 32 || a->c_out % 32 != 0)
        return LFFW_INVALID_ARGUMENT;
    const int64_t frames_out = a->frames_in / a->stride;
    if (a->y_row0 < 0 || a->y_rows < 1 || a->y_row0 + frames_out > a->y_rows)
        return LFFW_INVALID_ARGUMENT;
    // Tile bookkeeping is 32-bit: rows, tiles and K blocks stay well inside it.
    if (static_cast<int64_t>(a->streams) * (static_cast<int64_t>(a->frames_in) + 2) >= (int64_t(1) << 31) ||
        static_cast<int64_t>(a->streams) * a->y_rows >= (int64_t(1) << 31) || a->c_in > (1 << 20) ||
        a->c_out > (1 << 20))
        return LFFW_INVALID_ARGUMENT;
    if (a->x == nullptr || a->weight == nullptr || a->bias == nullptr || a->y == nullptr)
        return LFFW_INVALID_ARGUMENT;
    if (!aligned16(a->x) || !aligned16(a->weight) || !aligned16(a->bias) || !aligned16(a->positions) ||
        !aligned16(a->y))
        return LFFW_INVALID_ARGUMENT;
    lffw_status s = current_device_gate();
    if (s != LFFW_SUCCESS)
        return s;
    lffw::ConvLaunch L{};
    L.streams = a->streams;
    L.t_in = a->frames_in;
    L.c_in = a->c_in;
    L.c_out = a->c_out;
    L.stride = a->stride;
    L.x = a->x;
    L.w = a->weight;
    L.bias = a->bias;
    L.pos = a->positions;
    L.y = a->y;
    L.y_rows = a->y_rows;
    L.y_row0 = a->y_row0;
    return from_cuda(lffw::launch_conv_gelu(L, static_cast<cudaStream_t>(stream)));
}

lffw_status lffw_decoder_embed(const int32_t *tokens, const int32_t *lengths, const uint16_t *token_table,
                               const uint16_t *position_table, int32_t streams, int32_t width, int32_t vocab,
                               int32_t positions, uint16_t *x, void *stream) noexcept
{
    if (tokens == nullptr || lengths == nullptr || token_table == nullptr || position_table == nullptr ||
        x == nullptr || streams < 1 || streams > 65535 || width < 8 || width % 8 != 0 || vocab < 1 ||
        positions < 1 || !aligned16(token_table) || !aligned16(position_table) || !aligned16(x))
        return LFFW_INVALID_ARGUMENT;
    lffw_status s = current_device_gate();
    if (s != LFFW_SUCCESS)
        return s;
    return from_cuda(lffw::launch_decoder_embed(tokens, lengths, token_table, position_table, streams, width, vocab,
                                                positions, x, static_cast<cudaStream_t>(stream)));
}

lffw_status lffw_decoder_self_attention(const lffw_decoder_self_attention_args *a, void *stream) noexcept
{
    if (a == nullptr || a->struct_size < sizeof(lffw_decoder_self_attention_args))
        return a == nullptr ? LFFW_INVALID_ARGUMENT : LFFW_ABI_MISMATCH;
    if (a->head_dim != 64 || a->streams < 1 || a->heads < 1 || a->capacity < 1 ||
        a->capacity > lffw::kDecoderMaxCache)
        return LFFW_INVALID_ARGUMENT;
    const int64_t width = static_cast<int64_t>(a->heads) * 64;
    if (static_cast<int64_t>(a->streams) * a->heads >= (int64_t(1) << 31) || width > kMaxDim ||
        a->qkv_ld < 3 * width || a->qkv_ld % 8 != 0)
        return LFFW_INVALID_ARGUMENT;
    if (a->qkv == nullptr || a->cache_k == nullptr || a->cache_v == nullptr || a->lengths == nullptr ||
        (a->out == nullptr && a->out_codes == nullptr))
        return LFFW_INVALID_ARGUMENT;
    if (!aligned16(a->qkv) || !aligned16(a->cache_k) || !aligned16(a->cache_v) || !aligned16(a->out) ||
        !aligned16(a->out_codes) || (reinterpret_cast<uintptr_t>(a->lengths) & 3u) != 0)
        return LFFW_INVALID_ARGUMENT;
    if (a->out_codes != nullptr && !valid_scale(a->code_scale))
        return LFFW_INVALID_ARGUMENT;
    lffw_status s = current_device_gate();
    if (s != LFFW_SUCCESS)
        return s;
    lffw::DecoderAttentionLaunch L{};
    L.streams = a->streams;
    L.heads = a->heads;
    L.capacity = a->capacity;
    L.qkv = a->qkv;
    L.qkv_ld = a->qkv_ld;
    L.cache_k = a->cache_k;
    L.cache_v = a->cache_v;
    L.lengths = a->lengths;
    L.out = a->out;
    L.codes = a->out_codes;
    L.code_scale = a->code_scale;
    return from_cuda(lffw::launch_decoder_self_attention(L, static_cast<cudaStream_t>(stream)));
}

lffw_status lffw_greedy_select(const uint16_t *logits, int64_t logits_ld, const float *suppression,
                               int64_t suppression_ld, int32_t streams, int32_t vocab, int32_t *tokens,
                               int32_t *lengths, void *stream) noexcept
{
    if (logits == nullptr || suppression == nullptr || tokens == nullptr || streams < 1 || streams > 65535 ||
        vocab < 1 || logits_ld < vocab || suppression_ld < vocab)
        return LFFW_INVALID_ARGUMENT;
    if ((reinterpret_cast<uintptr_t>(logits) & 1u) != 0 || (reinterpret_cast<uintptr_t>(suppression) & 3u) != 0 ||
        (reinterpret_cast<uintptr_t>(tokens) & 3u) != 0 || (reinterpret_cast<uintptr_t>(lengths) & 3u) != 0)
        return LFFW_INVALID_ARGUMENT;
    lffw_status s = current_device_gate();
    if (s != LFFW_SUCCESS)
        return s;
    return from_cuda(lffw::launch_greedy_select(logits, logits_ld, suppression, suppression_ld, streams, vocab, tokens,
                                                lengths, static_cast<cudaStream_t>(stream)));
}

lffw_status lffw_decoder_error(int32_t *code) noexcept
{
    if (code == nullptr)
        return LFFW_INVALID_ARGUMENT;
    const int v = lffw::read_and_clear_decoder_error();
    if (v < 0) {
        cudaGetLastError();
        return LFFW_CUDA_ERROR;
    }
    *code = v;
    return LFFW_SUCCESS;
}

lffw_status lffw_fp8_linear_heads(const lffw_fp8_linear_heads_args *a, void *stream) noexcept
{
    if (a == nullptr || a->struct_size < sizeof(lffw_fp8_linear_heads_args))
        return a == nullptr ? LFFW_INVALID_ARGUMENT : LFFW_ABI_MISMATCH;
    if (a->streams < 1 || a->tokens < 1 || a->heads < 1 || a->k < 16 || a->k % 16 != 0 || a->k > kMaxDim ||
        a->n < 1 || a->n > kMaxDim)
        return LFFW_INVALID_ARGUMENT;
    const int64_t group = 64 * static_cast<int64_t>(a->heads);
    if (a->n % group != 0)
        return LFFW_INVALID_ARGUMENT;
    // 32-bit tile bookkeeping: rows and tiles (at most 128 rows x 256 columns each).
    const int64_t rows = static_cast<int64_t>(a->streams) * a->tokens;
    if (rows >= (int64_t(1) << 31) ||
        (static_cast<int64_t>(a->streams) * ((a->tokens + 127) / 128)) * ((a->n + 255) / 256) >= (int64_t(1) << 31))
        return LFFW_INVALID_ARGUMENT;
    if (a->x_codes == nullptr || a->w_codes == nullptr || a->w_scales == nullptr || a->y == nullptr)
        return LFFW_INVALID_ARGUMENT;
    if (!aligned16(a->x_codes) || !aligned16(a->w_codes) || !aligned16(a->w_scales) || !aligned16(a->bias) ||
        !aligned16(a->y) || (reinterpret_cast<uintptr_t>(a->act_scale_ptr) & 3u) != 0)
        return LFFW_INVALID_ARGUMENT;
    if (a->act_scale_ptr == nullptr && !positive_finite(a->act_scale))
        return LFFW_INVALID_ARGUMENT;
    if (a->y_streams != 0 && a->y_streams < a->streams)
        return LFFW_INVALID_ARGUMENT;
    lffw_status s = current_device_gate();
    if (s != LFFW_SUCCESS)
        return s;
    lffw::HeadsLinearLaunch L{};
    L.y_streams = a->y_streams != 0 ? a->y_streams : a->streams;
    L.streams = a->streams;
    L.tokens = a->tokens;
    L.heads = a->heads;
    L.n = a->n;
    L.k = a->k;
    L.x_codes = a->x_codes;
    L.act_scale = a->act_scale;
    L.act_scale_ptr = a->act_scale_ptr;
    L.w_codes = a->w_codes;
    L.w_scales = a->w_scales;
    L.bias = a->bias;
    L.y = a->y;
    return from_cuda(lffw::launch_fp8_linear_heads(L, static_cast<cudaStream_t>(stream)));
}

lffw_status lffw_fp8_quantize_rows(const uint16_t *w, int64_t rows, int64_t cols, const float *scales,
                                   uint8_t *codes, void *stream) noexcept
{
    if (w == nullptr || scales == nullptr || codes == nullptr || rows < 1 || cols < 1 ||
        rows > kMaxDim || cols > kMaxDim)
        return LFFW_INVALID_ARGUMENT;
    lffw_status s = current_device_gate();
    if (s != LFFW_SUCCESS)
        return s;
    return from_cuda(lffw::launch_quantize_rows(w, rows, cols, scales, codes,
                                                static_cast<cudaStream_t>(stream)));
}

lffw_status lffw_fp8_weight_scales(const uint16_t *w, int64_t rows, int64_t cols, float *scales,
                                   void *stream) noexcept
{
    if (w == nullptr || scales == nullptr || rows < 1 || cols < 1 || rows > kMaxDim)
        return LFFW_INVALID_ARGUMENT;
    lffw_status s = current_device_gate();
    if (s != LFFW_SUCCESS)
        return s;
    return from_cuda(lffw::launch_weight_scales(w, rows, cols, scales, static_cast<cudaStream_t>(stream)));
}

lffw_status lffw_fp8_dynamic_scale(const uint16_t *x, int64_t count, float *scale, float *amax_out,
                                   void *stream) noexcept
{
    if (x == nullptr || scale == nullptr || count < 1 ||
        (reinterpret_cast<uintptr_t>(scale) & 3u) != 0)
        return LFFW_INVALID_ARGUMENT;
    lffw_status s = current_device_gate();
    if (s != LFFW_SUCCESS)
        return s;
    return from_cuda(lffw::launch_dynamic_scale(x, count, scale, amax_out, static_cast<cudaStream_t>(stream)));
}

lffw_status lffw_fp16_fc1(const uint16_t *x, const uint16_t *weight, const uint16_t *bias, uint16_t *y,
                          int64_t rows, int64_t width, void *stream) noexcept
{
    if (x == nullptr || weight == nullptr || bias == nullptr || y == nullptr || rows < 1 ||
        width < 8 || width % 8 != 0 || rows > kMaxDim || width > kMaxDim || !aligned16(x) ||
        !aligned16(weight))
        return LFFW_INVALID_ARGUMENT;
    lffw_status s = current_device_gate();
    if (s != LFFW_SUCCESS)
        return s;
    return from_cuda(lffw::launch_fp16_fc1(x, weight, bias, y, rows, width, static_cast<cudaStream_t>(stream)));
}

lffw_status lffw_fp16_qkv(const uint16_t *x, const uint16_t *weight, const uint16_t *q_bias,
                          const uint16_t *v_bias, uint16_t *y, int64_t width, void *stream) noexcept
{
    if (x == nullptr || weight == nullptr || q_bias == nullptr || v_bias == nullptr || y == nullptr ||
        width < 8 || width % 8 != 0 || 3 * width > kMaxDim || !aligned16(x) || !aligned16(weight))
        return LFFW_INVALID_ARGUMENT;
    lffw_status s = current_device_gate();
    if (s != LFFW_SUCCESS)
        return s;
    return from_cuda(lffw::launch_fp16_qkv(x, weight, q_bias, v_bias, y, width, static_cast<cudaStream_t>(stream)));
}

lffw_status lffw_fp16_bias(const uint16_t *x, uint16_t bias_bits, uint16_t *y, int64_t count,
                           void *stream) noexcept
{
    if (x == nullptr || y == nullptr || count < 1 || count > kMaxDim)
        return LFFW_INVALID_ARGUMENT;
    lffw_status s = current_device_gate();
    if (s != LFFW_SUCCESS)
        return s;
    return from_cuda(lffw::launch_fp16_bias(x, bias_bits, y, count, static_cast<cudaStream_t>(stream)));
}

lffw_status lffw_fp16_linear(const uint16_t *x, const uint16_t *weight, const uint16_t *bias, uint16_t *y,
                             int64_t m, int64_t n, int64_t k, int32_t w_layout, void *stream) noexcept
{
    if (x == nullptr || weight == nullptr || y == nullptr || m < 1 || m > lffw::kSmallMaxRows || n < 1 ||
        n > kMaxDim || k < 8 || k % 8 != 0 || k > kMaxDim || !aligned16(x) || !aligned16(weight) ||
        (w_layout != LFFW_WEIGHTS_ROW_MAJOR && w_layout != LFFW_WEIGHTS_SKINNY_TILES))
        return LFFW_INVALID_ARGUMENT;
    lffw_status s = current_device_gate();
    if (s != LFFW_SUCCESS)
        return s;
    return from_cuda(lffw::launch_fp16_skinny(x, weight, bias, y, m, n, k, w_layout == LFFW_WEIGHTS_SKINNY_TILES,
                                              static_cast<cudaStream_t>(stream)));
}

int64_t lffw_skinny_packed_bytes(int64_t n, int64_t k, int32_t elem_bytes) noexcept
{
    if (n < 1 || k < 1 || (elem_bytes != 1 && elem_bytes != 2) || n > kMaxDim || k > kMaxDim)
        return 0;
    return lffw::skinny_packed_bytes(n, k * elem_bytes);
}

lffw_status lffw_pack_skinny_weights(const void *weight, int64_t n, int64_t k, int32_t elem_bytes, void *packed,
                                     void *stream) noexcept
{
    if (weight == nullptr || packed == nullptr || lffw_skinny_packed_bytes(n, k, elem_bytes) == 0 ||
        (k * elem_bytes) % 16 != 0 || !aligned16(weight) || !aligned16(packed))
        return LFFW_INVALID_ARGUMENT;
    lffw_status s = current_device_gate();
    if (s != LFFW_SUCCESS)
        return s;
    return from_cuda(lffw::launch_pack_skinny(weight, n, k * elem_bytes, packed, static_cast<cudaStream_t>(stream)));
}

lffw_status lffw_fp16_gelu(const uint16_t *x, uint16_t *y, int64_t count, void *stream) noexcept
{
    if (x == nullptr || y == nullptr || count < 1)
        return LFFW_INVALID_ARGUMENT;
    lffw_status s = current_device_gate();
    if (s != LFFW_SUCCESS)
        return s;
    return from_cuda(lffw::launch_fp16_gelu(x, y, count, static_cast<cudaStream_t>(stream)));
}

lffw_status lffw_device_supported(int32_t device) noexcept { return device_gate(device); }

lffw_status lffw_device_error(int32_t *where) noexcept
{
    int site = 0;
    cudaError_t err = lffw::read_and_clear_device_error(&site);
    if (where)
        *where = site;
    if (err != cudaSuccess)
        return from_cuda(err);
    return site != 0 ? LFFW_DEVICE_TIMEOUT : LFFW_SUCCESS;
}

uint64_t lffw_launch_count(void) noexcept { return lffw::launch_count(); }

const char *lffw_status_string(lffw_status status) noexcept
{
    switch (status) {
    case LFFW_SUCCESS: return "success";
    case LFFW_INVALID_ARGUMENT: return "invalid argument";
    case LFFW_ABI_MISMATCH: return "ABI mismatch";
    case LFFW_OUT_OF_MEMORY: return "out of memory";
    case LFFW_INTERNAL_ERROR: return "internal error";
    case LFFW_CUDA_ERROR: return "CUDA error";
    case LFFW_UNSUPPORTED_PRECISION: return "fp8 requires an sm_100 (B200) device";
    case LFFW_DEVICE_TIMEOUT: return "a bounded device-side wait expired";
    case LFFW_SCRATCH_TOO_SMALL: return "m * k exceeds the library's static scratch (LFFW_STATIC_SCRATCH_BYTES)";
    default: return "unknown status";
    }
}

void lffw_version(uint32_t *major, uint32_t *minor) noexcept
{
    if (major)
        *major = LFFW_FP8_ABI_MAJOR;
    if (minor)
        *minor = LFFW_FP8_ABI_MINOR;
}

} // extern "C"

// ===========================================================================
// Plugin surface.

namespace {

constexpr char kNamespace[] = "listenflow.fastest_whisper";
constexpr int64_t kWidth = 1280;       // cpp/fc1_plugin.cpp:22, cpp/qkv_plugin.cpp:22
constexpr int64_t kFc1Output = 5120;   // cpp/fc1_plugin.cpp:23

enum class Kind { Fc1, Qkv, Bias, Fp8Linear };

struct CreatorInfo {
    Kind kind;
    const char *name;
    const char *version;
    std::vector<lffw_plugin_field> fields;
};

const std::vector<CreatorInfo> &creators()
{
    static const std::vector<CreatorInfo> list = {
        {Kind::Bias, "LffwFp16Bias", "1",
         {{"bundle_sha256", nullptr, LFFW_FIELD_CHAR, 64}, {"bias", nullptr, LFFW_FIELD_FLOAT16, 1}}},
        {Kind::Qkv, "LffwFp16Qkv", "2", {{"bundle_sha256", nullptr, LFFW_FIELD_CHAR, 64}}},
        {Kind::Fc1, "LffwFp16Fc1", "1", {{"bundle_sha256", nullptr, LFFW_FIELD_CHAR, 64}}},
        {Kind::Fp8Linear, "LffwFp8Linear", "1",
         {{"bundle_sha256", nullptr, LFFW_FIELD_CHAR, 64},
          {"act_scale", nullptr, LFFW_FIELD_FLOAT32, 1},
          {"epilogue", nullptr, LFFW_FIELD_INT32, 1},
          {"output_scale", nullptr, LFFW_FIELD_FLOAT32, 1},
          {"has_bias", nullptr, LFFW_FIELD_INT32, 1}}},
    };
    return list;
}

struct FieldValue {
    std::string name;
    int32_t type;
    int32_t length;
    std::vector<uint8_t> bytes;
};

size_t field_element_size(int32_t type)
{
    switch (type) {
    case LFFW_FIELD_FLOAT16: return 2;
    case LFFW_FIELD_FLOAT32: return 4;
    case LFFW_FIELD_FLOAT64: return 8;
    case LFFW_FIELD_INT8: return 1;
    case LFFW_FIELD_INT16: return 2;
    case LFFW_FIELD_INT32: return 4;
    case LFFW_FIELD_CHAR: return 1;
    default: return 0;
    }
}

// Copy and check a field collection: names present and unique, data present,
// known element type.
bool parse_fields(const lffw_plugin_field *fields, int32_t count, std::vector<FieldValue> &out)
{
    if (count < 0 || (count > 0 && fields == nullptr))
        return false;
    for (int32_t i = 0; i < count; ++i) {
        const lffw_plugin_field &f = fields[i];
        const size_t elem = field_element_size(f.type);
        if (f.name == nullptr || f.data == nullptr || f.length < 0 || elem == 0)
            return false;
        for (const FieldValue &seen : out)
            if (seen.name == f.name)
                return false;
        FieldValue v{f.name, f.type, f.length, {}};
        v.bytes.assign(static_cast<const uint8_t *>(f.data),
                       static_cast<const uint8_t *>(f.data) + elem * static_cast<size_t>(f.length));
        out.push_back(std::move(v));
    }
    return true;
}

const FieldValue *find_field(const std::vector<FieldValue> &fields, const char *name)
{
    for (const FieldValue &f : fields)
        if (f.name == name)
            return &f;
    return nullptr;
}

} // namespace

struct lffw_plugin {
    Kind kind;
    std::vector<FieldValue> fields;
    uint16_t bias_bits = 0;     // LffwFp16Bias
    float act_scale = 0.0f;     // LffwFp8Linear
    int32_t epilogue = 0;       // LffwFp8Linear
    float output_scale = 0.0f;  // LffwFp8Linear: 0 -> fp16 output, > 0 -> E4M3 output
    int32_t has_bias = 0;       // LffwFp8Linear: 1 -> a 4th input holds the fp16 bias
};

namespace {

// Exactly the declared field set, with the library's own digest
// (cpp/fc1_plugin.cpp:32-37, cpp/plugin.cpp:33-41).
bool valid_fields(const CreatorInfo &info, lffw_plugin &plugin)
{
    const auto &fields = plugin.fields;
    if (fields.size() != info.fields.size())
        return false;
    for (const lffw_plugin_field &decl : info.fields) {
        const FieldValue *f = find_field(fields, decl.name);
        if (f == nullptr || f->type != decl.type || f->length != decl.length)
            return false;
    }
    const FieldValue *digest = find_field(fields, "bundle_sha256");
    if (std::memcmp(digest->bytes.data(), tensoracle_bundle_sha256, 64) != 0)
        return false;
    if (info.kind == Kind::Bias)
        std::memcpy(&plugin.bias_bits, find_field(fields, "bias")->bytes.data(), 2);
    if (info.kind == Kind::Fp8Linear) {
        std::memcpy(&plugin.act_scale, find_field(fields, "act_scale")->bytes.data(), 4);
        std::memcpy(&plugin.epilogue, find_field(fields, "epilogue")->bytes.data(), 4);
        std::memcpy(&plugin.output_scale, find_field(fields, "output_scale")->bytes.data(), 4);
        std::memcpy(&plugin.has_bias, find_field(fields, "has_bias")->bytes.data(), 4);
        if (plugin.has_bias != 0 && plugin.has_bias != 1)
            return false;
        if (!valid_scale(plugin.act_scale)) // network_graph.cpp:137-139 (+ normal reciprocal)
            return false;
        if (plugin.epilogue != LFFW_EPILOGUE_NONE && plugin.epilogue != LFFW_EPILOGUE_GELU)
            return false;
        if (!(plugin.output_scale == 0.0f || valid_scale(plugin.output_scale)))
            return false;
    }
    return true;
}

bool is(const lffw_tensor_desc &d, int32_t type)
{
    return d.type == type && d.format == LFFW_FORMAT_LINEAR;
}

bool dims_are(const lffw_tensor_desc &d, std::initializer_list<int64_t> expect)
{
    if (d.nb_dims != static_cast<int32_t>(expect.size()))
        return false;
    int i = 0;
    for (int64_t e : expect)
        if (d.dims[i++] != e)
            return false;
    return true;
}

int64_t rows_of(const lffw_tensor_desc &d)
{
    int64_t rows = 1;
    for (int i = 0; i + 1 < d.nb_dims; ++i)
        rows *= d.dims[i];
    return rows;
}

// The FP8 linear's accepted inputs: x HALF or FP8 [..., K] (rank 2-3),
// weight FP8 [N, K], weight scales FLOAT [N], optional bias HALF [N];
// output HALF (output_scale == 0) or FP8 (> 0) with x's leading dims and N.
int32_t validate_fp8_linear(const lffw_plugin &p, const lffw_tensor_desc *in, int32_t count,
                            const lffw_tensor_desc &out)
{
    if (count != 3 + p.has_bias)
        return -1;
    const lffw_tensor_desc &x = in[0], &w = in[1], &s = in[2];
    if (!(is(x, LFFW_DT_HALF) || is(x, LFFW_DT_FP8)) || x.nb_dims < 2 || x.nb_dims > 3)
        return -1;
    if (!is(w, LFFW_DT_FP8) || w.nb_dims != 2 || !is(s, LFFW_DT_FLOAT) || s.nb_dims != 1)
        return -1;
    const int64_t k = x.dims[x.nb_dims - 1], n = w.dims[0];
    if (w.dims[1] != k || s.dims[0] != n || k < 16 || n < 16 || k % 16 || n % 16)
        return -1;
    for (int i = 0; i < x.nb_dims; ++i)
        if (x.dims[i] < 1)
            return -1;
    if (count == 4 && (!is(in[3], LFFW_DT_HALF) || !dims_are(in[3], {n})))
        return -1;
    if (!is(out, p.output_scale > 0.0f ? LFFW_DT_FP8 : LFFW_DT_HALF) || out.nb_dims != x.nb_dims)
        return -1;
    for (int i = 0; i + 1 < x.nb_dims; ++i)
        if (out.dims[i] != x.dims[i])
            return -1;
    if (out.dims[out.nb_dims - 1] != n || rows_of(x) > kMaxDim)
        return -1;
    return 0;
}

int32_t validate(const lffw_plugin &p, const lffw_tensor_desc *in, int32_t count,
                 const lffw_tensor_desc *out)
{
    if (in == nullptr || out == nullptr)
        return -1;
    switch (p.kind) {
    case Kind::Fc1: // cpp/fc1_plugin.cpp:108-119
        if (count != 3)
            return -1;
        for (int i = 0; i < 3; ++i)
            if (!is(in[i], LFFW_DT_HALF))
                return -1;
        return is(*out, LFFW_DT_HALF) && dims_are(in[0], {1, 1, kWidth}) &&
                       dims_are(in[1], {kFc1Output, kWidth}) && dims_are(in[2], {kFc1Output}) &&
                       dims_are(*out, {1, 1, kFc1Output})
                   ? 0
                   : -1;
    case Kind::Qkv: // cpp/qkv_plugin.cpp:109-120
        if (count != 4)
            return -1;
        for (int i = 0; i < 4; ++i)
            if (!is(in[i], LFFW_DT_HALF))
                return -1;
        return is(*out, LFFW_DT_HALF) && dims_are(in[0], {1, 1, kWidth}) &&
                       dims_are(in[1], {3 * kWidth, kWidth}) && dims_are(in[2], {kWidth}) &&
                       dims_are(in[3], {kWidth}) && dims_are(*out, {1, 1, 3 * kWidth})
                   ? 0
                   : -1;
    case Kind::Bias: { // cpp/plugin.cpp:95-106 (-1 = dynamic length)
        if (count != 1 || !is(in[0], LFFW_DT_HALF) || !is(*out, LFFW_DT_HALF) || in[0].nb_dims != 1 ||
            out->nb_dims != 1)
            return -1;
        auto valid = [](int64_t length) { return length == -1 || (length > 0 && length <= kMaxDim); };
        const int64_t source = in[0].dims[0], target = out->dims[0];
        return valid(source) && valid(target) && (source == -1 || target == -1 || source == target) ? 0 : -1;
    }
    case Kind::Fp8Linear:
        return validate_fp8_linear(p, in, count, *out);
    }
    return -1;
}

int64_t workspace_bytes(const lffw_plugin &p, const lffw_tensor_desc *in, int32_t count)
{
    if (p.kind != Kind::Fp8Linear || in == nullptr || count < 1 || in[0].type != LFFW_DT_HALF)
        return 0;
    const int64_t bytes = rows_of(in[0]) * in[0].dims[in[0].nb_dims - 1];
    return (bytes + 255) / 256 * 256;
}

int32_t input_count(const lffw_plugin &p, const lffw_tensor_desc *in)
{
    switch (p.kind) {
    case Kind::Fc1: return 3;
    case Kind::Qkv: return 4;
    case Kind::Bias: return 1;
    case Kind::Fp8Linear: return 3 + p.has_bias;
    }
    (void)in;
    return 0;
}

} // namespace

extern "C" {

int32_t lffw_plugin_creator_count(void) noexcept { return static_cast<int32_t>(creators().size()); }

int32_t lffw_plugin_creator(int32_t index, const char **name, const char **version,
                            const char **plugin_namespace, const lffw_plugin_field **fields,
                            int32_t *field_count) noexcept
{
    if (index < 0 || index >= lffw_plugin_creator_count())
        return -1;
    const CreatorInfo &info = creators()[index];
    if (name)
        *name = info.name;
    if (version)
        *version = info.version;
    if (plugin_namespace)
        *plugin_namespace = kNamespace;
    if (fields)
        *fields = info.fields.data();
    if (field_count)
        *field_count = static_cast<int32_t>(info.fields.size());
    return 0;
}

lffw_plugin *lffw_plugin_create(const char *name, const char *version, const char *plugin_namespace,
                                const lffw_plugin_field *fields, int32_t count, int32_t phase) noexcept
{
    if (name == nullptr || version == nullptr || plugin_namespace == nullptr)
        return nullptr;
    if (phase != LFFW_PHASE_BUILD && phase != LFFW_PHASE_RUNTIME)
        return nullptr;
    if (std::strcmp(plugin_namespace, kNamespace) != 0)
        return nullptr;
    try {
        for (const CreatorInfo &info : creators()) {
            if (std::strcmp(info.name, name) != 0 || std::strcmp(info.version, version) != 0)
                continue;
            auto *plugin = new lffw_plugin{};
            plugin->kind = info.kind;
            if (!parse_fields(fields, count, plugin->fields) || !valid_fields(info, *plugin)) {
                delete plugin;
                return nullptr;
            }
            return plugin;
        }
    } catch (...) {
    }
    return nullptr;
}

lffw_plugin *lffw_plugin_clone(const lffw_plugin *plugin) noexcept
{
    if (plugin == nullptr)
        return nullptr;
    try {
        return new lffw_plugin(*plugin);
    } catch (...) {
        return nullptr;
    }
}

void lffw_plugin_destroy(lffw_plugin *plugin) noexcept { delete plugin; }

int32_t lffw_plugin_validate(const lffw_plugin *plugin, const lffw_tensor_desc *inputs,
                             int32_t count, const lffw_tensor_desc *output) noexcept
{
    if (plugin == nullptr)
        return -1;
    return validate(*plugin, inputs, count, output);
}

int64_t lffw_plugin_workspace_size(const lffw_plugin *plugin, const lffw_tensor_desc *inputs,
                                   int32_t count) noexcept
{
    if (plugin == nullptr)
        return 0;
    return workspace_bytes(*plugin, inputs, count);
}

int32_t lffw_plugin_enqueue(const lffw_plugin *plugin, const lffw_tensor_desc *input_desc,
                            const lffw_tensor_desc *output_desc, const void *const *inputs,
                            void *const *outputs, void *workspace, void *stream) noexcept
{
    if (plugin == nullptr || input_desc == nullptr || output_desc == nullptr || inputs == nullptr ||
        outputs == nullptr || outputs[0] == nullptr)
        return -1;
    const lffw_plugin &p = *plugin;
    const int32_t count = input_count(p, input_desc);
    for (int32_t i = 0; i < count; ++i)
        if (inputs[i] == nullptr)
            return -1;
    if (validate(p, input_desc, count, output_desc) != 0)
        return -1;
    if (p.kind == Kind::Bias && input_desc[0].dims[0] < 1)
        return -1;
    if (current_device_gate() != LFFW_SUCCESS)
        return -1;
    auto h = [](const void *ptr) { return static_cast<const uint16_t *>(ptr); };
    lffw_status s = LFFW_INTERNAL_ERROR;
    switch (p.kind) {
    case Kind::Fc1:
        s = lffw_fp16_fc1(h(inputs[0]), h(inputs[1]), h(inputs[2]), static_cast<uint16_t *>(outputs[0]),
                          kFc1Output, kWidth, stream);
        break;
    case Kind::Qkv:
        s = lffw_fp16_qkv(h(inputs[0]), h(inputs[1]), h(inputs[2]), h(inputs[3]),
                          static_cast<uint16_t *>(outputs[0]), kWidth, stream);
        break;
    case Kind::Bias:
        s = lffw_fp16_bias(h(inputs[0]), p.bias_bits, static_cast<uint16_t *>(outputs[0]),
                           input_desc[0].dims[0], stream);
        break;
    case Kind::Fp8Linear: {
        const lffw_tensor_desc &x = input_desc[0];
        const int64_t m = rows_of(x), k = x.dims[x.nb_dims - 1];
        const uint8_t *codes = static_cast<const uint8_t *>(inputs[0]);
        if (x.type == LFFW_DT_HALF) {
            if (workspace == nullptr)
                return -1;
            s = lffw_fp8_quantize(h(inputs[0]), m * k, p.act_scale, nullptr,
                                  static_cast<uint8_t *>(workspace), stream);
            if (s != LFFW_SUCCESS)
                return -1;
            codes = static_cast<const uint8_t *>(workspace);
        }
        lffw_fp8_linear_args a{};
        a.struct_size = sizeof(a);
        a.m = m;
        a.n = input_desc[1].dims[0];
        a.k = k;
        a.x_codes = codes;
        a.act_scale = p.act_scale;
        a.w_codes = static_cast<const uint8_t *>(inputs[1]);
        a.w_scales = static_cast<const float *>(inputs[2]);
        a.bias = count == 4 ? h(inputs[3]) : nullptr;
        a.epilogue = p.epilogue;
        if (p.output_scale > 0.0f) {
            a.next_scale = p.output_scale;
            a.next_codes = static_cast<uint8_t *>(outputs[0]);
        } else {
            a.y = static_cast<uint16_t *>(outputs[0]);
        }
        s = lffw_fp8_linear(&a, stream);
        break;
    }
    }
    return s == LFFW_SUCCESS ? 0 : -1;
}

} // extern "C"
