// Launchers for the reference's own fp16 projection kernels (cpp/kernels.cu,
// compiled from where it lies in the reference tree by oracle/Makefile with the
// constants its cubin bundle uses: WIDTH 1280, ROWS 4, DEPTH 2048, OUTPUT 5120
// for fc1; cpp/kernels.py:24-47).  BENCHMARK AND TEST INFRASTRUCTURE ONLY: the
// same-box baseline for lffw_fp16_fc1 / lffw_fp16_qkv; never linked by the product.
// Geometry as the plugins launch them: 128 threads, four output rows per block
// (cpp/fc1_plugin.cpp:105, cpp/qkv_plugin.cpp:105).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

extern "C" __global__ void qkv_fp16(half const *x_ptr, half const *weight_ptr, half const *q_bias_ptr,
                                    half const *v_bias_ptr, half *out_ptr);
extern "C" __global__ void fc1_fp16(half const *x_ptr, half const *weight_ptr, half const *bias_ptr, half *out_ptr);

extern "C" {

int ref_qkv_fp16_launch(const void *x, const void *weight, const void *q_bias, const void *v_bias, void *out,
                        void *stream)
{
    qkv_fp16<<<3 * 1280 / 4, 128, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const half *>(x), static_cast<const half *>(weight), static_cast<const half *>(q_bias),
        static_cast<const half *>(v_bias), static_cast<half *>(out));
    return static_cast<int>(cudaGetLastError());
}

int ref_fc1_fp16_launch(const void *x, const void *weight, const void *bias, void *out, void *stream)
{
    fc1_fp16<<<5120 / 4, 128, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const half *>(x), static_cast<const half *>(weight), static_cast<const half *>(bias),
        static_cast<half *>(out));
    return static_cast<int>(cudaGetLastError());
}

} // extern "C"
