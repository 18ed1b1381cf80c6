// C ABI around the reference's own CPU model of its fp16 projection plugins
// (cpp/tests/kernel_reference.hpp, compiled from where it lies in the
// reference tree).  TEST INFRASTRUCTURE ONLY: used to pin the oracle and to
// regenerate tests/golden/fp16_plugins.npz; never linked by the product.
#include "kernel_reference.hpp"

#include <algorithm>
#include <cstdint>

extern "C" {

// Fills the reference test's seeded data (mt19937(3318), kernel_reference.hpp:28-35)
// and its expected outputs (kernel_reference.hpp:36-50).  Buffers: x[1280],
// weight[rows*1280], bias[fc1 ? rows : 1280], v_bias[1280] (qkv only), expected[rows].
int ref_fp16_projection(int fc1, uint16_t *x, uint16_t *weight, uint16_t *bias, uint16_t *v_bias,
                        double *expected)
{
    lffw_test::Projection data(fc1 != 0);
    std::copy(data.x.begin(), data.x.end(), x);
    std::copy(data.weight.begin(), data.weight.end(), weight);
    std::copy(data.bias.begin(), data.bias.end(), bias);
    if (!fc1)
        std::copy(data.v_bias.begin(), data.v_bias.end(), v_bias);
    auto result = data.reference(fc1 != 0);
    std::copy(result.begin(), result.end(), expected);
    return data.rows;
}

// The reference's fp16-edge GELU applied to (dot, bias) (kernel_reference.hpp:20-25).
double ref_gelu(double dot, double bias) { return lffw_test::gelu(dot, bias); }

// The reference's IEEE-half rounding (kernel_reference.hpp:11-19).
uint16_t ref_half_bits(double value) { return lffw_test::half_bits(value); }
}
