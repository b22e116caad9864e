// The 16 KERNIX activations as device functions, shared by the GEMM/conv epilogues and the standalone
// activation kernel. Formulas and evaluation order follow the reference's kernix_act_chunk
// (include/kernix_model.h:468-517), which src/kernix_metal.m's bias_act kernel (:269-299) mirrors.
// Products and sums use explicit round-to-nearest intrinsics so that the compiler cannot contract them
// into fused multiply-adds; exp/tanh/expm1/log1p are CUDA's accurate library functions (max ~2 ulp), so
// results agree with the CPU reference to a few ulp, not bit for bit.
#pragma once
#include <cmath>

namespace kx {

enum {
    ACT_NONE = -1, ACT_RELU, ACT_GELU, ACT_SILU, ACT_SIGMOID, ACT_TANH, ACT_LEAKY_RELU, ACT_ELU, ACT_SELU,
    ACT_SOFTPLUS, ACT_RELU6, ACT_HARD_SIGMOID, ACT_HARD_SWISH, ACT_GELU_TANH, ACT_EXP, ACT_MISH, ACT_SOFTSIGN
};

__device__ __forceinline__ float relu6f(float v) { return v < 0.0f ? 0.0f : (v > 6.0f ? 6.0f : v); }
__device__ __forceinline__ float softplusf(float v) { return v > 20.0f ? v : log1pf(expf(v)); }

// GELU with the Abramowitz-Stegun 7.1.26 erf approximation (reference :485-496)
__device__ __forceinline__ float gelu_as(float x) {
    const float z = __fmul_rn(x, 0.70710678f);
    const float t = expf(__fmul_rn(-z, z));
    const float za = __fmul_rn(fabsf(x), 0.70710678f);
    const float k = __frcp_rn(__fadd_rn(1.0f, __fmul_rn(0.3275911f, za)));  // == 1 / d, correctly rounded
    float p = __fadd_rn(-1.453152027f, __fmul_rn(k, 1.061405429f));
    p = __fadd_rn(1.421413741f, __fmul_rn(k, p));
    p = __fadd_rn(-0.284496736f, __fmul_rn(k, p));
    p = __fadd_rn(0.254829592f, __fmul_rn(k, p));
    p = __fmul_rn(k, p);
    const float e = __fsub_rn(1.0f, __fmul_rn(p, t));
    return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, x < 0.0f ? -e : e));
}

__device__ __forceinline__ float sigmoidf_ref(float x) {
    return __frcp_rn(__fadd_rn(expf(-x), 1.0f));  // == 1 / d, correctly rounded
}

__device__ __forceinline__ float act_apply(int act, float x, float alpha) {
    switch (act) {
    case ACT_RELU: return x < 0.0f ? 0.0f : x;
    case ACT_GELU: return gelu_as(x);
    case ACT_SILU: return __fmul_rn(x, sigmoidf_ref(x));
    case ACT_SIGMOID: return sigmoidf_ref(x);
    case ACT_TANH: return tanhf(x);
    case ACT_LEAKY_RELU: return x < 0.0f ? __fmul_rn(alpha, x) : x;
    case ACT_ELU: return x < 0.0f ? __fmul_rn(alpha, expm1f(x)) : x;
    case ACT_SELU: return __fmul_rn(1.0507009873554805f, x < 0.0f ? __fmul_rn(1.6732632423543772f, expm1f(x)) : x);
    case ACT_SOFTPLUS: return softplusf(x);
    case ACT_RELU6: return relu6f(x);
    case ACT_HARD_SIGMOID: return __fdiv_rn(relu6f(__fadd_rn(x, 3.0f)), 6.0f);
    case ACT_HARD_SWISH: return __fdiv_rn(__fmul_rn(x, relu6f(__fadd_rn(x, 3.0f))), 6.0f);
    case ACT_GELU_TANH: {
        const float c = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, x), x), x);
        const float in = __fmul_rn(0.7978845608028654f, __fadd_rn(x, c));
        return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, tanhf(in)));
    }
    case ACT_EXP: return expf(x);
    case ACT_MISH: return __fmul_rn(x, tanhf(softplusf(x)));
    case ACT_SOFTSIGN: return __fdiv_rn(x, __fadd_rn(1.0f, fabsf(x)));
    default: return x;
    }
}

}  // namespace kx
