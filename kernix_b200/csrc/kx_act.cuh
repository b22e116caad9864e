// The 16 KERNIX activations as device functions, shared by the GEMM/conv epilogues and the standalone
// activation kernel. Formulas and evaluation order follow the reference's kernix_act_chunk
// (include/kernix_model.h:468-517), which src/kernix_metal.m's bias_act kernel (:269-299) mirrors.
// Products and sums use explicit round-to-nearest intrinsics so that the compiler cannot contract them
// into fused multiply-adds; exp/tanh/expm1/log1p are CUDA's accurate library functions (max ~2 ulp), so
// results agree with the CPU reference to a few ulp, not bit for bit. GELU is the exception (see gelu_as).
#pragma once
#include <cmath>

namespace kx {

enum {
    ACT_NONE = -1, ACT_RELU, ACT_GELU, ACT_SILU, ACT_SIGMOID, ACT_TANH, ACT_LEAKY_RELU, ACT_ELU, ACT_SELU,
    ACT_SOFTPLUS, ACT_RELU6, ACT_HARD_SIGMOID, ACT_HARD_SWISH, ACT_GELU_TANH, ACT_EXP, ACT_MISH, ACT_SOFTSIGN
};

__device__ __forceinline__ float relu6f(float v) { return v < 0.0f ? 0.0f : (v > 6.0f ? 6.0f : v); }
__device__ __forceinline__ float softplusf(float v) { return v > 20.0f ? v : log1pf(expf(v)); }

// Hardware approximations used by GELU: 2^a (ex2.approx) and 1/d (rcp.approx), both about 2 ulp.
__device__ __forceinline__ float ex2_approx(float a) {
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(a));
    return r;
}
__device__ __forceinline__ float rcp_approx(float d) {
    float r;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(d));
    return r;
}
__device__ __forceinline__ float2 f2(float v) { return make_float2(v, v); }

// max(m, |v|) on the bit patterns of non-negative floats (m: a previous result, 0 at first), NaN winning over every
// number (its bits exceed +inf's): one float max with NaN propagation instead of an and and an integer max
__device__ __forceinline__ uint32_t absmax_nan(uint32_t m, float v) {
    float r;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(__uint_as_float(m)), "f"(fabsf(v)));
    return __float_as_uint(r);
}

// Packed f32x2 arithmetic (sm_100): each component rounded to nearest like the scalar operation. The code
// generator may still contract a packed mul followed by a packed add into one fma (measured), so chains of
// these are not bitwise equal to chains of scalar __fmul_rn / __fadd_rn; exact dequantisation stays scalar.
__device__ __forceinline__ uint64_t pk2(float2 a) {
    return static_cast<uint64_t>(__float_as_uint(a.x)) | (static_cast<uint64_t>(__float_as_uint(a.y)) << 32);
}
__device__ __forceinline__ float2 upk2(uint64_t r) {
    return make_float2(__uint_as_float(static_cast<uint32_t>(r)), __uint_as_float(static_cast<uint32_t>(r >> 32)));
}
__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
    uint64_t r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(pk2(a)), "l"(pk2(b)));
    return upk2(r);
}
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(pk2(a)), "l"(pk2(b)));
    return upk2(r);
}
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(pk2(a)), "l"(pk2(b)), "l"(pk2(c)));
    return upk2(r);
}

// GELU with the Abramowitz-Stegun 7.1.26 erf approximation (reference :485-496): the same formula and
// constants, GELU(x) = x/2 (1 + sign(x) e) with e = 1 - k p(k) exp(-z^2), z = x/sqrt(2), k = 1/(1 + 0.3275911|z|),
// evaluated with fused multiply-adds, exp(-z^2) = 2^(-x^2 log2(e) / 2) on the hardware exp2 unit and the hardware
// reciprocal -- about 10 instructions per value instead of about 50 with correctly rounded steps. The constants
// of z are folded into the two uses of x (-x^2 log2(e)/2 and 0.3275911/sqrt(2) |x|), and sign(x) e is e with x's sign
// bit. The result differs from a step-by-step IEEE evaluation by at most about 1e-6 relative (GELU runs in the
// epilogue of every hidden layer of the int8 and Transformer configurations, where it bounds the epilogue's issue
// rate); the parity tests bound the end-to-end effect. +inf gives +inf and -inf NaN, as the reference's formula.
// gelu_as2 computes two GELUs with packed f32x2 arithmetic, the same steps as gelu_as.
__device__ __forceinline__ float sign_of(float v, float x) {  // |v| with the sign bit of x (v >= 0)
    return __int_as_float(__float_as_int(v) ^ (__float_as_int(x) & 0x80000000));
}
__device__ __forceinline__ float gelu_as(float x) {
    const float h = __fmul_rn(0.5f, x);
    const float t = ex2_approx(__fmul_rn(__fmul_rn(x, -0.72134752f), x));
    const float k = rcp_approx(__fmaf_rn(fabsf(x), 0.23164189f, 1.0f));
    float q = __fmaf_rn(k, -1.061405429f, 1.453152027f);
    q = __fmaf_rn(k, q, -1.421413741f);
    q = __fmaf_rn(k, q, 0.284496736f);
    q = __fmaf_rn(k, q, -0.254829592f);
    const float e = __fmaf_rn(__fmul_rn(k, q), t, 1.0f);  // 1 - k p(k) exp(-z^2), in [0, 1]
    return __fmul_rn(h, __fadd_rn(1.0f, sign_of(e, x)));
}
__device__ __forceinline__ float2 gelu_as2(float2 x) {
    const float2 h = mul2(x, f2(0.5f));
    const float2 a = mul2(mul2(x, f2(-0.72134752f)), x);
    const float2 t = make_float2(ex2_approx(a.x), ex2_approx(a.y));
    const float2 d = fma2(make_float2(fabsf(x.x), fabsf(x.y)), f2(0.23164189f), f2(1.0f));
    const float2 k = make_float2(rcp_approx(d.x), rcp_approx(d.y));
    float2 q = fma2(k, f2(-1.061405429f), f2(1.453152027f));
    q = fma2(k, q, f2(-1.421413741f));
    q = fma2(k, q, f2(0.284496736f));
    q = fma2(k, q, f2(-0.254829592f));
    const float2 e = fma2(mul2(k, q), t, f2(1.0f));
    return mul2(h, add2(f2(1.0f), make_float2(sign_of(e.x, x.x), sign_of(e.y, x.y))));
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
