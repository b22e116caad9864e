// KERNIX-B200 memory-bound graph ops, the int8 row quantiser, depthwise conv, attention core and fma_relu.
// Each kernel restates one reference computation (named on its kx_* entry in include/kx_kernels.h) with
// coalesced, vectorised (float4) accesses; row ops use one warp per row up to 1024 columns and one
// 256-thread block per row above that.
#include <cuda_runtime.h>

#include <cfloat>
#include <cmath>
#include <cstdint>

#include "kx_act.cuh"
#include "kx_kernels.h"
#include "kx_pdl.cuh"

namespace {

inline int launch_ok() { return cudaGetLastError() == cudaSuccess ? 0 : -1; }

inline unsigned grid_for(long n, int per_block) {
    long g = (n + per_block - 1) / per_block;
    if (g > 148L * 64) g = 148L * 64;  // grid-stride loops above this
    return static_cast<unsigned>(g < 1 ? 1 : g);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float u = __shfl_xor_sync(0xffffffffu, v, o);
        v = u > v ? u : v;
    }
    return v;
}
__device__ __forceinline__ uint32_t warp_umax(uint32_t v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// ---------------------------------------------------------------------------------- int8 quantise
// One 128-thread block per row. max|x| is reduced on the IEEE bit patterns of |x| (non-negative floats order
// like their bits; NaN > inf > finite), so a NaN anywhere makes the row's max NaN as in the reference.
// y = act(P[0] + P[1] + ... + bias) over m x n, planes P[z] of m x n floats added in plane order (split-K partial sums)
__global__ void k_add_planes(const float* __restrict__ part, int planes, int m, int n, const float* __restrict__ bias, int act,
                             float alpha, float* __restrict__ y, int ldy) {
    const long total = static_cast<long>(m) * n, plane = total;
    for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < total; i += static_cast<long>(gridDim.x) * blockDim.x) {
        float v[KX_SPLITK_MAX];
#pragma unroll
        for (int z = 0; z < KX_SPLITK_MAX; z++)
            if (z < planes) v[z] = __ldcg(part + z * plane + i);
        float s = v[0];
#pragma unroll
        for (int z = 1; z < KX_SPLITK_MAX; z++)
            if (z < planes) s = __fadd_rn(s, v[z]);
        const long r = i / n;
        const int c = static_cast<int>(i - r * n);
        if (bias) s = __fadd_rn(s, __ldg(bias + c));
        y[r * ldy + c] = kx::act_apply(act, s, alpha);
    }
}

constexpr int QT = 128;
constexpr int QV = 8;  // float4 per thread kept in registers (rows up to 4096 columns in one read)

__global__ void __launch_bounds__(QT) k_quant_rows(const float* __restrict__ x, int ldx, int k, int8_t* __restrict__ xq,
                                                   int ldq, float* __restrict__ sx, uint32_t* __restrict__ zero,
                                                   int zero_words) {
    kx::griddep_wait();  // launched as a dependent of the kernel before it: x is its output
    kx::griddep_launch_dependents();
    for (int i = blockIdx.x * QT + threadIdx.x; i < zero_words; i += gridDim.x * QT) zero[i] = 0;  // the next launch's counters
    const long row = blockIdx.x;
    const float* xr = x + row * ldx;
    int8_t* qr = xq + row * ldq;
    const bool vec = ((ldx & 3) == 0) && ((reinterpret_cast<uintptr_t>(x) & 15) == 0) && ((k & 3) == 0);
    __shared__ uint32_t red[QT / 32];
    __shared__ float s_inv;
    __shared__ float s_sx;
    float4 v[QV];
    uint32_t m = 0;
    const int nvec = vec ? (k >> 2) : 0;
#pragma unroll
    for (int i = 0; i < QV; i++) {
        const int c = threadIdx.x + i * QT;
        v[i] = c < nvec ? __ldg(reinterpret_cast<const float4*>(xr) + c) : make_float4(0.f, 0.f, 0.f, 0.f);
        m = max(m, max(max(__float_as_uint(fabsf(v[i].x)), __float_as_uint(fabsf(v[i].y))),
                       max(__float_as_uint(fabsf(v[i].z)), __float_as_uint(fabsf(v[i].w)))));
    }
    for (int c = threadIdx.x + QV * QT; c < nvec; c += QT) {  // columns beyond the register window
        const float4 t = __ldg(reinterpret_cast<const float4*>(xr) + c);
        m = max(m, max(max(__float_as_uint(fabsf(t.x)), __float_as_uint(fabsf(t.y))),
                       max(__float_as_uint(fabsf(t.z)), __float_as_uint(fabsf(t.w)))));
    }
    if (!vec)
        for (int c = threadIdx.x; c < k; c += QT) m = max(m, __float_as_uint(fabsf(__ldg(xr + c))));
    m = warp_umax(m);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t mm = red[0];
        for (int i = 1; i < QT / 32; i++) mm = max(mm, red[i]);
        const float mf = __uint_as_float(mm);
        if (mm >= 0x7F800000u) {  // NaN or infinite: the whole output row is NaN
            s_sx = __uint_as_float(0x7FC00000u);
            s_inv = 0.0f;
        } else {
            const float sxv = mf > 0.0f ? __fdiv_rn(mf, 127.0f) : 1.0f;
            s_sx = sxv;
            s_inv = __fdiv_rn(1.0f, sxv);
        }
        sx[row] = s_sx;
    }
    __syncthreads();
    const float inv = s_inv;
    auto q1 = [&](float a) -> int {
        float t = rintf(__fmul_rn(a, inv));
        t = t > 127.0f ? 127.0f : (t < -127.0f ? -127.0f : t);
        return t == t ? static_cast<int>(t) : 0;
    };
    if (vec) {
#pragma unroll
        for (int i = 0; i < QV; i++) {
            const int c = threadIdx.x + i * QT;
            if (c < nvec) {
                char4 o = make_char4(q1(v[i].x), q1(v[i].y), q1(v[i].z), q1(v[i].w));
                reinterpret_cast<char4*>(qr)[c] = o;
            }
        }
        for (int c = threadIdx.x + QV * QT; c < nvec; c += QT) {
            const float4 t = __ldg(reinterpret_cast<const float4*>(xr) + c);
            reinterpret_cast<char4*>(qr)[c] = make_char4(q1(t.x), q1(t.y), q1(t.z), q1(t.w));
        }
    } else {
        for (int c = threadIdx.x; c < k; c += QT) qr[c] = static_cast<int8_t>(q1(__ldg(xr + c)));
    }
    for (int c = k + threadIdx.x; c < ldq; c += QT) qr[c] = 0;
}

// ------------------------------------------------------------------------------------ bias + act
__global__ void k_bias_act(const float* x, float* y, long rows, int cols, const float* __restrict__ bias,
                           int act, float alpha) {
    const long n = rows * cols;
    const bool vec = (cols & 3) == 0;
    if (vec) {
        const long n4 = n >> 2;
        for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < n4; i += static_cast<long>(gridDim.x) * blockDim.x) {
            float4 v = reinterpret_cast<const float4*>(x)[i];
            const int c = static_cast<int>((i << 2) % cols);
            if (bias) {
                v.x = __fadd_rn(v.x, bias[c]);
                v.y = __fadd_rn(v.y, bias[c + 1]);
                v.z = __fadd_rn(v.z, bias[c + 2]);
                v.w = __fadd_rn(v.w, bias[c + 3]);
            }
            v.x = kx::act_apply(act, v.x, alpha);
            v.y = kx::act_apply(act, v.y, alpha);
            v.z = kx::act_apply(act, v.z, alpha);
            v.w = kx::act_apply(act, v.w, alpha);
            reinterpret_cast<float4*>(y)[i] = v;
        }
    } else {
        for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < n; i += static_cast<long>(gridDim.x) * blockDim.x) {
            float v = x[i];
            if (bias) v = __fadd_rn(v, bias[i % cols]);
            y[i] = kx::act_apply(act, v, alpha);
        }
    }
}

// ------------------------------------------------------------------------------------------ rows
// softmax: m = max (NaN-ignoring compare like vDSP_maxv), e = exp(x - m), s = sum e, y = e * (1/s)
template <int WARPS>
__global__ void k_softmax_warp(const float* x, float* y, long rows, int cols) {
    const long row = blockIdx.x * static_cast<long>(WARPS) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const float* xr = x + row * cols;
    float* yr = y + row * cols;
    float m = -INFINITY;
    for (int c = lane; c < cols; c += 32) {
        const float v = xr[c];
        m = v > m ? v : m;
    }
    m = warp_max(m);
    float s = 0.0f;
    for (int c = lane; c < cols; c += 32) {
        const float e = expf(__fsub_rn(xr[c], m));
        yr[c] = e;
        s = __fadd_rn(s, e);
    }
    s = warp_sum(s);
    const float inv = __fdiv_rn(1.0f, s);
    __syncwarp();
    for (int c = lane; c < cols; c += 32) yr[c] = __fmul_rn(yr[c], inv);
}

__global__ void k_softmax_block(const float* x, float* y, int cols) {
    const long row = blockIdx.x;
    const float* xr = x + row * cols;
    float* yr = y + row * cols;
    __shared__ float red[32];
    __shared__ float bc;
    float m = -INFINITY;
    for (int c = threadIdx.x; c < cols; c += blockDim.x) {
        const float v = xr[c];
        m = v > m ? v : m;
    }
    m = warp_max(m);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        float mm = red[0];
        for (int i = 1; i < static_cast<int>(blockDim.x >> 5); i++) mm = red[i] > mm ? red[i] : mm;
        bc = mm;
    }
    __syncthreads();
    m = bc;
    float s = 0.0f;
    for (int c = threadIdx.x; c < cols; c += blockDim.x) {
        const float e = expf(__fsub_rn(xr[c], m));
        yr[c] = e;
        s = __fadd_rn(s, e);
    }
    s = warp_sum(s);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        float ss = 0.0f;
        for (int i = 0; i < static_cast<int>(blockDim.x >> 5); i++) ss = __fadd_rn(ss, red[i]);
        bc = __fdiv_rn(1.0f, ss);
    }
    __syncthreads();
    const float inv = bc;
    for (int c = threadIdx.x; c < cols; c += blockDim.x) yr[c] = __fmul_rn(yr[c], inv);
}

// layer norm: mean = sum/cols, o = x - mean, rstd = 1/sqrt(sum(o^2)/cols + eps), y = o*rstd*g + b
template <int WARPS>
__global__ void k_layernorm_warp(const float* x, float* y, long rows, int cols, const float* __restrict__ g,
                                 const float* __restrict__ b, float eps) {
    const long row = blockIdx.x * static_cast<long>(WARPS) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const float* xr = x + row * cols;
    float* yr = y + row * cols;
    float s = 0.0f;
    for (int c = lane; c < cols; c += 32) s = __fadd_rn(s, xr[c]);
    const float mean = __fdiv_rn(warp_sum(s), static_cast<float>(cols));
    float ss = 0.0f;
    for (int c = lane; c < cols; c += 32) {
        const float o = __fsub_rn(xr[c], mean);
        ss = __fadd_rn(ss, __fmul_rn(o, o));
    }
    ss = warp_sum(ss);
    const float rstd = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(cols)), eps)));
    __syncwarp();
    for (int c = lane; c < cols; c += 32) {
        float o = __fmul_rn(__fsub_rn(xr[c], mean), rstd);
        if (g && b) o = __fadd_rn(__fmul_rn(o, g[c]), b[c]);
        else if (g) o = __fmul_rn(o, g[c]);
        else if (b) o = __fadd_rn(o, b[c]);
        yr[c] = o;
    }
}

__global__ void k_layernorm_block(const float* x, float* y, int cols, const float* __restrict__ g,
                                  const float* __restrict__ b, float eps) {
    const long row = blockIdx.x;
    const float* xr = x + row * cols;
    float* yr = y + row * cols;
    __shared__ float red[32];
    __shared__ float bc;
    const int nw = blockDim.x >> 5;
    float s = 0.0f;
    for (int c = threadIdx.x; c < cols; c += blockDim.x) s = __fadd_rn(s, xr[c]);
    s = warp_sum(s);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.0f;
        for (int i = 0; i < nw; i++) t = __fadd_rn(t, red[i]);
        bc = __fdiv_rn(t, static_cast<float>(cols));
    }
    __syncthreads();
    const float mean = bc;
    float ss = 0.0f;
    for (int c = threadIdx.x; c < cols; c += blockDim.x) {
        const float o = __fsub_rn(xr[c], mean);
        ss = __fadd_rn(ss, __fmul_rn(o, o));
    }
    ss = warp_sum(ss);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.0f;
        for (int i = 0; i < nw; i++) t = __fadd_rn(t, red[i]);
        bc = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, static_cast<float>(cols)), eps)));
    }
    __syncthreads();
    const float rstd = bc;
    for (int c = threadIdx.x; c < cols; c += blockDim.x) {
        float o = __fmul_rn(__fsub_rn(xr[c], mean), rstd);
        if (g && b) o = __fadd_rn(__fmul_rn(o, g[c]), b[c]);
        else if (g) o = __fmul_rn(o, g[c]);
        else if (b) o = __fadd_rn(o, b[c]);
        yr[c] = o;
    }
}

// ------------------------------------------------------------------------------ elementwise misc
__global__ void k_affine(const float* x, float* y, long n, int cols, const float* __restrict__ g,
                         const float* __restrict__ b) {
    for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < n; i += static_cast<long>(gridDim.x) * blockDim.x) {
        const int c = static_cast<int>(i % cols);
        y[i] = __fadd_rn(__fmul_rn(x[i], g[c]), b[c]);
    }
}

__global__ void k_add_const(const float* x, float* y, long n, long per, const float* __restrict__ cst) {
    for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < n; i += static_cast<long>(gridDim.x) * blockDim.x)
        y[i] = __fadd_rn(x[i], cst[i % per]);
}

__device__ __forceinline__ float bin1(int op, float a, float b) {
    switch (op) {
    case 0: return __fadd_rn(a, b);
    case 1: return __fsub_rn(a, b);
    case 2: return __fmul_rn(a, b);
    case 3: return __fdiv_rn(a, b);
    case 4: return a > b ? a : b;
    default: return a < b ? a : b;
    }
}

__global__ void k_binary(const float* a, int ra, int ca, const float* b, int rb, int cb, float* y,
                         long samples, int R, int C, int op) {
    const long n = samples * R * C;
    for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < n; i += static_cast<long>(gridDim.x) * blockDim.x) {
        const int c = static_cast<int>(i % C);
        const long rr = i / C;
        const int r = static_cast<int>(rr % R);
        const long s = rr / R;
        const float av = a[(s * ra + (ra == 1 ? 0 : r)) * ca + (ca == 1 ? 0 : c)];
        const float bv = b[(s * rb + (rb == 1 ? 0 : r)) * cb + (cb == 1 ? 0 : c)];
        y[i] = bin1(op, av, bv);
    }
}

__global__ void k_binary_same4(const float4* a, const float4* b, float4* y, long n4, int op) {
    for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < n4; i += static_cast<long>(gridDim.x) * blockDim.x) {
        const float4 u = a[i], v = b[i];
        y[i] = make_float4(bin1(op, u.x, v.x), bin1(op, u.y, v.y), bin1(op, u.z, v.z), bin1(op, u.w, v.w));
    }
}

// one thread per output (b, oy, ox, c); max starts at -inf, average multiplies by 1/count
__global__ void k_pool2d(const float* __restrict__ x, float* __restrict__ y, int B, int H, int W, int C, int Ho, int Wo,
                         int kh, int kw, int sh, int sw, int pt, int pl, int type, int count_pad) {
    const long n = static_cast<long>(B) * Ho * Wo * C;
    for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < n; i += static_cast<long>(gridDim.x) * blockDim.x) {
        const int c = static_cast<int>(i % C);
        long r = i / C;
        const int ox = static_cast<int>(r % Wo);
        r /= Wo;
        const int oy = static_cast<int>(r % Ho);
        const long b = r / Ho;
        float acc = type == 0 ? -INFINITY : 0.0f;
        int cnt = 0;
        for (int ky = 0; ky < kh; ky++) {
            const int iy = oy * sh - pt + ky;
            if (iy < 0 || iy >= H) continue;
            for (int kx2 = 0; kx2 < kw; kx2++) {
                const int ix = ox * sw - pl + kx2;
                if (ix < 0 || ix >= W) continue;
                const float v = x[((b * H + iy) * W + ix) * C + c];
                acc = type == 0 ? (acc > v ? acc : v) : __fadd_rn(acc, v);
                cnt++;
            }
        }
        if (type == 1) acc = __fmul_rn(acc, __fdiv_rn(1.0f, static_cast<float>(count_pad ? kh * kw : (cnt ? cnt : 1))));
        y[i] = acc;
    }
}

// the same windows four channels at a time (C % 4 == 0, 16-byte aligned rows, fewer than 2^31 float4 outputs):
// one float4 per thread with 32-bit index arithmetic; each component combines exactly as k_pool2d does
__global__ void k_pool2d_v4(const float4* __restrict__ x, float4* __restrict__ y, int B, int H, int W, int C4, int Ho, int Wo,
                            int kh, int kw, int sh, int sw, int pt, int pl, int type, int count_pad) {
    const int n = B * Ho * Wo * C4;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const int c = i % C4;
        int r = i / C4;
        const int ox = r % Wo;
        r /= Wo;
        const int oy = r % Ho;
        const int b = r / Ho;
        const float init = type == 0 ? -INFINITY : 0.0f;
        float4 acc = make_float4(init, init, init, init);
        int cnt = 0;
        for (int ky = 0; ky < kh; ky++) {
            const int iy = oy * sh - pt + ky;
            if (iy < 0 || iy >= H) continue;
            for (int kx2 = 0; kx2 < kw; kx2++) {
                const int ix = ox * sw - pl + kx2;
                if (ix < 0 || ix >= W) continue;
                const float4 v = __ldg(x + (static_cast<long>(b * H + iy) * W + ix) * C4 + c);
                if (type == 0) {
                    acc.x = acc.x > v.x ? acc.x : v.x;
                    acc.y = acc.y > v.y ? acc.y : v.y;
                    acc.z = acc.z > v.z ? acc.z : v.z;
                    acc.w = acc.w > v.w ? acc.w : v.w;
                } else {
                    acc.x = __fadd_rn(acc.x, v.x);
                    acc.y = __fadd_rn(acc.y, v.y);
                    acc.z = __fadd_rn(acc.z, v.z);
                    acc.w = __fadd_rn(acc.w, v.w);
                }
                cnt++;
            }
        }
        if (type == 1) {
            const float inv = __fdiv_rn(1.0f, static_cast<float>(count_pad ? kh * kw : (cnt ? cnt : 1)));
            acc = make_float4(__fmul_rn(acc.x, inv), __fmul_rn(acc.y, inv), __fmul_rn(acc.z, inv), __fmul_rn(acc.w, inv));
        }
        y[i] = acc;
    }
}

// sequential over the R rows of each sample, like the reference (first row copied, then combined)
__global__ void k_global_pool(const float* __restrict__ x, float* __restrict__ y, long B, int R, int C, int type) {
    const long n = B * C;
    for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < n; i += static_cast<long>(gridDim.x) * blockDim.x) {
        const int c = static_cast<int>(i % C);
        const long b = i / C;
        const float* xs = x + b * R * C + c;
        float acc = xs[0];
        for (int r = 1; r < R; r++) {
            const float v = xs[static_cast<long>(r) * C];
            acc = type == 0 ? (acc > v ? acc : v) : __fadd_rn(acc, v);
        }
        if (type == 1) acc = __fmul_rn(acc, __fdiv_rn(1.0f, static_cast<float>(R)));
        y[i] = acc;
    }
}

struct PermGeom {
    int nd;
    long od[4];   // output dims
    long ist[4];  // input stride of the input axis that feeds output axis k
    long per;
};

__global__ void k_permute(const float* __restrict__ x, float* __restrict__ y, long B, PermGeom g) {
    const long n = B * g.per;
    for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < n; i += static_cast<long>(gridDim.x) * blockDim.x) {
        const long b = i / g.per;
        long rem = i % g.per, src = 0;
        for (int k = g.nd - 1; k >= 0; k--) {
            src += (rem % g.od[k]) * g.ist[k];
            rem /= g.od[k];
        }
        y[i] = x[b * g.per + src];
    }
}

__global__ void k_copy_cols(const float* __restrict__ x, long ldx, float* __restrict__ y, long ldy, long yoff, long rows,
                            long cols) {
    const long n = rows * cols;
    for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < n; i += static_cast<long>(gridDim.x) * blockDim.x) {
        const long r = i / cols, c = i % cols;
        y[r * ldy + yoff + c] = x[r * ldx + c];
    }
}

__global__ void k_pad2d(const float* __restrict__ x, float* __restrict__ y, int B, int H, int W, int C, int Ho, int Wo,
                        int pt, int pl) {
    const long n = static_cast<long>(B) * Ho * Wo * C;
    for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < n; i += static_cast<long>(gridDim.x) * blockDim.x) {
        const int c = static_cast<int>(i % C);
        long r = i / C;
        const int ox = static_cast<int>(r % Wo);
        r /= Wo;
        const int oy = static_cast<int>(r % Ho);
        const long b = r / Ho;
        const int iy = oy - pt, ix = ox - pl;
        y[i] = (iy >= 0 && iy < H && ix >= 0 && ix < W) ? x[((b * H + iy) * W + ix) * C + c] : 0.0f;
    }
}

__global__ void k_upsample2d(const float* __restrict__ x, float* __restrict__ y, int B, int H, int W, int C, int Ho, int Wo,
                             int sh, int sw) {
    const long n = static_cast<long>(B) * Ho * Wo * C;
    for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < n; i += static_cast<long>(gridDim.x) * blockDim.x) {
        const int c = static_cast<int>(i % C);
        long r = i / C;
        const int ox = static_cast<int>(r % Wo);
        r /= Wo;
        const int oy = static_cast<int>(r % Ho);
        const long b = r / Ho;
        y[i] = x[((b * H + oy / sh) * W + ox / sw) * C + c];
    }
}

__global__ void k_embedding(const float* __restrict__ ids, long n, const float* __restrict__ table, int vocab, int dim,
                            float* __restrict__ y) {
    const long total = n * dim;
    for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < total; i += static_cast<long>(gridDim.x) * blockDim.x) {
        const long t = i / dim;
        const int d = static_cast<int>(i % dim);
        const float id = ids[t];
        y[i] = (id >= 0.0f && id < static_cast<float>(vocab) && id == floorf(id)) ? table[static_cast<long>(id) * dim + d]
                                                                                   : __uint_as_float(0x7FC00000u);
    }
}

// depthwise: output channel co = ci*mult + mi reads input channel ci; out = bias then += x*w per valid tap
__global__ void k_conv_dw(const float* __restrict__ x, const float* __restrict__ w, const float* __restrict__ bias,
                          float* __restrict__ y, int B, int H, int W, int C, int Co, int Ho, int Wo, int kh, int kw, int sh,
                          int sw, int dh, int dw, int pt, int pl, int act, float alpha) {
    const long n = static_cast<long>(B) * Ho * Wo * Co;
    const int mult = Co / C;
    for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < n; i += static_cast<long>(gridDim.x) * blockDim.x) {
        const int co = static_cast<int>(i % Co);
        long r = i / Co;
        const int ox = static_cast<int>(r % Wo);
        r /= Wo;
        const int oy = static_cast<int>(r % Ho);
        const long b = r / Ho;
        const int ci = co / mult;
        float acc = bias ? bias[co] : 0.0f;
        for (int ky = 0; ky < kh; ky++) {
            const int iy = oy * sh - pt + ky * dh;
            if (iy < 0 || iy >= H) continue;
            for (int kx2 = 0; kx2 < kw; kx2++) {
                const int ix = ox * sw - pl + kx2 * dw;
                if (ix < 0 || ix >= W) continue;
                acc = __fadd_rn(__fmul_rn(x[((b * H + iy) * W + ix) * C + ci], w[(ky * kw + kx2) * Co + co]), acc);
            }
        }
        y[i] = kx::act_apply(act, acc, alpha);
    }
}

// ----------------------------------------------------------------------------------- attention
// One block per (sample, head, tile of T query rows); one thread per query row. Scores for the thread's row
// live in shared memory (transposed so that a key index is one bank row), K/V stream through shared memory
// in chunks of KC keys. Two passes over the scores as the reference: max, then exp/sum, then P = e * (1/s)
// and ctx = P V.
template <int D>
__global__ void k_attention(const float* __restrict__ q, int ldq, const float* __restrict__ k, int ldk,
                            const float* __restrict__ v, int ldv, float* __restrict__ ctx, int ldc, int Rq, int S, int H,
                            int dk, int dv, int causal, float scale, int T) {
    constexpr int KC = 32;
    extern __shared__ float sm[];
    float* sc = sm;                          // S x T scores
    float* kv = sm + static_cast<size_t>(S) * T;  // KC x D chunk
    const int h = blockIdx.y, b = blockIdx.z;
    const int r = blockIdx.x * T + threadIdx.x;
    const bool live = r < Rq;
    float qr[D];
#pragma unroll
    for (int d = 0; d < D; d++) qr[d] = (live && d < dk) ? q[(static_cast<long>(b) * Rq + r) * ldq + h * dk + d] : 0.0f;
    const float* kb = k + static_cast<long>(b) * S * ldk + h * dk;
    const float* vb = v + static_cast<long>(b) * S * ldv + h * dv;
    float m = -INFINITY;
    for (int j0 = 0; j0 < S; j0 += KC) {
        const int nj = min(KC, S - j0);
        __syncthreads();
        for (int t = threadIdx.x; t < KC * D; t += blockDim.x) {
            const int jj = t / D, d = t % D;
            kv[t] = (jj < nj && d < dk) ? kb[static_cast<long>(j0 + jj) * ldk + d] : 0.0f;
        }
        __syncthreads();
        for (int jj = 0; jj < nj; jj++) {
            float s = 0.0f;
#pragma unroll
            for (int d = 0; d < D; d++) s = __fadd_rn(s, __fmul_rn(qr[d], kv[jj * D + d]));
            s = __fmul_rn(s, scale);
            if (causal && j0 + jj > r) s = -INFINITY;
            sc[static_cast<size_t>(j0 + jj) * T + threadIdx.x] = s;
            m = s > m ? s : m;
        }
    }
    float sum = 0.0f;
    for (int j = 0; j < S; j++) {
        const float e = expf(__fsub_rn(sc[static_cast<size_t>(j) * T + threadIdx.x], m));
        sc[static_cast<size_t>(j) * T + threadIdx.x] = e;
        sum = __fadd_rn(sum, e);
    }
    const float inv = __fdiv_rn(1.0f, sum);
    float acc[D];
#pragma unroll
    for (int d = 0; d < D; d++) acc[d] = 0.0f;
    for (int j0 = 0; j0 < S; j0 += KC) {
        const int nj = min(KC, S - j0);
        __syncthreads();
        for (int t = threadIdx.x; t < KC * D; t += blockDim.x) {
            const int jj = t / D, d = t % D;
            kv[t] = (jj < nj && d < dv) ? vb[static_cast<long>(j0 + jj) * ldv + d] : 0.0f;
        }
        __syncthreads();
        for (int jj = 0; jj < nj; jj++) {
            const float p = __fmul_rn(sc[static_cast<size_t>(j0 + jj) * T + threadIdx.x], inv);
#pragma unroll
            for (int d = 0; d < D; d++) acc[d] = __fadd_rn(acc[d], __fmul_rn(p, kv[jj * D + d]));
        }
    }
    if (live) {
        float* dst = ctx + (static_cast<long>(b) * Rq + r) * ldc + h * dv;
#pragma unroll
        for (int d = 0; d < D; d++)
            if (d < dv) dst[d] = acc[d];
    }
}

// Attention for short key sequences (S <= ATT_SMAX, head dims <= 64), register-tiled on the CUDA cores: one block of
// 128 threads per (sample, head, tile of 64 query rows). Q^T (d x 64), K^T (d x SP) and V (SP x 64) are staged in
// shared memory; thread (ty, tx) owns queries 8 ty .. 8 ty + 7 and, per 128-key chunk, keys 8 tx .. 8 tx + 7, so each
// step of the score loop reads two float4 of Q^T (a broadcast within the half-warp) and two of K^T (contiguous
// across the half-warp) for 64 fmas. s = (q . k) * scale (fma over d, then the scale, as alpha * (Q K^T)); the 16
// threads of a row reduce its max and sum with shuffles; P^T = exp(s - max) * (1 / sum) (keys x queries) replaces
// K^T in shared memory; thread (ty, tx) then owns ctx rows 8 ty .. +7 x columns 4 tx .. +3 (one float4 of V and two
// of P^T per key for 32 fmas).
constexpr int ATT_TQ = 64, ATT_D = 64, ATT_SMAX = 256, ATT_KC = 128;
__host__ __device__ constexpr int att_smem_floats(int SP) {
    return SP * ATT_D + ATT_D * ATT_TQ + (ATT_D > ATT_TQ ? ATT_D : ATT_TQ) * SP;
}
__global__ void __launch_bounds__(128) k_attention_tiled(const float* __restrict__ q, int ldq, const float* __restrict__ k,
                                                         int ldk, const float* __restrict__ v, int ldv, float* __restrict__ ctx,
                                                         int ldc, int Rq, int S, int dk, int dv, int causal, float scale) {
    extern __shared__ __align__(16) float sm[];
    const int SP = (S + 15) / 16 * 16;  // keys padded to a multiple of 16
    float* vs = sm;                      // SP x ATT_D
    float* qT = vs + SP * ATT_D;         // ATT_D x ATT_TQ
    float* kT = qT + ATT_D * ATT_TQ;     // ATT_D x SP, then P^T: SP x ATT_TQ
    float* pT = kT;
    const int h = blockIdx.y, b = blockIdx.z, r0 = blockIdx.x * ATT_TQ;
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const float* qb = q + static_cast<long>(b) * Rq * ldq + h * dk;
    const float* kb = k + static_cast<long>(b) * S * ldk + h * dk;
    const float* vb = v + static_cast<long>(b) * S * ldv + h * dv;
    const bool v4 = ((ldq | ldk | ldv | dk | dv) & 3) == 0 &&
                    ((reinterpret_cast<uintptr_t>(qb) | reinterpret_cast<uintptr_t>(kb) | reinterpret_cast<uintptr_t>(vb)) & 15) == 0;
    auto load4 = [&](const float* src, int d, int dmax, bool live) -> float4 {
        if (!live || d >= dmax) return make_float4(0.f, 0.f, 0.f, 0.f);
        if (v4) return __ldg(reinterpret_cast<const float4*>(src + d));
        return make_float4(src[d], d + 1 < dmax ? src[d + 1] : 0.f, d + 2 < dmax ? src[d + 2] : 0.f, d + 3 < dmax ? src[d + 3] : 0.f);
    };
    // staging, 4 consecutive d of one row per float4; loads are issued U at a time before their stores so that
    // their latencies overlap
    constexpr int U = 8;
    for (int t0 = 0; t0 < ATT_TQ * ATT_D / 4; t0 += 128 * U) {
        float4 x[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int t = t0 + u * 128 + tid, row = t / (ATT_D / 4), d = 4 * (t - row * (ATT_D / 4));
            x[u] = load4(qb + static_cast<long>(r0 + row) * ldq, d, dk, t < ATT_TQ * ATT_D / 4 && r0 + row < Rq);
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int t = t0 + u * 128 + tid, row = t / (ATT_D / 4), d = 4 * (t - row * (ATT_D / 4));
            if (t < ATT_TQ * ATT_D / 4)
                qT[d * ATT_TQ + row] = x[u].x, qT[(d + 1) * ATT_TQ + row] = x[u].y, qT[(d + 2) * ATT_TQ + row] = x[u].z,
                qT[(d + 3) * ATT_TQ + row] = x[u].w;
        }
    }
    for (int t0 = 0; t0 < SP * ATT_D / 4; t0 += 128 * U) {
        float4 x[U], y[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int t = t0 + u * 128 + tid, j = t / (ATT_D / 4), d = 4 * (t - j * (ATT_D / 4));
            const bool live = t < SP * ATT_D / 4 && j < S;
            x[u] = load4(kb + static_cast<long>(j) * ldk, d, dk, live);
            y[u] = load4(vb + static_cast<long>(j) * ldv, d, dv, live);
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int t = t0 + u * 128 + tid, j = t / (ATT_D / 4), d = 4 * (t - j * (ATT_D / 4));
            if (t < SP * ATT_D / 4) {
                kT[d * SP + j] = x[u].x, kT[(d + 1) * SP + j] = x[u].y, kT[(d + 2) * SP + j] = x[u].z, kT[(d + 3) * SP + j] = x[u].w;
                *reinterpret_cast<float4*>(vs + j * ATT_D + d) = y[u];
            }
        }
    }
    __syncthreads();
    // scores of rows 8 ty + i: key chunks of 128, keys 8 tx + c of each
    constexpr int NCH = ATT_SMAX / ATT_KC;
    float sc[NCH][8][8];
    const int nch = (SP + ATT_KC - 1) / ATT_KC;
#pragma unroll
    for (int ch = 0; ch < NCH; ch++) {
        if (ch >= nch) break;
        const int j0 = ch * ATT_KC + 8 * tx;
        const bool kin = j0 < SP;  // keys of this thread's group exist in the padded range
#pragma unroll
        for (int i = 0; i < 8; i++)
#pragma unroll
            for (int c = 0; c < 8; c++) sc[ch][i][c] = 0.0f;
        if (kin)
            for (int d = 0; d < dk; d++) {
                const float4 qa = *reinterpret_cast<const float4*>(qT + d * ATT_TQ + 8 * ty);
                const float4 qc = *reinterpret_cast<const float4*>(qT + d * ATT_TQ + 8 * ty + 4);
                const float4 ka = *reinterpret_cast<const float4*>(kT + d * SP + j0);
                const float4 kc = *reinterpret_cast<const float4*>(kT + d * SP + j0 + 4);
                const float qv[8] = {qa.x, qa.y, qa.z, qa.w, qc.x, qc.y, qc.z, qc.w};
                const float kv[8] = {ka.x, ka.y, ka.z, ka.w, kc.x, kc.y, kc.z, kc.w};
#pragma unroll
                for (int i = 0; i < 8; i++)
#pragma unroll
                    for (int c = 0; c < 8; c++) sc[ch][i][c] = __fmaf_rn(qv[i], kv[c], sc[ch][i][c]);
            }
    }
    __syncthreads();  // every thread is done reading K^T before P^T overwrites it
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int row = r0 + 8 * ty + i;
        float m = -INFINITY;
#pragma unroll
        for (int ch = 0; ch < NCH; ch++) {
            if (ch >= nch) break;
#pragma unroll
            for (int c = 0; c < 8; c++) {
                const int j = ch * ATT_KC + 8 * tx + c;
                float s = __fmul_rn(sc[ch][i][c], scale);
                if (j >= S || (causal && j > row)) s = -INFINITY;
                sc[ch][i][c] = s;
                m = fmaxf(m, s);
            }
        }
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        float sum = 0.0f;
#pragma unroll
        for (int ch = 0; ch < NCH; ch++) {
            if (ch >= nch) break;
#pragma unroll
            for (int c = 0; c < 8; c++) {
                const float e = expf(__fsub_rn(sc[ch][i][c], m));
                sc[ch][i][c] = e;
                sum = __fadd_rn(sum, e);
            }
        }
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, o));
        const float inv = __fdiv_rn(1.0f, sum);
#pragma unroll
        for (int ch = 0; ch < NCH; ch++) {
            if (ch >= nch) break;
#pragma unroll
            for (int c = 0; c < 8; c++) {
                const int j = ch * ATT_KC + 8 * tx + c;
                if (j < SP) pT[j * ATT_TQ + 8 * ty + i] = __fmul_rn(sc[ch][i][c], inv);
            }
        }
    }
    __syncthreads();
    // ctx rows 8 ty + i, columns 4 tx + e
    float acc[8][4];
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
        for (int e = 0; e < 4; e++) acc[i][e] = 0.0f;
    for (int j = 0; j < S; j++) {
        const float4 vv = *reinterpret_cast<const float4*>(vs + j * ATT_D + 4 * tx);
        const float4 pa = *reinterpret_cast<const float4*>(pT + j * ATT_TQ + 8 * ty);
        const float4 pc = *reinterpret_cast<const float4*>(pT + j * ATT_TQ + 8 * ty + 4);
        const float pv[8] = {pa.x, pa.y, pa.z, pa.w, pc.x, pc.y, pc.z, pc.w};
#pragma unroll
        for (int i = 0; i < 8; i++) {
            acc[i][0] = __fmaf_rn(pv[i], vv.x, acc[i][0]);
            acc[i][1] = __fmaf_rn(pv[i], vv.y, acc[i][1]);
            acc[i][2] = __fmaf_rn(pv[i], vv.z, acc[i][2]);
            acc[i][3] = __fmaf_rn(pv[i], vv.w, acc[i][3]);
        }
    }
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int row = r0 + 8 * ty + i;
        if (row >= Rq) continue;
        float* dst = ctx + (static_cast<long>(b) * Rq + row) * ldc + h * dv;
#pragma unroll
        for (int e = 0; e < 4; e++)
            if (4 * tx + e < dv) dst[4 * tx + e] = acc[i][e];
    }
}

__global__ void k_fma_relu(const float* __restrict__ a, const float* __restrict__ x, const float* __restrict__ b,
                           float* __restrict__ y, size_t n) {
    const size_t n4 = n >> 2;
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n4; i += stride) {
        const float4 u = reinterpret_cast<const float4*>(a)[i], v = reinterpret_cast<const float4*>(x)[i],
                     w = reinterpret_cast<const float4*>(b)[i];
        reinterpret_cast<float4*>(y)[i] = make_float4(fmaxf(__fmaf_rn(u.x, v.x, w.x), 0.0f), fmaxf(__fmaf_rn(u.y, v.y, w.y), 0.0f),
                                                      fmaxf(__fmaf_rn(u.z, v.z, w.z), 0.0f), fmaxf(__fmaf_rn(u.w, v.w, w.w), 0.0f));
    }
    for (size_t i = (n4 << 2) + blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n; i += stride)
        y[i] = fmaxf(__fmaf_rn(a[i], x[i], b[i]), 0.0f);
}

// [world][rows][slice] -> rows x (world * slice), one float4 (slice % 4 == 0) or one float per thread
template <int V>
__global__ void k_unshard_cols(const float* __restrict__ src, int world, long rows, int slice, float* __restrict__ y, int ldy) {
    const long per_row = static_cast<long>(world) * slice / V;
    const long n = rows * per_row;
    for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < n; i += static_cast<long>(gridDim.x) * blockDim.x) {
        const long r = i / per_row;
        const int c = static_cast<int>(i - r * per_row) * V;
        const int g = c / slice, j = c - g * slice;
        const float* s = src + (static_cast<long>(g) * rows + r) * slice + j;
        float* d = y + r * ldy + c;
        if (V == 4) *reinterpret_cast<float4*>(d) = __ldg(reinterpret_cast<const float4*>(s));
        else *d = __ldg(s);
    }
}

// One time step of an LSTM / GRU / SimpleRNN direction (kernix_rnn_dir, include/kernix_model.h:560-634).
// Block: RB sequences x TU hidden units; the RB previous states sit in shared memory, each thread accumulates
// h . U for its unit in every gate (U is units x gates*units row-major, reads coalesced across the block), then
// applies the gates in the reference's order with IEEE steps:
//   LSTM (i, f, g, o): z = x.W + b + h.U; c = i*g + f*c (c = i*g at step 0); h = act(c)*o
//   GRU (z, r, h~):    zh = b_rec + h.U (b_rec at step 0); z, r = sigmoid(x_z,r + zh_z,r);
//                      h~ = act(r*zh_h + x_h); h = (h - h~)*z + h~ (h = -h~*z + h~ at step 0)
//   RNN:               h = act(x.W + b + h.U)
// zx holds x.W + b for all steps ((B*T) x gu). Writes h_next, c (LSTM), and the state at time t to
// out + (b*T + t)*stride (ret_seq) or, at the last step, to out + b*stride.
template <int KIND>  // 0 LSTM, 1 GRU, 2 RNN
__global__ void k_rnn_step(const float* __restrict__ zx, const float* __restrict__ U, const float* __restrict__ brec,
                           const float* __restrict__ hp, float* __restrict__ hn, float* __restrict__ c, float* __restrict__ out,
                           long stride, int B, int T, int t, int u, int first, int ret_seq, int last, int act, float alpha,
                           int RB) {
    constexpr int G = KIND == 0 ? 4 : (KIND == 1 ? 3 : 1);
    constexpr int RBM = 8;
    extern __shared__ float hs[];  // RB x u
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    const int b0 = blockIdx.y * RB;
    const int nb = min(RB, B - b0);
    if (!first)
        for (int i = threadIdx.x; i < nb * u; i += blockDim.x) hs[i] = hp[static_cast<long>(b0) * u + i];
    __syncthreads();
    if (j >= u) return;
    const long gu = static_cast<long>(G) * u;
    float acc[RBM][G];
#pragma unroll
    for (int r = 0; r < RBM; r++)
#pragma unroll
        for (int g = 0; g < G; g++) acc[r][g] = 0.0f;
    if (!first)
        for (int k = 0; k < u; k++) {
            float w[G];
#pragma unroll
            for (int g = 0; g < G; g++) w[g] = __ldg(U + k * gu + g * u + j);
#pragma unroll
            for (int r = 0; r < RBM; r++) {
                if (r >= nb) break;
                const float hv = hs[r * u + k];
#pragma unroll
                for (int g = 0; g < G; g++) acc[r][g] = __fmaf_rn(hv, w[g], acc[r][g]);
            }
        }
#pragma unroll
    for (int r = 0; r < RBM; r++) {
        if (r >= nb) break;
        const int b = b0 + r;
        const float* z = zx + (static_cast<long>(b) * T + t) * gu;
        float h;
        if (KIND == 0) {
            float zg[4];
#pragma unroll
            for (int g = 0; g < 4; g++) zg[g] = first ? z[g * u + j] : __fadd_rn(z[g * u + j], acc[r][g]);
            const float ig = kx::act_apply(kx::ACT_SIGMOID, zg[0], 0.0f), fg = kx::act_apply(kx::ACT_SIGMOID, zg[1], 0.0f);
            const float gg = kx::act_apply(act, zg[2], alpha), og = kx::act_apply(kx::ACT_SIGMOID, zg[3], 0.0f);
            float* cb = c + static_cast<long>(b) * u + j;
            const float cn = first ? __fmul_rn(ig, gg) : __fadd_rn(__fmul_rn(ig, gg), __fmul_rn(fg, *cb));
            *cb = cn;
            h = __fmul_rn(kx::act_apply(act, cn, alpha), og);
        } else if (KIND == 1) {
            float zh[3];
#pragma unroll
            for (int g = 0; g < 3; g++) zh[g] = first ? brec[g * u + j] : __fadd_rn(acc[r][g], brec[g * u + j]);
            const float zgt = kx::act_apply(kx::ACT_SIGMOID, __fadd_rn(z[j], zh[0]), 0.0f);
            const float rgt = kx::act_apply(kx::ACT_SIGMOID, __fadd_rn(z[u + j], zh[1]), 0.0f);
            const float hh = kx::act_apply(act, __fadd_rn(__fmul_rn(rgt, zh[2]), z[2 * u + j]), alpha);
            const float d = first ? -hh : __fsub_rn(hs[r * u + j], hh);
            h = __fadd_rn(__fmul_rn(d, zgt), hh);
        } else {
            h = kx::act_apply(act, first ? z[j] : __fadd_rn(z[j], acc[r][0]), alpha);
        }
        hn[static_cast<long>(b) * u + j] = h;
        if (ret_seq) out[(static_cast<long>(b) * T + t) * stride + j] = h;
        else if (last) out[static_cast<long>(b) * stride + j] = h;
    }
}

// Elementwise merge of two directions (kernix_rnn_run :641-646): y = y * bw, y + bw, or (y + bw) * 0.5.
__global__ void k_rnn_merge(float* __restrict__ y, const float* __restrict__ bw, long n, int merge) {
    for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < n; i += static_cast<long>(gridDim.x) * blockDim.x) {
        const float a = y[i], b = bw[i];
        y[i] = merge == 2 ? __fmul_rn(a, b) : (merge == 3 ? __fmul_rn(__fadd_rn(a, b), 0.5f) : __fadd_rn(a, b));
    }
}

// Skinny dense layer (M <= 16 rows) on the CUDA cores, for weight streaming: fp32 W k x n row-major as in the
// file. Block = 256 threads x CPT consecutive columns each (16-, 8- or 4-byte loads of W, coalesced across the
// block) over one K slice; the slice of the M input rows is staged in shared memory in pieces of 256 K; each thread
// keeps MT x CPT (<= 32) fp32 fma accumulators and eight K steps of W loads in flight. Partial sums
// [slice][row][column] are reduced in slice order by k_skinny_reduce, which adds the bias and applies the
// activation (act(x.W + b), as the reference's sgemm then bias_act).
constexpr int SK_THREADS = 256, SK_KC = 256;
template <int CPT> struct SkVec;
template <> struct SkVec<4> { using T = float4; };
template <> struct SkVec<2> { using T = float2; };
template <> struct SkVec<1> { using T = float; };
template <int CPT>
__device__ __forceinline__ void sk_unpack(const typename SkVec<CPT>::T& v, float (&o)[CPT]) {
    if constexpr (CPT == 4) { o[0] = v.x; o[1] = v.y; o[2] = v.z; o[3] = v.w; }
    else if constexpr (CPT == 2) { o[0] = v.x; o[1] = v.y; }
    else { o[0] = v; }
}

template <int MT, int CPT>
__global__ void __launch_bounds__(SK_THREADS, 2) k_skinny(const float* __restrict__ x, int ldx, const float* __restrict__ w,
                                                         int n, float* __restrict__ part, int M, int K, int kslice) {
    using V = typename SkVec<CPT>::T;
    __shared__ float xs[MT][SK_KC];
    const int col = (blockIdx.x * SK_THREADS + threadIdx.x) * CPT;
    const int k0 = blockIdx.y * kslice, k1 = min(K, k0 + kslice);
    float acc[MT][CPT];
#pragma unroll
    for (int m = 0; m < MT; m++)
#pragma unroll
        for (int c = 0; c < CPT; c++) acc[m][c] = 0.0f;
    for (int kc = k0; kc < k1; kc += SK_KC) {
        const int nk = min(SK_KC, k1 - kc);
        __syncthreads();
        for (int i = threadIdx.x; i < MT * SK_KC; i += SK_THREADS) {
            const int m = i / SK_KC, kk = i - m * SK_KC;
            xs[m][kk] = (m < M && kk < nk) ? x[static_cast<long>(m) * ldx + kc + kk] : 0.0f;
        }
        __syncthreads();
        if (col < n) {
            const float* wp = w + static_cast<long>(kc) * n + col;
#pragma unroll 8
            for (int kk = 0; kk < nk; kk++) {
                float wv[CPT];
                sk_unpack<CPT>(__ldg(reinterpret_cast<const V*>(wp + static_cast<long>(kk) * n)), wv);
#pragma unroll
                for (int m = 0; m < MT; m++)
#pragma unroll
                    for (int c = 0; c < CPT; c++) acc[m][c] = __fmaf_rn(xs[m][kk], wv[c], acc[m][c]);
            }
        }
    }
    if (col < n) {
#pragma unroll
        for (int m = 0; m < MT; m++) {
            if (m >= M) break;
#pragma unroll
            for (int c = 0; c < CPT; c++) part[(static_cast<long>(blockIdx.y) * M + m) * n + col + c] = acc[m][c];
        }
    }
}

__global__ void k_skinny_reduce(const float* __restrict__ part, int S, int M, int n, const float* __restrict__ bias,
                                float* __restrict__ y, int ldy, int act, float alpha) {
    const long total = static_cast<long>(M) * n;
    for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < total; i += static_cast<long>(gridDim.x) * blockDim.x) {
        const int m = static_cast<int>(i / n), c = static_cast<int>(i - static_cast<long>(m) * n);
        float v = part[i];
        for (int sl = 1; sl < S; sl++) v = __fadd_rn(v, part[static_cast<long>(sl) * total + i]);
        if (bias) v = __fadd_rn(v, bias[c]);
        y[static_cast<long>(m) * ldy + c] = kx::act_apply(act, v, alpha);
    }
}

}  // namespace

// tensor-core attention core (kx_attn.cu): 0 done, 1 shape not covered, -1 launch error
int kx_attention_tc(const float* q, int ldq, const float* k, int ldk, const float* v, int ldv, float* ctx, int ldc, int B,
                    int Rq, int S, int H, int dk, int dv, int causal, float scale, int* status, cudaStream_t st);

extern "C" {

// columns per thread of the skinny kernel for m rows and n columns (m * CPT accumulators <= 32; n divisible)
static int sk_cpt(int m, int n) {
    const int c = m <= 8 ? 4 : 2;
    return n % c == 0 ? c : 1;
}

int kx_skinny_slices(int n, int k) {
    const int nblk = (n + 4 * SK_THREADS - 1) / (4 * SK_THREADS);  // column blocks at four columns per thread (the fewest)
    int S = (2 * 148 + nblk - 1) / nblk;  // about two blocks per SM
    const int smax = (k + SK_KC - 1) / SK_KC;
    if (S > smax) S = smax;
    return S < 1 ? 1 : S;
}

int kx_gemm_f32_skinny(const float* x, int ldx, const float* w, const float* bias, float* y, int ldy, int m, int n, int k, int act,
                       float alpha, float* part, size_t part_floats, void* stream) {
    if (m <= 0 || n <= 0) return 0;
    if (m > KX_SKINNY_MAX_ROWS || k <= 0 || ldx < k || ldy < n || part == nullptr) return -1;
    if (reinterpret_cast<uintptr_t>(w) & 15) return -1;
    const int S = kx_skinny_slices(n, k);
    if (static_cast<size_t>(S) * m * n > part_floats) return -1;
    const int cpt = sk_cpt(m, n);
    const int kslice = ((k + S - 1) / S + SK_KC - 1) / SK_KC * SK_KC;
    const int S_used = (k + kslice - 1) / kslice;
    dim3 grid((n + SK_THREADS * cpt - 1) / (SK_THREADS * cpt), S_used);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (m <= 8) {
        if (cpt == 4) k_skinny<8, 4><<<grid, SK_THREADS, 0, st>>>(x, ldx, w, n, part, m, k, kslice);
        else k_skinny<8, 1><<<grid, SK_THREADS, 0, st>>>(x, ldx, w, n, part, m, k, kslice);
    } else {
        if (cpt == 2) k_skinny<16, 2><<<grid, SK_THREADS, 0, st>>>(x, ldx, w, n, part, m, k, kslice);
        else k_skinny<16, 1><<<grid, SK_THREADS, 0, st>>>(x, ldx, w, n, part, m, k, kslice);
    }
    if (cudaGetLastError() != cudaSuccess) return -1;
    k_skinny_reduce<<<grid_for(static_cast<long>(m) * n, 256), 256, 0, st>>>(part, S_used, m, n, bias, y, ldy, act, alpha);
    return launch_ok();
}


int kx_rnn_step(int kind, const float* zx, const float* U, const float* brec, const float* h_prev, float* h_next, float* c,
                float* out, long stride, int B, int T, int t, int u, int first, int ret_seq, int last, int act, float alpha,
                void* stream) {
    if (B <= 0) return 0;
    if (u <= 0 || T <= 0 || t < 0 || t >= T || kind < 0 || kind > 2 || (kind == 1 && brec == nullptr) || (kind == 0 && c == nullptr))
        return -1;
    int RB = 8;
    while (RB > 1 && static_cast<long>(RB) * u * 4 > 48 * 1024) RB >>= 1;
    if (static_cast<long>(u) * 4 > 48 * 1024) return -1;  // one state row must fit the block's shared memory
    const int TU = u >= 128 ? 128 : (u + 31) / 32 * 32;
    dim3 grid((u + TU - 1) / TU, (B + RB - 1) / RB);
    const size_t smem = static_cast<size_t>(RB) * u * sizeof(float);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (kind == 0) k_rnn_step<0><<<grid, TU, smem, st>>>(zx, U, brec, h_prev, h_next, c, out, stride, B, T, t, u, first, ret_seq, last, act, alpha, RB);
    else if (kind == 1) k_rnn_step<1><<<grid, TU, smem, st>>>(zx, U, brec, h_prev, h_next, c, out, stride, B, T, t, u, first, ret_seq, last, act, alpha, RB);
    else k_rnn_step<2><<<grid, TU, smem, st>>>(zx, U, brec, h_prev, h_next, c, out, stride, B, T, t, u, first, ret_seq, last, act, alpha, RB);
    return launch_ok();
}

int kx_rnn_merge(float* y, const float* bw, long n, int merge, void* stream) {
    if (n <= 0) return 0;
    if (merge < 1 || merge > 3) return -1;
    k_rnn_merge<<<grid_for(n, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(y, bw, n, merge);
    return launch_ok();
}


int kx_unshard_cols(const float* src, int world, long rows, int slice, float* y, int ldy, void* stream) {
    if (rows <= 0 || world <= 0 || slice <= 0) return 0;
    if (ldy < world * slice) return -1;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const bool vec = (slice % 4 == 0) && (ldy % 4 == 0) && ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(y)) % 16 == 0);
    const long n = rows * world * slice;
    if (vec) k_unshard_cols<4><<<grid_for(n / 4, 256), 256, 0, st>>>(src, world, rows, slice, y, ldy);
    else k_unshard_cols<1><<<grid_for(n, 256), 256, 0, st>>>(src, world, rows, slice, y, ldy);
    return launch_ok();
}


int kx_add_planes(const float* part, int planes, int m, int n, const float* bias, int act, float alpha, float* y, int ldy,
                  void* stream) {
    const long total = static_cast<long>(m) * n;
    if (total <= 0) return 0;
    if (planes < 1 || planes > KX_SPLITK_MAX || part == nullptr || y == nullptr) return -1;
    k_add_planes<<<grid_for(total, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(part, planes, m, n, bias, act, alpha, y, ldy);
    return launch_ok();
}

int kx_quant_rows_z(const float* x, int ldx, int rows, int k, int8_t* xq, int ldq, float* sx, uint32_t* zero, int zero_words,
                    void* stream) {
    if (rows <= 0) return 0;
    if (k <= 0 || ldq < k || ldx < k || (zero_words > 0 && zero == nullptr)) return -1;
    if (kx::launch_pdl(k_quant_rows, dim3(rows), dim3(QT), 0, static_cast<cudaStream_t>(stream), x, ldx, k, xq, ldq, sx, zero,
                       zero_words) != 0)
        return -1;
    return launch_ok();
}

int kx_quant_rows(const float* x, int ldx, int rows, int k, int8_t* xq, int ldq, float* sx, void* stream) {
    return kx_quant_rows_z(x, ldx, rows, k, xq, ldq, sx, nullptr, 0, stream);
}

int kx_bias_act(const float* x, float* y, long rows, int cols, const float* bias, int act, float alpha, void* stream) {
    const long n = rows * cols;
    if (n <= 0) return 0;
    const bool vec = (cols % 4 == 0) && ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) % 16 == 0);
    if (!vec) {
        k_bias_act<<<grid_for(n, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(x, y, rows, cols, bias, act, alpha);
    } else {
        k_bias_act<<<grid_for(n / 4, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(x, y, rows, cols, bias, act, alpha);
    }
    return launch_ok();
}

int kx_softmax_rows(const float* x, float* y, long rows, int cols, void* stream) {
    if (rows <= 0 || cols <= 0) return 0;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (cols <= 1024) k_softmax_warp<8><<<static_cast<unsigned>((rows + 7) / 8), 256, 0, st>>>(x, y, rows, cols);
    else k_softmax_block<<<static_cast<unsigned>(rows), 256, 0, st>>>(x, y, cols);
    return launch_ok();
}

int kx_layernorm_rows(const float* x, float* y, long rows, int cols, const float* gamma, const float* beta, float eps,
                      void* stream) {
    if (rows <= 0 || cols <= 0) return 0;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (cols <= 1024)
        k_layernorm_warp<8><<<static_cast<unsigned>((rows + 7) / 8), 256, 0, st>>>(x, y, rows, cols, gamma, beta, eps);
    else k_layernorm_block<<<static_cast<unsigned>(rows), 256, 0, st>>>(x, y, cols, gamma, beta, eps);
    return launch_ok();
}

int kx_affine_rows(const float* x, float* y, long rows, int cols, const float* g, const float* b, void* stream) {
    const long n = rows * cols;
    if (n <= 0) return 0;
    k_affine<<<grid_for(n, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(x, y, n, cols, g, b);
    return launch_ok();
}

int kx_add_const(const float* x, float* y, long samples, long per, const float* cst, void* stream) {
    const long n = samples * per;
    if (n <= 0) return 0;
    k_add_const<<<grid_for(n, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(x, y, n, per, cst);
    return launch_ok();
}

int kx_binary(const float* a, int ra, int ca, const float* b, int rb, int cb, float* y, long samples, int R, int C, int op,
              void* stream) {
    const long n = samples * R * C;
    if (n <= 0) return 0;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const bool same = ra == R && rb == R && ca == C && cb == C;
    const bool al = ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) | reinterpret_cast<uintptr_t>(y)) & 15) == 0;
    if (same && al && (n & 3) == 0) {
        k_binary_same4<<<grid_for(n / 4, 256), 256, 0, st>>>(reinterpret_cast<const float4*>(a),
                                                             reinterpret_cast<const float4*>(b),
                                                             reinterpret_cast<float4*>(y), n / 4, op);
    } else {
        k_binary<<<grid_for(n, 256), 256, 0, st>>>(a, ra, ca, b, rb, cb, y, samples, R, C, op);
    }
    return launch_ok();
}

int kx_pool2d(const float* x, float* y, int B, int H, int W, int C, int Ho, int Wo, int kh, int kw, int sh, int sw, int pt,
              int pl, int type, int count_pad, void* stream) {
    const long n = static_cast<long>(B) * Ho * Wo * C;
    if (n <= 0) return 0;
    if (C % 4 == 0 && ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15) == 0 && n / 4 < INT32_MAX &&
        static_cast<long>(B) * H * W * (C / 4) < INT32_MAX) {
        k_pool2d_v4<<<grid_for(n / 4, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
            reinterpret_cast<const float4*>(x), reinterpret_cast<float4*>(y), B, H, W, C / 4, Ho, Wo, kh, kw, sh, sw, pt, pl,
            type, count_pad);
        return launch_ok();
    }
    k_pool2d<<<grid_for(n, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(x, y, B, H, W, C, Ho, Wo, kh, kw, sh, sw, pt,
                                                                               pl, type, count_pad);
    return launch_ok();
}

int kx_global_pool(const float* x, float* y, long B, int R, int C, int type, void* stream) {
    const long n = B * C;
    if (n <= 0) return 0;
    k_global_pool<<<grid_for(n, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(x, y, B, R, C, type);
    return launch_ok();
}

int kx_permute(const float* x, float* y, long B, int nd, const int* dims, const int* perm, void* stream) {
    if (nd < 1 || nd > 4) return -1;
    PermGeom g;
    long ist[4], n = 1;
    for (int k = nd - 1; k >= 0; k--) {
        ist[k] = n;
        n *= dims[k];
    }
    g.nd = nd;
    g.per = n;
    for (int k = 0; k < nd; k++) {
        g.od[k] = dims[perm[k]];
        g.ist[k] = ist[perm[k]];
    }
    if (B * n <= 0) return 0;
    k_permute<<<grid_for(B * n, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(x, y, B, g);
    return launch_ok();
}

int kx_copy_cols(const float* x, long ldx, float* y, long ldy, long yoff, long rows, long cols, void* stream) {
    if (rows * cols <= 0) return 0;
    k_copy_cols<<<grid_for(rows * cols, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(x, ldx, y, ldy, yoff, rows, cols);
    return launch_ok();
}

int kx_pad2d(const float* x, float* y, int B, int H, int W, int C, int Ho, int Wo, int pt, int pl, void* stream) {
    const long n = static_cast<long>(B) * Ho * Wo * C;
    if (n <= 0) return 0;
    k_pad2d<<<grid_for(n, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(x, y, B, H, W, C, Ho, Wo, pt, pl);
    return launch_ok();
}

int kx_upsample2d(const float* x, float* y, int B, int H, int W, int C, int Ho, int Wo, int sh, int sw, void* stream) {
    const long n = static_cast<long>(B) * Ho * Wo * C;
    if (n <= 0) return 0;
    k_upsample2d<<<grid_for(n, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(x, y, B, H, W, C, Ho, Wo, sh, sw);
    return launch_ok();
}

int kx_embedding(const float* ids, long n, const float* table, int vocab, int dim, float* y, void* stream) {
    if (n * dim <= 0) return 0;
    k_embedding<<<grid_for(n * dim, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(ids, n, table, vocab, dim, y);
    return launch_ok();
}

int kx_conv_depthwise(const float* x, const float* w, const float* bias, float* y, int B, int H, int W, int C, int Co,
                      int Ho, int Wo, int kh, int kw, int sh, int sw, int dh, int dw, int pt, int pl, int act, float alpha,
                      void* stream) {
    const long n = static_cast<long>(B) * Ho * Wo * Co;
    if (n <= 0) return 0;
    if (C <= 0 || Co % C) return -1;
    k_conv_dw<<<grid_for(n, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(x, w, bias, y, B, H, W, C, Co, Ho, Wo, kh, kw,
                                                                                sh, sw, dh, dw, pt, pl, act, alpha);
    return launch_ok();
}

int kx_attention(const float* q, int ldq, const float* k, int ldk, const float* v, int ldv, float* ctx, int ldc, int B,
                 int Rq, int S, int H, int dk, int dv, int causal, int* status, void* stream) {
    if (B <= 0 || Rq <= 0) return 0;
    if (S <= 0 || dk <= 0 || dv <= 0 || dk > 128 || dv > 128) return -1;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    {  // tensor cores (kx_attn.cu) when the shape fits one CTA per (sample, head)
        const int rc = kx_attention_tc(q, ldq, k, ldk, v, ldv, ctx, ldc, B, Rq, S, H, dk, dv, causal,
                                       1.0f / sqrtf(static_cast<float>(dk)), status, st);
        if (rc <= 0) return rc;
    }
    if (S <= ATT_SMAX && dk <= ATT_D && dv <= ATT_D) {
        const int SP = (S + 15) / 16 * 16;
        const size_t smem = static_cast<size_t>(att_smem_floats(SP)) * sizeof(float);
        static unsigned long long devs_set = 0;  // devices whose kernel attribute holds the largest size (S = ATT_SMAX)
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess) return -1;
        const unsigned long long bit = 1ull << (dev & 63);
        if (!(__atomic_load_n(&devs_set, __ATOMIC_ACQUIRE) & bit)) {
            if (cudaFuncSetAttribute(k_attention_tiled, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     att_smem_floats(ATT_SMAX) * 4) != cudaSuccess)
                return -1;
            __atomic_fetch_or(&devs_set, bit, __ATOMIC_RELEASE);
        }
        const float scale = 1.0f / sqrtf(static_cast<float>(dk));
        dim3 grid((Rq + ATT_TQ - 1) / ATT_TQ, H, B);
        k_attention_tiled<<<grid, 128, smem, st>>>(q, ldq, k, ldk, v, ldv, ctx, ldc, Rq, S, dk, dv, causal, scale);
        return launch_ok();
    }
    int T = 128;
    while (T > 32 && static_cast<size_t>(S) * T * 4 > 160 * 1024) T >>= 1;
    const int D = (dk <= 64 && dv <= 64) ? 64 : 128;
    const size_t smem = (static_cast<size_t>(S) * T + 32 * static_cast<size_t>(D)) * sizeof(float);
    if (smem > 220 * 1024) return -1;
    const float scale = 1.0f / sqrtf(static_cast<float>(dk)); /* IEEE on the host, as the reference's 1.0f / sqrtf */
    dim3 grid((Rq + T - 1) / T, H, B);
    if (D == 64) {
        if (cudaFuncSetAttribute(k_attention<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess)
            return -1;
        k_attention<64><<<grid, T, smem, st>>>(q, ldq, k, ldk, v, ldv, ctx, ldc, Rq, S, H, dk, dv, causal, scale, T);
    } else {
        if (cudaFuncSetAttribute(k_attention<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess)
            return -1;
        k_attention<128><<<grid, T, smem, st>>>(q, ldq, k, ldk, v, ldv, ctx, ldc, Rq, S, H, dk, dv, causal, scale, T);
    }
    return launch_ok();
}

int kx_fma_relu(const float* a, const float* x, const float* b, float* y, size_t n, void* stream) {
    if (n == 0) return 0;
    if (((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(b) |
          reinterpret_cast<uintptr_t>(y)) & 15) != 0)
        return -1;
    k_fma_relu<<<grid_for(static_cast<long>((n + 3) / 4), 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(a, x, b, y, n);
    return launch_ok();
}

}  // extern "C"
