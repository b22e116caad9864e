/* Plain-C stand-ins for the Apple Accelerate calls the KERNIX reference headers use.
 *
 * TEST INFRASTRUCTURE ONLY: force-included (-include) when oracle/ref/Makefile compiles the
 * reference's own CPU forward into oracle/_ref/. Never linked into the product library.
 *
 * Each function restates the documented vDSP / vForce semantics with a scalar loop, honouring
 * strides. Argument order follows Accelerate: vDSP_vsub(B, IB, A, IA, C, IC, N) gives C = A - B and
 * vDSP_vdiv(B, IB, A, IA, C, IC, N) gives C = A / B, which include/kernix.h:498-500 relies on.
 * cblas_sgemm forwards to the ILP64 OpenBLAS that numpy bundles (exported as scipy_cblas_sgemm64_);
 * the library is called by name only. vvexpf/vvtanhf/... call glibc's expf/tanhf/..., so
 * transcendental results match glibc, not Apple's libm (parity with M1 runs is tolerance-only).
 */
#ifndef KX_ACCELERATE_SHIM_H
#define KX_ACCELERATE_SHIM_H

#include <math.h>
#include <stddef.h>

#define KERNIX_ACCELERATE_ENABLED 1

typedef unsigned long vDSP_Length;
typedef long vDSP_Stride;

#define KX_LOOP(n) for (vDSP_Length i = 0; i < (n); i++)

static inline void vDSP_vadd(const float* a, vDSP_Stride ia, const float* b, vDSP_Stride ib, float* c, vDSP_Stride ic, vDSP_Length n)
{ KX_LOOP(n) c[i * ic] = a[i * ia] + b[i * ib]; }
static inline void vDSP_vsub(const float* b, vDSP_Stride ib, const float* a, vDSP_Stride ia, float* c, vDSP_Stride ic, vDSP_Length n)
{ KX_LOOP(n) c[i * ic] = a[i * ia] - b[i * ib]; }
static inline void vDSP_vmul(const float* a, vDSP_Stride ia, const float* b, vDSP_Stride ib, float* c, vDSP_Stride ic, vDSP_Length n)
{ KX_LOOP(n) c[i * ic] = a[i * ia] * b[i * ib]; }
static inline void vDSP_vdiv(const float* b, vDSP_Stride ib, const float* a, vDSP_Stride ia, float* c, vDSP_Stride ic, vDSP_Length n)
{ KX_LOOP(n) c[i * ic] = a[i * ia] / b[i * ib]; }
static inline void vDSP_vmax(const float* a, vDSP_Stride ia, const float* b, vDSP_Stride ib, float* c, vDSP_Stride ic, vDSP_Length n)
{ KX_LOOP(n) c[i * ic] = a[i * ia] > b[i * ib] ? a[i * ia] : b[i * ib]; }
static inline void vDSP_vmin(const float* a, vDSP_Stride ia, const float* b, vDSP_Stride ib, float* c, vDSP_Stride ic, vDSP_Length n)
{ KX_LOOP(n) c[i * ic] = a[i * ia] < b[i * ib] ? a[i * ia] : b[i * ib]; }
/* d = a*b + c */
static inline void vDSP_vma(const float* a, vDSP_Stride ia, const float* b, vDSP_Stride ib, const float* c, vDSP_Stride ic,
                            float* d, vDSP_Stride id, vDSP_Length n)
{ KX_LOOP(n) d[i * id] = a[i * ia] * b[i * ib] + c[i * ic]; }
static inline void vDSP_vsadd(const float* a, vDSP_Stride ia, const float* s, float* c, vDSP_Stride ic, vDSP_Length n)
{ const float v = *s; KX_LOOP(n) c[i * ic] = a[i * ia] + v; }
static inline void vDSP_vsmul(const float* a, vDSP_Stride ia, const float* s, float* c, vDSP_Stride ic, vDSP_Length n)
{ const float v = *s; KX_LOOP(n) c[i * ic] = a[i * ia] * v; }
static inline void vDSP_vneg(const float* a, vDSP_Stride ia, float* c, vDSP_Stride ic, vDSP_Length n)
{ KX_LOOP(n) c[i * ic] = -a[i * ia]; }
static inline void vDSP_vabs(const float* a, vDSP_Stride ia, float* c, vDSP_Stride ic, vDSP_Length n)
{ KX_LOOP(n) c[i * ic] = fabsf(a[i * ia]); }
/* threshold: c = a >= t ? a : t (NaN stays NaN) */
static inline void vDSP_vthr(const float* a, vDSP_Stride ia, const float* t, float* c, vDSP_Stride ic, vDSP_Length n)
{ const float v = *t; KX_LOOP(n) c[i * ic] = a[i * ia] < v ? v : a[i * ia]; }
static inline void vDSP_vclip(const float* a, vDSP_Stride ia, const float* lo, const float* hi, float* c, vDSP_Stride ic, vDSP_Length n)
{ KX_LOOP(n) { const float x = a[i * ia]; c[i * ic] = x < *lo ? *lo : x > *hi ? *hi : x; } }
static inline void vDSP_vfill(const float* s, float* c, vDSP_Stride ic, vDSP_Length n)
{ const float v = *s; KX_LOOP(n) c[i * ic] = v; }
static inline void vDSP_maxv(const float* a, vDSP_Stride ia, float* r, vDSP_Length n)
{ float m = -INFINITY; KX_LOOP(n) m = a[i * ia] > m ? a[i * ia] : m; *r = m; }
static inline void vDSP_minv(const float* a, vDSP_Stride ia, float* r, vDSP_Length n)
{ float m = INFINITY; KX_LOOP(n) m = a[i * ia] < m ? a[i * ia] : m; *r = m; }
static inline void vDSP_maxvi(const float* a, vDSP_Stride ia, float* r, vDSP_Length* ix, vDSP_Length n)
{ float m = -INFINITY; vDSP_Length k = 0; KX_LOOP(n) if (a[i * ia] > m) { m = a[i * ia]; k = i * (vDSP_Length)ia; } *r = m; *ix = k; }
static inline void vDSP_sve(const float* a, vDSP_Stride ia, float* r, vDSP_Length n)
{ float s = 0.0f; KX_LOOP(n) s += a[i * ia]; *r = s; }
static inline void vDSP_svesq(const float* a, vDSP_Stride ia, float* r, vDSP_Length n)
{ float s = 0.0f; KX_LOOP(n) s += a[i * ia] * a[i * ia]; *r = s; }
static inline void vDSP_meanv(const float* a, vDSP_Stride ia, float* r, vDSP_Length n)
{ float s = 0.0f; KX_LOOP(n) s += a[i * ia]; *r = n ? s / (float)n : 0.0f; }
/* c (m x n) = transpose of a (n x m) */
static inline void vDSP_mtrans(const float* a, vDSP_Stride ia, float* c, vDSP_Stride ic, vDSP_Length m, vDSP_Length n)
{
    for (vDSP_Length r = 0; r < m; r++)
        for (vDSP_Length k = 0; k < n; k++) c[(r * n + k) * ic] = a[(k * m + r) * ia];
}

static inline void vvexpf(float* y, const float* x, const int* n) { for (int i = 0; i < *n; i++) y[i] = expf(x[i]); }
static inline void vvlogf(float* y, const float* x, const int* n) { for (int i = 0; i < *n; i++) y[i] = logf(x[i]); }
static inline void vvsqrtf(float* y, const float* x, const int* n) { for (int i = 0; i < *n; i++) y[i] = sqrtf(x[i]); }
static inline void vvtanhf(float* y, const float* x, const int* n) { for (int i = 0; i < *n; i++) y[i] = tanhf(x[i]); }
static inline void vvrecf(float* y, const float* x, const int* n) { for (int i = 0; i < *n; i++) y[i] = 1.0f / x[i]; }

typedef enum { CblasRowMajor = 101, CblasColMajor = 102 } CBLAS_ORDER;
typedef enum { CblasNoTrans = 111, CblasTrans = 112 } CBLAS_TRANSPOSE;
/* numpy's bundled OpenBLAS (ILP64, symbol-suffixed build) */
void scipy_cblas_sgemm64_(int order, int ta, int tb, long m, long n, long k, float alpha, const float* a, long lda,
                          const float* b, long ldb, float beta, float* c, long ldc);
static inline void cblas_sgemm(CBLAS_ORDER o, CBLAS_TRANSPOSE ta, CBLAS_TRANSPOSE tb, int m, int n, int k, float alpha,
                               const float* a, int lda, const float* b, int ldb, float beta, float* c, int ldc)
{
    scipy_cblas_sgemm64_(o, ta, tb, m, n, k, alpha, a, lda, b, ldb, beta, c, ldc);
}

#endif
