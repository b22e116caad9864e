/* KERNIX-B200: the GPU backend of the reference's 2-D tensor library, on CUDA.
 *
 * The reference's include/kernix.h routes large tensor operations to a GPU through a small backend interface that a
 * build with KERNIX_USE_METAL links against (declarations include/kernix.h:30-37, 409-423, 936-990; implementation
 * src/kernix_metal.m). These are those functions, with the same names, arguments and return conventions, so the
 * reference's header-only tensor library uses B200 kernels unchanged:
 *
 *   kernix_metal_alloc / _free / _release_cache   tensor storage of >= 64 KB (include/kernix.h:156-160, 212-216):
 *                                                  here page-locked host memory mapped into the device address space
 *                                                  (the CPU code reads and writes it at host speed, kernels read and
 *                                                  write it directly over PCIe), freed buffers kept for reuse up to
 *                                                  256 MB as the reference keeps its Metal buffers (:36-37)
 *   kernix_metal_map        element-wise ops KERNIX_GPU_NEG .. KERNIX_GPU_DIV (include/kernix.h:409-414): the
 *                           float4-aligned prefix of n elements when n >= 2^22, bcols % 4 == 0 and y is backend
 *                           storage; returns the number of elements done (0: the caller's CPU code does them all)
 *   kernix_metal_rows       row softmax (mode 0), log_softmax (1), layer_norm (2) over rows x cols >= 2^22 into
 *                           backend storage; 1 if done, 0 if not
 *   kernix_metal_transpose  rows x cols -> cols x rows for rows * cols >= 2^22 into backend storage; 1 / 0
 *   kernix_matmul_ep_into   c = act(a . b + bias) (include/kernix.h:944-951): every row on the GPU (3xTF32), so
 *                           cpu_ep is called only when the inner dimension is 0 (all rows, as the reference does)
 *   float_matmul_metal      a . b into a new tensor (src/kernix_metal.m:319-328)
 *   floats_fma_relu_metal   y = max(a*x + b, 0) into a new tensor (include/kernix.h:990)
 * Inputs that are not backend storage are copied to the device first (the reference wraps them likewise). Results
 * are complete when a call returns. Tensors from float_matmul_metal / floats_fma_relu_metal are freed with
 * float_free (include/kernix.h), which hands backend storage back through kernix_metal_free.
 */
#ifndef KERNIX_GPU_H
#define KERNIX_GPU_H

#include <stddef.h>

#include "kernix.h"

#ifdef __cplusplus
extern "C" {
#endif

/* element-wise op codes (include/kernix.h:409-414) */
enum {
    KERNIX_GPU_NEG, KERNIX_GPU_ABS, KERNIX_GPU_EXP, KERNIX_GPU_LOG, KERNIX_GPU_SQRT, KERNIX_GPU_TANH,
    KERNIX_GPU_RELU, KERNIX_GPU_SIGMOID, KERNIX_GPU_SILU, KERNIX_GPU_GELU,
    KERNIX_GPU_ADD_SCALAR, KERNIX_GPU_MUL_SCALAR, KERNIX_GPU_CLAMP,
    KERNIX_GPU_ADD, KERNIX_GPU_SUB, KERNIX_GPU_MUL, KERNIX_GPU_DIV
};

/* the post-processing callback of kernix_matmul_ep_into for rows [r0, r1) computed on the CPU (the reference's
 * kernix_rows_fn, a block in the Apple build, a function pointer here) */
typedef void (*kernix_rows_fn)(size_t r0, size_t r1);

KERNIX_API void* kernix_metal_alloc(size_t bytes);
KERNIX_API int kernix_metal_free(void* p);
KERNIX_API void kernix_metal_release_cache(void);
KERNIX_API size_t kernix_metal_map(int op, const float* x, const float* b, size_t bcols, float* y, size_t n, float p0, float p1);
KERNIX_API int kernix_metal_rows(int mode, const float* x, const float* g, const float* b, float eps, float* y, size_t rows,
                                 size_t cols);
KERNIX_API int kernix_metal_transpose(const float* x, float* y, size_t rows, size_t cols);
KERNIX_API int kernix_matmul_ep_into(const float_tensor* a, const float_tensor* b, float_tensor* c, const float* bias, int act,
                                     float alpha, kernix_rows_fn cpu_ep);
KERNIX_API float_tensor* float_matmul_metal(const float_tensor* a, const float_tensor* b);
KERNIX_API float_tensor* floats_fma_relu_metal(const float_tensor* a, const float_tensor* x, const float_tensor* b);

#ifdef __cplusplus
}
#endif
#endif
