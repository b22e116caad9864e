/* KERNIX-B200: the tensor type and activation numbering shared by the model API.
 *
 * Replaces the parts of the reference's include/kernix.h that the .knx model path exposes:
 *   float_tensor           include/kernix.h:39-43   (row-major rows x col floats, host memory)
 *   KERNIX_ACT_*           include/kernix.h:928-942 (numbering is part of the .knx format)
 *   floats_fma_relu        include/kernix.h:990     (fused y = max(a*x + b, 0); reference name floats_fma_relu_metal)
 * The reference header's 2-D tensor operations stay header-only; their GPU backend is include/kernix_gpu.h.
 */
#ifndef KERNIX_H
#define KERNIX_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(_WIN32)
#define KERNIX_API
#else
#define KERNIX_API __attribute__((visibility("default")))
#endif

typedef struct {
    int row;
    int col;
    float* tensor;
} float_tensor;

/* activation numbers (.knx format, docs/mlp-runtime-design.md); 0-4 exist in KNX1/KNX2 */
enum {
    KERNIX_ACT_NONE = -1, KERNIX_ACT_RELU, KERNIX_ACT_GELU, KERNIX_ACT_SILU, KERNIX_ACT_SIGMOID, KERNIX_ACT_TANH,
    KERNIX_ACT_LEAKY_RELU, KERNIX_ACT_ELU, KERNIX_ACT_SELU, KERNIX_ACT_SOFTPLUS, KERNIX_ACT_RELU6,
    KERNIX_ACT_HARD_SIGMOID, KERNIX_ACT_HARD_SWISH, KERNIX_ACT_GELU_TANH, KERNIX_ACT_EXP, KERNIX_ACT_MISH,
    KERNIX_ACT_SOFTSIGN,
    KERNIX_ACT_LAST = KERNIX_ACT_SOFTSIGN
};

/* y = max(a*x + b, 0) elementwise on the current CUDA device (fused multiply-add, then max, as the
 * reference's GPU kernel does, src/kernix_metal.m:331-338). a, x, b: same shape, host memory. Returns a
 * new host tensor (free with float_free) or NULL. Replaces floats_fma_relu_metal (include/kernix.h:990). */
KERNIX_API float_tensor* floats_fma_relu(const float_tensor* a, const float_tensor* x, const float_tensor* b);

/* frees a tensor returned by this library (NULL allowed) */
KERNIX_API void float_free(float_tensor* t);

#ifdef __cplusplus
}
#endif
#endif
