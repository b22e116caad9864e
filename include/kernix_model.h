/* KERNIX-B200 model runtime: load a .knx file (KNX1/KNX2/KNX3) and run its forward pass on a B200.
 *
 * Same API, argument meaning and error behaviour as the reference's header-only runtime
 * (include/kernix_model.h); here every function is exported from libkernix.so instead of static inline.
 * Each declaration names the reference interface it replaces (reference file:line).
 *
 * Values are per-sample channels-last shapes stored as (batch * leading dims) x channels rows, exactly
 * as in the reference; the forward pass takes and returns HOST float32 buffers and runs every step as
 * CUDA kernels on the model's device (the current CUDA device at load time, or $KERNIX_DEVICE).
 * There is no CPU fallback: a GPU failure makes forward return NULL with a message on stderr.
 */
#ifndef KERNIX_MODEL_H
#define KERNIX_MODEL_H

#include "kernix.h"

#ifdef __cplusplus
extern "C" {
#endif

/* op numbers of the .knx format (include/kernix_model.h:24-31); changing them breaks existing files */
enum {
    KERNIX_OP_LINEAR, KERNIX_OP_ACT, KERNIX_OP_LAYERNORM, KERNIX_OP_SOFTMAX, KERNIX_OP_LSTM,
    KERNIX_OP_GRU, KERNIX_OP_RNN, KERNIX_OP_CONV, KERNIX_OP_POOL, KERNIX_OP_GLOBAL_POOL,
    KERNIX_OP_RESHAPE, KERNIX_OP_PERMUTE, KERNIX_OP_BINARY, KERNIX_OP_CONCAT, KERNIX_OP_EMBEDDING,
    KERNIX_OP_AFFINE, KERNIX_OP_ADD_CONST, KERNIX_OP_ATTENTION, KERNIX_OP_SELECT, KERNIX_OP_PAD,
    KERNIX_OP_UPSAMPLE,
    KERNIX_OP_LAST = KERNIX_OP_UPSAMPLE
};
enum { KERNIX_BIN_ADD, KERNIX_BIN_SUB, KERNIX_BIN_MUL, KERNIX_BIN_DIV, KERNIX_BIN_MAX, KERNIX_BIN_MIN };
enum { KERNIX_POOL_MAX, KERNIX_POOL_AVG };
enum { KERNIX_AXIS_FIRST, KERNIX_AXIS_LAST };
#define KERNIX_MAX_DIMS 4
#define KERNIX_MAX_INPUTS 8
#define KERNIX_MAX_GEOM 65536
#define KERNIX_MODEL_MAX_OPS 1024
#define KERNIX_INT8_MAX_K 131072 /* 128*127*K < 2^31: int32 accumulators cannot overflow (reference :47) */

/* Default bound on the forward workspace in bytes. Here the workspace is device memory (HBM), so the
 * default is 4 GiB instead of the reference's 64 MiB of host memory (include/kernix_model.h:239-241);
 * a batch needing more runs in chunks, with results identical to an unchunked run. */
#ifndef KERNIX_WORKSPACE_LIMIT
#define KERNIX_WORKSPACE_LIMIT ((size_t)4 << 30)
#endif

struct kx_model_impl; /* parsed graph, device weights, workspace, stream (opaque) */

/* Public fields match the reference's kernix_model (include/kernix_model.h:263-291) by name and meaning. */
typedef struct kernix_model {
    int n_steps;           /* steps after ACT fusion into the preceding LINEAR/CONV */
    int in_dim, out_dim;   /* input channels; floats per sample of output */
    int seq_len;           /* input rows per sample (sequence T, image H*W, vector 1) */
    int batch;             /* input rows the workspace is sized for (one chunk), -1 = none */
    size_t ws_limit;       /* workspace bound in bytes, 0 = unlimited */
    size_t ws_per_sample;  /* device workspace floats per sample */
    size_t ws_fixed;       /* batch-independent workspace floats (0: no im2col buffer, no dequantised int8 copies) */
    int in_nd, in_shape[KERNIX_MAX_DIMS];   /* per-sample input shape, channels-last */
    int out_nd, out_shape[KERNIX_MAX_DIMS]; /* per-sample output shape, channels-last */
    int layout;            /* 0 = channels-last input, 1 = PyTorch channels-first (the binding moves the axis) */
    struct kx_model_impl* impl;
} kernix_model;

typedef struct { int segments, compiles, ane_runs, failures; } kernix_ane_info;

/* Replaces kernix_model_load (include/kernix_model.h:1448-1601): same format, same rejection rules.
 * Returns NULL with the reason on stderr for a bad file or when no CUDA device can hold the weights. */
KERNIX_API kernix_model* kernix_model_load(const char* path);

/* Replaces kernix_model_forward (include/kernix_model.h:2018-2064). x: (batch*seq_len) x in_dim host
 * floats (NHWC images, T x F sequences). Returns batch x out_dim host floats owned by the model and
 * overwritten by the next call (do not free). NULL on bad x (NULL, column mismatch, rows % seq_len != 0),
 * on x aliasing the model's own output, or on a GPU failure. batch 0 returns a 0 x out_dim view.
 * x is never modified. Not reentrant for one model; different models may run concurrently. */
KERNIX_API const float_tensor* kernix_model_forward(kernix_model* m, const float_tensor* x);

/* Replaces kernix_model_free (include/kernix_model.h:367-385); NULL allowed. */
KERNIX_API void kernix_model_free(kernix_model* m);

/* Replaces kernix_model_trim (include/kernix_model.h:343-357): releases the workspace (device arena and
 * pinned host output); weights stay. The next forward allocates again. */
KERNIX_API void kernix_model_trim(kernix_model* m);

/* Replaces kernix_model_set_workspace_limit (include/kernix_model.h:1691-1694). bytes 0 = unlimited. */
KERNIX_API void kernix_model_set_workspace_limit(kernix_model* m, size_t bytes);

/* Replaces kernix_model_set_ane (include/kernix_model.h:1815-1829). There is no Apple Neural Engine on a
 * B200 host: on = 1 returns -1 and the model keeps running on the GPU; on = 0 returns 0. */
KERNIX_API int kernix_model_set_ane(kernix_model* m, int on);

/* Replaces kernix_model_ane_info (include/kernix_model.h:1831-1841): always zeros. */
KERNIX_API void kernix_model_ane_info(const kernix_model* m, kernix_ane_info* out);

#ifdef __cplusplus
}
#endif
#endif
