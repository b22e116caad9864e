/* KERNIX-B200 host-only inspection of a .knx file (no GPU needed).
 *
 * No counterpart in the reference: the reference's loader (include/kernix_model.h:1448-1601) has no
 * device step, so its parsing can be tested anywhere. This entry runs the same parse / validate / shape
 * inference / activation fusion / storage plan as kernix_model_load, without copying weights to a GPU,
 * so CPU-only callers and tests can check files and compare the loader with the reference.
 */
#ifndef KX_INSPECT_H
#define KX_INSPECT_H

#include "kernix.h"

#ifdef __cplusplus
extern "C" {
#endif

/* info[0..11] = n_steps, in_dim, out_dim, seq_len, layout, in_nd, out_nd, n_storage, version,
 *               storage floats per sample, fused-ACT count, 0; shapes[0..7] = in_shape[4], out_shape[4].
 * kinds/acts (capacity cap): step kind and fused activation per step after fusion.
 * Returns 0, or -1 with the rejection reason copied into err (errlen bytes). */
KERNIX_API int kx_knx_inspect(const char* path, long* info, int* shapes, int* kinds, int* acts, int cap, char* err,
                              int errlen);

/* Trace hook (no counterpart in the reference, whose intermediate values are host arrays): run the forward of
 * `rows` host input rows as one chunk and, right after each step, copy its output value into outs[k] (host,
 * (batch * r) x c floats for step k's output after activation fusion; NULL entries are skipped). Values are
 * captured before the storage plan lets a later step reuse their buffer. Returns 0 or -1. */
/* Storage plan of a .knx file without a GPU: st[v] = storage buffer of value v (-1 = the model input),
 * last[v] = last step reading it. Returns the number of values or -1. */
KERNIX_API int kx_knx_plan(const char* path, int* st, int* last, int cap);

struct kernix_model;
KERNIX_API int kx_model_forward_trace(struct kernix_model* m, const float* x, int rows, float** outs);

#ifdef __cplusplus
}
#endif
#endif
