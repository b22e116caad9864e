/* Extra exports for the compiled reference (TEST INFRASTRUCTURE ONLY, built into oracle/_ref/).
 *
 * The reference keeps its int8 kernel static inline in include/kernix_model.h; these wrappers make
 * kernix_qweight_pack (:62-81) + kernix_qmatmul (:99-182) callable from the tests so that the
 * oracle's int8 restatement and the GPU kernel can be compared with the reference's own code on
 * the known-answer cases of test/model_test.c:363-446. */
#include "kernix_model.h"

#define KX_REF_API __attribute__((visibility("default")))

/* q: k x n row-major int8 (in x out), scale[n], bias[n] or NULL, x: rows x k, y: rows x n. 0 = ok */
KX_REF_API int kx_ref_qmatmul(const float* x, int rows, const int8_t* q, const float* scale, int k, int n,
                              const float* bias, int accumulate, float* y)
{
    kernix_qweight* w = kernix_qweight_pack(q, scale, k, n);
    if (w == NULL) return -1;
    const int rc = kernix_qmatmul(x, rows, w, bias, accumulate, y);
    kernix_qweight_free(w);
    return rc;
}

/* public model fields the reference's own tests read (test/model_test.c:54-55, :299-302) */
KX_REF_API void kx_ref_model_info(const kernix_model* m, long* out)
{
    out[0] = m->n_steps; out[1] = m->in_dim; out[2] = m->out_dim; out[3] = m->seq_len; out[4] = m->batch;
    out[5] = (long)m->ws_limit; out[6] = (long)m->ws_per_sample; out[7] = (long)m->ws_fixed; out[8] = m->layout;
}

/* step kinds and fused activations after load, for comparing the loader's fusion with ours */
KX_REF_API int kx_ref_model_steps(const kernix_model* m, int* kind, int* act, int cap)
{
    for (int i = 0; i < m->n_steps && i < cap; i++) { kind[i] = m->steps[i].kind; act[i] = m->steps[i].act; }
    return m->n_steps;
}

/* storage buffer of every value after planning (-1 = caller input), for comparing buffer plans */
KX_REF_API int kx_ref_model_plan(const kernix_model* m, int* st, int* last, int cap)
{
    for (int v = 0; v < m->n_vals && v < cap; v++) { st[v] = m->vals[v].st; last[v] = m->vals[v].last; }
    return m->n_vals;
}
