/* Internal structures of the KERNIX-B200 model runtime (host C). Not part of the public API. */
#ifndef KX_INTERNAL_H
#define KX_INTERNAL_H

#include <stddef.h>
#include <stdint.h>

#include "kernix_model.h"

/* weight dtypes of the .knx v2/v3 weight block (include/kernix_model.h:426) */
enum { KX_DT_F32, KX_DT_I8_COL, KX_DT_I8_ROW };

/* One graph value: per-sample channels-last shape; stored as (batch*r) x c rows */
typedef struct {
    int nd, d[KERNIX_MAX_DIMS];
    int r, c;   /* rows per sample (product of leading dims), channels */
    int st;     /* storage buffer, -1 = the model input buffer */
    int last;   /* last step reading this value (n_steps for the model output) */
} kx_val;

/* A weight block as read from the file and its device forms */
typedef struct {
    int present;
    int int8;          /* kept as int8 (I8_COL block of a LINEAR) */
    int k, n;          /* in x out */
    const float* f;    /* host float k x n: points into the mapped file (F32) or into `own` (dequantised) */
    float* own;        /* host buffer owned by this weight (dequantised int8 blocks), NULL otherwise */
    const int8_t* q;   /* host int8 k x n (kept int8), points into the mapped file */
    const float* scale_h; /* host scales (kept int8), points into the mapped file */
    /* device */
    int ldw;           /* K-major leading dimension of the device planes */
    float* d_hi;       /* n x ldw tf32 split planes (GEMM / conv operand B) */
    float* d_lo;
    int8_t* d_q;       /* n x ldw int8 */
    float* d_scale;    /* n */
    float* d_raw;      /* k x n as in the file (depthwise conv, embedding table) */
} kx_weight;

typedef struct {
    int kind, act;
    float alpha;
    int n_in, inp[KERNIX_MAX_INPUTS];
    int in, out;
    kx_weight w, wk, wv, wo;
    const float *bias, *bk, *bv, *bo, *gamma, *beta, *cst; /* host, into the mapped file */
    float eps;
    int kh, kw, sh, sw, dh, dw, pt, pb, pl, pr, groups;
    int ptype, count_pad;
    int perm[KERNIX_MAX_DIMS];
    int nd, d[KERNIX_MAX_DIMS];
    int axis, start, len, squeeze;
    int bop;
    int heads, dk, dv, causal;
    int seq, ret_seq, dirs, merge; /* LSTM / GRU / RNN: weights w (input) and wv (recurrent) of the forward
                                      * direction, wk and wo of the backward one; biases bias and bk */
    /* device */
    float *d_bias, *d_bk, *d_bv, *d_bo, *d_gamma, *d_beta, *d_cst;
    int qkv_fused;        /* ATTENTION with q = k = v: one GEMM with [Wq | Wk | Wv] */
    kx_weight wqkv;
    float* d_bqkv;
    size_t scratch_per_row; /* bytes of scratch per input row this step needs */
    int shard_c0, shard_n;  /* sharded LINEAR: this rank keeps output columns [shard_c0, shard_c0 + shard_n); 0 = whole */
    int fuse_add, fuse_res; /* fp32 LINEAR / ATTENTION whose output only feeds the next step, an elementwise ADD: the
                             * GEMM writes that ADD's output, adding value fuse_res (the ADD's other operand) */
    int i8c_n, i8c_in;      /* int8 LINEAR chains run as one launch (kx_i8_chain): i8c_n = its length on the first
                             * step (0 elsewhere); i8c_in = 1 on every step of such a chain */
    int mlp_n, mlp_layers;  /* first step of a fused small-MLP chain: mlp_layers fp32 LINEAR steps (+ a SOFTMAX when
                             * mlp_n > mlp_layers) run as one kx_mlp_chain launch for small batches; 0 = none */
    int qout, qin, qpar;    /* int8 LINEAR chains: qout = the GEMM writes the next int8 step's quantised input (its
                             * fp32 output is never materialised); qin = the input arrives quantised from the step
                             * before; qpar = which of the two scratch slots holds this step's quantised input */
} kx_step;

/* Parsed graph (host side), the output of kx_graph_load */
typedef struct {
    int ver, layout;
    int n_steps;     /* after ACT fusion */
    kx_step* steps;
    int n_vals, out_v;
    kx_val* vals;
    int n_st;
    size_t* st_cap;  /* floats per sample of each storage buffer */
    void* map;       /* mapped file */
    size_t map_len;
} kx_graph;

/* Parse, validate, infer shapes, fuse activations and plan storage, exactly as the reference loader does
 * (include/kernix_model.h:1448-1601). Returns NULL and sets *err (static string) on failure. */
kx_graph* kx_graph_load(const char* path, const char** err);
void kx_graph_free(kx_graph* g);

/* NCCL data plane (knx_nccl.c): a communicator on the current device, its release, and the all-gather of the
 * column-sharded forward over it (a kernix_allgather_fn with the communicator as its context) */
void* kx_nccl_comm_init(int rank, int world, const void* id);
void kx_nccl_comm_free(void* comm);
int kx_nccl_gather(void* ctx, const float* send, float* recv, size_t count, void* stream);

/* in-place capable kinds (include/kernix_model.h:1397-1401) */
int kx_inplace_ok(int kind);

#endif
