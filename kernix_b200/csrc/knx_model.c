/* KERNIX-B200 model runtime: device weights, device workspace, chunked forward, public API.
 *
 * Replaces the reference's executor (include/kernix_model.h: workspace kernix_model_shape :1629-1676,
 * kernix_model_alloc :1679-1688, per-step dispatch kernix_step_run :1844-1905, kernix_model_run :1995-2016,
 * kernix_model_forward :2023-2064). Each model owns one CUDA stream on one device; a forward copies each
 * chunk of input rows host -> device, launches one kernel chain over the chunk, and copies the output rows
 * back, all ordered on that stream. Storage buffers follow the loader's plan (knx_load.c), so in-place steps
 * and RESHAPE views behave as in the reference. The workspace is a single device arena sized for one chunk.
 */
#define _GNU_SOURCE
#include <cuda_runtime_api.h>
#include <limits.h>
#include <math.h>
#include <stdint.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "kernix_capi.h"
#include "kernix_cuda.h"
#include "kernix_gpu.h"
#include "kx_inspect.h"
#include "kernix_model.h"
#include "kx_internal.h"
#include "kx_kernels.h"

#define KX_ALIGN 256
#define KX_PIPE_MAX 8             /* pieces a chunk of host rows is split into, at most */
#define KX_PIPE_MIN_BYTES (1 << 20) /* input bytes of one piece, at least */

#define KX_MAX_REPLICAS 15

struct kx_model_impl {
    kx_graph* g;
    int device;
    cudaStream_t stream;  /* kernels */
    cudaStream_t s_in;    /* host -> device copies of the host-memory forward */
    cudaStream_t s_out;   /* device -> host copies of the host-memory forward */
    /* per piece: end of its input copy, kernels and output copy (dependencies between the three streams only:
     * created without timing, which keeps cross-stream waits short) */
    cudaEvent_t ev_in[KX_PIPE_MAX], ev_comp[KX_PIPE_MAX], ev_out[KX_PIPE_MAX];
    cudaEvent_t ev_t0, ev_t1; /* start of the first input copy / end of the last output copy of the last chunk (timed,
                               * to choose the piece count) */
    int pipe;             /* pieces per chunk when pipelining ($KERNIX_PIPELINE; default 4) */
    int pipe_fixed;       /* 1: $KERNIX_PIPELINE was given, use it as is */
    int pipe_now;         /* pieces per chunk for the current chunk size (tuned over the first calls) */
    int tune_calls;       /* calls made at the current chunk size, while tuning */
    int tune_best;        /* fastest piece count tried so far, and its span in ms */
    float tune_best_ms;
    int last_pieces;      /* pieces of the last chunk of the last call (0: no timed chunk yet) */
    /* workspace (one arena) */
    void* arena;
    size_t arena_bytes;
    float** st;           /* device storage buffers as the running steps see them (a piece's rows) */
    float** st_base;      /* the same buffers from their first sample */
    float* xin;           /* device input rows */
    float* yout;          /* when set, the model output value lives here (a device forward writes the caller's
                           * buffer directly), else in its storage buffer */
    uint8_t* scratch;     /* per-step scratch: int8 activations, attention Q/K/V/context */
    int* status;          /* device status word of bounded waits */
    float* skinny_part;   /* partial sums of the skinny dense path (LINEAR steps of <= KX_SKINNY_MAX_ROWS rows) */
    size_t skinny_floats;
    float* split_part;    /* partial-sum planes of split-K dense steps (kx_gemm_f32_split), NULL if none splits */
    int32_t* i8s_part;    /* int32 planes of the small-batch int8 chains (kx_gemm_i8_split_acc), NULL if none */
    int* status_h;        /* pinned host copy */
    size_t scratch_per_row_max;
    int no_qchain;        /* 1 while tracing: every int8 step writes its fp32 output (int8 chains off) */
    void* nccl_comm;      /* the communicator of kernix_model_load_sharded_nccl (owned), else NULL */
    float* mlp_scratch;   /* partial sums of the fused small-MLP chains (kx_mlp_chain), NULL if the model has none */
    uint32_t* mlp_bar;    /* their grid-barrier words (zeroed at load; reset after a timeout) */
    /* batch sharding over the devices of $KERNIX_GPUS: whole-model replicas on the other devices; a host-memory
     * forward gives each device a contiguous share of the samples */
    int n_rep;
    kernix_model* rep[KX_MAX_REPLICAS];
    /* output-column sharding (kernix_model_load_sharded) */
    int rank, world;
    kernix_allgather_fn gather;
    void* gather_ctx;
    /* host output owned by the model (pinned) */
    float* out_host;
    size_t out_host_floats;
    float_tensor out_t;
};

static int dev_guard_enter(const kernix_model* m, int* prev) {
    if (cudaGetDevice(prev) != cudaSuccess) *prev = -1;
    if (*prev != m->impl->device && cudaSetDevice(m->impl->device) != cudaSuccess) return -1;
    return 0;
}

static void dev_guard_leave(const kernix_model* m, int prev) {
    if (prev >= 0 && prev != m->impl->device) cudaSetDevice(prev);
}

static size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

/* wait for the model's three streams; the first error seen, or cudaSuccess */
static cudaError_t sync_all(struct kx_model_impl* im) {
    cudaError_t e = cudaSuccess, f;
    cudaStream_t ss[3] = {im->s_in, im->stream, im->s_out};
    for (int i = 0; i < 3; i++)
        if (ss[i] && (f = cudaStreamSynchronize(ss[i])) != cudaSuccess && e == cudaSuccess) e = f;
    return e;
}

/* ------------------------------------------------------------------------------- weight upload */
/* Every copy and preparation kernel of the load goes on the model's stream: a legacy-stream cudaMemcpy from
 * pageable memory may return before its DMA has landed, and the model's non-blocking stream is not ordered
 * after the legacy stream, so mixing the two lets a preparation kernel read a half-copied buffer. */
static int upload(void** dst, const void* src, size_t bytes, cudaStream_t st) {
    if (cudaMalloc(dst, bytes ? bytes : 4) != cudaSuccess) return -1;
    if (bytes && cudaMemcpyAsync(*dst, src, bytes, cudaMemcpyHostToDevice, st) != cudaSuccess) return -1;
    return 0;
}

static int upload_f(float** dst, const float* src, size_t n, cudaStream_t st) {
    if (src == NULL) {
        *dst = NULL;
        return 0;
    }
    return upload((void**)dst, src, n * sizeof(float), st);
}

/* float weight k x n -> tf32 split planes n x ldw at rows [row0, row0+n) of (hi, lo); the uploaded k x n copy is
 * kept in *keep_raw when given (the skinny dense path streams it), freed otherwise */
static int prep_f32_into(const kx_weight* w, float* hi, float* lo, int ldw, size_t row0, cudaStream_t st, float** keep_raw) {
    float* raw = NULL;
    if (upload((void**)&raw, w->f, (size_t)w->k * w->n * sizeof(float), st) != 0) {
        cudaFree(raw);
        return -1;
    }
    int rc = kx_prep_f32_weight(raw, w->k, w->n, hi + row0 * (size_t)ldw, lo + row0 * (size_t)ldw, ldw, st);
    if (cudaStreamSynchronize(st) != cudaSuccess) rc = -1;
    if (keep_raw) *keep_raw = raw;
    else cudaFree(raw);
    return rc;
}

/* columns [c0, c0 + n) of a float weight k x N -> tf32 split planes n x ldw (the weight of one output slice) */
static int prep_f32_cols(kx_weight* w, int c0, int n, cudaStream_t st) {
    w->ldw = (int)round_up((size_t)w->k, 32);
    const size_t bytes = (size_t)n * w->ldw * sizeof(float);
    if (cudaMalloc((void**)&w->d_hi, bytes) != cudaSuccess || cudaMalloc((void**)&w->d_lo, bytes) != cudaSuccess) return -1;
    float* raw = NULL;
    if (cudaMalloc((void**)&raw, (size_t)w->k * n * sizeof(float)) != cudaSuccess) return -1;
    int rc = cudaMemcpy2DAsync(raw, (size_t)n * sizeof(float), w->f + c0, (size_t)w->n * sizeof(float), (size_t)n * sizeof(float),
                               (size_t)w->k, cudaMemcpyHostToDevice, st) == cudaSuccess ? 0 : -1;
    if (rc == 0) rc = kx_prep_f32_weight(raw, w->k, n, w->d_hi, w->d_lo, w->ldw, st);
    if (cudaStreamSynchronize(st) != cudaSuccess) rc = -1;
    w->d_raw = raw; /* k x n fp32, kept for the skinny dense path */
    return rc;
}

static int prep_f32(kx_weight* w, cudaStream_t st, int keep_raw) {
    w->ldw = (int)round_up((size_t)w->k, 32);
    const size_t bytes = (size_t)w->n * w->ldw * sizeof(float);
    if (cudaMalloc((void**)&w->d_hi, bytes) != cudaSuccess || cudaMalloc((void**)&w->d_lo, bytes) != cudaSuccess) return -1;
    return prep_f32_into(w, w->d_hi, w->d_lo, w->ldw, 0, st, keep_raw ? &w->d_raw : NULL);
}

static int prep_i8(kx_weight* w, cudaStream_t st) {
    w->ldw = (int)round_up((size_t)w->k, 16);
    int8_t* raw = NULL;
    if (cudaMalloc((void**)&w->d_q, (size_t)w->n * w->ldw) != cudaSuccess) return -1;
    if (upload((void**)&raw, w->q, (size_t)w->k * w->n, st) != 0 || upload_f(&w->d_scale, w->scale_h, (size_t)w->n, st) != 0) {
        cudaFree(raw);
        return -1;
    }
    int rc = kx_prep_i8_weight(raw, w->k, w->n, w->d_q, w->ldw, st);
    if (cudaStreamSynchronize(st) != cudaSuccess) rc = -1;
    cudaFree(raw);
    return rc;
}

/* recurrent weights u x G*u as plain fp32 rows on the device (int8 blocks kept as int8 are dequantised first,
 * as the reference's float copy of them, kernix_qweight_unpack :91-95) */
static int upload_raw_f32(kx_weight* w, cudaStream_t st) {
    if (!w->int8) return upload_f(&w->d_raw, w->f, (size_t)w->k * w->n, st);
    const size_t cnt = (size_t)w->k * w->n;
    float* tmp = malloc(cnt * sizeof(float));
    if (tmp == NULL) return -1;
    for (size_t i = 0; i < (size_t)w->k; i++)
        for (size_t j = 0; j < (size_t)w->n; j++) {
            float sc;
            memcpy(&sc, w->scale_h + j, sizeof sc);
            tmp[i * w->n + j] = (float)w->q[i * w->n + j] * sc;
        }
    int rc = upload_f(&w->d_raw, tmp, cnt, st);
    if (rc == 0 && cudaStreamSynchronize(st) != cudaSuccess) rc = -1;
    free(tmp);
    return rc;
}

static size_t rnn_gates(int kind) { return kind == KERNIX_OP_LSTM ? 4 : kind == KERNIX_OP_GRU ? 3 : 1; }

static void weight_dev_free(kx_weight* w) {
    cudaFree(w->d_hi);
    cudaFree(w->d_lo);
    cudaFree(w->d_q);
    cudaFree(w->d_scale);
    cudaFree(w->d_raw);
    w->d_hi = w->d_lo = w->d_raw = w->d_scale = NULL;
    w->d_q = NULL;
}

static int conv_pointwise(const kx_step* s) {
    return s->kh == 1 && s->kw == 1 && s->sh == 1 && s->sw == 1 && s->pt == 0 && s->pb == 0 && s->pl == 0 && s->pr == 0;
}

static int conv_depthwise(const kx_step* s) { return s->groups > 1 && s->in / s->groups == 1; }

/* convolutions that kx_conv_f32_ws may run from tf32 planes of their input (scratch: two copies of the input) */
static int conv_planes(const kx_step* s) {
    return s->kind == KERNIX_OP_CONV && !conv_depthwise(s) && !(s->groups == 1 && conv_pointwise(s)) && s->sh == 1 &&
           s->sw == 1 && s->groups >= 1 && (s->in / s->groups) % 32 == 0 && s->out / s->groups <= 128;
}

/* device copies of one step's parameters, in the layouts the kernels want */
static int step_upload(kx_graph* g, kx_step* s, cudaStream_t st) {
    switch (s->kind) {
    case KERNIX_OP_LINEAR:
        if (s->shard_n > 0) { /* this rank's output columns only */
            if (prep_f32_cols(&s->w, s->shard_c0, s->shard_n, st)) return -1;
            return upload_f(&s->d_bias, s->bias ? s->bias + s->shard_c0 : NULL, (size_t)s->shard_n, st);
        }
        if (s->w.int8 ? prep_i8(&s->w, st) : prep_f32(&s->w, st, 1)) return -1;
        return upload_f(&s->d_bias, s->bias, (size_t)s->out, st);
    case KERNIX_OP_CONV:
        if (conv_depthwise(s)) {
            if (upload_f(&s->w.d_raw, s->w.f, (size_t)s->w.k * s->w.n, st) != 0) return -1;
        } else if (prep_f32(&s->w, st, 0) != 0) {
            return -1;
        }
        return upload_f(&s->d_bias, s->bias, (size_t)s->out, st);
    case KERNIX_OP_LAYERNORM:
        return upload_f(&s->d_gamma, s->gamma, (size_t)s->in, st) || upload_f(&s->d_beta, s->beta, (size_t)s->in, st) ? -1 : 0;
    case KERNIX_OP_LSTM:
    case KERNIX_OP_GRU:
    case KERNIX_OP_RNN: {
        const size_t gu = rnn_gates(s->kind) * (size_t)s->out, nb = s->kind == KERNIX_OP_GRU ? 2 * gu : gu;
        if (prep_f32(&s->w, st, 0) || upload_raw_f32(&s->wv, st) || upload_f(&s->d_bias, s->bias, nb, st)) return -1;
        if (s->dirs == 2 && (prep_f32(&s->wk, st, 0) || upload_raw_f32(&s->wo, st) || upload_f(&s->d_bk, s->bk, nb, st))) return -1;
        return 0;
    }
    case KERNIX_OP_AFFINE:
        return upload_f(&s->d_gamma, s->gamma, (size_t)s->in, st) || upload_f(&s->d_beta, s->beta, (size_t)s->in, st) ? -1 : 0;
    case KERNIX_OP_ADD_CONST:
        return upload_f(&s->d_cst, s->cst, (size_t)s->in, st);
    case KERNIX_OP_EMBEDDING:
        return upload_f(&s->w.d_raw, s->w.f, (size_t)s->w.k * s->w.n, st);
    case KERNIX_OP_ATTENTION: {
        const size_t hk = (size_t)s->heads * s->dk, hv = (size_t)s->heads * s->dv;
        s->qkv_fused = s->n_in == 1;
        if (s->qkv_fused) { /* one GEMM: rows [Wq^T; Wk^T; Wv^T], columns of the product = [Q | K | V] */
            kx_weight* f = &s->wqkv;
            f->k = s->w.k;
            f->n = (int)(2 * hk + hv);
            f->ldw = (int)round_up((size_t)f->k, 32);
            const size_t bytes = (size_t)f->n * f->ldw * sizeof(float);
            if (cudaMalloc((void**)&f->d_hi, bytes) != cudaSuccess || cudaMalloc((void**)&f->d_lo, bytes) != cudaSuccess)
                return -1;
            if (prep_f32_into(&s->w, f->d_hi, f->d_lo, f->ldw, 0, st, NULL) || prep_f32_into(&s->wk, f->d_hi, f->d_lo, f->ldw, hk, st, NULL) ||
                prep_f32_into(&s->wv, f->d_hi, f->d_lo, f->ldw, 2 * hk, st, NULL))
                return -1;
            if (s->bias) {
                if (cudaMalloc((void**)&s->d_bqkv, (2 * hk + hv) * sizeof(float)) != cudaSuccess) return -1;
                if (cudaMemcpyAsync(s->d_bqkv, s->bias, hk * 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
                    cudaMemcpyAsync(s->d_bqkv + hk, s->bk, hk * 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
                    cudaMemcpyAsync(s->d_bqkv + 2 * hk, s->bv, hv * 4, cudaMemcpyHostToDevice, st) != cudaSuccess)
                    return -1;
            }
        } else {
            if (prep_f32(&s->w, st, 0) || prep_f32(&s->wk, st, 0) || prep_f32(&s->wv, st, 0)) return -1;
            if (upload_f(&s->d_bias, s->bias, hk, st) || upload_f(&s->d_bk, s->bk, hk, st) || upload_f(&s->d_bv, s->bv, hv, st)) return -1;
        }
        if (prep_f32(&s->wo, st, 0) != 0) return -1;
        return upload_f(&s->d_bo, s->bo, (size_t)s->out, st);
    }
    default:
        (void)g;
        return 0;
    }
}

static void step_dev_free(kx_step* s) {
    weight_dev_free(&s->w);
    weight_dev_free(&s->wk);
    weight_dev_free(&s->wv);
    weight_dev_free(&s->wo);
    weight_dev_free(&s->wqkv);
    cudaFree(s->d_bias); cudaFree(s->d_bk); cudaFree(s->d_bv); cudaFree(s->d_bo);
    cudaFree(s->d_gamma); cudaFree(s->d_beta); cudaFree(s->d_cst); cudaFree(s->d_bqkv);
    s->d_bias = s->d_bk = s->d_bv = s->d_bo = s->d_gamma = s->d_beta = s->d_cst = s->d_bqkv = NULL;
}

/* row pitch of the int8 activation slots: the largest quantised row any int8 LINEAR step reads or writes */
static size_t int8_pitch(const kx_graph* g) {
    size_t q = 16;
    for (int i = 0; i < g->n_steps; i++) {
        const kx_step* s = &g->steps[i];
        if (s->kind != KERNIX_OP_LINEAR || !s->w.int8) continue;
        if (round_up((size_t)s->in, 16) > q) q = round_up((size_t)s->in, 16);
        if (round_up((size_t)s->out, 16) > q) q = round_up((size_t)s->out, 16);
    }
    return q;
}

/* scratch bytes per input row (per sample for attention) that a step needs during its launch */
static size_t step_scratch(const kx_graph* g, const kx_step* s, size_t* per_sample) {
    *per_sample = 0;
    const kx_val* vi = &g->vals[s->inp[0]];
    if (s->kind == KERNIX_OP_LINEAR && s->shard_n > 0) { /* local slice, then the gathered [world][rows][slice] */
        *per_sample = (size_t)vi->r * ((size_t)s->shard_n + (size_t)s->out) * sizeof(float) + 2 * KX_ALIGN;
    } else if (s->kind == KERNIX_OP_LINEAR && s->w.int8 && s->i8c_n > 0) { /* a one-launch chain: int8 input of every
                                                                               * layer + row scales, control words */
        size_t b = 0;
        for (int l = 0; l < s->i8c_n; l++) b += round_up((size_t)s[l].in, 16) + 4 + (l > 0 ? 3 * 4 : 0);
        *per_sample = (size_t)vi->r * b + 4 * (size_t)s->i8c_n * KX_ALIGN;
    } else if (s->kind == KERNIX_OP_LINEAR && s->w.int8) { /* two int8 slots (rows x pitch + row scales), two ctl arrays */
        *per_sample = (size_t)vi->r * (2 * (int8_pitch(g) + 4) + 2 * 8) + 8 * KX_ALIGN;
    } else if (s->kind == KERNIX_OP_LSTM || s->kind == KERNIX_OP_GRU || s->kind == KERNIX_OP_RNN) {
        /* input projections of all steps, two state buffers, the cell state, the second direction's output */
        const size_t T = (size_t)vi->r, u = (size_t)s->out, gu = rnn_gates(s->kind) * u;
        *per_sample = (T * gu + 3 * u + (s->dirs == 2 && s->merge != 0 ? (s->ret_seq ? T : 1) * u : 0)) * sizeof(float) +
                      4 * KX_ALIGN;
    } else if (conv_planes(s)) { /* tf32 hi / lo planes of the input */
        *per_sample = 2 * (size_t)vi->r * (size_t)vi->c * sizeof(float) + KX_ALIGN;
    } else if (s->kind == KERNIX_OP_ATTENTION) {
        const kx_val* vv = &g->vals[s->inp[s->n_in > 1 ? 1 : 0]];
        const size_t hk = (size_t)s->heads * s->dk, hv = (size_t)s->heads * s->dv;
        const size_t rq = (size_t)vi->r, S = (size_t)vv->r;
        *per_sample = (rq * hk + S * hk + S * hv + rq * hv) * sizeof(float) + 4 * KX_ALIGN;
    }
    return *per_sample;
}

static void model_release(kernix_model* m) {
    struct kx_model_impl* im = m->impl;
    if (im->arena) cudaFree(im->arena);
    im->arena = NULL;
    im->arena_bytes = 0;
    free(im->st);
    im->st = NULL;
    free(im->st_base);
    im->st_base = NULL;
    im->xin = NULL;
    im->scratch = NULL;
    im->status = NULL;
    if (im->out_host) cudaFreeHost(im->out_host);
    im->out_host = NULL;
    im->out_host_floats = 0;
    m->batch = -1;
}

/* arena for `rows` input rows: storage buffers, input rows, scratch, status word */
static int model_alloc(kernix_model* m, int rows);

static int model_alloc(kernix_model* m, int rows) {
    struct kx_model_impl* im = m->impl;
    kx_graph* g = im->g;
    float* keep_out = im->out_host;
    size_t keep_n = im->out_host_floats;
    im->out_host = NULL;
    model_release(m);
    im->out_host = keep_out;
    im->out_host_floats = keep_n;
    const size_t B = (size_t)rows / (size_t)m->seq_len;
    size_t off = 0;
    size_t* st_off = calloc((size_t)g->n_st + 1, sizeof(size_t));
    im->st = calloc((size_t)g->n_st + 1, sizeof(float*));
    im->st_base = calloc((size_t)g->n_st + 1, sizeof(float*));
    if (st_off == NULL || im->st == NULL || im->st_base == NULL) {
        free(st_off);
        return -1;
    }
    for (int k = 0; k < g->n_st; k++) {
        st_off[k] = off;
        off = round_up(off + B * g->st_cap[k] * sizeof(float), KX_ALIGN);
    }
    const size_t xin_off = off;
    off = round_up(off + (size_t)rows * m->in_dim * sizeof(float), KX_ALIGN);
    const size_t scr_off = off;
    off = round_up(off + B * im->scratch_per_row_max + KX_ALIGN, KX_ALIGN);
    const size_t status_off = off;
    off += KX_ALIGN;
    if (cudaMalloc(&im->arena, off) != cudaSuccess) {
        im->arena = NULL;
        free(st_off);
        fprintf(stderr, "forward: cannot allocate %zu bytes of device workspace\n", off);
        return -1;
    }
    im->arena_bytes = off;
    uint8_t* base = (uint8_t*)im->arena;
    for (int k = 0; k < g->n_st; k++) im->st[k] = im->st_base[k] = (float*)(base + st_off[k]);
    im->xin = (float*)(base + xin_off);
    im->scratch = base + scr_off;
    im->status = (int*)(base + status_off);
    free(st_off);
    if (cudaMemsetAsync(im->status, 0, sizeof(int), im->stream) != cudaSuccess) return -1;
    m->batch = rows;
    im->pipe_now = im->pipe;
    im->tune_calls = 0;
    im->tune_best = 0;
    return 0;
}

/* device pointer of value v in the current chunk */
static float* val_ptr(const struct kx_model_impl* im, int v) {
    if (v == im->g->out_v && im->yout != NULL) return im->yout;
    const kx_val* val = &im->g->vals[v];
    return val->st < 0 ? im->xin : im->st[val->st];
}

static void* align_ptr(void* p) { return (void*)round_up((uintptr_t)p, KX_ALIGN); }

/* Mark the fp32 LINEAR / ATTENTION steps whose output is read only by the next step, an ADD of two operands of the
 * same shape: the GEMM that produces the output adds the ADD's other operand in its epilogue and writes the ADD's
 * output (the same round-to-nearest add on the same values, so the same bits), and the ADD step is skipped. The
 * ADD's output must not share storage with the LINEAR's input, which the GEMM is still reading. */
static void plan_fusions(kx_graph* g) {
    for (int i = 0; i + 1 < g->n_steps; i++) {
        kx_step* s = &g->steps[i];
        const kx_step* t = &g->steps[i + 1];
        s->fuse_add = 0;
        const int gemm = (s->kind == KERNIX_OP_LINEAR && !s->w.int8 && s->shard_n == 0) || s->kind == KERNIX_OP_ATTENTION;
        if (!gemm || t->kind != KERNIX_OP_BINARY || t->bop != 0 || t->n_in != 2) continue;
        const int out = i + 1, res = t->inp[0] == out ? t->inp[1] : t->inp[0];
        if ((t->inp[0] == out) == (t->inp[1] == out)) continue; /* the output is not exactly one of the operands */
        const kx_val *vo = &g->vals[out], *vr = &g->vals[res], *vy = &g->vals[i + 2];
        if (vo->last != i + 1 || out == g->out_v) continue;
        if (vo->r != vr->r || vo->c != vr->c || vo->r != vy->r || vo->c != vy->c) continue;
        if (s->kind == KERNIX_OP_LINEAR && vy->st == g->vals[s->inp[0]].st) continue;
        s->fuse_add = 1;
        s->fuse_res = res;
    }
}

/* Chains of int8 LINEAR steps: a step whose output is read only by the next step, itself an int8 LINEAR taking that
 * output as its input, runs kx_gemm_i8_q: its epilogue writes the next step's quantised rows and row scales (the
 * kernix_qmatmul quantisation, bit for bit) instead of fp32 rows, so neither the fp32 intermediate nor a separate
 * quantiser pass exists. The quantised rows alternate between two scratch slots along the chain. Needs CTA-pair
 * tiles (more than 128 columns), at most 64 tiles of 256 columns (a row group's tiles are resident at once) and a
 * reduction of at least KX_QCHAIN_MIN_K (the two-pass epilogue must hide under the tile's MMAs). */
static int act_kind(int act) { return act == KERNIX_ACT_NONE || act == KERNIX_ACT_RELU || act == KERNIX_ACT_GELU ? act : 99; }

/* int8 chains for one launch (kx_i8_chain): 2 to 4 int8 LINEAR steps, each after the first reading only the previous
 * step's output, which nothing else reads; every layer on CTA-pair tiles (more than 128 outputs, at most 64 tiles of
 * 256), the hidden layers' activations of one kind */
static void plan_i8chain(kx_graph* g) {
    for (int i = 0; i < g->n_steps; i++) g->steps[i].i8c_n = g->steps[i].i8c_in = 0;
    const char* off = getenv("KERNIX_NO_I8_CHAIN"); /* 1: int8 layers launch one by one (tests compare the two) */
    if (off && *off && *off != '0') return;
    for (int i = 0; i < g->n_steps;) {
        int j = i;
        while (j < g->n_steps && j - i < 4) {
            const kx_step* s = &g->steps[j];
            if (s->kind != KERNIX_OP_LINEAR || !s->w.int8 || s->out <= 128 || (s->out + 255) / 256 > 64) break;
            if (j > i && (s->n_in != 1 || s->inp[0] != j || g->vals[j].last != j || g->out_v == j || s->in != g->steps[j - 1].out))
                break;
            if (j > i + 1 && act_kind(g->steps[j - 1].act) != act_kind(g->steps[i].act)) break;
            j++;
        }
        if (j - i >= 2) {
            g->steps[i].i8c_n = j - i;
            for (int l = i; l < j; l++) g->steps[l].i8c_in = 1;
            i = j;
        } else {
            i++;
        }
    }
}

#define KX_QCHAIN_MIN_K 2048 /* below this the epilogue, not the MMAs, paces a tile (measured: K = 1024 gains nothing) */
static void plan_qchain(kx_graph* g) {
    for (int i = 0; i < g->n_steps; i++) g->steps[i].qout = g->steps[i].qin = g->steps[i].qpar = 0;
    for (int i = 0; i + 1 < g->n_steps; i++) {
        kx_step* s = &g->steps[i];
        kx_step* t = &g->steps[i + 1];
        /* the fused epilogue pays only where the MMAs of a tile outlast it: long reductions */
        const int int8_pair = s->kind == KERNIX_OP_LINEAR && s->w.int8 && s->out > 128 && (s->out + 255) / 256 <= 64 &&
                              s->in >= KX_QCHAIN_MIN_K;
        if (!int8_pair || t->kind != KERNIX_OP_LINEAR || !t->w.int8 || t->n_in != 1 || t->inp[0] != i + 1) continue;
        if (s->i8c_in || t->i8c_in) continue; /* runs inside a one-launch chain */
        if (g->vals[i + 1].last != i + 1 || g->out_v == i + 1 || t->in != s->out) continue;
        s->qout = 1;
        t->qin = 1;
        t->qpar = 1 - s->qpar;
    }
}

/* Small MLPs: a run of fp32 LINEAR steps, each after the first reading only the previous step's output, which
 * nothing else reads, optionally followed by a SOFTMAX of the last output (at most 64 columns), runs as one
 * kx_mlp_chain launch when a chunk has at most KX_MLP_MAX_ROWS rows (the tensor-core GEMMs' per-launch costs
 * dominate there). Chains that end in a fused residual ADD are left to the GEMMs (their fusion keeps the forward
 * bit-identical to running the steps one by one). */
#define KX_MLP_MAX_WEIGHTS ((size_t)1 << 21) /* weight floats of a fused small-MLP chain (8 MB) */
static void plan_mlp(kx_graph* g) {
    for (int i = 0; i < g->n_steps; i++) g->steps[i].mlp_n = g->steps[i].mlp_layers = 0;
    const char* off = getenv("KERNIX_NO_MLP_CHAIN"); /* 1: always the per-step GEMMs (tests compare the two) */
    if (off && *off && *off != '0') return;
    for (int i = 0; i < g->n_steps;) {
        int j = i;
        while (j < g->n_steps && j - i < KX_MLP_MAX_LAYERS) {
            const kx_step* s = &g->steps[j];
            if (s->kind != KERNIX_OP_LINEAR || s->w.int8 || s->shard_n > 0 || s->fuse_add) break;
            if (j > i && (s->n_in != 1 || s->inp[0] != j || g->vals[j].last != j || g->out_v == j)) break;
            j++;
        }
        const int layers = j - i;
        int ok = layers >= 1 && g->steps[i].in % 4 == 0;
        size_t wfloats = 0;
        for (int l = i; l < j; l++) wfloats += (size_t)g->steps[l].in * (size_t)g->steps[l].out;
        ok = ok && wfloats <= KX_MLP_MAX_WEIGHTS; /* small weights only: larger layers belong on the tensor cores */
        for (int l = i; ok && l + 1 < j; l++) ok = g->steps[l].out % 4 == 0;
        int sm = 0;
        if (ok && j < g->n_steps) {
            const kx_step* t = &g->steps[j];
            sm = t->kind == KERNIX_OP_SOFTMAX && t->inp[0] == j && g->vals[j].last == j && g->out_v != j &&
                 g->steps[j - 1].out <= 64;
        }
        if (ok && layers + sm >= 2) {
            g->steps[i].mlp_layers = layers;
            g->steps[i].mlp_n = layers + sm;
            i = j + sm;
        } else {
            i++;
        }
    }
}

/* the fused small-MLP chain starting at step i over `rin` rows (kx_mlp_chain) */
static int mlp_run(kernix_model* m, int i, long rin) {
    struct kx_model_impl* im = m->impl;
    kx_graph* g = im->g;
    const kx_step* s0 = &g->steps[i];
    const float* w[KX_MLP_MAX_LAYERS];
    const float* b[KX_MLP_MAX_LAYERS];
    int k[KX_MLP_MAX_LAYERS], n[KX_MLP_MAX_LAYERS], act[KX_MLP_MAX_LAYERS];
    float alpha[KX_MLP_MAX_LAYERS];
    for (int l = 0; l < s0->mlp_layers; l++) {
        const kx_step* s = &g->steps[i + l];
        w[l] = s->w.d_raw;
        b[l] = s->d_bias;
        k[l] = s->in;
        n[l] = s->out;
        act[l] = s->act;
        alpha[l] = s->alpha;
    }
    return kx_mlp_chain(val_ptr(im, s0->inp[0]), s0->in, (int)rin, s0->mlp_layers, w, b, k, n, act, alpha,
                        s0->mlp_n > s0->mlp_layers, val_ptr(im, i + s0->mlp_n), im->mlp_scratch, im->mlp_bar, im->status,
                        im->stream);
}

#define KX_I8S_MAX_ROWS 64 /* measured on c2: the chain kernel wins from ~128 rows */
/* small batches of an int8 chain (KX_I8S_MAX_ROWS rows or fewer): each layer's reduction split over the SMs into int32
 * planes (kx_gemm_i8_split_acc), then one block per row adds them and dequantises, activates and quantises the row for
 * the next layer or stores the last layer's fp32 rows (kx_i8_rows). Few rows give the chain kernel few tiles, so its
 * layers stream their weights through a few SMs one after another; here every layer's weights spread over all SMs.
 * Bit for bit the chain kernel's result. */
static int i8split_planes(int m, int n, int k) {
    const int kbs = kx_i8_split_blocks(m, n, k), nk = (k + 127) / 128;
    return (nk + kbs - 1) / kbs;
}
static int i8split_ok(const kx_graph* g, int i) { /* every layer within kx_i8_rows' row width */
    for (int l = 0; l < g->steps[i].i8c_n; l++)
        if (round_up((size_t)g->steps[i + l].out, 16) > 8192) return 0;
    return 1;
}
static int i8split_run(struct kx_model_impl* im, int n, long rin, const int8_t* const* a, const int* lda, const float* const* sx,
                       const int8_t* const* wq, const int* ldw, const float* const* scale, const float* const* bias,
                       const int* k, const int* nn, const int* act, const float* alpha, float* const* sx_out, float* y) {
    for (int l = 0; l < n; l++) {
        const int kbs = kx_i8_split_blocks((int)rin, nn[l], k[l]), planes = ((k[l] + 127) / 128 + kbs - 1) / kbs;
        if (kx_gemm_i8_split_acc(a[l], lda[l], wq[l], ldw[l], (int)rin, nn[l], k[l], kbs, im->i8s_part, im->status,
                                 im->stream) != 0)
            return -1;
        const int last = l == n - 1;
        if (kx_i8_rows(im->i8s_part, planes, (int)rin, nn[l], sx[l], scale[l], bias[l], act[l], alpha[l], last ? y : NULL,
                       last ? nn[l] : 0, last ? NULL : (int8_t*)a[l + 1], last ? 0 : lda[l + 1], last ? NULL : sx_out[l],
                       im->stream) != 0)
            return -1;
    }
    return 0;
}

/* the one-launch int8 chain starting at step i over `rin` rows: quantise its input (clearing the chain's control
 * words), then kx_i8_chain; scratch: per layer its int8 input (rows x K rounded to 16) and row scales, then the
 * control words */
static int i8chain_run(kernix_model* m, int i, long rin) {
    struct kx_model_impl* im = m->impl;
    kx_graph* g = im->g;
    const kx_step* s0 = &g->steps[i];
    const int n = s0->i8c_n;
    const int8_t* a[4];
    int lda[4], k[4], nn[4], act[4], ldw[4];
    const float *sx[4], *scale[4], *bias[4];
    float* sx_out[4] = {NULL, NULL, NULL, NULL};
    float alpha[4];
    const int8_t* wq[4];
    uint8_t* p = (uint8_t*)align_ptr(im->scratch);
    for (int l = 0; l < n; l++) {
        const kx_step* s = &g->steps[i + l];
        lda[l] = (int)round_up((size_t)s->in, 16);
        a[l] = (const int8_t*)p;
        p = (uint8_t*)align_ptr(p + (size_t)rin * lda[l]);
        sx[l] = (const float*)p;
        if (l > 0) sx_out[l - 1] = (float*)p;
        p = (uint8_t*)align_ptr(p + (size_t)rin * sizeof(float));
        wq[l] = s->w.d_q;
        ldw[l] = s->w.ldw;
        scale[l] = s->w.d_scale;
        bias[l] = s->d_bias;
        k[l] = s->in;
        nn[l] = s->out;
        act[l] = s->act;
        alpha[l] = s->alpha;
    }
    uint32_t* ctl = (uint32_t*)p;
    if (rin <= KX_I8S_MAX_ROWS && im->i8s_part != NULL && i8split_ok(g, i)) {
        if (kx_quant_rows(val_ptr(im, s0->inp[0]), s0->in, (int)rin, s0->in, (int8_t*)a[0], lda[0], (float*)sx[0], im->stream) != 0)
            return -1;
        return i8split_run(im, n, rin, a, lda, sx, wq, ldw, scale, bias, k, nn, act, alpha, sx_out, val_ptr(im, i + n));
    }
    const size_t words = (size_t)(n - 1) * ((size_t)rin + 2 * (((size_t)rin + 127) / 128));
    if (kx_quant_rows_z(val_ptr(im, s0->inp[0]), s0->in, (int)rin, s0->in, (int8_t*)a[0], lda[0], (float*)sx[0], ctl, (int)words,
                        im->stream) != 0)
        return -1;
    return kx_i8_chain(n, (int)rin, a, lda, sx, wq, ldw, scale, bias, k, nn, act, alpha, sx_out, ctl, val_ptr(im, i + n),
                       im->status, im->stream);
}

/* one step over B samples; fused: the step's GEMM also performs the next step, an ADD (plan_fusions) */
static int step_run(kernix_model* m, int i, int B, int fused) {
    struct kx_model_impl* im = m->impl;
    kx_graph* g = im->g;
    kx_step* s = &g->steps[i];
    const kx_val* vi = &g->vals[s->inp[0]];
    const kx_val* vo = &g->vals[i + 1];
    const float* a = val_ptr(im, s->inp[0]);
    float* y = val_ptr(im, fused ? i + 2 : i + 1);
    const float* res = fused ? val_ptr(im, s->fuse_res) : NULL;
    const long rin = (long)B * vi->r, rout = (long)B * vo->r;
    cudaStream_t st = im->stream;
    switch (s->kind) {
    case KERNIX_OP_LINEAR:
        if (s->w.int8) { /* scratch: int8 slots 0 and 1 (rows x pitch, then the row scales), ctl arrays 0 and 1 */
            const int ldq = (int)round_up((size_t)s->in, 16);
            const size_t pitch = int8_pitch(g), q_bytes = round_up((size_t)rin * pitch, KX_ALIGN);
            const size_t slot = q_bytes + round_up((size_t)rin * sizeof(float), KX_ALIGN);
            const size_t cw = (size_t)rin + ((size_t)rin + 127) / 128;
            uint8_t* sc = (uint8_t*)align_ptr(im->scratch);
            int8_t* xq_slot[2] = {(int8_t*)sc, (int8_t*)(sc + slot)};
            float* sx_slot[2] = {(float*)(sc + q_bytes), (float*)(sc + slot + q_bytes)};
            uint32_t* ctl[2] = {(uint32_t*)(sc + 2 * slot), (uint32_t*)(sc + 2 * slot + round_up(cw * 4, KX_ALIGN))};
            const int chain = !im->no_qchain, p = s->qpar;
            const int qin = chain && s->qin, qout = chain && s->qout;
            if (!qin && kx_quant_rows_z(a, s->in, (int)rin, s->in, xq_slot[p], ldq, sx_slot[p], qout ? ctl[p] : NULL,
                                        qout ? (int)cw : 0, st) != 0)
                return -1;
            if (qout) { /* this GEMM's ctl[p] was cleared by the kernel before it; it clears the next one's */
                const int zn = g->steps[i + 1].qout;
                return kx_gemm_i8_q(xq_slot[p], ldq, sx_slot[p], s->w.d_q, s->w.ldw, s->w.d_scale, s->d_bias, (int)rin, s->out,
                                    s->in, s->act, s->alpha, xq_slot[1 - p], (int)round_up((size_t)s->out, 16), sx_slot[1 - p],
                                    ctl[p], zn ? ctl[1 - p] : NULL, zn ? (int)cw : 0, im->status, st);
            }
            return kx_gemm_i8(xq_slot[p], ldq, sx_slot[p], s->w.d_q, s->w.ldw, s->w.d_scale, s->d_bias, y, s->out, (int)rin,
                              s->out, s->in, s->act, s->alpha, im->status, st);
        }
        const int skinny = rin <= KX_SKINNY_MAX_ROWS && s->w.d_raw != NULL && im->skinny_part != NULL;
        const int ncols = s->shard_n > 0 ? s->shard_n : s->out;
        /* 17..128 rows of a layer with few output tiles: K split over the idle SMs, planes added in a fixed order */
        const int splits = !skinny && !res && im->split_part != NULL ? kx_gemm_f32_splits((int)rin, ncols, s->in) : 1;
        if (s->shard_n > 0) { /* this rank's columns, all-gather across ranks, re-interleave into full rows */
            float* yl = (float*)align_ptr(im->scratch);
            float* yg = (float*)align_ptr(yl + (size_t)rin * s->shard_n);
            if ((skinny ? kx_gemm_f32_skinny(a, s->in, s->w.d_raw, s->d_bias, yl, s->shard_n, (int)rin, s->shard_n, s->in, s->act,
                                             s->alpha, im->skinny_part, im->skinny_floats, st)
                        : kx_gemm_f32_split(a, s->in, s->w.d_hi, s->w.d_lo, s->w.ldw, s->d_bias, yl, s->shard_n, (int)rin,
                                            s->shard_n, s->in, s->act, s->alpha, splits, im->split_part, im->status, st)) != 0)
                return -1;
            if (im->gather(im->gather_ctx, yl, yg, (size_t)rin * s->shard_n, st) != 0) {
                fprintf(stderr, "forward: the all-gather of step %d failed\n", i);
                return -1;
            }
            return kx_unshard_cols(yg, im->world, rin, s->shard_n, y, s->out, st);
        }
        if (skinny) /* few rows: stream the fp32 weights on the CUDA cores, K split over the SMs (never fused) */
            return kx_gemm_f32_skinny(a, s->in, s->w.d_raw, s->d_bias, y, s->out, (int)rin, s->out, s->in, s->act, s->alpha,
                                      im->skinny_part, im->skinny_floats, st);
        if (res)
            return kx_gemm_f32_res(a, s->in, s->w.d_hi, s->w.d_lo, s->w.ldw, s->d_bias, y, s->out, (int)rin, s->out, s->in,
                                   s->act, s->alpha, res, s->out, im->status, st);
        if (splits > 1)
            return kx_gemm_f32_split(a, s->in, s->w.d_hi, s->w.d_lo, s->w.ldw, s->d_bias, y, s->out, (int)rin, s->out, s->in,
                                     s->act, s->alpha, splits, im->split_part, im->status, st);
        return kx_gemm_f32(a, s->in, s->w.d_hi, s->w.d_lo, s->w.ldw, s->d_bias, y, s->out, (int)rin, s->out, s->in, s->act,
                           s->alpha, im->status, st);
    case KERNIX_OP_ACT:
        return kx_bias_act(a, y, rout, vo->c, NULL, s->act, s->alpha, st);
    case KERNIX_OP_LAYERNORM:
        return kx_layernorm_rows(a, y, rout, vo->c, s->d_gamma, s->d_beta, s->eps, st);
    case KERNIX_OP_SOFTMAX:
        return kx_softmax_rows(a, y, rout, vo->c, st);
    case KERNIX_OP_CONV: {
        const int H = vi->d[0], W = vi->nd == 3 ? vi->d[1] : 1, Ho = vo->d[0], Wo = vo->nd == 3 ? vo->d[1] : 1;
        if (s->groups == 1 && conv_pointwise(s))
            return kx_gemm_f32(a, s->in, s->w.d_hi, s->w.d_lo, s->w.ldw, s->d_bias, y, s->out, (int)rin, s->out, s->in,
                               s->act, s->alpha, im->status, st);
        if (conv_depthwise(s))
            return kx_conv_depthwise(a, s->w.d_raw, s->d_bias, y, B, H, W, vi->c, vo->c, Ho, Wo, s->kh, s->kw, s->sh, s->sw,
                                     s->dh, s->dw, s->pt, s->pl, s->act, s->alpha, st);
        if (conv_planes(s))
            return kx_conv_f32_ws(a, s->w.d_hi, s->w.d_lo, s->w.ldw, s->d_bias, y, B, H, W, vi->c, vo->c, Ho, Wo, s->kh, s->kw,
                                  s->sh, s->sw, s->dh, s->dw, s->pt, s->pl, s->groups, s->act, s->alpha,
                                  (float*)align_ptr(im->scratch), 2 * (size_t)rin * (size_t)vi->c, im->status, st);
        return kx_conv_f32(a, s->w.d_hi, s->w.d_lo, s->w.ldw, s->d_bias, y, B, H, W, vi->c, vo->c, Ho, Wo, s->kh, s->kw, s->sh,
                           s->sw, s->dh, s->dw, s->pt, s->pl, s->groups, s->act, s->alpha, im->status, st);
    }
    case KERNIX_OP_POOL: {
        const int H = vi->d[0], W = vi->nd == 3 ? vi->d[1] : 1, Ho = vo->d[0], Wo = vo->nd == 3 ? vo->d[1] : 1;
        return kx_pool2d(a, y, B, H, W, vi->c, Ho, Wo, s->kh, s->kw, s->sh, s->sw, s->pt, s->pl, s->ptype, s->count_pad, st);
    }
    case KERNIX_OP_GLOBAL_POOL:
        return kx_global_pool(a, y, B, vi->r, vi->c, s->ptype, st);
    case KERNIX_OP_RESHAPE:
        return 0;
    case KERNIX_OP_PERMUTE:
        return kx_permute(a, y, B, vi->nd, vi->d, s->perm, st);
    case KERNIX_OP_BINARY: {
        const kx_val* vb = &g->vals[s->inp[1]];
        return kx_binary(a, vi->r, vi->c, val_ptr(im, s->inp[1]), vb->r, vb->c, y, B, vo->r, vo->c, s->bop, st);
    }
    case KERNIX_OP_CONCAT: {
        long off = 0;
        for (int k = 0; k < s->n_in; k++) {
            const kx_val* v = &g->vals[s->inp[k]];
            const float* src = val_ptr(im, s->inp[k]);
            if (s->axis == KERNIX_AXIS_LAST) {
                if (kx_copy_cols(src, v->c, y, vo->c, off, rout, v->c, st) != 0) return -1;
                off += v->c;
            } else {
                const long per = (long)v->r * v->c;
                if (kx_copy_cols(src, per, y, (long)vo->r * vo->c, off, B, per, st) != 0) return -1;
                off += per;
            }
        }
        return 0;
    }
    case KERNIX_OP_EMBEDDING:
        return kx_embedding(a, rin * vi->c, s->w.d_raw, s->w.k, s->w.n, y, st);
    case KERNIX_OP_AFFINE:
        return kx_affine_rows(a, y, rout, vo->c, s->d_gamma, s->d_beta, st);
    case KERNIX_OP_ADD_CONST:
        return kx_add_const(a, y, B, s->in, s->d_cst, st);
    case KERNIX_OP_SELECT:
        if (s->axis == KERNIX_AXIS_FIRST) {
            const long per = (long)vi->r * vi->c, blk = per / vi->d[0];
            return kx_copy_cols(a + (long)s->start * blk, per, y, blk * s->len, 0, B, blk * s->len, st);
        }
        return kx_copy_cols(a + s->start, vi->c, y, s->len, 0, rin, s->len, st);
    case KERNIX_OP_PAD: {
        const int H = vi->d[0], W = vi->nd == 3 ? vi->d[1] : 1, Ho = vo->d[0], Wo = vo->nd == 3 ? vo->d[1] : 1;
        return kx_pad2d(a, y, B, H, W, vi->c, Ho, Wo, s->pt, s->pl, st);
    }
    case KERNIX_OP_UPSAMPLE: {
        const int H = vi->d[0], W = vi->nd == 3 ? vi->d[1] : 1, Ho = vo->d[0], Wo = vo->nd == 3 ? vo->d[1] : 1;
        return kx_upsample2d(a, y, B, H, W, vi->c, Ho, Wo, s->sh, s->sw, st);
    }
    case KERNIX_OP_ATTENTION: {
        const int vid = s->inp[s->n_in > 1 ? 1 : 0], kid = s->inp[s->n_in > 2 ? 2 : s->n_in > 1 ? 1 : 0];
        const kx_val* vv = &g->vals[vid];
        const int hk = s->heads * s->dk, hv = s->heads * s->dv;
        const long S = (long)B * vv->r;
        float* ctx;
        if (s->qkv_fused) {
            const int nq = 2 * hk + hv;
            float* qkv = (float*)align_ptr(im->scratch);
            ctx = (float*)align_ptr(qkv + (size_t)rin * nq);
            if (kx_gemm_f32(a, s->in, s->wqkv.d_hi, s->wqkv.d_lo, s->wqkv.ldw, s->d_bqkv, qkv, nq, (int)rin, nq, s->in,
                            KERNIX_ACT_NONE, 0.0f, im->status, st) != 0 ||
                kx_attention(qkv, nq, qkv + hk, nq, qkv + 2 * hk, nq, ctx, hv, B, vi->r, vv->r, s->heads, s->dk, s->dv,
                             s->causal, im->status, st) != 0)
                return -1;
        } else {
            float* Q = (float*)align_ptr(im->scratch);
            float* K = (float*)align_ptr(Q + (size_t)rin * hk);
            float* V = (float*)align_ptr(K + (size_t)S * hk);
            ctx = (float*)align_ptr(V + (size_t)S * hv);
            const kx_val* vk = &g->vals[kid];
            if (kx_gemm_f32(a, vi->c, s->w.d_hi, s->w.d_lo, s->w.ldw, s->d_bias, Q, hk, (int)rin, hk, vi->c, KERNIX_ACT_NONE,
                            0.0f, im->status, st) != 0 ||
                kx_gemm_f32(val_ptr(im, kid), vk->c, s->wk.d_hi, s->wk.d_lo, s->wk.ldw, s->d_bk, K, hk, (int)S, hk, vk->c,
                            KERNIX_ACT_NONE, 0.0f, im->status, st) != 0 ||
                kx_gemm_f32(val_ptr(im, vid), vv->c, s->wv.d_hi, s->wv.d_lo, s->wv.ldw, s->d_bv, V, hv, (int)S, hv, vv->c,
                            KERNIX_ACT_NONE, 0.0f, im->status, st) != 0 ||
                kx_attention(Q, hk, K, hk, V, hv, ctx, hv, B, vi->r, vv->r, s->heads, s->dk, s->dv, s->causal, im->status,
                             st) != 0)
                return -1;
        }
        if (res)
            return kx_gemm_f32_res(ctx, hv, s->wo.d_hi, s->wo.d_lo, s->wo.ldw, s->d_bo, y, s->out, (int)rin, s->out, hv,
                                   KERNIX_ACT_NONE, 0.0f, res, s->out, im->status, st);
        return kx_gemm_f32(ctx, hv, s->wo.d_hi, s->wo.d_lo, s->wo.ldw, s->d_bo, y, s->out, (int)rin, s->out, hv,
                           KERNIX_ACT_NONE, 0.0f, im->status, st);
    }
    case KERNIX_OP_LSTM:
    case KERNIX_OP_GRU:
    case KERNIX_OP_RNN: { /* kernix_rnn_run (:636-648): per direction, input projections of all steps in one GEMM,
                           * then one fused kernel per time step */
        const int kind = s->kind == KERNIX_OP_LSTM ? 0 : (s->kind == KERNIX_OP_GRU ? 1 : 2);
        const int T = vi->r, u = s->out, gu = (int)rnn_gates(s->kind) * u;
        const int concat = s->dirs == 2 && s->merge == 0;
        const long uo = concat ? 2L * u : u;
        float* zx = (float*)align_ptr(im->scratch);
        float* h0 = (float*)align_ptr(zx + (size_t)rin * gu);
        float* h1 = (float*)align_ptr(h0 + (size_t)B * u);
        float* cst = (float*)align_ptr(h1 + (size_t)B * u);
        float* bw = (float*)align_ptr(cst + (size_t)B * u);
        for (int d = 0; d < s->dirs; d++) {
            const kx_weight* W = d ? &s->wk : &s->w;
            const kx_weight* U = d ? &s->wo : &s->wv;
            const float* bias = d ? s->d_bk : s->d_bias;
            float* dst = d == 0 ? y : (concat ? y + u : bw);
            const long stride = d == 0 ? uo : (concat ? uo : u);
            if (kx_gemm_f32(a, s->in, W->d_hi, W->d_lo, W->ldw, bias, zx, gu, (int)rin, gu, s->in, KERNIX_ACT_NONE, 0.0f,
                            im->status, st) != 0)
                return -1;
            float *hp = h0, *hn = h1;
            for (int step = 0; step < T; step++) {
                const int t = d ? T - 1 - step : step;
                if (kx_rnn_step(kind, zx, U->d_raw, kind == 1 ? bias + gu : NULL, hp, hn, cst, dst, stride, B, T, t, u, step == 0,
                                s->ret_seq, step == T - 1, s->act, s->alpha, st) != 0)
                    return -1;
                float* tmp = hp;
                hp = hn;
                hn = tmp;
            }
        }
        if (s->dirs == 2 && !concat) return kx_rnn_merge(y, bw, (long)B * (s->ret_seq ? T : 1) * u, s->merge, st);
        return 0;
    }
    default:
        return -1;
    }
}

static const char* kind_name(int k) {
    static const char* names[] = {"LINEAR", "ACT", "LAYERNORM", "SOFTMAX", "LSTM", "GRU", "RNN", "CONV", "POOL",
                                  "GLOBAL_POOL", "RESHAPE", "PERMUTE", "BINARY", "CONCAT", "EMBEDDING", "AFFINE",
                                  "ADD_CONST", "ATTENTION", "SELECT", "PAD", "UPSAMPLE"};
    return k >= 0 && k <= KERNIX_OP_LAST ? names[k] : "?";
}

static int chunk_run(kernix_model* m, int B) {
    struct kx_model_impl* im = m->impl;
    for (int i = 0; i < im->g->n_steps; i++) {
        const kx_step* s = &im->g->steps[i];
        /* a fused LINEAR must take the tensor-core path (the skinny path for few rows has no residual) */
        const long rin = (long)B * im->g->vals[s->inp[0]].r;
        if (s->i8c_n > 0 && !im->no_qchain) {
            if (i8chain_run(m, i, rin) != 0) {
                fprintf(stderr, "forward: the int8 chain at step %d failed to launch: %s\n", i,
                        cudaGetErrorString(cudaGetLastError()));
                return -1;
            }
            i += s->i8c_n - 1;
            continue;
        }
        if (s->mlp_n > 0 && rin <= KX_MLP_MAX_ROWS && im->mlp_scratch != NULL && !im->no_qchain) {
            if (mlp_run(m, i, rin) != 0) {
                fprintf(stderr, "forward: the fused dense chain at step %d failed to launch: %s\n", i,
                        cudaGetErrorString(cudaGetLastError()));
                return -1;
            }
            i += s->mlp_n - 1;
            continue;
        }
        const int fused = s->fuse_add && (s->kind == KERNIX_OP_ATTENTION || !(rin <= KX_SKINNY_MAX_ROWS && s->w.d_raw != NULL &&
                                                                              im->skinny_part != NULL));
        if (step_run(m, i, B, fused) != 0) {
            fprintf(stderr, "forward: step %d (%s) failed to launch: %s\n", i, kind_name(s->kind),
                    cudaGetErrorString(cudaGetLastError()));
            return -1;
        }
        if (fused) i++; /* the ADD is done */
    }
    return 0;
}

/* samples per chunk under the workspace limit (the reference's rule, include/kernix_model.h:2040-2050) */
static int chunk_samples(const kernix_model* m, int samples) {
    int chunk = samples;
    if (m->ws_limit > 0 && m->ws_per_sample > 0) {
        const size_t fixed = m->ws_fixed * sizeof(float), avail = m->ws_limit > fixed ? m->ws_limit - fixed : 0;
        size_t c = avail / (m->ws_per_sample * sizeof(float));
        if (c < 1) c = 1;
        if (c < (size_t)samples) chunk = (int)c;
    }
    return chunk;
}

/* Point the running steps at samples [a, a + n) of the chunk arena: the input rows and every storage buffer are
 * offset by a samples (a buffer holds st_cap floats per sample), so pieces of one chunk use disjoint memory and
 * can be in flight together. The per-step scratch is shared: pieces run one after another on the kernel stream. */
static void piece_view(struct kx_model_impl* im, float* xin_base, int a, size_t in_per_sample) {
    im->xin = xin_base + (size_t)a * in_per_sample;
    for (int k = 0; k < im->g->n_st; k++) im->st[k] = im->st_base[k] + (size_t)a * im->g->st_cap[k];
}

/* Enqueue the forward of device rows d_x into d_out (samples x out_dim) on im->stream, chunk by chunk. The model
 * input is never written (the plan keeps it read-only), so each chunk reads it in place. The step that produces the
 * model output writes the caller's rows directly unless that output is a RESHAPE view (then it is copied out). */
static int forward_enqueue_device(kernix_model* m, const float* x, int rows, float* out) {
    struct kx_model_impl* im = m->impl;
    const int samples = rows / m->seq_len;
    if (samples == 0) return 0;
    const int chunk = chunk_samples(m, samples);
    const int crow = chunk * m->seq_len;
    if (crow != m->batch && model_alloc(m, crow) != 0) return -1;
    const kx_graph* g = im->g;
    const int direct = g->out_v > 0 && g->steps[g->out_v - 1].kind != KERNIX_OP_RESHAPE && ((uintptr_t)out & 15) == 0;
    float* const xin_own = im->xin;
    for (int s0 = 0; s0 < samples; s0 += chunk) {
        const int n = samples - s0 < chunk ? samples - s0 : chunk;
        float* yo = out + (size_t)s0 * m->out_dim;
        im->xin = (float*)(x + (size_t)s0 * m->seq_len * m->in_dim);
        im->yout = direct ? yo : NULL;
        const int rc = chunk_run(m, n);
        const float* yc = val_ptr(im, g->out_v); /* the input itself when the graph is only views of it */
        im->xin = xin_own;
        im->yout = NULL;
        if (rc != 0) return -1;
        if (!direct && cudaMemcpyAsync(yo, yc, (size_t)n * m->out_dim * sizeof(float), cudaMemcpyDeviceToDevice,
                                       im->stream) != cudaSuccess)
            return -1;
    }
    return 0;
}

/* 1 if the host buffer p is page-locked (registered or allocated by CUDA), so that copies into it are asynchronous */
static int host_page_locked(const void* p) {
    struct cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return a.type == cudaMemoryTypeHost;
}

/* Enqueue the forward of host rows x into host out. Each chunk is cut into up to im->pipe_now pieces; piece p's host -> device copy (stream s_in), kernels (stream) and device
 * -> host copy (s_out) are ordered by events, so the copies of one piece overlap the kernels of its neighbours and
 * the two copy directions overlap each other. Piece p of every chunk reuses arena region p: its input copy waits
 * until the last user of region p has been computed and copied out, and its kernels wait for that copy-out too.
 * Rows never mix across pieces, so the result is the same for any cut (the chunking invariance of
 * include/kernix_model.h:1691-1694): bit for bit, except that a piece too small for the persistent 3xTF32 tiles
 * (which sum their three products in one accumulator) differs from a whole run by at most ~6e-6 of the scale. Into page-locked memory a piece's output copy is queued right after its
 * kernels, so that it never waits for the host to queue the later pieces; into pageable memory (a copy that returns
 * only when done) the copies of a chunk are queued after all of its kernels, so that they do not hold back the
 * later pieces' launches. */
static int forward_enqueue_host(kernix_model* m, const float* x, int rows, float* out) {
    struct kx_model_impl* im = m->impl;
    const int samples = rows / m->seq_len;
    if (samples == 0) return 0;
    const int chunk = chunk_samples(m, samples);
    const int crow = chunk * m->seq_len;
    if (crow != m->batch && model_alloc(m, crow) != 0) return -1;
    const size_t in_ps = (size_t)m->seq_len * m->in_dim; /* input floats per sample */
    const kx_val* vo = &im->g->vals[im->g->out_v];
    const int out_st = vo->st;
    float* const xin_own = im->xin;
    const int eager_out = host_page_locked(out);
    int rc = 0;
    for (int s0 = 0; s0 < samples && rc == 0; s0 += chunk) {
        const int n = samples - s0 < chunk ? samples - s0 : chunk;
        int P = im->pipe_now < n ? im->pipe_now : n;
        while (P > 1 && (size_t)(n / P) * in_ps * sizeof(float) < KX_PIPE_MIN_BYTES) P--;
        const int q = (n + P - 1) / P;
        P = (n + q - 1) / q;
        /* the output copy of piece p: its value is in its storage buffer at the piece's offset, or (a graph of views
         * only) in the piece's input rows */
        #define KX_QUEUE_OUT(p)                                                                                          \
            do {                                                                                                         \
                const int a_ = (p) * q, np_ = n - a_ < q ? n - a_ : q;                                                  \
                const float* yp = out_st < 0 ? xin_own + (size_t)a_ * in_ps                                               \
                                             : im->st_base[out_st] + (size_t)a_ * im->g->st_cap[out_st];                  \
                rc |= cudaStreamWaitEvent(im->s_out, im->ev_comp[(p)], 0) != cudaSuccess;                                \
                rc |= cudaMemcpyAsync(out + (size_t)(s0 + a_) * m->out_dim, yp, (size_t)np_ * m->out_dim * sizeof(float), \
                                      cudaMemcpyDeviceToHost, im->s_out) != cudaSuccess;                                 \
                rc |= cudaEventRecord(im->ev_out[(p)], im->s_out) != cudaSuccess;                                        \
            } while (0)
        for (int p = 0; p < P && rc == 0; p++) {
            const int a = p * q, np = n - a < q ? n - a : q;
            float* xr = xin_own + (size_t)a * in_ps;
            /* the waits see the previous chunk's (or call's) records of this piece's events */
            rc |= cudaStreamWaitEvent(im->s_in, im->ev_comp[p], 0) != cudaSuccess;
            rc |= cudaStreamWaitEvent(im->s_in, im->ev_out[p], 0) != cudaSuccess;
            if (p == 0) rc |= cudaEventRecord(im->ev_t0, im->s_in) != cudaSuccess;
            rc |= cudaMemcpyAsync(xr, x + (size_t)(s0 + a) * in_ps, (size_t)np * in_ps * sizeof(float),
                                  cudaMemcpyHostToDevice, im->s_in) != cudaSuccess;
            rc |= cudaEventRecord(im->ev_in[p], im->s_in) != cudaSuccess;
            rc |= cudaStreamWaitEvent(im->stream, im->ev_in[p], 0) != cudaSuccess;
            rc |= cudaStreamWaitEvent(im->stream, im->ev_out[p], 0) != cudaSuccess;
            if (rc) break;
            piece_view(im, xin_own, a, in_ps);
            rc |= chunk_run(m, np) != 0;
            rc |= cudaEventRecord(im->ev_comp[p], im->stream) != cudaSuccess;
            if (eager_out) KX_QUEUE_OUT(p);
        }
        if (!eager_out)
            for (int p = 0; p < P && rc == 0; p++) KX_QUEUE_OUT(p);
        #undef KX_QUEUE_OUT
        rc |= cudaEventRecord(im->ev_t1, im->s_out) != cudaSuccess;
        im->last_pieces = P;
    }
    piece_view(im, xin_own, 0, in_ps);
    return rc ? -1 : 0;
}

/* Choose the piece count by trying it: the calls after the first at a chunk size (the first also pays for loading
 * the kernels) run with 1, 2, 3, 4, 6 and 8 pieces in turn, each timed on the device from its last chunk's first
 * input copy to its last output copy, and the fastest count is kept from then on. How many pieces pay depends on
 * the model (kernels that are much longer than the copies want one, kernels that lose efficiency on small pieces
 * want few) and on the link, so it is measured rather than guessed. The result does not depend on the count (to
 * the bit, or within ~6e-6 where the persistent tiles apply to the whole but not to a piece). */
static const int kx_pipe_cand[] = {1, 2, 3, 4, 6, 8};
#define KX_PIPE_NCAND ((int)(sizeof kx_pipe_cand / sizeof kx_pipe_cand[0]))
static void pipe_tune(struct kx_model_impl* im) {
    if (im->pipe_fixed || im->tune_calls > KX_PIPE_NCAND) return;
    const int c = im->tune_calls++; /* call c at this chunk size ran with pipe_now pieces */
    if (c >= 1 && im->last_pieces > 0) {
        float v;
        if (cudaEventElapsedTime(&v, im->ev_t0, im->ev_t1) == cudaSuccess &&
            (c == 1 || v < im->tune_best_ms)) {
            im->tune_best_ms = v;
            im->tune_best = im->pipe_now;
        }
        cudaGetLastError();
    }
    im->pipe_now = c < KX_PIPE_NCAND ? kx_pipe_cand[c] : (im->tune_best > 0 ? im->tune_best : im->pipe);
}

/* host-memory forward: enqueue, then wait for every stream and check the status word */
static int forward_one(kernix_model* m, const float* x, int rows, float* out);

/* one device's share of a batch-sharded host forward, run on its own host thread */
typedef struct {
    kernix_model* m;
    const float* x;
    int rows;
    float* out;
    int rc;
} kx_share;

static void* share_run(void* arg) {
    kx_share* sh = (kx_share*)arg;
    int prev;
    sh->rc = dev_guard_enter(sh->m, &prev) == 0 ? forward_one(sh->m, sh->x, sh->rows, sh->out) : -1;
    dev_guard_leave(sh->m, prev);
    return NULL;
}

/* host-memory forward of a model with replicas: samples split in contiguous shares, one per device, each share's
 * input read and output written in place in the caller's buffers; every share must succeed */
static int forward_sharded_batch(kernix_model* m, const float* x, int rows, float* out) {
    struct kx_model_impl* im = m->impl;
    const int samples = rows / m->seq_len, parts = im->n_rep + 1 < samples ? im->n_rep + 1 : samples;
    kx_share sh[KX_MAX_REPLICAS + 1];
    pthread_t th[KX_MAX_REPLICAS + 1];
    int started[KX_MAX_REPLICAS + 1] = {0};
    for (int k = 0; k < parts; k++) {
        const int a = (int)((long)samples * k / parts), b = (int)((long)samples * (k + 1) / parts);
        sh[k] = (kx_share){k == 0 ? m : im->rep[k - 1], x + (size_t)a * m->seq_len * m->in_dim, (b - a) * m->seq_len,
                           out + (size_t)a * m->out_dim, -1};
    }
    for (int k = 1; k < parts; k++) started[k] = pthread_create(&th[k], NULL, share_run, &sh[k]) == 0;
    sh[0].rc = forward_one(m, sh[0].x, sh[0].rows, sh[0].out);
    int rc = sh[0].rc;
    for (int k = 1; k < parts; k++) {
        if (started[k]) pthread_join(th[k], NULL);
        else share_run(&sh[k]); /* no thread: run the share here */
        rc |= sh[k].rc;
    }
    return rc ? -1 : 0;
}

/* host-memory forward on the model's device(s) (the caller made the model's device current) */
static int forward_into(kernix_model* m, const float* x, int rows, float* out) {
    if (m->impl->n_rep > 0 && rows / m->seq_len > 1) return forward_sharded_batch(m, x, rows, out);
    return forward_one(m, x, rows, out);
}

/* host-memory forward on the model's own device */
static int forward_one(kernix_model* m, const float* x, int rows, float* out) {
    struct kx_model_impl* im = m->impl;
    if (rows / m->seq_len == 0) return 0;
    cudaStream_t st = im->stream;
    if (m->batch > 0 && cudaMemsetAsync(im->status, 0, sizeof(int), st) != cudaSuccess) return -1;
    const int rc = forward_enqueue_host(m, x, rows, out);
    if (rc == 0 && m->batch > 0) cudaMemcpyAsync(im->status_h, im->status, sizeof(int), cudaMemcpyDeviceToHost, st);
    const cudaError_t e = sync_all(im); /* also on failure: no copy may still be reading x or writing out */
    if (rc != 0 || m->batch <= 0) return -1;
    if (e != cudaSuccess) {
        fprintf(stderr, "forward: CUDA error %s\n", cudaGetErrorString(e));
        return -1;
    }
    if (*im->status_h != KX_STATUS_OK) {
        fprintf(stderr, "forward: a kernel gave up waiting (status %d)\n", *im->status_h);
        cudaMemsetAsync(im->status, 0, sizeof(int), st);
        if (im->mlp_bar) cudaMemsetAsync(im->mlp_bar, 0, 2 * sizeof(uint32_t), st);
        return -1;
    }
    pipe_tune(im);
    return 0;
}

/* workspace floats per sample: storage buffers, input rows, step scratch */
static size_t ws_count(kernix_model* m) {
    kx_graph* g = m->impl->g;
    size_t n = 0;
    for (int k = 0; k < g->n_st; k++) n += g->st_cap[k];
    n += (size_t)m->seq_len * m->in_dim;
    size_t mx = 0;
    for (int i = 0; i < g->n_steps; i++) {
        size_t ps;
        step_scratch(g, &g->steps[i], &ps);
        if (ps > mx) mx = ps;
    }
    m->impl->scratch_per_row_max = mx;
    return n + (mx + 3) / 4;
}

/* ------------------------------------------------------------------------------------ public API */
/* the device a model loads onto: `device` if >= 0, else $KERNIX_DEVICE, else the caller's current device */
static int pick_device(int device) {
    if (device >= 0) return device;
    const char* env = getenv("KERNIX_DEVICE");
    int cur = -1;
    cudaGetDevice(&cur);
    return env && *env ? atoi(env) : (cur >= 0 ? cur : 0);
}

static kernix_model* model_load(const char* path, int rank, int world, kernix_allgather_fn gather, void* ctx, int device) {
    const char* err = NULL;
    if (world < 1 || rank < 0 || rank >= world || (world > 1 && gather == NULL)) {
        fprintf(stderr, "model load failed (%s): bad shard arguments (rank %d of %d)\n", path ? path : "NULL", rank, world);
        return NULL;
    }
    kx_graph* g = kx_graph_load(path, &err);
    if (g == NULL) {
        fprintf(stderr, "model load failed (%s): %s\n", path ? path : "NULL", err);
        return NULL;
    }
    if (world > 1) /* wide fp32 LINEAR steps keep one output slice per rank */
        for (int i = 0; i < g->n_steps; i++) {
            kx_step* s = &g->steps[i];
            if (s->kind == KERNIX_OP_LINEAR && !s->w.int8 && s->out >= KERNIX_SHARD_MIN_COLS && s->out % world == 0) {
                s->shard_n = s->out / world;
                s->shard_c0 = s->shard_n * rank;
            }
        }
    plan_fusions(g);
    plan_i8chain(g);
    plan_qchain(g);
    plan_mlp(g);
    kernix_model* m = calloc(1, sizeof *m);
    struct kx_model_impl* im = calloc(1, sizeof *im);
    if (m == NULL || im == NULL) {
        free(m);
        free(im);
        kx_graph_free(g);
        fprintf(stderr, "model load failed (%s): out of memory\n", path);
        return NULL;
    }
    m->impl = im;
    im->g = g;
    im->rank = rank;
    im->world = world;
    im->gather = gather;
    im->gather_ctx = ctx;
    m->batch = -1;
    const kx_val* vin = &g->vals[0];
    const kx_val* vout = &g->vals[g->out_v];
    m->n_steps = g->n_steps;
    m->in_dim = vin->c;
    m->seq_len = vin->r;
    m->out_dim = vout->r * vout->c;
    m->in_nd = vin->nd;
    memcpy(m->in_shape, vin->d, sizeof m->in_shape);
    m->out_nd = vout->nd;
    memcpy(m->out_shape, vout->d, sizeof m->out_shape);
    m->layout = g->layout;
    m->ws_limit = KERNIX_WORKSPACE_LIMIT;
    m->ws_fixed = 0;
    m->ws_per_sample = ws_count(m);

    int prev = -1;
    cudaGetDevice(&prev);
    im->device = pick_device(device);
    const char* why = NULL;
    if (cudaSetDevice(im->device) != cudaSuccess) why = "no CUDA device";
    else if (cudaStreamCreateWithFlags(&im->stream, cudaStreamNonBlocking) != cudaSuccess ||
             cudaStreamCreateWithFlags(&im->s_in, cudaStreamNonBlocking) != cudaSuccess ||
             cudaStreamCreateWithFlags(&im->s_out, cudaStreamNonBlocking) != cudaSuccess)
        why = "cannot create a CUDA stream";
    for (int i = 0; why == NULL && i < KX_PIPE_MAX; i++)
        if (cudaEventCreateWithFlags(&im->ev_in[i], cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&im->ev_comp[i], cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&im->ev_out[i], cudaEventDisableTiming) != cudaSuccess)
            why = "cannot create a CUDA event";
    if (why == NULL && (cudaEventCreate(&im->ev_t0) != cudaSuccess || cudaEventCreate(&im->ev_t1) != cudaSuccess))
        why = "cannot create a CUDA event";
    if (why == NULL && cudaHostAlloc((void**)&im->status_h, sizeof(int), cudaHostAllocDefault) != cudaSuccess)
        why = "cannot allocate host memory";
    const char* pe = getenv("KERNIX_PIPELINE");
    im->pipe_fixed = (pe && *pe) || world > 1; /* sharded: the same pieces (collectives) on every rank */
    im->pipe = pe && *pe ? atoi(pe) : (world > 1 ? 1 : 4);
    if (im->pipe < 1) im->pipe = 1;
    if (im->pipe > KX_PIPE_MAX) im->pipe = KX_PIPE_MAX;
    im->pipe_now = im->pipe;
    for (int i = 0; why == NULL && i < g->n_steps; i++)
        if (step_upload(g, &g->steps[i], im->stream) != 0) why = "cannot copy the weights to the GPU";
    if (why == NULL && cudaStreamSynchronize(im->stream) != cudaSuccess) why = "cannot copy the weights to the GPU";
    if (why == NULL) { /* partial sums of the skinny dense path: slices x KX_SKINNY_MAX_ROWS x columns, the largest step */
        size_t mx = 0;
        for (int i = 0; i < g->n_steps; i++) {
            const kx_step* s = &g->steps[i];
            if (s->kind != KERNIX_OP_LINEAR || s->w.int8) continue;
            const int n = s->shard_n > 0 ? s->shard_n : s->out;
            const size_t f = (size_t)kx_skinny_slices(n, s->in) * KX_SKINNY_MAX_ROWS * n;
            if (f > mx) mx = f;
        }
        if (mx > 0 && cudaMalloc((void**)&im->skinny_part, mx * sizeof(float)) != cudaSuccess) why = "cannot allocate device memory";
        im->skinny_floats = mx;
    }
    const char* no_split = getenv("KERNIX_NO_SPLITK"); /* 1: dense steps never split K (tests compare the two) */
    if (why == NULL && !(no_split && *no_split && *no_split != '0')) { /* split-K planes: splits x 128 rows x columns, the largest step */
        size_t mx = 0;
        for (int i = 0; i < g->n_steps; i++) {
            const kx_step* s = &g->steps[i];
            if (s->kind != KERNIX_OP_LINEAR || s->w.int8 || s->fuse_add) continue;
            const int n = s->shard_n > 0 ? s->shard_n : s->out, sp = kx_gemm_f32_splits(128, n, s->in);
            if (sp > 1 && (size_t)sp * 128 * n > mx) mx = (size_t)sp * 128 * n;
        }
        if (mx > 0 && cudaMalloc((void**)&im->split_part, mx * sizeof(float)) != cudaSuccess) why = "cannot allocate device memory";
    }
    const char* no_i8s = getenv("KERNIX_NO_I8_SPLIT"); /* 1: small batches of int8 chains run the chain kernel too */
    if (why == NULL && !(no_i8s && *no_i8s && *no_i8s != '0')) { /* int8 chain planes: ranges x 128 rows x columns */
        size_t mx = 0;
        for (int i = 0; i < g->n_steps; i++) {
            const kx_step* s = &g->steps[i];
            if (s->i8c_n == 0 || !i8split_ok(g, i)) continue;
            for (int l = 0; l < s->i8c_n; l++) {
                const kx_step* t = &g->steps[i + l];
                const size_t f = (size_t)i8split_planes(KX_I8S_MAX_ROWS, t->out, t->in) * KX_I8S_MAX_ROWS * (size_t)t->out;
                if (f > mx) mx = f;
            }
        }
        if (mx > 0 && cudaMalloc((void**)&im->i8s_part, mx * sizeof(int32_t)) != cudaSuccess) why = "cannot allocate device memory";
    }
    if (why == NULL) { /* fused small-MLP chains: partial sums for up to KX_MLP_MAX_ROWS rows, the largest chain */
        size_t mx = 0;
        for (int i = 0; i < g->n_steps; i++) {
            const kx_step* s = &g->steps[i];
            if (s->mlp_n == 0) continue;
            int k[KX_MLP_MAX_LAYERS], n[KX_MLP_MAX_LAYERS];
            for (int l = 0; l < s->mlp_layers; l++) {
                k[l] = g->steps[i + l].in;
                n[l] = g->steps[i + l].out;
            }
            const size_t f = kx_mlp_chain_scratch_floats(KX_MLP_MAX_ROWS, k, n, s->mlp_layers);
            if (f > mx) mx = f;
        }
        if (mx > 0 && (cudaMalloc((void**)&im->mlp_scratch, mx * sizeof(float)) != cudaSuccess ||
                       cudaMalloc((void**)&im->mlp_bar, 2 * sizeof(uint32_t)) != cudaSuccess ||
                       cudaMemsetAsync(im->mlp_bar, 0, 2 * sizeof(uint32_t), im->stream) != cudaSuccess))
            why = "cannot allocate device memory";
    }
    if (prev >= 0 && prev != im->device) cudaSetDevice(prev);
    if (why != NULL) {
        fprintf(stderr, "model load failed (%s): %s (%s)\n", path, why, cudaGetErrorString(cudaGetLastError()));
        kernix_model_free(m);
        return NULL;
    }
    /* weights live on the device now: drop the file mapping and dequantised host copies */
    for (int i = 0; i < g->n_steps; i++) {
        kx_step* s = &g->steps[i];
        kx_weight* ws[4] = {&s->w, &s->wk, &s->wv, &s->wo};
        for (int k = 0; k < 4; k++) {
            free(ws[k]->own);
            ws[k]->own = NULL;
            ws[k]->f = NULL;
            ws[k]->q = NULL;
            ws[k]->scale_h = NULL;
        }
        s->bias = s->bk = s->bv = s->bo = s->gamma = s->beta = s->cst = NULL;
    }
    return m;
}

/* devices named by $KERNIX_GPUS ("0,1,2,3" or "all"): the count, at most KX_MAX_REPLICAS + 1, or 0 if unset */
static int gpus_from_env(int* dev) {
    const char* env = getenv("KERNIX_GPUS");
    if (env == NULL || *env == 0) return 0;
    int n = 0;
    if (strcmp(env, "all") == 0) {
        int count = 0;
        if (cudaGetDeviceCount(&count) != cudaSuccess) {
            cudaGetLastError();
            return 0;
        }
        for (int d = 0; d < count && n <= KX_MAX_REPLICAS; d++) dev[n++] = d;
        return n;
    }
    for (const char* p = env; *p && n <= KX_MAX_REPLICAS;) {
        char* end = NULL;
        const long v = strtol(p, &end, 10);
        if (end == p || v < 0) break;
        dev[n++] = (int)v;
        p = *end == ',' ? end + 1 : end;
        if (*end != ',' && *end != 0) break;
    }
    return n;
}

KERNIX_API kernix_model* kernix_model_load(const char* path) {
    int dev[KX_MAX_REPLICAS + 1];
    const int n = gpus_from_env(dev);
    kernix_model* m = model_load(path, 0, 1, NULL, NULL, n >= 2 ? dev[0] : -1);
    if (m == NULL || n < 2) return m;
    for (int k = 1; k < n; k++) { /* whole-model replicas; the load fails if any device cannot hold one */
        kernix_model* r = model_load(path, 0, 1, NULL, NULL, dev[k]);
        if (r == NULL) {
            fprintf(stderr, "model load failed (%s): no replica on device %d of $KERNIX_GPUS\n", path, dev[k]);
            kernix_model_free(m);
            return NULL;
        }
        m->impl->rep[m->impl->n_rep++] = r;
    }
    return m;
}

KERNIX_API kernix_model* kernix_model_load_sharded(const char* path, int rank, int world, kernix_allgather_fn gather,
                                                   void* ctx) {
    return model_load(path, rank, world, gather, ctx, -1);
}

KERNIX_API kernix_model* kernix_model_load_sharded_nccl(const char* path, int rank, int world, const void* nccl_id) {
    if (world == 1) return model_load(path, 0, 1, NULL, NULL, -1);
    if (world < 1 || rank < 0 || rank >= world || nccl_id == NULL) {
        fprintf(stderr, "model load failed (%s): bad shard arguments (rank %d of %d)\n", path ? path : "NULL", rank, world);
        return NULL;
    }
    const int device = pick_device(-1);
    int prev = -1;
    cudaGetDevice(&prev);
    if (cudaSetDevice(device) != cudaSuccess) {
        fprintf(stderr, "model load failed (%s): no CUDA device %d\n", path ? path : "NULL", device);
        return NULL;
    }
    void* comm = kx_nccl_comm_init(rank, world, nccl_id); /* collective: every rank of the group is here */
    if (prev >= 0 && prev != device) cudaSetDevice(prev);
    if (comm == NULL) return NULL;
    kernix_model* m = model_load(path, rank, world, kx_nccl_gather, comm, device);
    if (m == NULL) {
        kx_nccl_comm_free(comm);
        return NULL;
    }
    m->impl->nccl_comm = comm;
    return m;
}

KERNIX_API void kernix_model_free(kernix_model* m) {
    if (m == NULL) return;
    struct kx_model_impl* im = m->impl;
    if (im != NULL) {
        for (int k = 0; k < im->n_rep; k++) kernix_model_free(im->rep[k]);
        im->n_rep = 0;
        int prev = -1;
        cudaGetDevice(&prev);
        cudaSetDevice(im->device);
        sync_all(im);
        model_release(m);
        if (im->g != NULL)
            for (int i = 0; i < im->g->n_steps; i++) step_dev_free(&im->g->steps[i]);
        if (im->status_h) cudaFreeHost(im->status_h);
        cudaFree(im->skinny_part);
        cudaFree(im->split_part);
        cudaFree(im->i8s_part);
        cudaFree(im->mlp_scratch);
        cudaFree(im->mlp_bar);
        for (int i = 0; i < KX_PIPE_MAX; i++) {
            cudaEvent_t* evs[3] = {im->ev_in, im->ev_comp, im->ev_out};
            for (int k = 0; k < 3; k++)
                if (evs[k][i]) cudaEventDestroy(evs[k][i]);
        }
        if (im->ev_t0) cudaEventDestroy(im->ev_t0);
        if (im->ev_t1) cudaEventDestroy(im->ev_t1);
        if (im->s_in) cudaStreamDestroy(im->s_in);
        if (im->s_out) cudaStreamDestroy(im->s_out);
        if (im->stream) cudaStreamDestroy(im->stream);
        kx_graph_free(im->g);
        if (im->nccl_comm) kx_nccl_comm_free(im->nccl_comm);
        if (prev >= 0) cudaSetDevice(prev);
        free(im);
    }
    free(m);
}

KERNIX_API void kernix_model_trim(kernix_model* m) {
    if (m == NULL) return;
    for (int k = 0; k < m->impl->n_rep; k++) kernix_model_trim(m->impl->rep[k]);
    int prev;
    if (dev_guard_enter(m, &prev) != 0) return;
    sync_all(m->impl);
    model_release(m);
    dev_guard_leave(m, prev);
}

KERNIX_API void kernix_model_set_workspace_limit(kernix_model* m, size_t bytes) {
    if (m == NULL) return;
    m->ws_limit = bytes;
    for (int k = 0; k < m->impl->n_rep; k++) m->impl->rep[k]->ws_limit = bytes;
}

KERNIX_API int kernix_model_set_ane(kernix_model* m, int on) {
    if (m == NULL) return -1;
    return on ? -1 : 0;
}

KERNIX_API void kernix_model_ane_info(const kernix_model* m, kernix_ane_info* out) {
    (void)m;
    if (out) memset(out, 0, sizeof *out);
}

KERNIX_API const float_tensor* kernix_model_forward(kernix_model* m, const float_tensor* x) {
    if (m == NULL || x == NULL || x->tensor == NULL || x->row < 0 || x->col != m->in_dim || x->row % m->seq_len != 0)
        return NULL;
    struct kx_model_impl* im = m->impl;
    if (im->out_host != NULL && x->tensor == im->out_host) {
        fprintf(stderr, "forward: this model's output buffer cannot be its own input (copy it first)\n");
        return NULL;
    }
    const int samples = x->row / m->seq_len;
    const size_t need = (size_t)samples * m->out_dim;
    int prev;
    if (dev_guard_enter(m, &prev) != 0) return NULL;
    if (need > im->out_host_floats || im->out_host == NULL) {
        if (im->out_host) cudaFreeHost(im->out_host);
        im->out_host = NULL;
        im->out_host_floats = 0;
        if (cudaHostAlloc((void**)&im->out_host, need ? need * sizeof(float) : 4, cudaHostAllocPortable) != cudaSuccess) {
            im->out_host = NULL;
            dev_guard_leave(m, prev);
            return NULL;
        }
        im->out_host_floats = need;
    }
    const int rc = forward_into(m, x->tensor, x->row, im->out_host);
    dev_guard_leave(m, prev);
    if (rc != 0) return NULL;
    im->out_t.row = samples;
    im->out_t.col = m->out_dim;
    im->out_t.tensor = im->out_host;
    return &im->out_t;
}

/* ------------------------------------------------------------------------ device-memory forward */
KERNIX_API int kernix_model_forward_device(kernix_model* m, const float* d_x, int rows, float* d_out, void* stream) {
    if (m == NULL || d_x == NULL || d_out == NULL || rows <= 0 || rows % m->seq_len != 0) return -1;
    struct kx_model_impl* im = m->impl;
    int prev;
    if (dev_guard_enter(m, &prev) != 0) return -1;
    cudaStream_t own = im->stream;
    im->stream = (cudaStream_t)stream; /* as given: 0 is the legacy default stream */
    const int rc = forward_enqueue_device(m, d_x, rows, d_out);
    im->stream = own;
    dev_guard_leave(m, prev);
    return rc;
}

KERNIX_API int kernix_model_check(kernix_model* m) {
    if (m == NULL || m->impl->status == NULL) return 0;
    int prev, v = 0;
    if (dev_guard_enter(m, &prev) != 0) return -1;
    if (cudaMemcpy(&v, m->impl->status, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) v = -1;
    if (v != 0) {
        cudaMemset(m->impl->status, 0, sizeof(int));
        if (m->impl->mlp_bar) cudaMemset(m->impl->mlp_bar, 0, 2 * sizeof(uint32_t)); /* a barrier may have given up */
    }
    dev_guard_leave(m, prev);
    return v == 0 ? 0 : -1;
}

/* --------------------------------------------------------------------------------- trace hook */
KERNIX_API int kx_model_forward_trace(kernix_model* m, const float* x, int rows, float** outs) {
    if (m == NULL || x == NULL || outs == NULL || rows <= 0 || rows % m->seq_len != 0) return -1;
    struct kx_model_impl* im = m->impl;
    const int B = rows / m->seq_len;
    int prev;
    if (dev_guard_enter(m, &prev) != 0) return -1;
    int rc = -1;
    if (rows != m->batch && model_alloc(m, rows) != 0) goto done;
    cudaStream_t st = im->stream;
    if (cudaMemcpyAsync(im->xin, x, (size_t)rows * m->in_dim * sizeof(float), cudaMemcpyHostToDevice, st) != cudaSuccess)
        goto done;
    im->no_qchain = 1; /* every intermediate value is materialised */
    for (int i = 0; i < im->g->n_steps; i++) {
        if (step_run(m, i, B, 0) != 0) {
            im->no_qchain = 0;
            goto done;
        }
        if (outs[i] != NULL) {
            const kx_val* v = &im->g->vals[i + 1];
            if (cudaMemcpyAsync(outs[i], val_ptr(im, i + 1), (size_t)B * v->r * v->c * sizeof(float), cudaMemcpyDeviceToHost,
                                st) != cudaSuccess)
                goto done;
        }
    }
    rc = cudaStreamSynchronize(st) == cudaSuccess ? 0 : -1;
done:
    im->no_qchain = 0;
    dev_guard_leave(m, prev);
    return rc;
}

/* -------------------------------------------------------------------------------- C ABI (capi) */
KERNIX_API void* kernix_capi_load(const char* path) { return kernix_model_load(path); }
KERNIX_API void kernix_capi_free(void* m) { kernix_model_free((kernix_model*)m); }
KERNIX_API void kernix_capi_trim(void* m) { kernix_model_trim((kernix_model*)m); }
KERNIX_API void kernix_capi_set_workspace_limit(void* m, size_t bytes) { kernix_model_set_workspace_limit((kernix_model*)m, bytes); }

KERNIX_API void kernix_capi_dims(const void* mv, int* in_dim, int* out_dim, int* seq_len) {
    const kernix_model* m = (const kernix_model*)mv;
    *in_dim = m->in_dim;
    *out_dim = m->out_dim;
    *seq_len = m->seq_len;
}

KERNIX_API int kernix_capi_forward(void* mv, const float* x, int rows, float* out) {
    kernix_model* m = (kernix_model*)mv;
    if (m == NULL || x == NULL || out == NULL || rows <= 0 || rows % m->seq_len != 0) return -1;
    int prev;
    if (dev_guard_enter(m, &prev) != 0) return -1;
    const int rc = forward_into(m, x, rows, out);
    dev_guard_leave(m, prev);
    return rc;
}

KERNIX_API int kernix_capi_set_ane(void* m, int on) { return kernix_model_set_ane((kernix_model*)m, on); }

KERNIX_API void kernix_capi_ane_info(const void* m, int* out) {
    (void)m;
    out[0] = out[1] = out[2] = out[3] = 0;
}

KERNIX_API int kernix_capi_ane_dump(const void* m, int seg, int batch, const char* path) {
    (void)m; (void)seg; (void)batch; (void)path;
    return -1;
}

KERNIX_API void kernix_capi_shapes(const void* mv, int* in_nd, int* in_shape, int* out_nd, int* out_shape, int* layout) {
    const kernix_model* m = (const kernix_model*)mv;
    *in_nd = m->in_nd;
    *out_nd = m->out_nd;
    *layout = m->layout;
    for (int k = 0; k < KERNIX_MAX_DIMS; k++) {
        in_shape[k] = m->in_shape[k];
        out_shape[k] = m->out_shape[k];
    }
}

/* -------------------------------------------------------------------------------- kernix.h extras */
KERNIX_API void float_free(float_tensor* t) {
    if (t == NULL) return;
    if (!kernix_metal_free(t->tensor)) free(t->tensor); /* backend storage goes back to its cache (kernix_gpu.h) */
    free(t);
}

KERNIX_API float_tensor* floats_fma_relu(const float_tensor* a, const float_tensor* x, const float_tensor* b) {
    if (a == NULL || x == NULL || b == NULL || a->tensor == NULL || x->tensor == NULL || b->tensor == NULL ||
        a->row != x->row || a->col != x->col || b->row != x->row || b->col != x->col || x->row < 0 || x->col < 0)
        return NULL;
    const size_t n = (size_t)x->row * (size_t)x->col, np = round_up(n ? n : 1, 4); /* planes 16-byte aligned */
    float_tensor* y = malloc(sizeof *y);
    if (y == NULL) return NULL;
    y->row = x->row;
    y->col = x->col;
    y->tensor = malloc(np * sizeof(float));
    float* d = NULL;
    int ok = y->tensor != NULL && cudaMalloc((void**)&d, 4 * np * sizeof(float)) == cudaSuccess;
    if (ok && n) {
        ok = cudaMemcpy(d, a->tensor, n * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
             cudaMemcpy(d + np, x->tensor, n * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
             cudaMemcpy(d + 2 * np, b->tensor, n * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
             kx_fma_relu(d, d + np, d + 2 * np, d + 3 * np, n, NULL) == 0 && cudaDeviceSynchronize() == cudaSuccess &&
             cudaMemcpy(y->tensor, d + 3 * np, n * 4, cudaMemcpyDeviceToHost) == cudaSuccess;
    }
    cudaFree(d);
    if (!ok) {
        float_free(y);
        return NULL;
    }
    return y;
}
