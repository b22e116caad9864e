/* .knx reader for the KERNIX-B200 runtime: parse, validate, infer shapes, fuse activations, plan storage.
 *
 * The file is untrusted input. It is mapped read-only and every read is checked against the bytes left,
 * before any allocation, with the same acceptance rules as the reference loader (include/kernix_model.h:
 * header :1461-1487, op records kernix_parse_op :1082-1243, weight blocks kernix_load_weight :1059-1077 /
 * kernix_read_weight :434-460, legacy input shape :1516-1526, kernix_infer :1266-1394, ACT fusion
 * :1530-1555, storage plan kernix_plan :1405-1445). Weight and bias arrays stay in the mapping until the
 * device copies are made (knx_model.c); int8 blocks that are not kept as int8 are dequantised here.
 */
#define _GNU_SOURCE
#include <fcntl.h>
#include <float.h>
#include <limits.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include "kx_internal.h"
#include "kx_inspect.h"

#define KX_CHUNK 8192 /* RNN unit bound: two gates fit one activation chunk (reference :1116, :1129) */

typedef struct {
    const uint8_t* p;
    size_t left;
} kx_rd;

static int rd_u32(kx_rd* r, uint32_t* v) {
    if (r->left < 4) return -1;
    memcpy(v, r->p, 4);
    r->p += 4;
    r->left -= 4;
    return 0;
}

static int rd_u32s(kx_rd* r, uint32_t* v, int n) {
    for (int i = 0; i < n; i++)
        if (rd_u32(r, &v[i]) != 0) return -1;
    return 0;
}

static int rd_f32(kx_rd* r, float* v) {
    if (r->left < 4) return -1;
    memcpy(v, r->p, 4);
    r->p += 4;
    r->left -= 4;
    return 0;
}

/* pointer to n floats inside the mapping (possibly unaligned: only ever copied with memcpy/cudaMemcpy) */
static const float* rd_floats(kx_rd* r, size_t n) {
    if (n > r->left / 4) return NULL;
    const float* f = (const float*)r->p;
    r->p += n * 4;
    r->left -= n * 4;
    return f;
}

static float ld_f(const float* p, size_t i) {
    float v;
    memcpy(&v, (const uint8_t*)p + i * 4, 4);
    return v;
}

static int geom_ok(uint32_t v, uint32_t lo) { return v >= lo && v <= KERNIX_MAX_GEOM; }

static uint64_t weight_bytes(uint32_t dt, uint64_t k, uint64_t n) {
    return dt == KX_DT_F32 ? 4 * k * n : dt == KX_DT_I8_COL ? 4 * n + k * n : 4 * k + k * n;
}

/* one k x n weight block; keep_int8: an I8_COL block stays int8 (LINEAR weights, RNN recurrent weights) */
static int rd_weight(kx_rd* r, int ver, uint64_t k, uint64_t n, int keep_int8, kx_weight* w, const char** err) {
    if (k < 1 || n < 1 || k > INT_MAX || n > INT_MAX || k * n > (uint64_t)INT_MAX) {
        *err = "weight size out of range";
        return -1;
    }
    uint32_t dt = KX_DT_F32;
    if (ver >= 2 && rd_u32(r, &dt) != 0) return -1;
    if (dt > KX_DT_I8_ROW) {
        *err = "unknown weight dtype";
        return -1;
    }
    if (weight_bytes(dt, k, n) > r->left) return -1;
    w->present = 1;
    w->k = (int)k;
    w->n = (int)n;
    const size_t cnt = (size_t)k * (size_t)n;
    if (dt == KX_DT_F32) {
        w->f = rd_floats(r, cnt);
        return w->f ? 0 : -1;
    }
    if (keep_int8 && dt == KX_DT_I8_COL && k > KERNIX_INT8_MAX_K) {
        *err = "int8 weight input size out of range";
        return -1;
    }
    const size_t ns = dt == KX_DT_I8_COL ? (size_t)n : (size_t)k;
    const float* sc = rd_floats(r, ns);
    if (sc == NULL || cnt > r->left) return -1;
    const int8_t* q = (const int8_t*)r->p;
    r->p += cnt;
    r->left -= cnt;
    for (size_t i = 0; i < ns; i++) {
        const float s = ld_f(sc, i);
        if (!(s > 0.0f && s <= FLT_MAX)) {
            *err = "int8 scale is not positive and finite";
            return -1;
        }
    }
    if (keep_int8 && dt == KX_DT_I8_COL) {
        w->int8 = 1;
        w->q = q;
        w->scale_h = sc;
        return 0;
    }
    /* other int8 blocks become float at load: w = q * scale (per column for I8_COL, per row for I8_ROW) */
    w->own = (float*)malloc(cnt * sizeof(float));
    if (w->own == NULL) {
        *err = "out of memory";
        return -1;
    }
    for (size_t i = 0; i < (size_t)k; i++)
        for (size_t j = 0; j < (size_t)n; j++)
            w->own[i * n + j] = (float)q[i * n + j] * ld_f(sc, dt == KX_DT_I8_COL ? j : i);
    w->f = w->own;
    return 0;
}

static size_t rnn_gates(int kind) { return kind == KERNIX_OP_LSTM ? 4 : kind == KERNIX_OP_GRU ? 3 : 1; }

/* ------------------------------------------------------------------------------------------- op records
 *
 * An op record is: kind, (KNX3) its input value ids, a run of u32 header fields, then its data blocks (weight
 * blocks, float arrays, float parameters). Every kind has a descriptor: the accepted range of each header field
 * and the kx_step member the field fills, plus a reader for the data blocks that also applies the checks
 * involving several fields. Header fields are all read and range-checked before any data block is touched, and a
 * data block's size is checked against the bytes left before it is read (rd_weight / rd_floats), so a corrupt
 * record is rejected before anything is allocated for it. The accepted values are those of the reference's
 * loader (include/kernix_model.h kernix_parse_op :1082-1245), which the loader tests compare file by file. */

#define KX_MAX_FIELDS 14
#define TO_NONE (-1)
#define TO(member) ((short)offsetof(kx_step, member))

typedef struct {
    uint32_t lo, hi; /* accepted range */
    short to;        /* offset of the int member of kx_step the value goes to, or TO_NONE */
} kx_field;

typedef int (*kx_data_fn)(kx_rd* r, int ver, kx_step* s, const uint32_t* f, const char** err);

typedef struct {
    int n_fields;
    kx_field field[KX_MAX_FIELDS];
    const char* bad; /* rejection reason for a header field out of range */
    kx_data_fn data; /* data blocks and cross-field checks; NULL: none */
} kx_op_desc;

#define ANY_U32 {0, UINT32_MAX, TO_NONE}
#define FLAG {0, 1, TO_NONE}
#define SIZE_TO(m) {1, INT_MAX, TO(m)}
#define GEOM_TO(m) {1, KERNIX_MAX_GEOM, TO(m)}
#define EDGE_TO(m) {0, KERNIX_MAX_GEOM, TO(m)}

static int data_linear(kx_rd* r, int ver, kx_step* s, const uint32_t* f, const char** err) {
    if (rd_weight(r, ver, f[0], f[1], 1, &s->w, err) != 0) return -1;
    return f[2] && (s->bias = rd_floats(r, f[1])) == NULL ? -1 : 0;
}

static int data_act(kx_rd* r, int ver, kx_step* s, const uint32_t* f, const char** err) {
    if (ver >= 3 && rd_f32(r, &s->alpha) != 0) return -1;
    if (!isfinite(s->alpha)) {
        *err = "activation parameter is not finite";
        return -1;
    }
    return 0;
}

static int data_layernorm(kx_rd* r, int ver, kx_step* s, const uint32_t* f, const char** err) {
    if (rd_f32(r, &s->eps) != 0) return -1;
    if (!(s->eps >= 0.0f) || isinf(s->eps)) {
        *err = "LayerNorm epsilon out of range";
        return -1;
    }
    s->out = s->in;
    if (f[1] && ((s->gamma = rd_floats(r, f[0])) == NULL || (s->beta = rd_floats(r, f[0])) == NULL)) return -1;
    return 0;
}

/* recurrent layers: per direction an input weight (in x gates*units, made float), a recurrent weight (units x
 * gates*units, an I8_COL block stays int8) and the biases (GRU: input then recurrent, 2 * gates*units) */
static int data_recurrent(kx_rd* r, int ver, kx_step* s, const uint32_t* f, const char** err) {
    if (ver < 3) {
        if (s->act != KERNIX_ACT_RELU && s->act != KERNIX_ACT_TANH) {
            *err = "LSTM activation must be relu or tanh";
            return -1;
        }
        s->dirs = 1;
        s->merge = 0;
    }
    const uint64_t gu = rnn_gates(s->kind) * (uint64_t)s->out;
    const uint64_t nb = s->kind == KERNIX_OP_GRU ? 2 * gu : gu;
    kx_weight* in_w[2] = {&s->w, &s->wk};
    kx_weight* rec_w[2] = {&s->wv, &s->wo};
    const float** b[2] = {&s->bias, &s->bk};
    for (int d = 0; d < s->dirs; d++) {
        if (rd_weight(r, ver, (uint64_t)s->in, gu, 0, in_w[d], err) != 0 ||
            rd_weight(r, ver, (uint64_t)s->out, gu, 1, rec_w[d], err) != 0 || (*b[d] = rd_floats(r, nb)) == NULL)
            return -1;
    }
    return 0;
}

static int data_conv(kx_rd* r, int ver, kx_step* s, const uint32_t* f, const char** err) {
    if (s->in % s->groups != 0 || s->out % s->groups != 0) {
        *err = "conv channels do not split into the groups";
        return -1;
    }
    const uint64_t rows = (uint64_t)s->kh * (uint64_t)s->kw * (uint64_t)(s->in / s->groups);
    if (rd_weight(r, ver, rows, (uint64_t)s->out, 0, &s->w, err) != 0) return -1;
    return f[13] && (s->bias = rd_floats(r, f[1])) == NULL ? -1 : 0;
}

static int data_pool(kx_rd* r, int ver, kx_step* s, const uint32_t* f, const char** err) {
    if (s->pt >= s->kh || s->pb >= s->kh || s->pl >= s->kw || s->pr >= s->kw) {
        *err = "pooling padding not smaller than the window";
        return -1;
    }
    return 0;
}

/* RESHAPE: the target shape; PERMUTE: a permutation of the axes */
static int data_axes(kx_rd* r, int ver, kx_step* s, const uint32_t* f, const char** err) {
    uint32_t v[KERNIX_MAX_DIMS];
    if (rd_u32s(r, v, s->nd) != 0) return -1;
    unsigned used = 0;
    for (int k = 0; k < s->nd; k++) {
        if (s->kind == KERNIX_OP_RESHAPE) {
            if (v[k] < 1 || v[k] > INT_MAX) {
                *err = "Reshape dimension out of range";
                return -1;
            }
            s->d[k] = (int)v[k];
        } else {
            if (v[k] >= (uint32_t)s->nd || (used & (1u << v[k]))) {
                *err = "Permute order is not a permutation";
                return -1;
            }
            used |= 1u << v[k];
            s->perm[k] = (int)v[k];
        }
    }
    return 0;
}

static int data_embedding(kx_rd* r, int ver, kx_step* s, const uint32_t* f, const char** err) {
    s->in = f[0] > INT_MAX ? 0 : (int)f[0];
    s->out = f[1] > INT_MAX ? 0 : (int)f[1];
    return rd_weight(r, ver, f[0], f[1], 0, &s->w, err);
}

static int data_affine(kx_rd* r, int ver, kx_step* s, const uint32_t* f, const char** err) {
    s->out = s->in;
    return (s->gamma = rd_floats(r, f[0])) == NULL || (s->beta = rd_floats(r, f[0])) == NULL ? -1 : 0;
}

static int data_add_const(kx_rd* r, int ver, kx_step* s, const uint32_t* f, const char** err) {
    return (s->cst = rd_floats(r, f[0])) == NULL ? -1 : 0;
}

/* ATTENTION: Wq (cq x H*dk), Wk (ck x H*dk), Wv (cv x H*dv), Wo (H*dv x cout), each followed by its bias if any */
static int data_attention(kx_rd* r, int ver, kx_step* s, const uint32_t* f, const char** err) {
    const uint64_t hk = (uint64_t)f[0] * f[1], hv = (uint64_t)f[0] * f[2];
    const struct {
        uint64_t k, n;
        kx_weight* w;
        const float** b;
    } blk[4] = {{f[4], hk, &s->w, &s->bias}, {f[6], hk, &s->wk, &s->bk}, {f[5], hv, &s->wv, &s->bv}, {hv, f[7], &s->wo, &s->bo}};
    for (int i = 0; i < 4; i++) {
        if (rd_weight(r, ver, blk[i].k, blk[i].n, 0, blk[i].w, err) != 0) return -1;
        if (f[8] && (*blk[i].b = rd_floats(r, blk[i].n)) == NULL) return -1;
    }
    return 0;
}

static const kx_op_desc OP_LINEAR = {3, {SIZE_TO(in), SIZE_TO(out), FLAG}, "Linear size out of range", data_linear};
static const kx_op_desc OP_ACT_V12 = {1, {{0, KERNIX_ACT_TANH, TO(act)}}, "unknown activation", data_act};
static const kx_op_desc OP_ACT_V3 = {1, {{0, KERNIX_ACT_LAST, TO(act)}}, "unknown activation", data_act};
static const kx_op_desc OP_LAYERNORM = {2, {SIZE_TO(in), FLAG}, "LayerNorm size out of range", data_layernorm};
static const kx_op_desc OP_SOFTMAX = {0, {{0, 0, TO_NONE}}, NULL, NULL};
/* KNX1/2 LSTM: in, units, act, ret_seq, sequence length; KNX3 LSTM/GRU/RNN: in, units, act, ret_seq, dirs, merge */
static const kx_op_desc OP_LSTM_V12 = {5, {SIZE_TO(in), {1, KX_CHUNK / 2, TO(out)}, {0, KERNIX_ACT_TANH, TO(act)},
                                           {0, 1, TO(ret_seq)}, SIZE_TO(seq)},
                                       "LSTM value out of range", data_recurrent};
static const kx_op_desc OP_RECURRENT_V3 = {6, {SIZE_TO(in), {1, KX_CHUNK / 2, TO(out)}, {0, KERNIX_ACT_LAST, TO(act)},
                                               {0, 1, TO(ret_seq)}, {1, 2, TO(dirs)}, {0, 3, TO(merge)}},
                                           "RNN value out of range", data_recurrent};
/* cin, cout, kh, kw, sh, sw, dh, dw, pad top, bottom, left, right, groups, has_bias */
static const kx_op_desc OP_CONV = {14, {SIZE_TO(in), SIZE_TO(out), GEOM_TO(kh), GEOM_TO(kw), GEOM_TO(sh), GEOM_TO(sw),
                                        GEOM_TO(dh), GEOM_TO(dw), EDGE_TO(pt), EDGE_TO(pb), EDGE_TO(pl), EDGE_TO(pr),
                                        SIZE_TO(groups), FLAG},
                                   "conv value out of range", data_conv};
/* type, kh, kw, sh, sw, pad top, bottom, left, right, count_pad */
static const kx_op_desc OP_POOL = {10, {{0, KERNIX_POOL_AVG, TO(ptype)}, GEOM_TO(kh), GEOM_TO(kw), GEOM_TO(sh), GEOM_TO(sw),
                                        EDGE_TO(pt), EDGE_TO(pb), EDGE_TO(pl), EDGE_TO(pr), {0, 1, TO(count_pad)}},
                                   "pooling value out of range", data_pool};
static const kx_op_desc OP_GLOBAL_POOL = {1, {{0, KERNIX_POOL_AVG, TO(ptype)}}, "pooling value out of range", NULL};
static const kx_op_desc OP_AXES = {1, {{1, KERNIX_MAX_DIMS, TO(nd)}}, "axis count out of range", data_axes};
static const kx_op_desc OP_BINARY = {1, {{0, KERNIX_BIN_MIN, TO(bop)}}, "unknown binary op", NULL};
static const kx_op_desc OP_CONCAT = {1, {{0, KERNIX_AXIS_LAST, TO(axis)}}, "Concatenate axis out of range", NULL};
static const kx_op_desc OP_EMBEDDING = {2, {ANY_U32, ANY_U32}, NULL, data_embedding};
static const kx_op_desc OP_AFFINE = {1, {SIZE_TO(in)}, "Affine size out of range", data_affine};
static const kx_op_desc OP_ADD_CONST = {1, {SIZE_TO(in)}, "constant size out of range", data_add_const};
/* heads, dk, dv, causal, cq, cv, ck, cout, has_bias */
static const kx_op_desc OP_ATTENTION = {9, {{1, 4096, TO(heads)}, {1, 65536, TO(dk)}, {1, 65536, TO(dv)}, {0, 1, TO(causal)},
                                            SIZE_TO(in), {1, INT_MAX, TO_NONE}, {1, INT_MAX, TO_NONE}, SIZE_TO(out), FLAG},
                                        "attention value out of range", data_attention};
/* axis, start, length, squeeze */
static const kx_op_desc OP_SELECT = {4, {{0, KERNIX_AXIS_LAST, TO(axis)}, {0, INT_MAX, TO(start)}, SIZE_TO(len),
                                         {0, 1, TO(squeeze)}},
                                     "Select value out of range", NULL};
static const kx_op_desc OP_PAD = {4, {EDGE_TO(pt), EDGE_TO(pb), EDGE_TO(pl), EDGE_TO(pr)}, "padding value out of range", NULL};
static const kx_op_desc OP_UPSAMPLE = {2, {GEOM_TO(sh), GEOM_TO(sw)}, "UpSampling value out of range", NULL};

static const kx_op_desc* op_desc(int kind, int ver) {
    switch (kind) {
    case KERNIX_OP_LINEAR: return &OP_LINEAR;
    case KERNIX_OP_ACT: return ver >= 3 ? &OP_ACT_V3 : &OP_ACT_V12;
    case KERNIX_OP_LAYERNORM: return &OP_LAYERNORM;
    case KERNIX_OP_SOFTMAX: return &OP_SOFTMAX;
    case KERNIX_OP_LSTM: return ver >= 3 ? &OP_RECURRENT_V3 : &OP_LSTM_V12;
    case KERNIX_OP_GRU:
    case KERNIX_OP_RNN: return &OP_RECURRENT_V3;
    case KERNIX_OP_CONV: return &OP_CONV;
    case KERNIX_OP_POOL: return &OP_POOL;
    case KERNIX_OP_GLOBAL_POOL: return &OP_GLOBAL_POOL;
    case KERNIX_OP_RESHAPE:
    case KERNIX_OP_PERMUTE: return &OP_AXES;
    case KERNIX_OP_BINARY: return &OP_BINARY;
    case KERNIX_OP_CONCAT: return &OP_CONCAT;
    case KERNIX_OP_EMBEDDING: return &OP_EMBEDDING;
    case KERNIX_OP_AFFINE: return &OP_AFFINE;
    case KERNIX_OP_ADD_CONST: return &OP_ADD_CONST;
    case KERNIX_OP_ATTENTION: return &OP_ATTENTION;
    case KERNIX_OP_SELECT: return &OP_SELECT;
    case KERNIX_OP_PAD: return &OP_PAD;
    case KERNIX_OP_UPSAMPLE: return &OP_UPSAMPLE;
    default: return NULL;
    }
}

/* Read the header fields and data blocks of the op record at r into s (kind and inputs already set). */
static int read_op(kx_rd* r, int ver, kx_step* s, const char** err) {
    const kx_op_desc* d = op_desc(s->kind, ver);
    if (d == NULL) {
        *err = "unknown op";
        return -1;
    }
    s->act = KERNIX_ACT_NONE;
    s->dirs = 1;
    s->groups = 1;
    s->kh = s->kw = s->sh = s->sw = s->dh = s->dw = 1;
    uint32_t f[KX_MAX_FIELDS];
    if (rd_u32s(r, f, d->n_fields) != 0) return -1;
    for (int i = 0; i < d->n_fields; i++) {
        const kx_field* fd = &d->field[i];
        if (f[i] < fd->lo || f[i] > fd->hi) {
            *err = d->bad;
            return -1;
        }
        if (fd->to != TO_NONE) *(int*)((char*)s + fd->to) = (int)f[i];
    }
    return d->data ? d->data(r, ver, s, f, err) : 0;
}

/* ------------------------------------------------------------------------------------------ value shapes
 *
 * A value's per-sample shape has 1..4 axes, each >= 1, with at most INT_MAX elements; it is stored as r rows of
 * c channels (r = product of the leading axes). Each op kind has a shape rule computing its output shape from
 * its inputs' (the rules of the reference's kernix_infer, include/kernix_model.h:1266-1394). */

typedef struct {
    int nd, d[KERNIX_MAX_DIMS];
} kx_shape;

static int make_val(kx_val* v, const kx_shape* sh) {
    if (sh->nd < 1 || sh->nd > KERNIX_MAX_DIMS) return -1;
    uint64_t elems = 1;
    for (int k = 0; k < sh->nd; k++) {
        if (sh->d[k] < 1) return -1;
        elems *= (uint64_t)sh->d[k];
        if (elems > INT_MAX) return -1; /* every dim is >= 1: prefixes never exceed the total */
    }
    memset(v, 0, sizeof *v);
    v->nd = sh->nd;
    memcpy(v->d, sh->d, sizeof(int) * (size_t)sh->nd);
    v->c = sh->d[sh->nd - 1];
    v->r = (int)(elems / (uint64_t)v->c);
    v->st = -1;
    v->last = -1;
    return 0;
}

typedef int (*kx_shape_rule)(kx_step* s, int ver, const kx_val* vals, kx_shape* y, const char** err);

#define FAIL(msg) \
    do {          \
        *err = msg; \
        return -1; \
    } while (0)

static const kx_val* input(const kx_step* s, const kx_val* vals, int k) { return &vals[s->inp[k]]; }

static int rule_keep(kx_step* s, int ver, const kx_val* vals, kx_shape* y, const char** err) { return 0; }

static int rule_channels_in(kx_step* s, int ver, const kx_val* vals, kx_shape* y, const char** err) {
    if (input(s, vals, 0)->c != s->in) FAIL("input channels differ from the op's size");
    if (s->kind == KERNIX_OP_LINEAR) y->d[y->nd - 1] = s->out;
    return 0;
}

static int rule_recurrent(kx_step* s, int ver, const kx_val* vals, kx_shape* y, const char** err) {
    const kx_val* x = input(s, vals, 0);
    if (x->c != s->in) FAIL("recurrent input size differs from the previous output");
    if (ver < 3 && s->seq != x->r) FAIL("LSTM sequence length differs from the previous step");
    s->seq = x->r;
    const int units = s->dirs == 2 && s->merge == 0 ? 2 * s->out : s->out;
    if (s->ret_seq) {
        y->nd = 2;
        y->d[0] = x->r;
        y->d[1] = units;
    } else {
        y->nd = 1;
        y->d[0] = units;
    }
    return 0;
}

/* CONV / POOL / PAD / UPSAMPLE over a T x C or H x W x C value (a T x C value has W = 1 and 1-wide kernels) */
static int rule_spatial(kx_step* s, int ver, const kx_val* vals, kx_shape* y, const char** err) {
    const int two_d = y->nd == 3;
    if (y->nd != 2 && !two_d) FAIL("spatial op input must be T x C or H x W x C");
    if (!two_d && (s->kw != 1 || s->sw != 1 || s->dw != 1 || s->pl != 0 || s->pr != 0)) FAIL("2-D window on a T x C input");
    if (s->kind == KERNIX_OP_CONV && input(s, vals, 0)->c != s->in) FAIL("conv input channels differ from the previous output");
    const int64_t h = y->d[0], w = two_d ? y->d[1] : 1;
    int64_t oh, ow;
    switch (s->kind) {
    case KERNIX_OP_PAD:
        oh = h + s->pt + s->pb;
        ow = w + s->pl + s->pr;
        break;
    case KERNIX_OP_UPSAMPLE:
        oh = h * s->sh;
        ow = w * s->sw;
        break;
    default: { /* window: extent (k - 1) * dilation + 1 over the padded input, stepped by the stride */
        const int64_t room_h = h + s->pt + s->pb - ((int64_t)(s->kh - 1) * s->dh + 1);
        const int64_t room_w = w + s->pl + s->pr - ((int64_t)(s->kw - 1) * s->dw + 1);
        if (room_h < 0 || room_w < 0) FAIL("window larger than the padded input");
        oh = room_h / s->sh + 1;
        ow = room_w / s->sw + 1;
    }
    }
    if (oh > INT_MAX || ow > INT_MAX) FAIL("shape out of range");
    y->d[0] = (int)oh;
    if (two_d) y->d[1] = (int)ow;
    if (s->kind == KERNIX_OP_CONV) y->d[y->nd - 1] = s->out;
    return 0;
}

static int rule_global_pool(kx_step* s, int ver, const kx_val* vals, kx_shape* y, const char** err) {
    y->nd = 1;
    y->d[0] = input(s, vals, 0)->c;
    return 0;
}

static int rule_reshape(kx_step* s, int ver, const kx_val* vals, kx_shape* y, const char** err) {
    const kx_val* x = input(s, vals, 0);
    uint64_t elems = 1;
    for (int k = 0; k < s->nd; k++) elems *= (uint64_t)s->d[k];
    if (elems != (uint64_t)x->r * (uint64_t)x->c) FAIL("Reshape changes the element count");
    y->nd = s->nd;
    memcpy(y->d, s->d, sizeof y->d);
    return 0;
}

static int rule_permute(kx_step* s, int ver, const kx_val* vals, kx_shape* y, const char** err) {
    const kx_val* x = input(s, vals, 0);
    if (s->nd != x->nd) FAIL("Permute order has the wrong axis count");
    for (int k = 0; k < x->nd; k++) y->d[k] = x->d[s->perm[k]];
    return 0;
}

/* elementwise op of two values; either may broadcast along rows or channels (size 1); the output takes the
 * shape of the operand with more elements (the first on a tie) with the broadcast channel count */
static int rule_binary(kx_step* s, int ver, const kx_val* vals, kx_shape* y, const char** err) {
    const kx_val* a = input(s, vals, 0);
    const kx_val* b = input(s, vals, 1);
    const int rows = a->r > b->r ? a->r : b->r, chans = a->c > b->c ? a->c : b->c;
    const kx_val* larger = (int64_t)b->r * b->c > (int64_t)a->r * a->c ? b : a;
    const int rows_ok = (a->r == rows || a->r == 1) && (b->r == rows || b->r == 1);
    const int chans_ok = (a->c == chans || a->c == 1) && (b->c == chans || b->c == 1);
    if (!rows_ok || !chans_ok || larger->r != rows) FAIL("binary op operands do not broadcast");
    y->nd = larger->nd;
    memcpy(y->d, larger->d, sizeof y->d);
    y->d[y->nd - 1] = chans;
    return 0;
}

static int rule_concat(kx_step* s, int ver, const kx_val* vals, kx_shape* y, const char** err) {
    const kx_val* first = input(s, vals, 0);
    const int ax = s->axis == KERNIX_AXIS_FIRST ? 0 : y->nd - 1;
    int64_t total = 0;
    for (int k = 0; k < s->n_in; k++) {
        const kx_val* v = input(s, vals, k);
        if (v->nd != first->nd) FAIL("Concatenate inputs differ in rank");
        for (int j = 0; j < v->nd; j++)
            if (j != ax && v->d[j] != first->d[j]) FAIL("Concatenate inputs differ off the joined axis");
        total += v->d[ax];
    }
    if (total > INT_MAX) FAIL("shape out of range");
    y->d[ax] = (int)total;
    return 0;
}

static int rule_embedding(kx_step* s, int ver, const kx_val* vals, kx_shape* y, const char** err) {
    if (y->nd >= KERNIX_MAX_DIMS) FAIL("axis count out of range");
    y->d[y->nd++] = s->out;
    return 0;
}

static int rule_add_const(kx_step* s, int ver, const kx_val* vals, kx_shape* y, const char** err) {
    const kx_val* x = input(s, vals, 0);
    if ((int64_t)x->r * x->c != s->in) FAIL("constant size differs from the previous output");
    return 0;
}

/* inputs: query; then value (default: the query); then key (default: the value) */
static int rule_attention(kx_step* s, int ver, const kx_val* vals, kx_shape* y, const char** err) {
    const kx_val* q = input(s, vals, 0);
    const kx_val* v = input(s, vals, s->n_in > 1 ? 1 : 0);
    const kx_val* k = s->n_in > 2 ? input(s, vals, 2) : v;
    if (q->c != s->w.k || v->c != s->wv.k || k->c != s->wk.k || k->r != v->r) FAIL("attention inputs do not fit the weights");
    y->d[y->nd - 1] = s->out;
    return 0;
}

static int rule_select(kx_step* s, int ver, const kx_val* vals, kx_shape* y, const char** err) {
    const int ax = s->axis == KERNIX_AXIS_FIRST ? 0 : y->nd - 1;
    if ((int64_t)s->start + s->len > y->d[ax]) FAIL("Select range outside the input");
    y->d[ax] = s->len;
    if (s->squeeze && s->len == 1 && y->nd > 1) {
        for (int j = ax; j + 1 < y->nd; j++) y->d[j] = y->d[j + 1];
        y->nd--;
    }
    return 0;
}

static const kx_shape_rule SHAPE_RULE[KERNIX_OP_LAST + 1] = {
    [KERNIX_OP_LINEAR] = rule_channels_in,   [KERNIX_OP_ACT] = rule_keep,
    [KERNIX_OP_LAYERNORM] = rule_channels_in, [KERNIX_OP_SOFTMAX] = rule_keep,
    [KERNIX_OP_LSTM] = rule_recurrent,        [KERNIX_OP_GRU] = rule_recurrent,
    [KERNIX_OP_RNN] = rule_recurrent,         [KERNIX_OP_CONV] = rule_spatial,
    [KERNIX_OP_POOL] = rule_spatial,          [KERNIX_OP_GLOBAL_POOL] = rule_global_pool,
    [KERNIX_OP_RESHAPE] = rule_reshape,       [KERNIX_OP_PERMUTE] = rule_permute,
    [KERNIX_OP_BINARY] = rule_binary,         [KERNIX_OP_CONCAT] = rule_concat,
    [KERNIX_OP_EMBEDDING] = rule_embedding,   [KERNIX_OP_AFFINE] = rule_channels_in,
    [KERNIX_OP_ADD_CONST] = rule_add_const,   [KERNIX_OP_ATTENTION] = rule_attention,
    [KERNIX_OP_SELECT] = rule_select,         [KERNIX_OP_PAD] = rule_spatial,
    [KERNIX_OP_UPSAMPLE] = rule_spatial,
};

/* output value of step s: its first input's shape, transformed by the kind's rule */
static int step_output(kx_step* s, int ver, const kx_val* vals, kx_val* out, const char** err) {
    const kx_val* x = input(s, vals, 0);
    kx_shape y = {x->nd, {0}};
    memcpy(y.d, x->d, sizeof y.d);
    if (SHAPE_RULE[s->kind](s, ver, vals, &y, err) != 0) return -1;
    if (make_val(out, &y) != 0) FAIL("shape out of range");
    return 0;
}

int kx_inplace_ok(int kind) {
    return kind == KERNIX_OP_ACT || kind == KERNIX_OP_LAYERNORM || kind == KERNIX_OP_SOFTMAX || kind == KERNIX_OP_AFFINE ||
           kind == KERNIX_OP_ADD_CONST || kind == KERNIX_OP_BINARY;
}

/* ------------------------------------------------------------------------------------------ storage plan
 *
 * Storage buffers form a pool; a buffer is held until the last step that reads any value placed in it, and a
 * step's output goes, in order of preference, (1) for RESHAPE, into its input's buffer (a view); (2) for a step
 * that works row by row in place, into the buffer of an input it reads last if the sizes match; (3) into the
 * free buffer the pool ranks first: the smallest one large enough, else the largest one (grown); a new buffer
 * when none is free. Ties go to the older buffer. This is the reference's plan (kernix_plan :1405-1445): buffer
 * numbers and sizes come out the same, which the loader tests check value by value. */

typedef struct {
    int n;
    size_t* cap;     /* floats per sample */
    int* held_until; /* last step that reads a value in the buffer (or writes one) */
} kx_pool;

/* rank of buffer k for a value of `need` floats: lower is better */
static int pool_better(const kx_pool* p, int k, int than, size_t need) {
    const int k_fits = p->cap[k] >= need, t_fits = p->cap[than] >= need;
    if (k_fits != t_fits) return k_fits;
    return k_fits ? p->cap[k] < p->cap[than] : p->cap[k] > p->cap[than];
}

static int pool_take(kx_pool* p, size_t need, int step) {
    int pick = -1;
    for (int k = 0; k < p->n; k++)
        if (p->held_until[k] < step && (pick < 0 || pool_better(p, k, pick, need))) pick = k;
    if (pick < 0) pick = p->n++;
    if (p->cap[pick] < need) p->cap[pick] = need;
    return pick;
}

static int plan(kx_graph* g) {
    const int n = g->n_steps;
    kx_pool pool = {0, calloc((size_t)n + 1, sizeof(size_t)), calloc((size_t)n + 1, sizeof(int))};
    if (pool.cap == NULL || pool.held_until == NULL) {
        free(pool.cap);
        free(pool.held_until);
        return -1;
    }
    for (int i = 0; i < n; i++) {
        const kx_step* s = &g->steps[i];
        kx_val* v = &g->vals[i + 1];
        const size_t need = (size_t)v->r * (size_t)v->c;
        int buf = -2; /* -1 is the caller's input buffer (a RESHAPE view of the model input) */
        if (s->kind == KERNIX_OP_RESHAPE) {
            buf = g->vals[s->inp[0]].st;
        } else if (kx_inplace_ok(s->kind)) {
            const int n_cand = s->kind == KERNIX_OP_BINARY ? 2 : 1;
            for (int k = 0; k < n_cand && buf == -2; k++) {
                const kx_val* u = &g->vals[s->inp[k]];
                const int last_reader = u->st >= 0 && pool.held_until[u->st] <= i;
                if (last_reader && (size_t)u->r * (size_t)u->c == need) buf = u->st;
            }
        }
        if (buf == -2) buf = pool_take(&pool, need, i);
        v->st = buf;
        if (buf >= 0) {
            const int until = v->last > i ? v->last : i;
            if (pool.held_until[buf] < until) pool.held_until[buf] = until;
        }
    }
    free(pool.held_until);
    g->n_st = pool.n;
    g->st_cap = pool.cap;
    return 0;
}

static void weight_free(kx_weight* w) { free(w->own); }

void kx_graph_free(kx_graph* g) {
    if (g == NULL) return;
    for (int i = 0; g->steps != NULL && i < g->n_steps; i++) {
        kx_step* s = &g->steps[i];
        weight_free(&s->w);
        weight_free(&s->wk);
        weight_free(&s->wv);
        weight_free(&s->wo);
    }
    free(g->steps);
    free(g->vals);
    free(g->st_cap);
    if (g->map != NULL) munmap(g->map, g->map_len);
    free(g);
}

kx_graph* kx_graph_load(const char* path, const char** err) {
    *err = "file shorter than declared";
    int fd = path ? open(path, O_RDONLY | O_CLOEXEC) : -1;
    if (fd < 0) {
        *err = "cannot open the file";
        return NULL;
    }
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size < 0) {
        close(fd);
        *err = "cannot open the file";
        return NULL;
    }
    kx_graph* g = calloc(1, sizeof *g);
    int* cons = NULL;
    int* map = NULL;
    if (g == NULL) {
        close(fd);
        *err = "out of memory";
        return NULL;
    }
    g->map_len = (size_t)st.st_size;
    if (g->map_len > 0) {
        g->map = mmap(NULL, g->map_len, PROT_READ, MAP_PRIVATE, fd, 0);
        if (g->map == MAP_FAILED) {
            g->map = NULL;
            close(fd);
            free(g);
            *err = "cannot map the file";
            return NULL;
        }
        madvise(g->map, g->map_len, MADV_SEQUENTIAL);
    }
    close(fd);
    kx_rd r = {(const uint8_t*)g->map, g->map_len};
    uint32_t magic_n, n_ops, hdr[2 + KERNIX_MAX_DIMS];
    if (rd_u32(&r, &magic_n) != 0 || rd_u32(&r, &n_ops) != 0) goto fail;
    char magic[4];
    memcpy(magic, &magic_n, 4);
    const int ver = memcmp(magic, "KNX1", 4) == 0 ? 1 : memcmp(magic, "KNX2", 4) == 0 ? 2 : memcmp(magic, "KNX3", 4) == 0 ? 3 : 0;
    if (ver == 0) { *err = "not a KNX1/KNX2/KNX3 file"; goto fail; }
    if (n_ops < 1 || n_ops > KERNIX_MODEL_MAX_OPS) { *err = "op count out of range"; goto fail; }
    g->ver = ver;
    g->steps = calloc(n_ops, sizeof(kx_step));
    g->vals = calloc((size_t)n_ops + 1, sizeof(kx_val));
    cons = calloc((size_t)n_ops + 1, sizeof(int));
    map = calloc((size_t)n_ops + 1, sizeof(int));
    if (g->steps == NULL || g->vals == NULL || cons == NULL || map == NULL) { *err = "out of memory"; goto fail; }
    if (ver == 3) { /* layout, input rank, per-sample input shape (channels-last) */
        if (rd_u32s(&r, hdr, 2) != 0) goto fail;
        if (hdr[0] > 1 || hdr[1] < 1 || hdr[1] > KERNIX_MAX_DIMS) { *err = "input shape out of range"; goto fail; }
        kx_shape in = {(int)hdr[1], {0}};
        if (rd_u32s(&r, hdr + 2, (int)hdr[1]) != 0) goto fail;
        for (uint32_t k = 0; k < hdr[1]; k++) in.d[k] = hdr[2 + k] > INT_MAX ? 0 : (int)hdr[2 + k];
        if (make_val(&g->vals[0], &in) != 0) { *err = "input shape out of range"; goto fail; }
        g->layout = (int)hdr[0];
    }
    for (uint32_t i = 0; i < n_ops; i++) {
        kx_step* s = &g->steps[i];
        uint32_t kind;
        if (rd_u32(&r, &kind) != 0) goto fail;
        if (kind > (uint32_t)(ver == 3 ? KERNIX_OP_LAST : KERNIX_OP_LSTM)) { *err = "unknown op"; goto fail; }
        s->kind = (int)kind;
        if (ver == 3) { /* input value ids: 0 = model input, k+1 = output of op k (earlier ops only) */
            uint32_t n_in;
            if (rd_u32(&r, &n_in) != 0) goto fail;
            const uint32_t lo = (kind == KERNIX_OP_BINARY || kind == KERNIX_OP_CONCAT) ? 2 : 1;
            const uint32_t hi = kind == KERNIX_OP_BINARY ? 2 : kind == KERNIX_OP_CONCAT ? KERNIX_MAX_INPUTS
                                                             : kind == KERNIX_OP_ATTENTION ? 3 : 1;
            if (n_in < lo || n_in > hi) { *err = "op input count out of range"; goto fail; }
            s->n_in = (int)n_in;
            for (uint32_t k = 0; k < n_in; k++) {
                uint32_t id;
                if (rd_u32(&r, &id) != 0) goto fail;
                if (id > i) { *err = "op input refers to a later op"; goto fail; }
                s->inp[k] = (int)id;
            }
        } else {
            s->n_in = 1;
            s->inp[0] = (int)i;
        }
        g->n_steps = (int)i + 1; /* steps parsed so far are freed on failure */
        if (read_op(&r, ver, s, err) != 0) goto fail;
    }
    if (r.left != 0) { *err = "data left after the last op"; goto fail; }
    if (ver < 3) { /* input: first sized op's width; with an LSTM, its sequence length x that width */
        int in_dim = 0, seq = 0;
        for (uint32_t i = 0; i < n_ops; i++) {
            const kx_step* s = &g->steps[i];
            if (in_dim == 0 && (s->kind == KERNIX_OP_LINEAR || s->kind == KERNIX_OP_LAYERNORM || s->kind == KERNIX_OP_LSTM))
                in_dim = s->in;
            if (seq == 0 && s->kind == KERNIX_OP_LSTM) seq = s->seq;
        }
        if (in_dim == 0) { *err = "no Linear or LayerNorm gives the input size"; goto fail; }
        const kx_shape in = seq ? (kx_shape){2, {seq, in_dim}} : (kx_shape){1, {in_dim}};
        if (make_val(&g->vals[0], &in) != 0) { *err = "input shape out of range"; goto fail; }
    }
    for (uint32_t i = 0; i < n_ops; i++)
        if (step_output(&g->steps[i], ver, g->vals, &g->vals[i + 1], err) != 0) goto fail;

    /* fuse an ACT into the LINEAR/CONV whose output only it reads */
    for (uint32_t i = 0; i < n_ops; i++)
        for (int k = 0; k < g->steps[i].n_in; k++) cons[g->steps[i].inp[k]]++;
    cons[n_ops]++;
    int n = 0;
    for (uint32_t i = 0; i < n_ops; i++) {
        kx_step s = g->steps[i];
        for (int k = 0; k < s.n_in; k++) s.inp[k] = map[s.inp[k]];
        if (s.kind == KERNIX_OP_ACT && s.inp[0] > 0 && cons[g->steps[i].inp[0]] == 1) {
            kx_step* p = &g->steps[s.inp[0] - 1];
            if ((p->kind == KERNIX_OP_LINEAR || p->kind == KERNIX_OP_CONV) && p->act == KERNIX_ACT_NONE) {
                p->act = s.act;
                p->alpha = s.alpha;
                map[i + 1] = s.inp[0];
                continue;
            }
        }
        g->steps[n] = s;
        g->vals[n + 1] = g->vals[i + 1];
        map[i + 1] = n + 1;
        n++;
    }
    if (n < (int)n_ops) memset(&g->steps[n], 0, sizeof(kx_step) * (n_ops - (uint32_t)n));
    g->n_steps = n;
    g->n_vals = n + 1;
    g->out_v = map[n_ops];
    for (int i = 0; i < n; i++)
        for (int k = 0; k < g->steps[i].n_in; k++) g->vals[g->steps[i].inp[k]].last = i;
    g->vals[g->out_v].last = n;
    if (plan(g) != 0) { *err = "out of memory"; goto fail; }
    free(cons);
    free(map);
    return g;
fail:
    free(cons);
    free(map);
    kx_graph_free(g);
    return NULL;
}

/* ---------------------------------------------------------------------------- host-only inspection */

KERNIX_API int kx_knx_inspect(const char* path, long* info, int* shapes, int* kinds, int* acts, int cap, char* err,
                              int errlen) {
    const char* e = NULL;
    kx_graph* g = kx_graph_load(path, &e);
    if (g == NULL) {
        if (err && errlen > 0) snprintf(err, (size_t)errlen, "%s", e ? e : "?");
        return -1;
    }
    const kx_val* vin = &g->vals[0];
    const kx_val* vout = &g->vals[g->out_v];
    size_t per = 0;
    for (int k = 0; k < g->n_st; k++) per += g->st_cap[k];
    long v[12] = {g->n_steps, vin->c, (long)vout->r * vout->c, vin->r, g->layout, vin->nd, vout->nd, g->n_st, g->ver,
                  (long)per, 0, 0};
    for (int i = 0; i < 12; i++) info[i] = v[i];
    for (int k = 0; k < KERNIX_MAX_DIMS; k++) {
        shapes[k] = k < vin->nd ? vin->d[k] : 0;
        shapes[4 + k] = k < vout->nd ? vout->d[k] : 0;
    }
    for (int i = 0; i < g->n_steps && i < cap; i++) {
        kinds[i] = g->steps[i].kind;
        acts[i] = g->steps[i].act;
    }
    kx_graph_free(g);
    return 0;
}

KERNIX_API int kx_knx_plan(const char* path, int* st, int* last, int cap) {
    const char* e = NULL;
    kx_graph* g = kx_graph_load(path, &e);
    if (g == NULL) return -1;
    for (int v = 0; v < g->n_vals && v < cap; v++) {
        st[v] = g->vals[v].st;
        last[v] = g->vals[v].last;
    }
    const int n = g->n_vals;
    kx_graph_free(g);
    return n;
}
