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

static int parse_op(kx_rd* r, int ver, kx_step* s, const char** err) {
    uint32_t a[16];
    s->act = KERNIX_ACT_NONE;
    s->dirs = 1;
    s->groups = 1;
    s->kh = s->kw = s->sh = s->sw = s->dh = s->dw = 1;
    switch (s->kind) {
    case KERNIX_OP_LINEAR:
        if (rd_u32s(r, a, 3) != 0) return -1;
        if (a[0] < 1 || a[1] < 1 || a[0] > INT_MAX || a[1] > INT_MAX || a[2] > 1) {
            *err = "Linear size out of range";
            return -1;
        }
        s->in = (int)a[0];
        s->out = (int)a[1];
        if (rd_weight(r, ver, a[0], a[1], 1, &s->w, err) != 0) return -1;
        if (a[2] && (s->bias = rd_floats(r, a[1])) == NULL) return -1;
        return 0;
    case KERNIX_OP_ACT:
        if (rd_u32(r, &a[0]) != 0 || (ver >= 3 && rd_f32(r, &s->alpha) != 0)) return -1;
        if (a[0] > (uint32_t)(ver >= 3 ? KERNIX_ACT_LAST : KERNIX_ACT_TANH) || !isfinite(s->alpha)) {
            *err = "unknown activation";
            return -1;
        }
        s->act = (int)a[0];
        return 0;
    case KERNIX_OP_LAYERNORM:
        if (rd_u32s(r, a, 2) != 0 || rd_f32(r, &s->eps) != 0) return -1;
        if (a[0] < 1 || a[0] > INT_MAX || a[1] > 1 || !(s->eps >= 0.0f) || isinf(s->eps)) {
            *err = "LayerNorm value out of range";
            return -1;
        }
        s->in = s->out = (int)a[0];
        if (a[1] && ((s->gamma = rd_floats(r, a[0])) == NULL || (s->beta = rd_floats(r, a[0])) == NULL)) return -1;
        return 0;
    case KERNIX_OP_SOFTMAX:
        return 0;
    case KERNIX_OP_LSTM:
    case KERNIX_OP_GRU:
    case KERNIX_OP_RNN: {
        if (ver < 3) { /* in, units, act (relu/tanh), ret_seq, seq */
            if (rd_u32s(r, a, 5) != 0) return -1;
            if (a[0] < 1 || a[0] > INT_MAX || a[1] < 1 || a[1] > KX_CHUNK / 2 || a[3] > 1 || a[4] < 1 || a[4] > INT_MAX ||
                (a[2] != KERNIX_ACT_RELU && a[2] != KERNIX_ACT_TANH)) {
                *err = "LSTM value out of range";
                return -1;
            }
            s->seq = (int)a[4];
            a[4] = 1;
            a[5] = 0;
        } else { /* in, units, act, ret_seq, dirs, merge */
            if (rd_u32s(r, a, 6) != 0) return -1;
            if (a[0] < 1 || a[0] > INT_MAX || a[1] < 1 || a[1] > KX_CHUNK / 2 || a[2] > KERNIX_ACT_LAST || a[3] > 1 ||
                a[4] < 1 || a[4] > 2 || a[5] > 3) {
                *err = "RNN value out of range";
                return -1;
            }
        }
        s->in = (int)a[0];
        s->out = (int)a[1];
        s->act = (int)a[2];
        s->ret_seq = (int)a[3];
        s->dirs = (int)a[4];
        s->merge = (int)a[5];
        const uint64_t gu = rnn_gates(s->kind) * (uint64_t)a[1], nb = s->kind == KERNIX_OP_GRU ? 2 * gu : gu;
        for (int d = 0; d < s->dirs; d++) {
            kx_weight* wx = d ? &s->wk : &s->w; /* input and recurrent weights, per direction */
            kx_weight* wr = d ? &s->wo : &s->wv;
            if (rd_weight(r, ver, a[0], gu, 0, wx, err) != 0 || rd_weight(r, ver, a[1], gu, 1, wr, err) != 0) return -1;
            const float** bp = d ? &s->bk : &s->bias; /* input bias (gu), then for GRU the recurrent bias (gu) */
            if ((*bp = rd_floats(r, nb)) == NULL) return -1;
        }
        return 0;
    }
    case KERNIX_OP_CONV: /* cin, cout, kh, kw, sh, sw, dh, dw, pt, pb, pl, pr, groups, has_bias */
        if (rd_u32s(r, a, 14) != 0) return -1;
        if (a[0] < 1 || a[0] > INT_MAX || a[1] < 1 || a[1] > INT_MAX || !geom_ok(a[2], 1) || !geom_ok(a[3], 1) ||
            !geom_ok(a[4], 1) || !geom_ok(a[5], 1) || !geom_ok(a[6], 1) || !geom_ok(a[7], 1) || !geom_ok(a[8], 0) ||
            !geom_ok(a[9], 0) || !geom_ok(a[10], 0) || !geom_ok(a[11], 0) || a[12] < 1 || a[0] % a[12] != 0 ||
            a[1] % a[12] != 0 || a[13] > 1) {
            *err = "conv value out of range";
            return -1;
        }
        s->in = (int)a[0];
        s->out = (int)a[1];
        s->kh = (int)a[2]; s->kw = (int)a[3]; s->sh = (int)a[4]; s->sw = (int)a[5]; s->dh = (int)a[6]; s->dw = (int)a[7];
        s->pt = (int)a[8]; s->pb = (int)a[9]; s->pl = (int)a[10]; s->pr = (int)a[11]; s->groups = (int)a[12];
        if (rd_weight(r, ver, (uint64_t)a[2] * a[3] * (a[0] / a[12]), a[1], 0, &s->w, err) != 0) return -1;
        if (a[13] && (s->bias = rd_floats(r, a[1])) == NULL) return -1;
        return 0;
    case KERNIX_OP_POOL: /* type, kh, kw, sh, sw, pt, pb, pl, pr, count_pad */
        if (rd_u32s(r, a, 10) != 0) return -1;
        if (a[0] > KERNIX_POOL_AVG || !geom_ok(a[1], 1) || !geom_ok(a[2], 1) || !geom_ok(a[3], 1) || !geom_ok(a[4], 1) ||
            a[5] >= a[1] || a[6] >= a[1] || a[7] >= a[2] || a[8] >= a[2] || a[9] > 1) {
            *err = "pooling value out of range";
            return -1;
        }
        s->ptype = (int)a[0]; s->kh = (int)a[1]; s->kw = (int)a[2]; s->sh = (int)a[3]; s->sw = (int)a[4];
        s->pt = (int)a[5]; s->pb = (int)a[6]; s->pl = (int)a[7]; s->pr = (int)a[8]; s->count_pad = (int)a[9];
        return 0;
    case KERNIX_OP_GLOBAL_POOL:
        if (rd_u32(r, &a[0]) != 0) return -1;
        if (a[0] > KERNIX_POOL_AVG) {
            *err = "pooling value out of range";
            return -1;
        }
        s->ptype = (int)a[0];
        return 0;
    case KERNIX_OP_RESHAPE:
    case KERNIX_OP_PERMUTE: {
        if (rd_u32(r, &a[0]) != 0) return -1;
        if (a[0] < 1 || a[0] > KERNIX_MAX_DIMS) {
            *err = "axis count out of range";
            return -1;
        }
        s->nd = (int)a[0];
        if (rd_u32s(r, a + 1, s->nd) != 0) return -1;
        int seen = 0;
        for (int k = 0; k < s->nd; k++) {
            const uint32_t v = a[1 + k];
            if (s->kind == KERNIX_OP_RESHAPE) {
                if (v < 1 || v > INT_MAX) {
                    *err = "Reshape shape out of range";
                    return -1;
                }
                s->d[k] = (int)v;
            } else {
                if (v >= (uint32_t)s->nd || ((seen >> v) & 1)) {
                    *err = "Permute axis order is wrong";
                    return -1;
                }
                s->perm[k] = (int)v;
                seen |= 1 << v;
            }
        }
        return 0;
    }
    case KERNIX_OP_BINARY:
        if (rd_u32(r, &a[0]) != 0) return -1;
        if (a[0] > KERNIX_BIN_MIN) {
            *err = "unknown binary op";
            return -1;
        }
        s->bop = (int)a[0];
        return 0;
    case KERNIX_OP_CONCAT:
        if (rd_u32(r, &a[0]) != 0) return -1;
        if (a[0] > KERNIX_AXIS_LAST) {
            *err = "Concatenate axis out of range";
            return -1;
        }
        s->axis = (int)a[0];
        return 0;
    case KERNIX_OP_EMBEDDING:
        if (rd_u32s(r, a, 2) != 0) return -1;
        s->in = (int)(a[0] > INT_MAX ? 0 : a[0]);
        s->out = (int)(a[1] > INT_MAX ? 0 : a[1]);
        return rd_weight(r, ver, a[0], a[1], 0, &s->w, err);
    case KERNIX_OP_AFFINE:
        if (rd_u32(r, &a[0]) != 0) return -1;
        if (a[0] < 1 || a[0] > INT_MAX) {
            *err = "Affine size out of range";
            return -1;
        }
        s->in = s->out = (int)a[0];
        if ((s->gamma = rd_floats(r, a[0])) == NULL || (s->beta = rd_floats(r, a[0])) == NULL) return -1;
        return 0;
    case KERNIX_OP_ADD_CONST:
        if (rd_u32(r, &a[0]) != 0) return -1;
        if (a[0] < 1 || a[0] > INT_MAX) {
            *err = "constant size out of range";
            return -1;
        }
        s->in = (int)a[0];
        return (s->cst = rd_floats(r, a[0])) == NULL ? -1 : 0;
    case KERNIX_OP_ATTENTION: { /* heads, dk, dv, causal, cq, cv, ck, cout, has_bias */
        if (rd_u32s(r, a, 9) != 0) return -1;
        if (a[0] < 1 || a[0] > 4096 || a[1] < 1 || a[1] > 65536 || a[2] < 1 || a[2] > 65536 || a[3] > 1 || a[8] > 1 ||
            a[4] < 1 || a[4] > INT_MAX || a[5] < 1 || a[5] > INT_MAX || a[6] < 1 || a[6] > INT_MAX || a[7] < 1 ||
            a[7] > INT_MAX) {
            *err = "attention value out of range";
            return -1;
        }
        s->heads = (int)a[0]; s->dk = (int)a[1]; s->dv = (int)a[2]; s->causal = (int)a[3];
        s->in = (int)a[4];
        s->out = (int)a[7];
        const uint64_t hk = (uint64_t)a[0] * a[1], hv = (uint64_t)a[0] * a[2];
        if (rd_weight(r, ver, a[4], hk, 0, &s->w, err) != 0 || (a[8] && (s->bias = rd_floats(r, hk)) == NULL) ||
            rd_weight(r, ver, a[6], hk, 0, &s->wk, err) != 0 || (a[8] && (s->bk = rd_floats(r, hk)) == NULL) ||
            rd_weight(r, ver, a[5], hv, 0, &s->wv, err) != 0 || (a[8] && (s->bv = rd_floats(r, hv)) == NULL) ||
            rd_weight(r, ver, hv, a[7], 0, &s->wo, err) != 0 || (a[8] && (s->bo = rd_floats(r, a[7])) == NULL))
            return -1;
        return 0;
    }
    case KERNIX_OP_SELECT: /* axis, start, len, squeeze */
        if (rd_u32s(r, a, 4) != 0) return -1;
        if (a[0] > KERNIX_AXIS_LAST || a[1] > INT_MAX || a[2] < 1 || a[2] > INT_MAX || a[3] > 1) {
            *err = "Select value out of range";
            return -1;
        }
        s->axis = (int)a[0]; s->start = (int)a[1]; s->len = (int)a[2]; s->squeeze = (int)a[3];
        return 0;
    case KERNIX_OP_PAD:
        if (rd_u32s(r, a, 4) != 0) return -1;
        if (!geom_ok(a[0], 0) || !geom_ok(a[1], 0) || !geom_ok(a[2], 0) || !geom_ok(a[3], 0)) {
            *err = "padding value out of range";
            return -1;
        }
        s->pt = (int)a[0]; s->pb = (int)a[1]; s->pl = (int)a[2]; s->pr = (int)a[3];
        return 0;
    case KERNIX_OP_UPSAMPLE:
        if (rd_u32s(r, a, 2) != 0) return -1;
        if (!geom_ok(a[0], 1) || !geom_ok(a[1], 1)) {
            *err = "UpSampling value out of range";
            return -1;
        }
        s->sh = (int)a[0]; s->sw = (int)a[1];
        return 0;
    default:
        *err = "unknown op";
        return -1;
    }
}

static int val_set(kx_val* v, int nd, const int* d) {
    if (nd < 1 || nd > KERNIX_MAX_DIMS) return -1;
    uint64_t r = 1;
    for (int k = 0; k < nd; k++) {
        if (d[k] < 1) return -1;
        if (k < nd - 1 && (r *= (uint64_t)d[k]) > INT_MAX) return -1;
    }
    if (r * (uint64_t)d[nd - 1] > INT_MAX) return -1;
    memset(v, 0, sizeof *v);
    v->nd = nd;
    memcpy(v->d, d, sizeof(int) * (size_t)nd);
    v->r = (int)r;
    v->c = d[nd - 1];
    v->st = -1;
    v->last = -1;
    return 0;
}

static int infer(kx_step* s, int ver, const kx_val* fv, kx_val* out, const char** err) {
    const kx_val* x = &fv[s->inp[0]];
    int nd = x->nd, d[KERNIX_MAX_DIMS];
    memcpy(d, x->d, sizeof d);
    switch (s->kind) {
    case KERNIX_OP_LINEAR:
        if (x->c != s->in) { *err = "Linear input size differs from the previous output"; return -1; }
        d[nd - 1] = s->out;
        break;
    case KERNIX_OP_ACT:
    case KERNIX_OP_SOFTMAX:
        break;
    case KERNIX_OP_LAYERNORM:
        if (x->c != s->in) { *err = "LayerNorm size differs from the previous output"; return -1; }
        break;
    case KERNIX_OP_LSTM:
    case KERNIX_OP_GRU:
    case KERNIX_OP_RNN: {
        if (x->c != s->in) { *err = "RNN input size differs from the previous output"; return -1; }
        if (ver < 3 && s->seq != x->r) { *err = "LSTM sequence length differs from the previous step"; return -1; }
        s->seq = x->r;
        const int uo = s->dirs == 2 && s->merge == 0 ? 2 * s->out : s->out;
        if (s->ret_seq) { nd = 2; d[0] = x->r; d[1] = uo; }
        else { nd = 1; d[0] = uo; }
        break;
    }
    case KERNIX_OP_CONV:
    case KERNIX_OP_POOL:
    case KERNIX_OP_PAD:
    case KERNIX_OP_UPSAMPLE: {
        if (nd != 2 && nd != 3) { *err = "conv/pool input must be T x C or H x W x C"; return -1; }
        if (nd == 2 && (s->kw != 1 || s->sw != 1 || s->dw != 1 || s->pl != 0 || s->pr != 0)) {
            *err = "2-D kernel on a 1-D (T x C) input";
            return -1;
        }
        if (s->kind == KERNIX_OP_CONV && x->c != s->in) { *err = "conv input channels differ from the previous output"; return -1; }
        const int64_t H = d[0], W = nd == 3 ? d[1] : 1;
        int64_t Ho, Wo;
        if (s->kind == KERNIX_OP_PAD) { Ho = H + s->pt + s->pb; Wo = W + s->pl + s->pr; }
        else if (s->kind == KERNIX_OP_UPSAMPLE) { Ho = H * s->sh; Wo = W * s->sw; }
        else {
            const int64_t nh = H + s->pt + s->pb - ((int64_t)s->dh * (s->kh - 1) + 1);
            const int64_t nw = W + s->pl + s->pr - ((int64_t)s->dw * (s->kw - 1) + 1);
            if (nh < 0 || nw < 0) { *err = "conv/pool output size <= 0"; return -1; }
            Ho = nh / s->sh + 1;
            Wo = nw / s->sw + 1;
        }
        if (Ho > INT_MAX || Wo > INT_MAX) { *err = "shape out of range"; return -1; }
        d[0] = (int)Ho;
        if (nd == 3) d[1] = (int)Wo;
        if (s->kind == KERNIX_OP_CONV) d[nd - 1] = s->out;
        break;
    }
    case KERNIX_OP_GLOBAL_POOL:
        nd = 1;
        d[0] = x->c;
        break;
    case KERNIX_OP_RESHAPE: {
        uint64_t n = 1;
        for (int k = 0; k < s->nd; k++) n *= (uint64_t)s->d[k];
        if (n != (uint64_t)x->r * (uint64_t)x->c) { *err = "Reshape size differs from the input"; return -1; }
        nd = s->nd;
        memcpy(d, s->d, sizeof d);
        break;
    }
    case KERNIX_OP_PERMUTE:
        if (s->nd != nd) { *err = "Permute axis count differs from the input"; return -1; }
        for (int k = 0; k < nd; k++) d[k] = x->d[s->perm[k]];
        break;
    case KERNIX_OP_BINARY: {
        const kx_val* y = &fv[s->inp[1]];
        const int R = x->r > y->r ? x->r : y->r, C = x->c > y->c ? x->c : y->c;
        const kx_val* big = (int64_t)x->r * x->c >= (int64_t)y->r * y->c ? x : y;
        if ((x->r != R && x->r != 1) || (y->r != R && y->r != 1) || (x->c != C && x->c != 1) || (y->c != C && y->c != 1) ||
            big->r != R) {
            *err = "binary op input shapes do not match";
            return -1;
        }
        nd = big->nd;
        memcpy(d, big->d, sizeof d);
        d[nd - 1] = C;
        break;
    }
    case KERNIX_OP_CONCAT: {
        int64_t sum = 0;
        const int ax = s->axis == KERNIX_AXIS_FIRST ? 0 : nd - 1;
        for (int k = 0; k < s->n_in; k++) {
            const kx_val* v = &fv[s->inp[k]];
            int same = v->nd == nd;
            for (int j = 0; same && j < nd; j++)
                if (j != ax) same = v->d[j] == x->d[j];
            if (!same) { *err = "Concatenate input shapes do not match"; return -1; }
            sum += v->d[ax];
        }
        if (sum > INT_MAX) { *err = "shape out of range"; return -1; }
        d[ax] = (int)sum;
        break;
    }
    case KERNIX_OP_EMBEDDING:
        if (nd >= KERNIX_MAX_DIMS) { *err = "axis count out of range"; return -1; }
        d[nd++] = s->out;
        break;
    case KERNIX_OP_AFFINE:
        if (x->c != s->in) { *err = "Affine size differs from the previous output"; return -1; }
        break;
    case KERNIX_OP_ADD_CONST:
        if ((int64_t)x->r * x->c != s->in) { *err = "constant size differs from the previous output"; return -1; }
        break;
    case KERNIX_OP_ATTENTION: {
        const kx_val* v = &fv[s->inp[s->n_in > 1 ? 1 : 0]];
        const kx_val* k = &fv[s->inp[s->n_in > 2 ? 2 : s->n_in > 1 ? 1 : 0]];
        if (x->c != s->w.k || v->c != s->wv.k || k->c != s->wk.k || k->r != v->r) {
            *err = "attention input sizes differ from the weights";
            return -1;
        }
        d[nd - 1] = s->out;
        break;
    }
    case KERNIX_OP_SELECT: {
        const int ax = s->axis == KERNIX_AXIS_FIRST ? 0 : nd - 1;
        if ((int64_t)s->start + s->len > d[ax]) { *err = "Select range outside the input"; return -1; }
        d[ax] = s->len;
        if (s->squeeze && s->len == 1 && nd > 1) {
            memmove(d + ax, d + ax + 1, sizeof(int) * (size_t)(nd - 1 - ax));
            nd--;
        }
        break;
    }
    default:
        break;
    }
    if (val_set(out, nd, d) != 0) { *err = "shape out of range"; return -1; }
    return 0;
}

int kx_inplace_ok(int kind) {
    return kind == KERNIX_OP_ACT || kind == KERNIX_OP_LAYERNORM || kind == KERNIX_OP_SOFTMAX || kind == KERNIX_OP_AFFINE ||
           kind == KERNIX_OP_ADD_CONST || kind == KERNIX_OP_BINARY;
}

/* Storage plan: a value reuses a buffer whose values are all dead; RESHAPE views its input's buffer; an
 * in-place capable step that is the last reader of an input of the same size writes over it. Among free
 * buffers the smallest one that is large enough wins, else the largest one grows. */
static int plan(kx_graph* g) {
    const int n = g->n_steps;
    size_t* cap = calloc((size_t)n + 1, sizeof(size_t));
    int* busy = calloc((size_t)n + 1, sizeof(int));
    if (cap == NULL || busy == NULL) {
        free(cap);
        free(busy);
        return -1;
    }
    int ns = 0;
    for (int i = 0; i < n; i++) {
        const kx_step* s = &g->steps[i];
        kx_val* v = &g->vals[i + 1];
        const size_t need = (size_t)v->r * (size_t)v->c;
        int st = -2;
        if (s->kind == KERNIX_OP_RESHAPE) {
            st = g->vals[s->inp[0]].st;
        } else if (kx_inplace_ok(s->kind)) {
            for (int k = 0; k < (s->kind == KERNIX_OP_BINARY ? 2 : 1) && st == -2; k++) {
                const kx_val* u = &g->vals[s->inp[k]];
                if (u->st >= 0 && busy[u->st] <= i && (size_t)u->r * (size_t)u->c == need) st = u->st;
            }
        }
        if (st == -2) {
            int best = -1;
            for (int k = 0; k < ns; k++) {
                if (busy[k] >= i) continue;
                if (best < 0) best = k;
                else if (cap[k] >= need ? (cap[best] < need || cap[k] < cap[best]) : (cap[best] < need && cap[k] > cap[best]))
                    best = k;
            }
            if (best < 0) best = ns++;
            if (cap[best] < need) cap[best] = need;
            st = best;
        }
        v->st = st;
        if (st >= 0 && busy[st] < v->last) busy[st] = v->last;
        if (st >= 0 && busy[st] < i) busy[st] = i;
    }
    free(busy);
    g->n_st = ns;
    g->st_cap = cap;
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
        int d[KERNIX_MAX_DIMS];
        if (rd_u32s(&r, hdr + 2, (int)hdr[1]) != 0) goto fail;
        for (uint32_t k = 0; k < hdr[1]; k++) d[k] = hdr[2 + k] > INT_MAX ? 0 : (int)hdr[2 + k];
        if (val_set(&g->vals[0], (int)hdr[1], d) != 0) { *err = "input shape out of range"; goto fail; }
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
        if (parse_op(&r, ver, s, err) != 0) goto fail;
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
        const int d[2] = {seq ? seq : in_dim, in_dim};
        if (val_set(&g->vals[0], seq ? 2 : 1, d) != 0) { *err = "input shape out of range"; goto fail; }
    }
    for (uint32_t i = 0; i < n_ops; i++)
        if (infer(&g->steps[i], ver, g->vals, &g->vals[i + 1], err) != 0) goto fail;

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
