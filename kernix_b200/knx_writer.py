"""Write `.knx` model files (KNX1 / KNX2 / KNX3) from numpy arrays, without torch.

The format is the reference's (little-endian u32 records; weight blocks F32 / I8_COL / I8_ROW):
KNX1 sequential float32 (docs/mlp-runtime-design.md), KNX2 = KNX1 + a dtype word per weight block
(docs/int8-quantization-design.md), KNX3 graph with per-op input value ids and a channels-last input
shape (docs/graph-runtime-design.md, tools/knx3.py:242-276 writes the same layout). The reader is
kernix_b200/csrc/knx_load.c. The int8 weight quantiser restates tools/knx_quant.py:18-25: symmetric
per output column, scale = max|w| / 127 (1 when the column is all zero), q = clip(rint(w / scale), +-127),
computed in float64.
"""
import struct

import numpy as np

OP = dict(LINEAR=0, ACT=1, LAYERNORM=2, SOFTMAX=3, LSTM=4, GRU=5, RNN=6, CONV=7, POOL=8, GLOBAL_POOL=9, RESHAPE=10,
          PERMUTE=11, BINARY=12, CONCAT=13, EMBEDDING=14, AFFINE=15, ADD_CONST=16, ATTENTION=17, SELECT=18, PAD=19,
          UPSAMPLE=20)
ACT = dict(relu=0, gelu=1, silu=2, sigmoid=3, tanh=4, leaky_relu=5, elu=6, selu=7, softplus=8, relu6=9,
           hard_sigmoid=10, hard_swish=11, gelu_tanh=12, exp=13, mish=14, softsign=15)
BIN = dict(add=0, sub=1, mul=2, div=3, max=4, min=5)
DT = dict(f32=0, i8_col=1, i8_row=2)


def _f32(a):
    return np.ascontiguousarray(a, dtype="<f4").tobytes()


def quantize_int8(w, axis="col"):
    """Symmetric int8 of w (in x out). axis "col": one scale per output column. Returns (scale f32, q int8)."""
    w = np.asarray(w, np.float64)
    m = np.abs(w).max(axis=0 if axis == "col" else 1)
    scale = np.where(m > 0, m / 127.0, 1.0).astype(np.float32)
    s = scale[None, :] if axis == "col" else scale[:, None]
    q = np.clip(np.rint(w / s), -127, 127).astype(np.int8)
    return scale, q


def weight_block(w, mode, with_dtype):
    """Bytes of one weight block. with_dtype False = KNX1 (float32 values only)."""
    if not with_dtype:
        if mode != "f32":
            raise ValueError("KNX1 holds float32 weights only")
        return _f32(w)
    head = struct.pack("<I", DT[mode])
    if mode == "f32":
        return head + _f32(w)
    scale, q = quantize_int8(w, "col" if mode == "i8_col" else "row")
    return head + _f32(scale) + np.ascontiguousarray(q).tobytes()


class Sequential:
    """KNX1 (float) / KNX2 (int8 Linear weights) sequential model: linear, act, layernorm, softmax."""

    def __init__(self, int8=False):
        self.int8 = int8
        self.ops = []

    def linear(self, w, b=None):
        w = np.asarray(w)
        op = struct.pack("<4I", OP["LINEAR"], w.shape[0], w.shape[1], b is not None)
        op += weight_block(w, "i8_col" if self.int8 else "f32", self.int8)
        if b is not None:
            op += _f32(b)
        self.ops.append(op)
        return self

    def act(self, name):
        if ACT[name] > ACT["tanh"]:
            raise ValueError("KNX1/KNX2 activations are relu, gelu, silu, sigmoid, tanh")
        self.ops.append(struct.pack("<2I", OP["ACT"], ACT[name]))
        return self

    def layernorm(self, cols, gamma=None, beta=None, eps=1e-5):
        op = struct.pack("<3If", OP["LAYERNORM"], cols, gamma is not None, eps)
        if gamma is not None:
            op += _f32(gamma) + _f32(beta if beta is not None else np.zeros(cols))
        self.ops.append(op)
        return self

    def softmax(self):
        self.ops.append(struct.pack("<I", OP["SOFTMAX"]))
        return self

    def tobytes(self):
        return (b"KNX2" if self.int8 else b"KNX1") + struct.pack("<I", len(self.ops)) + b"".join(self.ops)

    def write(self, path):
        with open(path, "wb") as f:
            f.write(self.tobytes())


class Graph:
    """KNX3 graph. Value ids: 0 = model input, k + 1 = output of op k. Shapes are per sample, channels-last."""

    def __init__(self, in_shape, layout=0, int8=False):
        self.layout = layout
        self.int8 = int8
        self.shapes = [tuple(int(v) for v in in_shape)]
        self.ops = []

    def _add(self, kind, inp, u32, blobs, shape):
        rec = struct.pack("<2I", OP[kind], len(inp)) + struct.pack(f"<{len(inp)}I", *inp)
        rec += struct.pack(f"<{len(u32)}I", *[int(v) for v in u32])
        for b in blobs:
            if b[0] == "w":
                rec += weight_block(b[1], b[2] if self.int8 else "f32", True)
            elif b[0] == "fl":
                rec += struct.pack("<f", b[1])
            else:
                rec += _f32(b[1])
        self.ops.append(rec)
        self.shapes.append(tuple(int(v) for v in shape))
        return len(self.ops)

    def shape(self, v):
        return self.shapes[v]

    def act(self, x, name, alpha=0.0):
        return self._add("ACT", [x], [ACT[name]], [("fl", alpha)], self.shape(x))

    def linear(self, x, w, b=None):
        s = self.shape(x)
        blobs = [("w", w, "i8_col")] + ([("f", b)] if b is not None else [])
        return self._add("LINEAR", [x], [w.shape[0], w.shape[1], b is not None], blobs, s[:-1] + (w.shape[1],))

    def layernorm(self, x, gamma, beta, eps=1e-5):
        c = self.shape(x)[-1]
        return self._add("LAYERNORM", [x], [c, 1], [("fl", eps), ("f", gamma), ("f", beta)], self.shape(x))

    def softmax(self, x):
        return self._add("SOFTMAX", [x], [], [], self.shape(x))

    def conv(self, x, w, b, k, stride=(1, 1), dil=(1, 1), pads=(0, 0, 0, 0), groups=1):
        """w: (kh*kw*cin/groups) x cout, rows ordered (ky, kx, ci). pads: top, bottom, left, right."""
        s = self.shape(x)
        H, W = s[0], (s[1] if len(s) == 3 else 1)
        oh = (H + pads[0] + pads[1] - dil[0] * (k[0] - 1) - 1) // stride[0] + 1
        ow = (W + pads[2] + pads[3] - dil[1] * (k[1] - 1) - 1) // stride[1] + 1
        out = (oh, ow, w.shape[1]) if len(s) == 3 else (oh, w.shape[1])
        blobs = [("w", w, "i8_col")] + ([("f", b)] if b is not None else [])
        return self._add("CONV", [x], [s[-1], w.shape[1], k[0], k[1], *stride, *dil, *pads, groups, b is not None], blobs, out)

    def pool(self, x, kind, k, stride, pads=(0, 0, 0, 0), count_pad=False):
        s = self.shape(x)
        H, W = s[0], (s[1] if len(s) == 3 else 1)
        oh = (H + pads[0] + pads[1] - k[0]) // stride[0] + 1
        ow = (W + pads[2] + pads[3] - k[1]) // stride[1] + 1
        out = (oh, ow, s[-1]) if len(s) == 3 else (oh, s[-1])
        return self._add("POOL", [x], [{"max": 0, "avg": 1}[kind], *k, *stride, *pads, int(count_pad)], [], out)

    def global_pool(self, x, kind):
        return self._add("GLOBAL_POOL", [x], [{"max": 0, "avg": 1}[kind]], [], (self.shape(x)[-1],))

    def reshape(self, x, shape):
        return self._add("RESHAPE", [x], [len(shape), *shape], [], shape)

    def permute(self, x, perm):
        s = self.shape(x)
        return self._add("PERMUTE", [x], [len(perm), *perm], [], tuple(s[p] for p in perm))

    def binary(self, a, b, op):
        sa, sb = self.shape(a), self.shape(b)
        big = sa if np.prod(sa) >= np.prod(sb) else sb
        return self._add("BINARY", [a, b], [BIN[op]], [], big[:-1] + (max(sa[-1], sb[-1]),))

    def concat(self, xs, axis):
        s0 = list(self.shape(xs[0]))
        ax = 0 if axis == 0 else len(s0) - 1
        s0[ax] = sum(self.shape(v)[ax] for v in xs)
        return self._add("CONCAT", xs, [axis], [], s0)

    def rnn(self, x, kind, units, weights, act="tanh", ret_seq=False, merge="concat"):
        """LSTM / GRU / RNN over the sequence axis of x (T x in). weights: one (W in x gu, U units x gu, bias) per
        direction (two = bidirectional), gu = gates * units with gates 4 (LSTM: i, f, g, o), 3 (GRU: z, r, h~)
        or 1; bias has gu values (GRU: 2 * gu, input then recurrent). merge of two directions: concat, sum, mul,
        ave. In int8 mode the recurrent weights are written I8_COL (kept int8) and the input weights I8_COL too
        (dequantised at load)."""
        T, cin = self.shape(x)[-2], self.shape(x)[-1]
        dirs = len(weights)
        mg = dict(concat=0, sum=1, mul=2, ave=3)[merge]
        blobs = []
        for w, u, b in weights:
            blobs += [("w", w, "i8_col"), ("w", u, "i8_col"), ("f", b)]
        uo = 2 * units if dirs == 2 and mg == 0 else units
        return self._add(kind.upper(), [x], [cin, units, ACT[act], int(ret_seq), dirs, mg], blobs,
                         (T, uo) if ret_seq else (uo,))

    def embedding(self, x, table):
        return self._add("EMBEDDING", [x], [table.shape[0], table.shape[1]], [("w", table, "i8_row")],
                         self.shape(x) + (table.shape[1],))

    def affine(self, x, scale, shift):
        return self._add("AFFINE", [x], [self.shape(x)[-1]], [("f", scale), ("f", shift)], self.shape(x))

    def add_const(self, x, c):
        return self._add("ADD_CONST", [x], [c.size], [("f", c)], self.shape(x))

    def attention(self, q, heads, wq, bq, wk, bk, wv, bv, wo, bo, v=None, k=None, causal=False):
        inp = [q] + ([v] if v is not None else []) + ([k] if k is not None else [])
        dk, dv = wq.shape[1] // heads, wv.shape[1] // heads
        cv = self.shape(v if v is not None else q)[-1]
        ck = self.shape(k if k is not None else (v if v is not None else q))[-1]
        hb = bq is not None
        blobs = []
        for w, b in ((wq, bq), (wk, bk), (wv, bv), (wo, bo)):
            blobs.append(("w", w, "i8_col"))
            if hb:
                blobs.append(("f", b))
        return self._add("ATTENTION", inp, [heads, dk, dv, int(causal), wq.shape[0], cv, ck, wo.shape[1], int(hb)], blobs,
                         self.shape(q)[:-1] + (wo.shape[1],))

    def select(self, x, axis, start, length, squeeze=False):
        s = list(self.shape(x))
        ax = 0 if axis == 0 else len(s) - 1
        s[ax] = length
        if squeeze and length == 1 and len(s) > 1:
            del s[ax]
        return self._add("SELECT", [x], [axis, start, length, int(squeeze)], [], s)

    def pad(self, x, pads):
        s = self.shape(x)
        out = (s[0] + pads[0] + pads[1],) + ((s[1] + pads[2] + pads[3],) if len(s) == 3 else ()) + (s[-1],)
        return self._add("PAD", [x], list(pads), [], out)

    def upsample(self, x, sh, sw=1):
        s = self.shape(x)
        out = (s[0] * sh,) + ((s[1] * sw,) if len(s) == 3 else ()) + (s[-1],)
        return self._add("UPSAMPLE", [x], [sh, sw], [], out)

    def tobytes(self):
        s = self.shapes[0]
        head = b"KNX3" + struct.pack(f"<{3 + len(s)}I", len(self.ops), self.layout, len(s), *s)
        return head + b"".join(self.ops)

    def write(self, path):
        with open(path, "wb") as f:
            f.write(self.tobytes())
