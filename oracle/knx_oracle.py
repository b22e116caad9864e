"""CPU oracle for the KERNIX `.knx` forward path: a numpy restatement of the reference runtime.

TEST INFRASTRUCTURE ONLY. Nothing in kernix_b200/ imports this module; only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline leg use it, always as the checker.

What it restates (file:line in the KERNIX reference, include/kernix_model.h unless noted):
  * the .knx v1/v2/v3 reader: header :1461-1487, op records kernix_parse_op :1082-1243,
    weight blocks kernix_read_weight :434-460 (F32 / I8_COL / I8_ROW), legacy v1/v2 input shape
    :1516-1526, shape inference kernix_infer :1266-1394;
  * every graph op's arithmetic, in float32 and in the reference's operation order:
    activations kernix_act_chunk :468-517, dense + bias + act kernix_dense/kernix_bias_act :528-550,
    int8 kernix_qmatmul :99-182, conv kernix_conv_run :711-771, pooling :773-830, permute :833-862,
    binary :877-906, concat :908-930, select :932-947, pad :949-966, upsample :968-983, embedding
    :986-1000, attention kernix_attention_run :1005-1048, layer_norm / softmax include/kernix.h:652-677,
    affine / add_const kernix_step_run :1882-1895.
  * The int8 LINEAR uses the reference's int8 semantics everywhere: per-row dynamic int8 activations,
    int32 accumulators (exact, computed in float64 BLAS: |acc| < 2^53), dequant ((float)acc*sx)*scale + bias
    with two roundings. The reference itself runs this kernel for chunks of <= 2 rows
    (KERNIX_INT8_MAX_ROWS, :50, :1854-1857), which includes config 2 at its default workspace limit.

Float32 sums (sgemm, softmax/LN sums) follow numpy's/OpenBLAS's summation order, so agreement with the
reference is to rounding (tests pin it at 1e-5 relative); integer work (int8 quantisation and
accumulators) is bit-exact. LSTM/GRU/RNN steps follow kernix_rnn_dir / kernix_rnn_run (:560-648).
"""
import struct

import numpy as np

F32 = np.float32
FLT_MAX = np.finfo(np.float32).max

OP_NAMES = ["LINEAR", "ACT", "LAYERNORM", "SOFTMAX", "LSTM", "GRU", "RNN", "CONV", "POOL", "GLOBAL_POOL",
            "RESHAPE", "PERMUTE", "BINARY", "CONCAT", "EMBEDDING", "AFFINE", "ADD_CONST", "ATTENTION",
            "SELECT", "PAD", "UPSAMPLE"]
OP = {n: i for i, n in enumerate(OP_NAMES)}
ACT_NONE = -1
ACT_NAMES = ["relu", "gelu", "silu", "sigmoid", "tanh", "leaky_relu", "elu", "selu", "softplus", "relu6",
             "hard_sigmoid", "hard_swish", "gelu_tanh", "exp", "mish", "softsign"]
ACT_LAST = len(ACT_NAMES) - 1
DT_F32, DT_I8_COL, DT_I8_ROW = 0, 1, 2
MAX_DIMS = 4
MAX_GEOM = 65536
INT8_MAX_K = 131072
INT_MAX = 2**31 - 1


class KnxError(ValueError):
    pass


# --------------------------------------------------------------------------------------------- reader
class _Reader:
    def __init__(self, data):
        self.b = memoryview(data)
        self.p = 0

    def left(self):
        return len(self.b) - self.p

    def u32(self, n=1):
        if self.left() < 4 * n:
            raise KnxError("file shorter than declared")
        v = struct.unpack_from(f"<{n}I", self.b, self.p)
        self.p += 4 * n
        return v if n > 1 else v[0]

    def f32(self, n):
        if self.left() < 4 * n:
            raise KnxError("file shorter than declared")
        a = np.frombuffer(self.b, "<f4", n, self.p).astype(F32)
        self.p += 4 * n
        return a

    def i8(self, n):
        if self.left() < n:
            raise KnxError("file shorter than declared")
        a = np.frombuffer(self.b, np.int8, n, self.p).copy()
        self.p += n
        return a


def _weight(r, ver, k, n, keep_int8):
    """kernix_load_weight/kernix_read_weight (:434-460, :1059-1077). Returns ("f32", W k x n) or
    ("i8", q k x n int8, scale[n]) for an I8_COL block kept as int8."""
    if k < 1 or n < 1 or k * n > INT_MAX:
        raise KnxError("weight size out of range")
    dt = r.u32() if ver >= 2 else DT_F32
    if dt > DT_I8_ROW:
        raise KnxError("unknown weight dtype")
    if dt == DT_F32:
        return ("f32", r.f32(k * n).reshape(k, n))
    if keep_int8 and dt == DT_I8_COL and k > INT8_MAX_K:
        raise KnxError("int8 weight input size out of range")
    ns = n if dt == DT_I8_COL else k
    sc = r.f32(ns)
    q = r.i8(k * n).reshape(k, n)
    if not np.all((sc > 0) & (sc <= FLT_MAX)):
        raise KnxError("int8 scale <= 0 or not finite")
    if keep_int8 and dt == DT_I8_COL:
        return ("i8", q, sc)
    w = q.astype(F32) * (sc[None, :] if dt == DT_I8_COL else sc[:, None])
    return ("f32", w.astype(F32))


def _geom_ok(v, lo):
    return lo <= v <= MAX_GEOM


def _parse_op(r, ver, kind):
    """kernix_parse_op (:1082-1243): arguments and weights of one record."""
    s = dict(kind=kind, act=ACT_NONE, alpha=0.0)
    if kind == OP["LINEAR"]:
        i, o, hb = r.u32(3)
        if i < 1 or o < 1 or i > INT_MAX or o > INT_MAX or hb > 1:
            raise KnxError("Linear size out of range")
        s.update(inp_c=i, out=o, w=_weight(r, ver, i, o, True), bias=r.f32(o) if hb else None)
    elif kind == OP["ACT"]:
        a = r.u32()
        alpha = float(r.f32(1)[0]) if ver >= 3 else 0.0
        if a > (ACT_LAST if ver >= 3 else 4) or not np.isfinite(alpha):
            raise KnxError("unknown activation")
        s.update(act=a, alpha=alpha)
    elif kind == OP["LAYERNORM"]:
        c, aff = r.u32(2)
        eps = float(r.f32(1)[0])
        if c < 1 or c > INT_MAX or aff > 1 or not (eps >= 0) or np.isinf(eps):
            raise KnxError("LayerNorm value out of range")
        s.update(inp_c=c, out=c, eps=F32(eps), gamma=r.f32(c) if aff else None, beta=r.f32(c) if aff else None)
    elif kind == OP["SOFTMAX"]:
        pass
    elif kind in (OP["LSTM"], OP["GRU"], OP["RNN"]):
        if ver < 3:
            a = list(r.u32(5))
            if a[2] not in (0, 4) or a[0] < 1 or a[1] < 1 or a[1] > 4096 or a[3] > 1 or a[4] < 1:
                raise KnxError("LSTM value out of range")
            seq, dirs, merge = a[4], 1, 0
        else:
            a = list(r.u32(6))
            if a[0] < 1 or a[1] < 1 or a[1] > 4096 or a[2] > ACT_LAST or a[3] > 1 or not 1 <= a[4] <= 2 or a[5] > 3:
                raise KnxError("RNN value out of range")
            seq, dirs, merge = None, a[4], a[5]
        g = {OP["LSTM"]: 4, OP["GRU"]: 3, OP["RNN"]: 1}[kind]
        gu = g * a[1]
        nb = 2 * gu if kind == OP["GRU"] else gu
        s["rnn"] = [(_weight(r, ver, a[0], gu, False), _weight(r, ver, a[1], gu, True), r.f32(nb)) for _ in range(dirs)]
        s.update(inp_c=a[0], out=a[1], act=a[2], ret_seq=a[3], dirs=dirs, merge=merge, seq=seq)
    elif kind == OP["CONV"]:
        a = r.u32(14)
        ok = a[0] >= 1 and a[1] >= 1 and all(_geom_ok(a[j], 1) for j in range(2, 8)) and \
            all(_geom_ok(a[j], 0) for j in range(8, 12)) and a[12] >= 1 and a[0] % a[12] == 0 and a[1] % a[12] == 0 and a[13] <= 1
        if not ok:
            raise KnxError("conv value out of range")
        s.update(inp_c=a[0], out=a[1], kh=a[2], kw=a[3], sh=a[4], sw=a[5], dh=a[6], dw=a[7],
                 pt=a[8], pb=a[9], pl=a[10], pr=a[11], groups=a[12])
        s["w"] = _weight(r, ver, a[2] * a[3] * (a[0] // a[12]), a[1], False)
        s["bias"] = r.f32(a[1]) if a[13] else None
    elif kind == OP["POOL"]:
        a = r.u32(10)
        if a[0] > 1 or not all(_geom_ok(a[j], 1) for j in range(1, 5)) or a[5] >= a[1] or a[6] >= a[1] or \
                a[7] >= a[2] or a[8] >= a[2] or a[9] > 1:
            raise KnxError("pooling value out of range")
        s.update(ptype=a[0], kh=a[1], kw=a[2], sh=a[3], sw=a[4], pt=a[5], pb=a[6], pl=a[7], pr=a[8], count_pad=a[9],
                 dh=1, dw=1)
    elif kind == OP["GLOBAL_POOL"]:
        a = r.u32()
        if a > 1:
            raise KnxError("pooling value out of range")
        s.update(ptype=a)
    elif kind in (OP["RESHAPE"], OP["PERMUTE"]):
        nd = r.u32()
        if nd < 1 or nd > MAX_DIMS:
            raise KnxError("axis count out of range")
        d = [r.u32() for _ in range(nd)]
        if kind == OP["RESHAPE"]:
            if any(v < 1 or v > INT_MAX for v in d):
                raise KnxError("Reshape shape out of range")
            s.update(nd=nd, d=d)
        else:
            if sorted(d) != list(range(nd)):
                raise KnxError("bad Permute order")
            s.update(nd=nd, perm=d)
    elif kind == OP["BINARY"]:
        a = r.u32()
        if a > 5:
            raise KnxError("unknown binary op")
        s.update(bop=a)
    elif kind == OP["CONCAT"]:
        a = r.u32()
        if a > 1:
            raise KnxError("Concatenate axis out of range")
        s.update(axis=a)
    elif kind == OP["EMBEDDING"]:
        v, d = r.u32(2)
        s.update(inp_c=v, out=d, w=_weight(r, ver, v, d, False))
    elif kind == OP["AFFINE"]:
        c = r.u32()
        if c < 1 or c > INT_MAX:
            raise KnxError("Affine size out of range")
        s.update(inp_c=c, out=c, gamma=r.f32(c), beta=r.f32(c))
    elif kind == OP["ADD_CONST"]:
        c = r.u32()
        if c < 1 or c > INT_MAX:
            raise KnxError("constant size out of range")
        s.update(inp_c=c, cst=r.f32(c))
    elif kind == OP["ATTENTION"]:
        a = r.u32(9)
        if not (1 <= a[0] <= 4096 and 1 <= a[1] <= 65536 and 1 <= a[2] <= 65536 and a[3] <= 1 and a[8] <= 1 and
                all(a[j] >= 1 for j in range(4, 8))):
            raise KnxError("attention value out of range")
        H, dk, dv, causal, cq, cv, ck, co, hb = a
        s.update(heads=H, dk=dk, dv=dv, causal=causal, inp_c=cq, out=co)
        s["wq"] = _weight(r, ver, cq, H * dk, False)
        s["bq"] = r.f32(H * dk) if hb else None
        s["wk"] = _weight(r, ver, ck, H * dk, False)
        s["bk"] = r.f32(H * dk) if hb else None
        s["wv"] = _weight(r, ver, cv, H * dv, False)
        s["bv"] = r.f32(H * dv) if hb else None
        s["wo"] = _weight(r, ver, H * dv, co, False)
        s["bo"] = r.f32(co) if hb else None
    elif kind == OP["SELECT"]:
        a = r.u32(4)
        if a[0] > 1 or a[2] < 1 or a[3] > 1:
            raise KnxError("Select value out of range")
        s.update(axis=a[0], start=a[1], len=a[2], squeeze=a[3])
    elif kind == OP["PAD"]:
        a = r.u32(4)
        if not all(_geom_ok(v, 0) for v in a):
            raise KnxError("padding value out of range")
        s.update(pt=a[0], pb=a[1], pl=a[2], pr=a[3])
    elif kind == OP["UPSAMPLE"]:
        a = r.u32(2)
        if not all(_geom_ok(v, 1) for v in a):
            raise KnxError("UpSampling value out of range")
        s.update(sh=a[0], sw=a[1])
    else:
        raise KnxError("unknown op")
    return s


def _val(d):
    d = [int(v) for v in d]
    if not 1 <= len(d) <= MAX_DIMS or min(d) < 1:
        raise KnxError("shape out of range")
    r = int(np.prod(d[:-1])) if len(d) > 1 else 1
    if r * d[-1] > INT_MAX:
        raise KnxError("shape out of range")
    return dict(nd=len(d), d=d, r=r, c=d[-1])


def _hw(v):
    return v["d"][0], (v["d"][1] if v["nd"] == 3 else 1)


def _infer(s, vals):
    """kernix_infer (:1266-1394): output shape of one step."""
    x = vals[s["inp"][0]]
    d = list(x["d"])
    k = s["kind"]
    if k == OP["LINEAR"]:
        if x["c"] != s["inp_c"]:
            raise KnxError("Linear input size differs from previous output")
        d[-1] = s["out"]
    elif k in (OP["LAYERNORM"], OP["AFFINE"]):
        if x["c"] != s["inp_c"]:
            raise KnxError("size differs from previous output")
    elif k in (OP["CONV"], OP["POOL"], OP["PAD"], OP["UPSAMPLE"]):
        if x["nd"] not in (2, 3):
            raise KnxError("conv/pool input must be TxC or HxWxC")
        if x["nd"] == 2 and (s.get("kw", 1) != 1 or s.get("sw", 1) != 1 or s.get("dw", 1) != 1 or s.get("pl", 0) or s.get("pr", 0)):
            raise KnxError("2-D kernel on 1-D input")
        if k == OP["CONV"] and x["c"] != s["inp_c"]:
            raise KnxError("conv input channels differ")
        H, W = _hw(x)
        if k == OP["PAD"]:
            Ho, Wo = H + s["pt"] + s["pb"], W + s["pl"] + s["pr"]
        elif k == OP["UPSAMPLE"]:
            Ho, Wo = H * s["sh"], W * s["sw"]
        else:
            nh = H + s["pt"] + s["pb"] - (s["dh"] * (s["kh"] - 1) + 1)
            nw = W + s["pl"] + s["pr"] - (s["dw"] * (s["kw"] - 1) + 1)
            if nh < 0 or nw < 0:
                raise KnxError("conv/pool output size <= 0")
            Ho, Wo = nh // s["sh"] + 1, nw // s["sw"] + 1
        d[0] = Ho
        if x["nd"] == 3:
            d[1] = Wo
        if k == OP["CONV"]:
            d[-1] = s["out"]
    elif k == OP["GLOBAL_POOL"]:
        d = [x["c"]]
    elif k == OP["RESHAPE"]:
        if int(np.prod(s["d"])) != x["r"] * x["c"]:
            raise KnxError("Reshape size differs")
        d = list(s["d"])
    elif k == OP["PERMUTE"]:
        if s["nd"] != x["nd"]:
            raise KnxError("Permute axis count differs")
        d = [x["d"][p] for p in s["perm"]]
    elif k == OP["BINARY"]:
        y = vals[s["inp"][1]]
        R, C = max(x["r"], y["r"]), max(x["c"], y["c"])
        big = x if x["r"] * x["c"] >= y["r"] * y["c"] else y
        if x["r"] not in (R, 1) or y["r"] not in (R, 1) or x["c"] not in (C, 1) or y["c"] not in (C, 1) or big["r"] != R:
            raise KnxError("binary input shapes do not match")
        d = list(big["d"])
        d[-1] = C
    elif k == OP["CONCAT"]:
        ax = 0 if s["axis"] == 0 else x["nd"] - 1
        tot = 0
        for i in s["inp"]:
            v = vals[i]
            if v["nd"] != x["nd"] or any(v["d"][j] != x["d"][j] for j in range(x["nd"]) if j != ax):
                raise KnxError("Concatenate shapes do not match")
            tot += v["d"][ax]
        d[ax] = tot
    elif k == OP["EMBEDDING"]:
        if x["nd"] >= MAX_DIMS:
            raise KnxError("axis count out of range")
        d = d + [s["out"]]
    elif k == OP["ADD_CONST"]:
        if x["r"] * x["c"] != s["inp_c"]:
            raise KnxError("constant size differs")
    elif k == OP["ATTENTION"]:
        n = len(s["inp"])
        v = vals[s["inp"][1 if n > 1 else 0]]
        kk = vals[s["inp"][2 if n > 2 else (1 if n > 1 else 0)]]
        if x["c"] != s["wq"][1].shape[0] or v["c"] != s["wv"][1].shape[0] or kk["c"] != s["wk"][1].shape[0] or kk["r"] != v["r"]:
            raise KnxError("attention input size differs from weights")
        d[-1] = s["out"]
    elif k == OP["SELECT"]:
        ax = 0 if s["axis"] == 0 else x["nd"] - 1
        if s["start"] + s["len"] > d[ax]:
            raise KnxError("Select range outside input")
        d[ax] = s["len"]
        if s["squeeze"] and s["len"] == 1 and len(d) > 1:
            del d[ax]
    elif k in (OP["LSTM"], OP["GRU"], OP["RNN"]):
        if x["c"] != s["inp_c"]:
            raise KnxError("RNN input size differs")
        uo = 2 * s["out"] if s["dirs"] == 2 and s["merge"] == 0 else s["out"]
        d = [x["r"], uo] if s["ret_seq"] else [uo]
    return _val(d)


def load(path_or_bytes):
    """Parse a .knx file (kernix_model_load :1448-1601 minus buffer planning). Returns a model dict with
    'steps' (each with 'inp' value ids; value 0 = model input, k+1 = step k), 'vals' (per-sample shapes),
    'layout', 'in_shape', 'out_shape', 'in_dim', 'out_dim', 'seq_len', 'n_fused_steps' (steps after
    the reference's ACT-into-LINEAR/CONV fusion :1530-1555)."""
    data = path_or_bytes if isinstance(path_or_bytes, (bytes, bytearray)) else open(path_or_bytes, "rb").read()
    r = _Reader(data)
    magic = bytes(r.b[0:4]) if r.left() >= 4 else b""
    r.u32()
    n_ops = r.u32()
    ver = {b"KNX1": 1, b"KNX2": 2, b"KNX3": 3}.get(magic, 0)
    if ver == 0:
        raise KnxError("not a KNX1/KNX2/KNX3 file")
    if n_ops < 1 or n_ops > 1024:
        raise KnxError("op count out of range")
    layout = 0
    vals = [None]
    if ver == 3:
        layout, nd = r.u32(2)
        if layout > 1 or nd < 1 or nd > MAX_DIMS:
            raise KnxError("input shape out of range")
        vals[0] = _val([r.u32() for _ in range(nd)])
    steps = []
    for i in range(n_ops):
        kind = r.u32()
        if kind > (len(OP_NAMES) - 1 if ver == 3 else OP["LSTM"]):
            raise KnxError("unknown op")
        if ver == 3:
            n_in = r.u32()
            lo = 2 if kind in (OP["BINARY"], OP["CONCAT"]) else 1
            hi = 2 if kind == OP["BINARY"] else 8 if kind == OP["CONCAT"] else 3 if kind == OP["ATTENTION"] else 1
            if not lo <= n_in <= hi:
                raise KnxError("op input count out of range")
            inp = [r.u32() for _ in range(n_in)]
            if any(v > i for v in inp):
                raise KnxError("op input refers to a later op")
        else:
            inp = [i]
        s = _parse_op(r, ver, kind)
        s["inp"] = inp
        steps.append(s)
    if r.left() != 0:
        raise KnxError("data left after the last op")
    if ver < 3:
        in_dim, seq = 0, 0
        for s in steps:
            if in_dim == 0 and s["kind"] in (OP["LINEAR"], OP["LAYERNORM"], OP["LSTM"]):
                in_dim = s["inp_c"]
            if seq == 0 and s["kind"] == OP["LSTM"]:
                seq = s["seq"]
        if in_dim == 0:
            raise KnxError("no Linear or LayerNorm to give the input size")
        vals[0] = _val([seq, in_dim] if seq else [in_dim])
    for s in steps:
        vals.append(_infer(s, vals))
    # ACT fusion (:1530-1555): an ACT whose input is a LINEAR/CONV output read only by it merges into that step.
    # fused_map[v] = value id of original value v in the fused graph (the runtime's numbering).
    cons = [0] * (n_ops + 1)
    for s in steps:
        for i in s["inp"]:
            cons[i] += 1
    cons[n_ops] += 1
    fmap = [0] * (n_ops + 1)
    kept = []  # (kind, act) of fused steps
    for i, s in enumerate(steps):
        inp = [fmap[v] for v in s["inp"]]
        if s["kind"] == OP["ACT"] and inp[0] > 0 and cons[s["inp"][0]] == 1:
            pk, pa = kept[inp[0] - 1]
            if pk in (OP["LINEAR"], OP["CONV"]) and pa == ACT_NONE:
                kept[inp[0] - 1] = (pk, s["act"])
                fmap[i + 1] = inp[0]
                continue
        kept.append((s["kind"], s["act"]))
        fmap[i + 1] = len(kept)
    fused = n_ops - len(kept)
    vin, vout = vals[0], vals[n_ops]
    return dict(ver=ver, layout=layout, steps=steps, vals=vals, in_shape=vin["d"], out_shape=vout["d"],
                in_dim=vin["c"], seq_len=vin["r"], out_dim=vout["r"] * vout["c"], n_fused_steps=n_ops - fused,
                fused_map=fmap, fused_steps=kept)


# ------------------------------------------------------------------------------------------ arithmetic
def act(x, a, alpha=0.0):
    """kernix_act_chunk (:468-517), float32, same operation order."""
    x = x.astype(F32, copy=True)
    one = F32(1)
    with np.errstate(all="ignore"):
        if a == ACT_NONE:
            return x
        if a == 0:  # vDSP_vthr(x, 0): x < 0 ? 0 : x
            return np.where(x < 0, F32(0), x).astype(F32)
        if a == 4:
            return np.tanh(x).astype(F32)
        if a == 3:
            return (one / (np.exp(-x) + one)).astype(F32)
        if a == 2:
            t = (one / (np.exp(-x) + one)).astype(F32)
            return (x * t).astype(F32)
        if a == 1:
            z = x * F32(0.70710678)
            t = np.exp(-(z * z)).astype(F32)
            z = np.abs(x) * F32(0.70710678)
            k = one / (one + F32(0.3275911) * z)
            p = k * (F32(0.254829592) + k * (F32(-0.284496736) + k * (F32(1.421413741)
                                                                       + k * (F32(-1.453152027) + k * F32(1.061405429)))))
            e = one - p * t
            return (F32(0.5) * x * (one + np.where(x < 0, -e, e))).astype(F32)
        if a == 5:
            return np.where(x < 0, F32(alpha) * x, x).astype(F32)
        if a == 6:
            return np.where(x < 0, F32(alpha) * np.expm1(x), x).astype(F32)
        if a == 7:
            return (F32(1.0507009873554805) * np.where(x < 0, F32(1.6732632423543772) * np.expm1(x), x)).astype(F32)
        if a == 8:
            return np.where(x > 20, x, np.log1p(np.exp(x))).astype(F32)
        relu6 = lambda v: np.where(v < 0, F32(0), np.where(v > 6, F32(6), v)).astype(F32)  # noqa: E731
        if a == 9:
            return relu6(x)
        if a == 10:
            return (relu6(x + F32(3)) / F32(6)).astype(F32)
        if a == 11:
            return ((x * relu6(x + F32(3))) / F32(6)).astype(F32)
        if a == 12:
            inner = F32(0.7978845608028654) * (x + F32(0.044715) * x * x * x)
            return (F32(0.5) * x * (one + np.tanh(inner))).astype(F32)
        if a == 13:
            return np.exp(x).astype(F32)
        if a == 14:
            sp = np.where(x > 20, x, np.log1p(np.exp(x))).astype(F32)
            return (x * np.tanh(sp)).astype(F32)
        if a == 15:
            return (x / (one + np.abs(x))).astype(F32)
    raise KnxError(f"unknown activation {a}")


def quantize_rows(x):
    """Per-row dynamic int8 quantisation of kernix_qmatmul (:115-142). Returns (xq int8, sx float32, bad)
    where bad marks rows whose max |x| is NaN or infinite (those output rows are all NaN)."""
    x = np.asarray(x, F32)
    with np.errstate(all="ignore"):
        m = np.max(np.abs(x), axis=1) if x.shape[1] else np.zeros(x.shape[0], F32)
        bad = ~(m <= FLT_MAX)
        sx = np.where(m > 0, m / F32(127), F32(1)).astype(F32)
        inv = (F32(1) / sx).astype(F32)
        v = np.rint((x * inv[:, None]).astype(F32))
        v = np.clip(v, -127, 127)
        v = np.where(np.isnan(v), 0, v)
    return v.astype(np.int8), sx, bad


def int8_acc(xq, q):
    """int32 accumulators sum_t xq[r,t] * q[t,c], exact (float64 BLAS, every partial sum < 2^53)."""
    return (xq.astype(np.float64) @ q.astype(np.float64)).astype(np.int64).astype(np.int32)


def qlinear(x, q, scale, bias):
    """kernix_qmatmul (:99-182) with accumulate = 0: ((float)acc*sx)*scale + bias, NaN rows for NaN/Inf inputs."""
    xq, sx, bad = quantize_rows(x)
    acc = int8_acc(xq, q)
    with np.errstate(all="ignore"):
        y = (acc.astype(F32) * sx[:, None]).astype(F32)
        y = (y * scale[None, :].astype(F32)).astype(F32)
        y = (y + (bias[None, :] if bias is not None else F32(0))).astype(F32)
    y[bad] = np.nan
    return y


def dense(x, w, b, a, alpha):
    """kernix_dense (:544-550): sgemm, then in-place bias add and activation."""
    y = np.matmul(x.astype(F32), w.astype(F32)).astype(F32)
    if b is not None:
        y = (y + b[None, :]).astype(F32)
    return act(y, a, alpha)


def softmax_rows(x):
    """floats_softmax_into (include/kernix.h:652-657)."""
    with np.errstate(all="ignore"):
        m = np.max(x, axis=1, keepdims=True) if x.shape[1] else x
        o = np.exp((x - m).astype(F32)).astype(F32)
        s = np.sum(o, axis=1, keepdims=True, dtype=F32)
        return (o * (F32(1) / s)).astype(F32)


def layer_norm_rows(x, g, b, eps):
    """kernix_layer_norm_rows_into (include/kernix.h:667-677): two-pass mean, biased variance."""
    cols = x.shape[1]
    mean = (np.sum(x, axis=1, keepdims=True, dtype=F32) / F32(cols)).astype(F32)
    o = (x - mean).astype(F32)
    ss = np.sum(o * o, axis=1, keepdims=True, dtype=F32)
    rstd = (F32(1) / np.sqrt((ss / F32(cols) + F32(eps)).astype(F32))).astype(F32)
    o = (o * rstd).astype(F32)
    if g is not None and b is not None:
        o = (o * g[None, :] + b[None, :]).astype(F32)
    elif g is not None:
        o = (o * g[None, :]).astype(F32)
    elif b is not None:
        o = (o + b[None, :]).astype(F32)
    return o


def _wf(w):
    """float weights of a parsed block (int8 kept blocks dequantised as kernix_qweight_unpack :91-95)."""
    if w[0] == "f32":
        return w[1]
    return (w[1].astype(F32) * w[2][None, :]).astype(F32)


def conv(s, vi, vo, x2):
    """kernix_conv_run (:711-771). x2: (B*H*W) x C channels-last."""
    H, W = _hw(vi)
    Ho, Wo = _hw(vo)
    C, Co, g = vi["c"], vo["c"], s["groups"]
    cg, cog = C // g, Co // g
    B = x2.shape[0] // (H * W)
    x = x2.reshape(B, H, W, C)
    w = _wf(s["w"])
    kh, kw = s["kh"], s["kw"]
    xp = np.zeros((B, H + s["pt"] + s["pb"] + s["dh"] * kh, W + s["pl"] + s["pr"] + s["dw"] * kw, C), F32)
    xp[:, s["pt"]:s["pt"] + H, s["pl"]:s["pl"] + W, :] = x
    oy = np.arange(Ho) * s["sh"]
    ox = np.arange(Wo) * s["sw"]
    out = np.empty((B, Ho, Wo, Co), F32)
    if g > 1 and cg == 1:  # depthwise: out = bias, then taps in (ky, kx) order, vDSP_vma per tap
        mult = Co // C
        acc = np.broadcast_to(s["bias"] if s["bias"] is not None else np.zeros(Co, F32), (B, Ho, Wo, Co)).astype(F32)
        for ky in range(kh):
            iy = oy - s["pt"] + ky * s["dh"]
            vy = (iy >= 0) & (iy < H)
            for kx in range(kw):
                ix = ox - s["pl"] + kx * s["dw"]
                vx = (ix >= 0) & (ix < W)
                tap = xp[:, oy + ky * s["dh"]][:, :, ox + kx * s["dw"]]
                tap = np.repeat(tap, mult, axis=3)
                m = (vy[:, None] & vx[None, :])[None, :, :, None]
                acc = np.where(m, (tap * w[ky * kw + kx][None, None, None, :] + acc).astype(F32), acc).astype(F32)
        return act(acc.reshape(-1, Co), s["act"], s["alpha"])
    cols = []
    for ky in range(kh):
        for kx in range(kw):
            cols.append(xp[:, oy + ky * s["dh"]][:, :, ox + kx * s["dw"]])  # B x Ho x Wo x C
    colm = np.stack(cols, axis=3)  # B x Ho x Wo x (kh*kw) x C
    for gi in range(g):
        a = colm[..., gi * cg:(gi + 1) * cg].reshape(B * Ho * Wo, kh * kw * cg)
        out.reshape(-1, Co)[:, gi * cog:(gi + 1) * cog] = np.matmul(a, w[:, gi * cog:(gi + 1) * cog]).astype(F32)
    y = out.reshape(-1, Co)
    if s["bias"] is not None:
        y = (y + s["bias"][None, :]).astype(F32)
    return act(y, s["act"], s["alpha"])


def pool(s, vi, vo, x2):
    """kernix_pooling_run (:773-807)."""
    H, W = _hw(vi)
    Ho, Wo = _hw(vo)
    C = vi["c"]
    B = x2.shape[0] // (H * W)
    x = x2.reshape(B, H, W, C)
    mx = s["ptype"] == 0
    out = np.full((B, Ho, Wo, C), -np.inf if mx else 0, F32)
    cnt = np.zeros((Ho, Wo), np.int64)
    for ky in range(s["kh"]):
        iy = np.arange(Ho) * s["sh"] - s["pt"] + ky
        for kx in range(s["kw"]):
            ix = np.arange(Wo) * s["sw"] - s["pl"] + kx
            m = ((iy >= 0) & (iy < H))[:, None] & ((ix >= 0) & (ix < W))[None, :]
            tap = x[:, np.clip(iy, 0, H - 1)][:, :, np.clip(ix, 0, W - 1)]
            mm = m[None, :, :, None]
            if mx:
                out = np.where(mm, np.where(out > tap, out, tap), out).astype(F32)
            else:
                out = np.where(mm, out + tap, out).astype(F32)
            cnt += m
    if not mx:
        n = np.full((Ho, Wo), s["kh"] * s["kw"]) if s["count_pad"] else np.where(cnt > 0, cnt, 1)
        out = (out * (F32(1) / n.astype(F32))[None, :, :, None]).astype(F32)
    return out.reshape(-1, C)


def global_pool(s, vi, x2):
    """kernix_global_pool_run (:810-830): sequential over rows, mean = sum * (1/R)."""
    R, C = vi["r"], vi["c"]
    x = x2.reshape(-1, R, C)
    o = x[:, 0].copy()
    for i in range(1, R):
        o = (np.where(o > x[:, i], o, x[:, i]) if s["ptype"] == 0 else o + x[:, i]).astype(F32)
    if s["ptype"] == 1:
        o = (o * (F32(1) / F32(R))).astype(F32)
    return o


def permute(s, vi, x2):
    """kernix_permute_run (:833-862): output axis k = input axis perm[k], per sample."""
    per = vi["r"] * vi["c"]
    x = x2.reshape(-1, *vi["d"])
    y = np.transpose(x, [0] + [p + 1 for p in s["perm"]])
    return np.ascontiguousarray(y).reshape(-1, per // 1)


def binary(s, va, a2, vb, b2, vo):
    """kernix_binary_run (:877-906) with row/column size-1 broadcast inside a sample."""
    R, C = vo["r"], vo["c"]
    a = a2.reshape(-1, va["r"], va["c"])
    b = b2.reshape(-1, vb["r"], vb["c"])
    with np.errstate(all="ignore"):
        op = s["bop"]
        if op == 0:
            y = a + b
        elif op == 1:
            y = a - b
        elif op == 2:
            y = a * b
        elif op == 3:
            y = a / b
        elif op == 4:
            y = np.where(a > b, a, b)
        else:
            y = np.where(a < b, a, b)
    return np.broadcast_to(y, (y.shape[0], R, C)).astype(F32).reshape(-1, C)


def attention(s, q2, vq, k2, v2, vv):
    """kernix_attention_run (:1005-1048)."""
    Rq, S = vq["r"], vv["r"]
    H, dk, dv = s["heads"], s["dk"], s["dv"]
    B = q2.shape[0] // Rq
    Q = dense(q2, _wf(s["wq"]), s["bq"], ACT_NONE, 0).reshape(B, Rq, H, dk).transpose(0, 2, 1, 3)
    K = dense(k2, _wf(s["wk"]), s["bk"], ACT_NONE, 0).reshape(B, S, H, dk).transpose(0, 2, 1, 3)
    V = dense(v2, _wf(s["wv"]), s["bv"], ACT_NONE, 0).reshape(B, S, H, dv).transpose(0, 2, 1, 3)
    scale = F32(1) / np.sqrt(F32(dk))
    P = (np.matmul(Q, K.transpose(0, 1, 3, 2)) * scale).astype(F32)
    if s["causal"]:
        P = np.where(np.triu(np.ones((Rq, S), bool), 1)[None, None], F32(-np.inf), P)
    m = np.max(P, axis=-1, keepdims=True)
    with np.errstate(all="ignore"):
        E = np.exp((P - m).astype(F32)).astype(F32)
    P = (E * (F32(1) / np.sum(E, axis=-1, keepdims=True, dtype=F32))).astype(F32)
    ctx = np.matmul(P, V).astype(F32).transpose(0, 2, 1, 3).reshape(B * Rq, H * dv)
    return dense(ctx, _wf(s["wo"]), s["bo"], ACT_NONE, 0)


INT8_MAX_ROWS = 2  # KERNIX_INT8_MAX_ROWS (:50)
MERGE_CONCAT, MERGE_SUM, MERGE_MUL, MERGE_AVE = 0, 1, 2, 3  # KERNIX_MERGE_* (:35)
ACT_SIGMOID = ACT_NAMES.index("sigmoid")


def rnn_dir(s, d, x, B, T):
    """kernix_rnn_dir (:560-634): one direction of an LSTM / GRU / SimpleRNN over B sequences of T rows (x is
    (B*T) x in). The input projection x.W + b is one dense for all steps; each step adds h.U (sgemm with beta = 1,
    or kernix_qmatmul when U is int8 and B <= 2) and applies the gates in the reference's operation order:
    LSTM (i, f, g, o): c = i*g + f*c (c = i*g at step 0), h = act(c)*o; GRU (z, r, h~, recurrent bias after the
    reset gate): h~ = act(x_h + r*(h.U_h + b_h)), h = (h - h~)*z + h~; RNN: h = act(x.W + b + h.U).
    The backward direction reads t = T-1 .. 0 and writes each state at its own time position. Returns
    (B, T, u) states when ret_seq, else (B, u) final states."""
    kind, u, a, alpha = s["kind"], s["out"], s["act"], F32(s["alpha"])
    g = {OP["LSTM"]: 4, OP["GRU"]: 3, OP["RNN"]: 1}[kind]
    gu = g * u
    Ww, Uw, bias = s["rnn"][d]
    gru = kind == OP["GRU"]
    brec = bias[gu:2 * gu] if gru else None
    zx = dense(x, _wf(Ww), bias[:gu], ACT_NONE, 0.0).reshape(B, T, gu)
    h = np.zeros((B, u), F32)
    c = np.zeros((B, u), F32)
    out = np.zeros((B, T, u), F32) if s["ret_seq"] else None
    q8 = Uw[0] == "i8"
    with np.errstate(all="ignore"):
        for step in range(T):
            t = T - 1 - step if d else step
            z = zx[:, t, :].copy()
            zh = None
            if step == 0:
                if gru:
                    zh = np.broadcast_to(brec, (B, gu)).astype(F32)
            elif q8 and B <= INT8_MAX_ROWS:
                v = qlinear(h, Uw[1], Uw[2], brec)
                if gru:
                    zh = v
                else:
                    z = (z + v).astype(F32)
            else:
                hu = np.matmul(h, _wf(Uw)).astype(F32)
                if gru:
                    zh = (hu + brec[None, :]).astype(F32)
                else:
                    z = (z + hu).astype(F32)
            if kind == OP["LSTM"]:
                i_ = act(z[:, 0:u], ACT_SIGMOID, 0.0)
                f_ = act(z[:, u:2 * u], ACT_SIGMOID, 0.0)
                g_ = act(z[:, 2 * u:3 * u], a, alpha)
                o_ = act(z[:, 3 * u:4 * u], ACT_SIGMOID, 0.0)
                c = (i_ * g_).astype(F32) if step == 0 else ((i_ * g_).astype(F32) + (f_ * c).astype(F32)).astype(F32)
                h = (act(c, a, alpha) * o_).astype(F32)
            elif gru:
                zr = act((z[:, :2 * u] + zh[:, :2 * u]).astype(F32), ACT_SIGMOID, 0.0)
                hh = act(((zr[:, u:] * zh[:, 2 * u:]).astype(F32) + z[:, 2 * u:]).astype(F32), a, alpha)
                dh = -hh if step == 0 else (h - hh).astype(F32)
                h = ((dh * zr[:, :u]).astype(F32) + hh).astype(F32)
            else:
                h = act(z, a, alpha)
            if out is not None:
                out[:, t] = h
    return out if out is not None else h


def rnn(s, x, B, T):
    """kernix_rnn_run (:636-648): one or two directions; two are concatenated per position or merged
    elementwise (sum, product, average = (fw + bw) * 0.5)."""
    fw = rnn_dir(s, 0, x, B, T)
    if s["dirs"] == 1:
        return fw
    bw = rnn_dir(s, 1, x, B, T)
    if s["merge"] == MERGE_CONCAT:
        return np.concatenate([fw, bw], axis=-1)
    if s["merge"] == MERGE_MUL:
        return (fw * bw).astype(F32)
    y = (fw + bw).astype(F32)
    return (y * F32(0.5)).astype(F32) if s["merge"] == MERGE_AVE else y


def forward(model, x, trace=None):
    """kernix_model_forward on (rows, in_dim) float32, rows a multiple of seq_len. Returns (B, out_dim).
    trace: optional list that receives every value (index = original value id, (B*r) x c arrays)."""
    vals = model["vals"]
    x = np.ascontiguousarray(x, F32).reshape(-1, model["in_dim"])
    B = x.shape[0] // model["seq_len"]
    views = [x]
    for i, s in enumerate(model["steps"]):
        k = s["kind"]
        a = views[s["inp"][0]]
        vi, vo = vals[s["inp"][0]], vals[i + 1]
        if k == OP["LINEAR"]:
            if s["w"][0] == "i8":
                y = act(qlinear(a, s["w"][1], s["w"][2], s["bias"]), s["act"], s["alpha"])
            else:
                y = dense(a, s["w"][1], s["bias"], s["act"], s["alpha"])
        elif k == OP["ACT"]:
            y = act(a, s["act"], s["alpha"])
        elif k == OP["LAYERNORM"]:
            y = layer_norm_rows(a, s["gamma"], s["beta"], s["eps"])
        elif k == OP["SOFTMAX"]:
            y = softmax_rows(a)
        elif k == OP["CONV"]:
            y = conv(s, vi, vo, a)
        elif k == OP["POOL"]:
            y = pool(s, vi, vo, a)
        elif k == OP["GLOBAL_POOL"]:
            y = global_pool(s, vi, a)
        elif k == OP["RESHAPE"]:
            y = a.reshape(-1, vo["c"])
        elif k == OP["PERMUTE"]:
            y = permute(s, vi, a).reshape(-1, vo["c"])
        elif k == OP["BINARY"]:
            y = binary(s, vi, a, vals[s["inp"][1]], views[s["inp"][1]], vo)
        elif k == OP["CONCAT"]:
            if s["axis"] == 1:
                y = np.concatenate([views[j].reshape(B * vo["r"], -1) for j in s["inp"]], axis=1)
            else:
                y = np.concatenate([views[j].reshape(B, -1) for j in s["inp"]], axis=1).reshape(-1, vo["c"])
        elif k == OP["EMBEDDING"]:
            ids = a.reshape(-1)
            V = s["inp_c"]
            table = _wf(s["w"])
            ok = (ids >= 0) & (ids < V) & (ids == np.floor(ids))
            y = np.full((ids.size, s["out"]), np.nan, F32)
            y[ok] = table[ids[ok].astype(np.int64)]
        elif k == OP["AFFINE"]:
            y = (a * s["gamma"][None, :] + s["beta"][None, :]).astype(F32)
        elif k == OP["ADD_CONST"]:
            y = (a.reshape(B, -1) + s["cst"][None, :]).astype(F32).reshape(-1, vo["c"])
        elif k == OP["ATTENTION"]:
            n = len(s["inp"])
            vid = s["inp"][1 if n > 1 else 0]
            kid = s["inp"][2 if n > 2 else (1 if n > 1 else 0)]
            y = attention(s, a, vi, views[kid], views[vid], vals[vid])
        elif k == OP["SELECT"]:
            if s["axis"] == 0:
                per = vi["r"] * vi["c"]
                blk = per // vi["d"][0]
                y = a.reshape(B, per)[:, s["start"] * blk:(s["start"] + s["len"]) * blk].reshape(-1, vo["c"])
            else:
                y = a[:, s["start"]:s["start"] + s["len"]].reshape(-1, vo["c"])
        elif k == OP["PAD"]:
            H, W = _hw(vi)
            Ho, Wo = _hw(vo)
            xx = a.reshape(B, H, W, vi["c"])
            y = np.zeros((B, Ho, Wo, vi["c"]), F32)
            y[:, s["pt"]:s["pt"] + H, s["pl"]:s["pl"] + W] = xx
            y = y.reshape(-1, vo["c"])
        elif k in (OP["LSTM"], OP["GRU"], OP["RNN"]):
            y = rnn(s, a, B, vi["r"])
        elif k == OP["UPSAMPLE"]:
            H, W = _hw(vi)
            Ho, Wo = _hw(vo)
            xx = a.reshape(B, H, W, vi["c"])
            y = xx[:, np.arange(Ho) // s["sh"]][:, :, np.arange(Wo) // s["sw"]].reshape(-1, vo["c"])
        else:
            raise NotImplementedError(f"{OP_NAMES[k]} is outside the GPU path")
        views.append(np.ascontiguousarray(y, F32).reshape(B * vo["r"], vo["c"]))
    if trace is not None:
        trace.extend(views)
    return views[-1].reshape(B, -1)


def forward_file(path, x):
    return forward(load(path), x)
