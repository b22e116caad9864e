"""The five benchmark configurations as seeded synthetic `.knx` models (random-init weights, no checkpoints).

Shapes, activations and value distributions follow the benchmark definition of the KERNIX .knx forward
path; weights are drawn with numpy's PCG64 from the given seed (they are not the torch draws of the same
seed, which only matters for the exact values, not for shapes, op lists or throughput). `params_cN` returns a
configuration's draws and `build_cN` writes them with knx_writer; the bytes written are the bytes the reference
exporters write for a PyTorch model holding the same parameters (tools/export_torch.py for the sequential MLPs,
--quantize int8 for c2, tools/torch_graph.py + tools/knx3.py for the CNN, whose BatchNorms are folded, and the
Transformer): tests/test_cpu_exporters.py exports each one through the reference tools and compares.

  c1  fp32 MLP 784-512-256-10, ReLU, softmax out            x ~ U[0,1)       (B, 784)
  c2  int8 MLP 1024-4096-4096-1024, GELU (I8_COL weights)    x ~ N(0,1)       (B, 1024)
  c3  fp32 CNN 3x32x32 (conv64 x2, pool, conv128 x2 + residual, pool, conv256, GAP, dense 10)
                                                            x ~ N(0,1)       (B, 3, 32, 32) channels-first
  c4  fp32 Transformer encoder 6 x (pre-LN, MHA 8 heads, FFN 2048 GELU), d 512, seq 128
                                                            x ~ N(0,1)       (B, 128, 512)
  c5  wide fp32 MLP 8192-16384-16384-8192, ReLU             x ~ U[-1,1)      (B, 8192)
"""
import math
import os

import numpy as np

from . import knx_writer as kw

F32 = np.float32


def _he(rng, fan_in, shape):
    return (rng.standard_normal(shape, dtype=F32) * F32(math.sqrt(2.0 / fan_in))).astype(F32)


def _unif(rng, fan_in, n):
    b = 1.0 / math.sqrt(fan_in)
    return rng.uniform(-b, b, n).astype(F32)


def params_c1(seed=0, dims=(784, 512, 256, 10)):
    """Per layer (w in x out, b): W ~ N(0, sqrt(2/fan_in)), b = 0.01."""
    rng = np.random.default_rng(seed)
    return [(_he(rng, dims[i], (dims[i], dims[i + 1])), np.full(dims[i + 1], 0.01, F32)) for i in range(len(dims) - 1)]


def build_c1(path, seed=0):
    m = kw.Sequential()
    layers = params_c1(seed)
    for i, (w, b) in enumerate(layers):
        m.linear(w, b)
        if i < len(layers) - 1:
            m.act("relu")
    m.softmax().write(path)


def params_c2(seed=1, dims=(1024, 4096, 4096, 1024)):
    """Per layer (w in x out, float32 before quantisation, b): W ~ N(0, 0.02), b ~ U(+-1/sqrt(fan_in))."""
    rng = np.random.default_rng(seed)
    out = []
    for i in range(len(dims) - 1):
        w = (rng.standard_normal((dims[i], dims[i + 1]), dtype=F32) * F32(0.02)).astype(F32)
        out.append((w, _unif(rng, dims[i], dims[i + 1])))
    return out


def build_c2(path, seed=1, dims=(1024, 4096, 4096, 1024)):
    m = kw.Sequential(int8=True)
    layers = params_c2(seed, dims)
    for i, (w, b) in enumerate(layers):
        m.linear(w, b)
        if i < len(layers) - 1:
            m.act("gelu")
    m.write(path)


def params_c3(seed=2):
    """The CNN's convolutions in graph order: dict(cin, cout, w (9*cin x cout, rows (ky, kx, ci)), b, bn), bn =
    (gamma, beta, running mean, running var) of a BatchNorm2d(eval) with non-default statistics or None; then the
    dense layer (w 256 x 10, b)."""
    rng = np.random.default_rng(seed)
    convs = []
    for cin, cout, bn in ((3, 64, True), (64, 64, True), (64, 128, False), (128, 128, False), (128, 256, False)):
        w = _he(rng, cin * 9, (9 * cin, cout))
        b = _unif(rng, cin * 9, cout)
        stats = None
        if bn:
            stats = (rng.uniform(0.5, 1.5, cout).astype(F32), rng.uniform(-0.2, 0.2, cout).astype(F32),
                     rng.uniform(-0.3, 0.3, cout).astype(F32), rng.uniform(0.5, 2.0, cout).astype(F32))
        convs.append(dict(cin=cin, cout=cout, w=w, b=b, bn=stats))
    return convs, (_he(rng, 256, (256, 10)), _unif(rng, 256, 10))


def fold_bn(w, b, bn, eps=1e-5):
    """BatchNorm(eval) after a convolution folded into its weights, in float64 as the reference exporter does
    (tools/torch_graph.py:372-377 scale / shift, tools/knx3.py:209-240 fold): scale = gamma / sqrt(var + eps),
    shift = beta - mean * scale, w' = w * scale, b' = b * scale + shift, then stored as float32."""
    gamma, beta, mean, var = (np.asarray(a, np.float64) for a in bn)
    scale = gamma / np.sqrt(var + eps)
    shift = beta - mean * scale
    return ((np.asarray(w, np.float64) * scale[None, :]).astype(F32),
            (np.asarray(b, np.float64) * scale + shift).astype(F32))


def build_c3(path, seed=2):
    convs, (wd, bd) = params_c3(seed)
    g = kw.Graph((32, 32, 3), layout=1)

    def conv(x, c):
        w, b = fold_bn(c["w"], c["b"], c["bn"]) if c["bn"] is not None else (c["w"], c["b"])
        return g.act(g.conv(x, w, b, (3, 3), pads=(1, 1, 1, 1)), "relu")

    x = conv(0, convs[0])
    x = conv(x, convs[1])
    x = g.pool(x, "max", (2, 2), (2, 2))
    h = conv(x, convs[2])
    x = g.binary(h, conv(h, convs[3]), "add")
    x = g.pool(x, "max", (2, 2), (2, 2))
    x = conv(x, convs[4])
    x = g.global_pool(x, "avg")
    x = g.reshape(x, (1, 1, 256))
    x = g.permute(x, (2, 0, 1))
    x = g.reshape(x, (256,))
    g.linear(x, wd, bd)
    g.write(path)


def params_c4(seed=3, layers=6, d=512, ffn=2048):
    """Per encoder layer: dict(wq, wk, wv, wo (d x d, in x out), w1 (d x ffn), b1, w2 (ffn x d), b2); attention
    biases are zero and the LayerNorms are the identity affine (gamma 1, beta 0)."""
    rng = np.random.default_rng(seed)
    nrm = lambda *s: (rng.standard_normal(s, dtype=F32) * F32(0.02)).astype(F32)  # noqa: E731
    out = []
    for _ in range(layers):
        p = dict(wq=nrm(d, d), wk=nrm(d, d), wv=nrm(d, d), wo=nrm(d, d))
        p["w1"] = nrm(d, ffn)
        p["b1"] = _unif(rng, d, ffn)
        p["w2"] = nrm(ffn, d)
        p["b2"] = _unif(rng, ffn, d)
        out.append(p)
    return out


def build_c4(path, seed=3, layers=6, d=512, heads=8, ffn=2048, seq=128):
    g = kw.Graph((seq, d))
    ones, zeros = np.ones(d, F32), np.zeros(d, F32)
    x = 0
    for p in params_c4(seed, layers, d, ffn):
        h = g.layernorm(x, ones, zeros)
        a = g.attention(h, heads, p["wq"], zeros, p["wk"], zeros, p["wv"], zeros, p["wo"], zeros)
        x = g.binary(x, a, "add")
        h = g.layernorm(x, ones, zeros)
        h = g.act(g.linear(h, p["w1"], p["b1"]), "gelu")
        h = g.linear(h, p["w2"], p["b2"])
        x = g.binary(x, h, "add")
    g.write(path)


def params_c5(seed=4, dims=(8192, 16384, 16384, 8192)):
    """Per layer (w in x out, b): W ~ N(0, sqrt(2/fan_in)), b = 0.01."""
    return params_c1(seed, dims)


def build_c5(path, seed=4, dims=(8192, 16384, 16384, 8192)):
    m = kw.Sequential()
    layers = params_c5(seed, dims)
    for i, (w, b) in enumerate(layers):
        m.linear(w, b)
        if i < len(layers) - 1:
            m.act("relu")
    m.write(path)


BUILDERS = dict(c1=build_c1, c2=build_c2, c3=build_c3, c4=build_c4, c5=build_c5)


def inputs(cfg, batch, seed=100):
    """Seeded synthetic input rows (rows x in_dim, channels-last) for a config."""
    rng = np.random.default_rng(seed)
    if cfg == "c1":
        return rng.random((batch, 784), dtype=F32)
    if cfg == "c2":
        return rng.standard_normal((batch, 1024), dtype=F32)
    if cfg == "c3":
        return rng.standard_normal((batch * 1024, 3), dtype=F32)
    if cfg == "c4":
        return rng.standard_normal((batch * 128, 512), dtype=F32)
    if cfg == "c5":
        return rng.uniform(-1, 1, (batch, 8192)).astype(F32)
    raise ValueError(cfg)


def model_path(cfg, directory=None):
    """Build (once) and return the path of a config's .knx under directory (default: $KERNIX_MODEL_DIR or /tmp)."""
    directory = directory or os.environ.get("KERNIX_MODEL_DIR", "/tmp/kernix_models")
    os.makedirs(directory, exist_ok=True)
    p = os.path.join(directory, f"{cfg}.knx")
    if not os.path.exists(p):
        tmp = p + f".tmp{os.getpid()}"
        BUILDERS[cfg](tmp)
        os.replace(tmp, p)
    return p
