"""The five benchmark configurations as seeded synthetic `.knx` models (random-init weights, no checkpoints).

Shapes, activations and value distributions follow the benchmark definition of the KERNIX .knx forward
path; weights are drawn with numpy's PCG64 from the given seed (they are not the torch draws of the same
seed, which only matters for the exact values, not for shapes, op lists or throughput). The op lists are
the ones the reference exporters emit for the same architectures (tools/export_torch.py for sequential
MLPs, tools/torch_graph.py + tools/knx3.py for the CNN and Transformer, BatchNorm folded into the conv).

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


def build_c1(path, seed=0):
    rng = np.random.default_rng(seed)
    m = kw.Sequential()
    dims = [784, 512, 256, 10]
    for i in range(3):
        m.linear(_he(rng, dims[i], (dims[i], dims[i + 1])), np.full(dims[i + 1], 0.01, F32))
        if i < 2:
            m.act("relu")
    m.softmax().write(path)


def build_c2(path, seed=1):
    rng = np.random.default_rng(seed)
    m = kw.Sequential(int8=True)
    dims = [1024, 4096, 4096, 1024]
    for i in range(3):
        w = (rng.standard_normal((dims[i], dims[i + 1]), dtype=F32) * F32(0.02)).astype(F32)
        m.linear(w, _unif(rng, dims[i], dims[i + 1]))
        if i < 2:
            m.act("gelu")
    m.write(path)


def build_c3(path, seed=2):
    rng = np.random.default_rng(seed)
    g = kw.Graph((32, 32, 3), layout=1)

    def conv(x, cin, cout, bn):
        w = _he(rng, cin * 9, (9 * cin, cout))
        b = _unif(rng, cin * 9, cout)
        if bn:  # BatchNorm2d(eval) with non-default running stats, folded as tools/knx3.py:209-240 does
            gamma = rng.uniform(0.5, 1.5, cout).astype(F32)
            beta = rng.uniform(-0.2, 0.2, cout).astype(F32)
            mean = rng.uniform(-0.3, 0.3, cout).astype(F32)
            var = rng.uniform(0.5, 2.0, cout).astype(F32)
            sc = (gamma / np.sqrt(var + 1e-5)).astype(np.float64)
            w = (w.astype(np.float64) * sc[None, :]).astype(F32)
            b = (b.astype(np.float64) * sc + (beta - mean * sc)).astype(F32)
        return g.act(g.conv(x, w, b, (3, 3), pads=(1, 1, 1, 1)), "relu")

    x = conv(0, 3, 64, True)
    x = conv(x, 64, 64, True)
    x = g.pool(x, "max", (2, 2), (2, 2))
    h = conv(x, 64, 128, False)
    x = g.binary(h, conv(h, 128, 128, False), "add")
    x = g.pool(x, "max", (2, 2), (2, 2))
    x = conv(x, 128, 256, False)
    x = g.global_pool(x, "avg")
    x = g.reshape(x, (1, 1, 256))
    x = g.permute(x, (2, 0, 1))
    x = g.reshape(x, (256,))
    g.linear(x, _he(rng, 256, (256, 10)), _unif(rng, 256, 10))
    g.write(path)


def build_c4(path, seed=3, layers=6, d=512, heads=8, ffn=2048, seq=128):
    rng = np.random.default_rng(seed)
    g = kw.Graph((seq, d))
    nrm = lambda *s: (rng.standard_normal(s, dtype=F32) * F32(0.02)).astype(F32)  # noqa: E731
    ones, zeros = np.ones(d, F32), np.zeros(d, F32)
    x = 0
    for _ in range(layers):
        h = g.layernorm(x, ones, zeros)
        a = g.attention(h, heads, nrm(d, d), np.zeros(d, F32), nrm(d, d), np.zeros(d, F32),
                        nrm(d, d), np.zeros(d, F32), nrm(d, d), np.zeros(d, F32))
        x = g.binary(x, a, "add")
        h = g.layernorm(x, ones, zeros)
        h = g.act(g.linear(h, nrm(d, ffn), _unif(rng, d, ffn)), "gelu")
        h = g.linear(h, nrm(ffn, d), _unif(rng, ffn, d))
        x = g.binary(x, h, "add")
    g.write(path)


def build_c5(path, seed=4):
    rng = np.random.default_rng(seed)
    m = kw.Sequential()
    dims = [8192, 16384, 16384, 8192]
    for i in range(3):
        m.linear(_he(rng, dims[i], (dims[i], dims[i + 1])), np.full(dims[i + 1], 0.01, F32))
        if i < 2:
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
