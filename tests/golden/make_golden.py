"""Regenerate the golden fixtures in tests/golden/ (run in the build container, where the reference checkout exists).

    python tests/golden/make_golden.py [--reference /root/reference]

Every model here is exported by the REFERENCE's own tools (tools/export_torch.py, tools/torch_graph.py,
tools/knx3.py) and every expected output `y_ref` is computed by the REFERENCE's own forward, compiled from its
sources into oracle/_ref/libkernix_ref.so (make -C oracle/ref). `y_torch` is PyTorch's output of the same module,
as the reference's own tests compare against. Fixtures:

  small, wide, inplace_first   the golden MLPs of the reference's test/mlp_bench.py:35-62 (torch seed 0)
  small_int8                   `small` exported with --quantize int8; y_ref from the reference's int8 path
                               (workspace forced to one sample per chunk, so every LINEAR runs kernix_qmatmul)
  q8_s                         int8 MLP 64-128-128-32 GELU (config 2's family, reduced)
  cnn_s, tfm_s                 config 3's CNN and config 4's pre-LN Transformer families, reduced
  g_cnn, g_attn, g_rnn         the three graphs of the reference's test/knx_fuzz_test.py:20-40 (conv kinds, pad,
                               upsample, pools; embedding, causal attention, reshape/permute, affine; RNNs -- the
                               RNN graph is a loader fixture only)
"""
import argparse
import contextlib
import io
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default="/root/reference")
    a = ap.parse_args()
    sys.path.insert(0, os.path.join(a.reference, "tools"))
    import torch
    import torch.nn as nn
    from export_torch import export  # noqa: E402  (reference tool)
    from knx3 import FIRST, LAST, Graph  # noqa: E402  (reference tool)
    from torch_graph import export_graph  # noqa: E402  (reference tool)

    from oracle import ref_lib

    out = {}

    def save(name, path_knx, xs, ys_torch=None, int8=False):
        m = ref_lib.RefModel(path_knx)
        if int8:  # one sample per chunk: the reference's int8 kernel runs for every LINEAR (include/kernix_model.h:1854)
            m.set_workspace_limit(1)
        data = {}
        for i, x in enumerate(xs):
            data[f"x{i}"] = x.astype(np.float32)
            data[f"y_ref{i}"] = m.forward(x)
            if ys_torch is not None:
                data[f"y_torch{i}"] = ys_torch[i].astype(np.float32)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **data)
        out[name] = (os.path.getsize(path_knx), len(xs))
        m.close()

    def knx(name):
        return os.path.join(HERE, f"{name}.knx")

    quiet = contextlib.redirect_stdout(io.StringIO())

    # ---- reference golden MLPs (test/mlp_bench.py:35-62)
    torch.manual_seed(0)
    small = nn.Sequential(
        nn.Linear(64, 128), nn.GELU(), nn.LayerNorm(128),
        nn.Linear(128, 96, bias=False), nn.SiLU(),
        nn.Linear(96, 96), nn.Tanh(),
        nn.Linear(96, 80), nn.Sigmoid(),
        nn.Linear(80, 32), nn.ReLU(), nn.LayerNorm(32, elementwise_affine=False),
        nn.Linear(32, 10), nn.Softmax(dim=-1),
    )
    nn.init.normal_(small[2].weight, 1.0, 0.5)
    nn.init.normal_(small[2].bias, 0.0, 0.5)
    wide = nn.Sequential(nn.Linear(4, 9000), nn.SiLU(), nn.GELU(), nn.Linear(9000, 3))
    inplace_first = nn.Sequential(nn.Tanh(), nn.Linear(8, 4))
    with torch.no_grad():
        for name, model, in_dim, batches in (("small", small, 64, (1, 37)), ("wide", wide, 4, (5,)),
                                             ("inplace_first", inplace_first, 8, (3,))):
            export(model, knx(name))
            xs = [torch.randn(b, in_dim) for b in batches]
            save(name, knx(name), [x.numpy() for x in xs], [model(x).numpy() for x in xs])
        export(small, knx("small_int8"), quantize="int8")
        x = torch.randn(37, 64)
        save("small_int8", knx("small_int8"), [x.numpy()], [small(x).numpy()], int8=True)

        # ---- config families, reduced
        torch.manual_seed(1)
        q8 = nn.Sequential(nn.Linear(64, 128), nn.GELU(), nn.Linear(128, 128), nn.GELU(), nn.Linear(128, 32))
        for layer in q8:
            if isinstance(layer, nn.Linear):
                nn.init.normal_(layer.weight, 0, 0.02)
        export(q8, knx("q8_s"), quantize="int8")
        x = torch.randn(8, 64)
        save("q8_s", knx("q8_s"), [x.numpy()], [q8(x).numpy()], int8=True)

        class CNN(nn.Module):
            def __init__(s):
                super().__init__()
                C = lambda i, o: nn.Conv2d(i, o, 3, padding=1)  # noqa: E731
                s.c1, s.b1, s.c2, s.b2, s.c3, s.c4, s.c5 = C(3, 8), nn.BatchNorm2d(8), C(8, 8), nn.BatchNorm2d(8), C(8, 16), C(16, 16), C(16, 32)
                s.mp = nn.MaxPool2d(2)
                s.gap = nn.AdaptiveAvgPool2d(1)
                s.fc = nn.Linear(32, 10)
                for layer in s.modules():
                    if isinstance(layer, (nn.Conv2d, nn.Linear)):
                        nn.init.kaiming_normal_(layer.weight)
                for bn in (s.b1, s.b2):
                    bn.running_mean.uniform_(-0.5, 0.5)
                    bn.running_var.uniform_(0.5, 2.0)
                    bn.weight.data.uniform_(0.5, 1.5)
                    bn.bias.data.uniform_(-0.5, 0.5)

            def forward(s, x):
                x = torch.relu(s.b1(s.c1(x)))
                x = torch.relu(s.b2(s.c2(x)))
                x = s.mp(x)
                h = torch.relu(s.c3(x))
                x = h + torch.relu(s.c4(h))
                x = s.mp(x)
                x = torch.relu(s.c5(x))
                return s.fc(torch.flatten(s.gap(x), 1))

        torch.manual_seed(2)
        cnn = CNN().eval()
        with quiet:
            export_graph(cnn, knx("cnn_s"), (3, 16, 16))
        x = torch.randn(2, 3, 16, 16)
        save("cnn_s", knx("cnn_s"), [x.permute(0, 2, 3, 1).reshape(-1, 3).numpy()], [cnn(x).numpy()])

        class Wrap(nn.Module):
            def __init__(s, e):
                super().__init__()
                s.e = e

            def forward(s, x):
                return s.e(x)

        torch.manual_seed(3)
        enc = nn.TransformerEncoder(nn.TransformerEncoderLayer(32, 4, 64, dropout=0.0, activation="gelu", batch_first=True,
                                                               norm_first=True), 2, enable_nested_tensor=False)
        for p in enc.parameters():
            if p.dim() > 1:
                nn.init.normal_(p, 0, 0.1)
        tfm = Wrap(enc).eval()
        with quiet:
            export_graph(tfm, knx("tfm_s"), (8, 32))
        x = torch.randn(2, 8, 32)
        save("tfm_s", knx("tfm_s"), [x.reshape(-1, 32).numpy()], [tfm(x).reshape(2, -1).numpy()])

    # ---- the reference fuzz test's graphs (test/knx_fuzz_test.py:20-40), built with its own knx3.Graph
    rng = np.random.default_rng(0)
    W = lambda *s: rng.normal(0, 0.3, s)  # noqa: E731
    g = Graph((9, 8, 3))
    x = g.conv(0, W(27, 6), W(6), (3, 3), pads=(1, 1, 1, 1), act="relu")
    y = g.conv(x, W(9, 6), None, (3, 3), pads=(1, 1, 1, 1), groups=6)
    y = g.conv(y, W(27, 6), W(6), (3, 3), pads=(1, 1, 1, 1), groups=2)
    x = g.binary(x, y, "add")
    x = g.upsample(g.pad(g.pool(x, "max", (2, 2), (2, 2)), (1, 0, 0, 1)), 2, 2)
    x = g.pool(x, "avg", (3, 3), (1, 1), (1, 1, 1, 1), True)
    g.write(knx("g_cnn"), g.linear(g.global_pool(x, "avg"), W(6, 4), W(4), act="softmax"))
    save("g_cnn", knx("g_cnn"), [rng.standard_normal((3 * 72, 3)).astype(np.float32)])
    g = Graph((7, 5))
    a_ = g.rnn(0, "GRU", 4, [(W(5, 12), W(4, 12), W(24)), (W(5, 12), W(4, 12), W(24))], ret_seq=True)
    b_ = g.rnn(0, "LSTM", 3, [(W(5, 12), W(3, 12), W(12))], act="relu", ret_seq=True)
    c_ = g.concat([a_, b_], LAST)
    c_ = g.rnn(c_, "RNN", 4, [(W(11, 4), W(4, 4), W(4)), (W(11, 4), W(4, 4), W(4))], ret_seq=False, merge="ave")
    g.write(knx("g_rnn"), g.concat([c_, g.select(a_, FIRST, 6, 1, True)], LAST))
    save("g_rnn", knx("g_rnn"), [rng.standard_normal((2 * 7, 5)).astype(np.float32)])
    g = Graph((6,))
    e = g.add_const(g.embedding(0, W(10, 8)), W(48))
    h = g.layernorm(g.binary(e, g.attention(e, 2, W(8, 6), W(6), W(8, 6), W(6), W(8, 4), W(4), W(4, 8), W(8), causal=True), "add"),
                    W(8), W(8), 1e-5)
    h = g.permute(g.reshape(h, (6, 2, 4)), (1, 0, 2))
    g.write(knx("g_attn"), g.affine(g.reshape(h, (2, 24)), W(24), W(24)))
    ids = rng.integers(0, 10, (4, 6)).astype(np.float32)
    save("g_attn", knx("g_attn"), [ids])

    for k, (sz, n) in out.items():
        print(f"{k:14s} {sz / 1024:8.1f} KB  {n} input(s)")


if __name__ == "__main__":
    main()
