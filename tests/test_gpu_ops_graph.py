"""GPU: one-op and few-op KNX3 graphs through the full runtime (loader, plan, executor, kernels) against the
oracle -- each graph op in isolation at the shapes the benchmark configurations use, plus the edge cases of the
reference's op semantics (broadcasting, pooling padding, views, concat/select axes)."""
import numpy as np
import pytest

from conftest import rel_err
from oracle import knx_oracle as ko

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu
F32 = np.float32
# tcgen05 accumulates fp32 with truncation, so 3xTF32 results drift by ~5e-9 * K relative to the output scale:
# 1e-5 holds up to K ~ 1000; layers with K in the thousands (attention on 512 channels, FFN 2048, conv 128x9)
# are checked at 3e-5, well inside the 1e-4 bound of the configurations that contain them.
TF32_LONG_K = 3e-5


@pytest.fixture(scope="module")
def run(libkx, tmp_path_factory):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from kernix_b200 import Model
    d = tmp_path_factory.mktemp("ops")
    counter = [0]

    def _run(graph, x, tol=1e-5):
        counter[0] += 1
        p = str(d / f"g{counter[0]}.knx")
        graph.write(p)
        got = Model(p)(x)
        want = ko.forward(ko.load(p), x)
        err = rel_err(got.reshape(want.shape), want)
        assert err <= tol, f"max rel err {err:.3e}"
        return got
    return _run


def G(shape, layout=0):
    from kernix_b200.knx_writer import Graph
    return Graph(shape, layout)


def rnd(*s, scale=1.0, seed=0):
    return (np.random.default_rng(seed + sum(s)).standard_normal(s) * scale).astype(F32)


@pytest.mark.parametrize("H,W,C,Co,B", [(16, 16, 64, 128, 3), (8, 8, 128, 256, 2), (32, 32, 3, 64, 2), (16, 16, 128, 128, 2)])
def test_conv3x3_shapes_of_c3(run, H, W, C, Co, B):
    g = G((H, W, C))
    g.act(g.conv(0, rnd(9 * C, Co, scale=1 / np.sqrt(9 * C)), rnd(Co, scale=0.1), (3, 3), pads=(1, 1, 1, 1)), "relu")
    run(g, rnd(B * H * W, C), tol=1e-5)


def test_conv_strided_dilated_grouped_depthwise(run):
    g = G((12, 10, 8))
    a = g.conv(0, rnd(9 * 4, 12, scale=0.2), rnd(12), (3, 3), stride=(2, 1), dil=(1, 2), pads=(1, 1, 2, 2), groups=2)
    b = g.conv(a, rnd(9, 24, scale=0.3), None, (3, 3), pads=(1, 1, 1, 1), groups=12)  # depthwise, multiplier 2
    g.act(g.conv(b, rnd(24, 5, scale=0.3), rnd(5), (1, 1)), "silu")  # pointwise -> GEMM
    run(g, rnd(2 * 12 * 10, 8), tol=1e-5)


def test_attention_self_c4_shape(run):
    d, h = 512, 8
    g = G((128, d))
    w = [rnd(d, d, scale=0.02, seed=i) for i in range(4)]
    b = [rnd(d, scale=0.1, seed=10 + i) for i in range(4)]
    g.attention(0, h, w[0], b[0], w[1], b[1], w[2], b[2], w[3], b[3])
    run(g, rnd(2 * 128, d), tol=TF32_LONG_K)


@pytest.mark.parametrize("d,h,S,B", [(64, 4, 16, 3), (512, 8, 128, 1), (128, 2, 40, 2)])
def test_attention_self_fused_projection(run, d, h, S, B):
    g = G((S, d))
    w = [rnd(d, d, scale=0.05, seed=i) for i in range(4)]
    b = [rnd(d, scale=0.1, seed=10 + i) for i in range(4)]
    g.attention(0, h, w[0], b[0], w[1], b[1], w[2], b[2], w[3], b[3])
    run(g, rnd(B * S, d), tol=TF32_LONG_K)


def test_linear_as_fused_qkv(run):
    d = 512
    g = G((128, d))
    g.linear(0, rnd(d, 3 * d, scale=0.02), rnd(3 * d, scale=0.1))
    run(g, rnd(2 * 128, d), tol=1e-5)


def test_attention_cross_causal_no_bias(run):
    g = G((10, 16))
    kv = g.linear(0, rnd(16, 24, scale=0.3), None)
    g.attention(0, 4, rnd(16, 32, scale=0.3), None, rnd(24, 32, scale=0.3), None, rnd(24, 40, scale=0.3), None,
                rnd(40, 16, scale=0.3), None, v=kv, k=kv, causal=True)
    run(g, rnd(3 * 10, 16), tol=1e-5)


def test_residual_layernorm_ffn(run):
    d = 64
    g = G((16, d))
    h = g.layernorm(0, rnd(d, scale=0.5) + 1, rnd(d, scale=0.1))
    h = g.act(g.linear(h, rnd(d, 4 * d, scale=0.05), rnd(4 * d, scale=0.1)), "gelu")
    h = g.linear(h, rnd(4 * d, d, scale=0.05), rnd(d, scale=0.1))
    g.binary(0, h, "add")
    run(g, rnd(4 * 16, d), tol=1e-5)


def test_pool_gap_reshape_permute_linear(run):
    g = G((8, 8, 16))
    x = g.pool(0, "max", (2, 2), (2, 2))
    y = g.pool(0, "avg", (3, 3), (2, 2), pads=(1, 1, 1, 1), count_pad=True)
    z = g.binary(x, y, "sub")
    z = g.global_pool(z, "avg")
    z = g.reshape(z, (1, 1, 16))
    z = g.permute(z, (2, 0, 1))
    z = g.reshape(z, (16,))
    g.softmax(g.linear(z, rnd(16, 7), rnd(7)))
    run(g, rnd(5 * 64, 16), tol=1e-6)


def test_broadcast_binary_ops(run):
    g = G((6, 5))
    c = g.linear(0, rnd(5, 1), None)         # (6, 1): channel broadcast
    r = g.global_pool(0, "max")              # (5,): row broadcast against (6, 5)
    a = g.binary(0, c, "mul")
    a = g.binary(a, r, "add")
    a = g.binary(a, c, "max")
    a = g.binary(r, a, "min")
    g.binary(a, g.act(c, "exp"), "div")
    run(g, rnd(4 * 6, 5), tol=1e-5)


def test_concat_select_pad_upsample_affine_addconst_embedding(run):
    g = G((4, 6, 3))
    a = g.concat([0, g.act(0, "tanh")], 1)                      # channel concat -> (4, 6, 6)
    b = g.concat([a, a], 0)                                     # first-axis concat -> (8, 6, 6)
    b = g.select(b, 0, 2, 4)                                    # rows 2..5 -> (4, 6, 6)
    b = g.select(b, 1, 1, 4)                                    # channels 1..4 -> (4, 6, 4)
    b = g.pad(b, (1, 2, 0, 1))                                  # (7, 7, 4)
    b = g.upsample(b, 2, 1)                                     # (14, 7, 4)
    b = g.affine(b, rnd(4), rnd(4))
    b = g.add_const(b, rnd(14 * 7 * 4, scale=0.1))
    run(g, rnd(3 * 24, 3), tol=1e-6)
    e = G((5,))
    e.embedding(0, rnd(10, 3))
    ids = np.array([[0, 1, 9, 3, 4], [2, 2, 7, 8, 5]], F32)
    run(e, ids, tol=0)


@pytest.mark.parametrize("act", ["relu", "gelu", "silu", "sigmoid", "tanh", "leaky_relu", "elu", "selu", "softplus", "relu6",
                                 "hard_sigmoid", "hard_swish", "gelu_tanh", "exp", "mish", "softsign"])
def test_every_activation_fused_and_standalone(run, act):
    g = G((12,))
    a = g.act(g.linear(0, rnd(12, 40, scale=0.5), rnd(40, scale=0.2)), act, 0.2)  # fused into the GEMM epilogue
    g.act(g.layernorm(a, np.ones(40, F32), np.zeros(40, F32)), act, 0.3)          # standalone ACT step
    run(g, rnd(9, 12), tol=2e-6)


def test_c3_prefix_conv_pool_conv(run):
    """the first four steps of config c3: conv(3->64)+relu, conv(64->64)+relu, maxpool 2, conv(64->128)+relu"""
    g = G((32, 32, 3))
    a = g.act(g.conv(0, rnd(27, 64, scale=0.3), rnd(64, scale=0.1), (3, 3), pads=(1, 1, 1, 1)), "relu")
    a = g.act(g.conv(a, rnd(576, 64, scale=0.05), rnd(64, scale=0.1), (3, 3), pads=(1, 1, 1, 1)), "relu")
    a = g.pool(a, "max", (2, 2), (2, 2))
    g.act(g.conv(a, rnd(576, 128, scale=0.05), rnd(128, scale=0.1), (3, 3), pads=(1, 1, 1, 1)), "relu")
    run(g, rnd(3 * 1024, 3), tol=1e-5)


def test_pool_then_conv(run):
    g = G((32, 32, 64))
    a = g.pool(0, "max", (2, 2), (2, 2))
    g.conv(a, rnd(576, 128, scale=0.05), rnd(128, scale=0.1), (3, 3), pads=(1, 1, 1, 1))
    run(g, rnd(3 * 1024, 64), tol=1e-5)


@pytest.mark.parametrize("B", [1, 2, 3])
def test_attention_composition_by_hand(libkx, B):
    """fused QKV GEMM -> packed attention core -> output GEMM, driven through the kernel ABI with torch buffers"""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from kernix_b200 import kx_abi as kx
    keep = []

    def dev(a):
        t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
        keep.append(t)
        return t

    def prep(w):
        k, n = w.shape
        ldw = (k + 31) // 32 * 32
        hi = torch.empty((n, ldw), device="cuda")
        lo = torch.empty((n, ldw), device="cuda")
        keep.extend([hi, lo])
        kx.call("kx_prep_f32_weight", dev(w).data_ptr(), k, n, hi.data_ptr(), lo.data_ptr(), ldw, None)
        return hi, lo, ldw

    d, H, S = 512, 8, 128
    dk = d // H
    x = rnd(B * S, d)
    w = [rnd(d, d, scale=0.05, seed=i) for i in range(4)]
    b = [rnd(d, scale=0.1, seed=10 + i) for i in range(4)]
    wqkv = np.concatenate(w[:3], axis=1)
    bqkv = np.concatenate(b[:3])
    hi, lo, ldw = prep(wqkv)
    qkv = torch.empty((B * S, 3 * d), device="cuda")
    kx.call("kx_gemm_f32", dev(x).data_ptr(), d, hi.data_ptr(), lo.data_ptr(), ldw, dev(bqkv).data_ptr(), qkv.data_ptr(), 3 * d,
            B * S, 3 * d, d, -1, 0.0, None, None)
    torch.cuda.synchronize()
    want_qkv = x.astype(np.float64) @ wqkv + bqkv
    assert rel_err(qkv.cpu().numpy(), want_qkv) <= 1e-5, "QKV GEMM"
    ctx = torch.empty((B * S, d), device="cuda")
    base = qkv.data_ptr()
    kx.call("kx_attention", base, 3 * d, base + 4 * d, 3 * d, base + 8 * d, 3 * d, ctx.data_ptr(), d, B, S, S, H, dk, dk, 0, None,
            None)
    torch.cuda.synchronize()
    Q, K, V = (want_qkv[:, i * d:(i + 1) * d].reshape(B, S, H, dk).transpose(0, 2, 1, 3) for i in range(3))
    P = Q @ K.transpose(0, 1, 3, 2) / np.sqrt(dk)
    P = np.exp(P - P.max(-1, keepdims=True))
    P /= P.sum(-1, keepdims=True)
    want_ctx = (P @ V).transpose(0, 2, 1, 3).reshape(B * S, d)
    assert rel_err(ctx.cpu().numpy(), want_ctx) <= TF32_LONG_K, "attention core"
    hi2, lo2, ldw2 = prep(w[3])
    y = torch.empty((B * S, d), device="cuda")
    kx.call("kx_gemm_f32", ctx.data_ptr(), d, hi2.data_ptr(), lo2.data_ptr(), ldw2, dev(b[3]).data_ptr(), y.data_ptr(), d,
            B * S, d, d, -1, 0.0, None, None)
    torch.cuda.synchronize()
    assert rel_err(y.cpu().numpy(), want_ctx @ w[3].astype(np.float64) + b[3]) <= TF32_LONG_K, "output GEMM"


@pytest.mark.parametrize("variant", ["conv2_pool_conv3", "conv1_conv2_conv3", "conv1_pool_conv3", "conv3_conv3"])
def test_conv_sequences(run, variant):
    w1, b1 = rnd(27, 64, scale=0.3), rnd(64, scale=0.1)
    w2, b2 = rnd(576, 64, scale=0.05), rnd(64, scale=0.1)
    w3, b3 = rnd(576, 128, scale=0.05), rnd(128, scale=0.1)
    w4, b4 = rnd(1152, 128, scale=0.03), rnd(128, scale=0.1)
    pads = (1, 1, 1, 1)
    if variant == "conv2_pool_conv3":
        g = G((32, 32, 64))
        a = g.act(g.conv(0, w2, b2, (3, 3), pads=pads), "relu")
        a = g.pool(a, "max", (2, 2), (2, 2))
        g.conv(a, w3, b3, (3, 3), pads=pads)
        x = rnd(2 * 1024, 64)
    elif variant == "conv1_conv2_conv3":
        g = G((32, 32, 3))
        a = g.act(g.conv(0, w1, b1, (3, 3), pads=pads), "relu")
        a = g.act(g.conv(a, w2, b2, (3, 3), pads=pads), "relu")
        g.conv(a, w3, b3, (3, 3), pads=pads)
        x = rnd(2 * 1024, 3)
    elif variant == "conv1_pool_conv3":
        g = G((32, 32, 3))
        a = g.act(g.conv(0, w1, b1, (3, 3), pads=pads), "relu")
        a = g.pool(a, "max", (2, 2), (2, 2))
        g.conv(a, w3, b3, (3, 3), pads=pads)
        x = rnd(2 * 1024, 3)
    else:
        g = G((16, 16, 64))
        a = g.act(g.conv(0, w3, b3, (3, 3), pads=pads), "relu")
        g.conv(a, w4, b4, (3, 3), pads=pads)
        x = rnd(2 * 256, 64)
    run(g, x, tol=TF32_LONG_K)


def test_conv_sequence_by_hand(libkx):
    """conv(64->64) then conv(64->128) with the same kernel template, driven through the kernel ABI"""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from kernix_b200 import kx_abi as kx
    keep = []

    def dev(a):
        t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
        keep.append(t)
        return t

    def prep(w):
        k, n = w.shape
        ldw = (k + 31) // 32 * 32
        hi = torch.empty((n, ldw), device="cuda")
        lo = torch.empty((n, ldw), device="cuda")
        keep.extend([hi, lo])
        kx.call("kx_prep_f32_weight", dev(w).data_ptr(), k, n, hi.data_ptr(), lo.data_ptr(), ldw, None)
        return hi, lo, ldw

    B, H = 2, 16
    x = rnd(B * H * H, 64)
    w2, b2 = rnd(576, 64, scale=0.05), rnd(64, scale=0.1)
    w3, b3 = rnd(576, 128, scale=0.05), rnd(128, scale=0.1)
    h2, l2, ld2 = prep(w2)
    h3, l3, ld3 = prep(w3)
    y2 = torch.empty((B * H * H, 64), device="cuda")
    y3 = torch.empty((B * H * H, 128), device="cuda")
    dx = dev(x)
    db2, db3 = dev(b2), dev(b3)
    kx.call("kx_conv_f32", dx.data_ptr(), h2.data_ptr(), l2.data_ptr(), ld2, db2.data_ptr(), y2.data_ptr(), B, H, H, 64, 64,
            H, H, 3, 3, 1, 1, 1, 1, 1, 1, 1, 0, 0.0, None, None)
    kx.call("kx_conv_f32", y2.data_ptr(), h3.data_ptr(), l3.data_ptr(), ld3, db3.data_ptr(), y3.data_ptr(), B, H, H, 64, 128,
            H, H, 3, 3, 1, 1, 1, 1, 1, 1, 1, -1, 0.0, None, None)
    torch.cuda.synchronize()
    mk = lambda w, b, act: dict(groups=1, kh=3, kw=3, sh=1, sw=1, dh=1, dw=1, pt=1, pb=1, pl=1, pr=1, w=("f32", w), bias=b,  # noqa: E731
                                act=act, alpha=0.0)
    want2 = ko.conv(mk(w2, b2, 0), ko._val([H, H, 64]), ko._val([H, H, 64]), x)
    assert rel_err(y2.cpu().numpy(), want2) <= 1e-5, "first conv"
    want3 = ko.conv(mk(w3, b3, -1), ko._val([H, H, 64]), ko._val([H, H, 128]), want2)
    assert rel_err(y3.cpu().numpy(), want3) <= 1e-5, "second conv"


def test_conv_three_launches_by_hand(libkx):
    """conv(3->64), conv(64->64), conv(64->128): three launches of one kernel template, through the kernel ABI"""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from kernix_b200 import kx_abi as kx
    keep = []

    def dev(a):
        t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
        keep.append(t)
        return t

    def prep(w):
        k, n = w.shape
        ldw = (k + 31) // 32 * 32
        hi = torch.empty((n, ldw), device="cuda")
        lo = torch.empty((n, ldw), device="cuda")
        keep.extend([hi, lo])
        kx.call("kx_prep_f32_weight", dev(w).data_ptr(), k, n, hi.data_ptr(), lo.data_ptr(), ldw, None)
        return hi, lo, ldw

    B, H = 2, 32
    x = rnd(B * H * H, 3)
    specs = [(3, 64, rnd(27, 64, scale=0.3), rnd(64, scale=0.1)), (64, 64, rnd(576, 64, scale=0.05), rnd(64, scale=0.1)),
             (64, 128, rnd(576, 128, scale=0.05), rnd(128, scale=0.1))]
    cur, want = dev(x), x
    mk = lambda w, b: dict(groups=1, kh=3, kw=3, sh=1, sw=1, dh=1, dw=1, pt=1, pb=1, pl=1, pr=1, w=("f32", w), bias=b,  # noqa: E731
                           act=0, alpha=0.0)
    for i, (ci, co, w, b) in enumerate(specs):
        hi, lo, ldw = prep(w)
        y = torch.empty((B * H * H, co), device="cuda")
        keep.append(y)
        kx.call("kx_conv_f32", cur.data_ptr(), hi.data_ptr(), lo.data_ptr(), ldw, dev(b).data_ptr(), y.data_ptr(), B, H, H, ci,
                co, H, H, 3, 3, 1, 1, 1, 1, 1, 1, 1, 0, 0.0, None, None)
        torch.cuda.synchronize()
        want = ko.conv(mk(w, b), ko._val([H, H, ci]), ko._val([H, H, co]), want)
        assert rel_err(y.cpu().numpy(), want) <= 2e-5, f"conv {i}"
        cur = y
