"""GPU backend of the reference's 2-D tensor library (include/kernix_gpu.h; reference include/kernix.h:30-37, 409-423,
936-990 and src/kernix_metal.m): the element-wise map ops, the row ops and the transpose on backend storage, the
hand-over rules (what the backend leaves to the caller's CPU code), the matmul entries and the storage cache.
Expected values are numpy restatements of the reference's formulas."""
import ctypes

import numpy as np
import pytest

from conftest import rel_err

F32 = np.float32

pytestmark = pytest.mark.gpu

N_MIN = 1 << 22  # the reference's GPU threshold (elements)
NEG, ABS, EXP, LOG, SQRT, TANH, RELU, SIGMOID, SILU, GELU, ADD_S, MUL_S, CLAMP, ADD, SUB, MUL, DIV = range(17)


class FloatTensor(ctypes.Structure):
    _fields_ = [("row", ctypes.c_int), ("col", ctypes.c_int), ("tensor", ctypes.POINTER(ctypes.c_float))]


ROWS_FN = ctypes.CFUNCTYPE(None, ctypes.c_size_t, ctypes.c_size_t)


@pytest.fixture(scope="module")
def L():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from kernix_b200 import kernix
    L = kernix.lib()
    vp, sz, f, i = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_float, ctypes.c_int
    L.kernix_metal_alloc.argtypes, L.kernix_metal_alloc.restype = [sz], vp
    L.kernix_metal_free.argtypes, L.kernix_metal_free.restype = [vp], i
    L.kernix_metal_release_cache.argtypes, L.kernix_metal_release_cache.restype = [], None
    L.kernix_metal_map.argtypes, L.kernix_metal_map.restype = [i, vp, vp, sz, vp, sz, f, f], sz
    L.kernix_metal_rows.argtypes, L.kernix_metal_rows.restype = [i, vp, vp, vp, f, vp, sz, sz], i
    L.kernix_metal_transpose.argtypes, L.kernix_metal_transpose.restype = [vp, vp, sz, sz], i
    pt = ctypes.POINTER(FloatTensor)
    L.kernix_matmul_ep_into.argtypes, L.kernix_matmul_ep_into.restype = [pt, pt, pt, vp, i, f, ROWS_FN], i
    L.float_matmul_metal.argtypes, L.float_matmul_metal.restype = [pt, pt], pt
    L.floats_fma_relu_metal.argtypes, L.floats_fma_relu_metal.restype = [pt, pt, pt], pt
    L.float_free.argtypes, L.float_free.restype = [pt], None
    return L


def backend(L, n, fill=None):
    """n floats of backend storage as (pointer, numpy view)."""
    p = L.kernix_metal_alloc(n * 4)
    assert p
    a = np.ctypeslib.as_array((ctypes.c_float * n).from_address(p))
    if fill is not None:
        a[:] = fill
    return p, a


def tensor(a):
    a = np.ascontiguousarray(a, dtype=F32)
    t = FloatTensor(a.shape[0], a.shape[1], a.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
    t._keep = a
    return t


def gelu_as(x):
    x = x.astype(np.float64)
    z = np.abs(x) * 0.70710678
    k = 1.0 / (1.0 + 0.3275911 * z)
    p = k * (0.254829592 + k * (-0.284496736 + k * (1.421413741 + k * (-1.453152027 + k * 1.061405429))))
    return 0.5 * x * (1.0 + np.copysign(1.0 - p * np.exp(-z * z), x))


@pytest.mark.parametrize("op", range(17))
def test_map_ops(L, op):
    n = N_MIN + 6
    rng = np.random.default_rng(op)
    xv = rng.standard_normal(n).astype(F32) * 3
    if op in (LOG, SQRT):
        xv = np.abs(xv) + 0.01
    px, x = backend(L, n, xv)
    py, y = backend(L, n, -7.0)
    bcols = 1024 if op in (ADD, MUL) else 0  # row broadcast for two of the binary ops
    bv = rng.standard_normal(bcols or n).astype(F32)
    if op == DIV:
        bv = np.where(np.abs(bv) < 0.1, 0.5, bv).astype(F32)
    b = np.ascontiguousarray(bv)  # ordinary host memory: the backend copies it
    done = L.kernix_metal_map(op, px, b.ctypes.data if op >= ADD else None, bcols, py, n, 0.75, 1.5)
    assert done == n - 2, "the float4 prefix is done on the GPU, the tail is left to the caller"
    assert np.all(y[done:] == -7.0)
    xs, ys = x[:done], y[:done]
    bb = np.tile(bv, done // bcols + 1)[:done] if bcols else bv[:done]
    exact = {NEG: -xs, ABS: np.abs(xs), RELU: np.maximum(xs, 0), ADD_S: xs + F32(0.75), MUL_S: xs * F32(0.75),
             CLAMP: np.clip(xs, F32(0.75), F32(1.5)), ADD: xs + bb, SUB: xs - bb, MUL: xs * bb, DIV: xs / bb, SQRT: np.sqrt(xs)}
    if op in exact:
        assert np.array_equal(ys, exact[op].astype(F32))
    else:
        x64 = xs.astype(np.float64)
        want = {EXP: np.exp(x64), LOG: np.log(x64), TANH: np.tanh(x64), SIGMOID: 1 / (1 + np.exp(-x64)),
                SILU: x64 / (1 + np.exp(-x64)), GELU: gelu_as(xs)}[op]
        if op == GELU:  # 1 + copysign(1 - p e^-z^2, x) cancels for x << 0 in fp32: compare against the output scale
            assert rel_err(ys, want) <= 2e-6
        else:
            assert np.max(np.abs(ys - want) / np.maximum(np.abs(want), 1e-30)) <= 2e-6
    assert L.kernix_metal_free(px) == 1 and L.kernix_metal_free(py) == 1


def test_map_hand_over_rules(L):
    """Below 2^22 elements, with a broadcast width not a multiple of 4, or into memory that is not backend storage,
    the backend does nothing and returns 0 (the caller's CPU code computes every element)."""
    n = N_MIN
    px, x = backend(L, n, 1.0)
    py, y = backend(L, n, 0.0)
    host = np.zeros(n, F32)
    b = np.ones(6, F32)
    assert L.kernix_metal_map(NEG, px, None, 0, py, n - 4, 0, 0) == 0
    assert L.kernix_metal_map(ADD, px, b.ctypes.data, 6, py, n, 0, 0) == 0
    assert L.kernix_metal_map(NEG, px, None, 0, host.ctypes.data, n, 0, 0) == 0
    assert np.all(y == 0) and np.all(host == 0)
    assert L.kernix_metal_map(NEG, host.ctypes.data, None, 0, py, n, 0, 0) == n  # a host input is copied in
    assert np.all(y == 0.0)
    L.kernix_metal_free(px)
    L.kernix_metal_free(py)


@pytest.mark.parametrize("mode,affine", [(0, False), (1, False), (2, False), (2, True)])
def test_rows(L, mode, affine):
    rows, cols = 4096, 1030
    rng = np.random.default_rng(mode)
    xv = (rng.standard_normal((rows, cols)) * 4).astype(F32)
    px, x = backend(L, rows * cols, xv.ravel())
    py, y = backend(L, rows * cols, 0.0)
    g = rng.standard_normal(cols).astype(F32) if affine else None
    bt = rng.standard_normal(cols).astype(F32) if affine else None
    ok = L.kernix_metal_rows(mode, px, g.ctypes.data if affine else None, bt.ctypes.data if affine else None, 1e-5, py,
                             rows, cols)
    assert ok == 1
    x64 = xv.astype(np.float64)
    if mode < 2:
        m = x64.max(1, keepdims=True)
        s = np.exp(x64 - m).sum(1, keepdims=True)
        want = np.exp(x64 - m) / s if mode == 0 else x64 - m - np.log(s)
    else:
        mu = x64.mean(1, keepdims=True)
        want = (x64 - mu) / np.sqrt(((x64 - mu) ** 2).mean(1, keepdims=True) + 1e-5)
        if affine:
            want = want * g + bt
    assert rel_err(y.reshape(rows, cols), want) <= 2e-6
    assert L.kernix_metal_rows(mode, px, None, None, 1e-5, px, rows, cols) == 0  # in place: left to the CPU
    L.kernix_metal_free(px)
    L.kernix_metal_free(py)


def test_transpose(L):
    rows, cols = 2049, 2050
    xv = np.arange(rows * cols, dtype=np.float64).astype(F32)
    px, x = backend(L, rows * cols, xv)
    py, y = backend(L, rows * cols, 0.0)
    assert L.kernix_metal_transpose(px, py, rows, cols) == 1
    assert np.array_equal(y.reshape(cols, rows), xv.reshape(rows, cols).T)
    assert L.kernix_metal_transpose(px, py, 100, 100) == 0
    L.kernix_metal_free(px)
    L.kernix_metal_free(py)


@pytest.mark.parametrize("m,k,n,act,bias", [(300, 700, 520, 0, True), (5, 3, 7, -1, False), (1024, 2048, 64, 1, True)])
def test_matmul_ep_into(L, m, k, n, act, bias):
    """c = act(a . b + bias) entirely on the GPU (3xTF32): within 1e-5 of float64, cpu_ep never called."""
    rng = np.random.default_rng(m + k + n)
    a = rng.standard_normal((m, k)).astype(F32)
    b = (rng.standard_normal((k, n)) / np.sqrt(k)).astype(F32)
    bv = rng.standard_normal(n).astype(F32) if bias else None
    c = np.zeros((m, n), F32)
    calls = []
    cb = ROWS_FN(lambda r0, r1: calls.append((r0, r1)))
    ta, tb, tc = tensor(a), tensor(b), tensor(c)
    assert L.kernix_matmul_ep_into(ctypes.byref(ta), ctypes.byref(tb), ctypes.byref(tc), bv.ctypes.data if bias else None, act,
                                   0.0, cb) == 0
    want = a.astype(np.float64) @ b + (bv if bias else 0)
    if act == 0:
        want = np.maximum(want, 0)
    elif act == 1:
        want = gelu_as(want.astype(F32))
    assert rel_err(tc._keep, want) <= 1e-5 and calls == []


def test_matmul_inner_zero_and_mismatch(L):
    calls = []
    cb = ROWS_FN(lambda r0, r1: calls.append((r0, r1)))
    a, b, c = tensor(np.zeros((4, 0), F32).reshape(4, 0)), tensor(np.zeros((0, 3), F32).reshape(0, 3)), tensor(np.full((4, 3), 9, F32))
    assert L.kernix_matmul_ep_into(ctypes.byref(a), ctypes.byref(b), ctypes.byref(c), None, -1, 0.0, cb) == 0
    assert np.all(c._keep == 0) and calls == [(0, 4)]
    a2, b2 = tensor(np.ones((2, 3), F32)), tensor(np.ones((4, 2), F32))
    assert L.kernix_matmul_ep_into(ctypes.byref(a2), ctypes.byref(b2), ctypes.byref(c), None, -1, 0.0, cb) == -1


def test_float_matmul_and_fma_relu(L):
    rng = np.random.default_rng(9)
    a = rng.standard_normal((130, 300)).astype(F32)
    b = rng.standard_normal((300, 200)).astype(F32)
    r = L.float_matmul_metal(ctypes.byref(tensor(a)), ctypes.byref(tensor(b)))
    assert r and r.contents.row == 130 and r.contents.col == 200
    got = np.ctypeslib.as_array(r.contents.tensor, shape=(130 * 200,)).reshape(130, 200).copy()
    L.float_free(r)
    assert rel_err(got, a.astype(np.float64) @ b) <= 1e-5
    for shape in ((3, 5), (1024, 2048)):  # below and above the backend-storage size
        va, vx, vb = (rng.standard_normal(shape).astype(F32) for _ in range(3))
        r = L.floats_fma_relu_metal(ctypes.byref(tensor(va)), ctypes.byref(tensor(vx)), ctypes.byref(tensor(vb)))
        assert r
        got = np.ctypeslib.as_array(r.contents.tensor, shape=(shape[0] * shape[1],)).reshape(shape).copy()
        L.float_free(r)
        want = np.maximum(va.astype(np.float64) * vx + vb, 0)
        assert rel_err(got, want) <= 1e-7


def test_storage_cache(L):
    p = L.kernix_metal_alloc(1 << 20)
    assert p and L.kernix_metal_free(p) == 1
    q = L.kernix_metal_alloc(1 << 20)
    assert q == p  # a freed buffer of the same size is reused
    host = np.zeros(4, F32)
    assert L.kernix_metal_free(host.ctypes.data) == 0 and L.kernix_metal_free(None) == 0
    L.kernix_metal_free(q)
    L.kernix_metal_release_cache()
