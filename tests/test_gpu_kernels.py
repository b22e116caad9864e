"""GPU parity of each kernel, called through the kernel-level C ABI (include/kx_kernels.h), against the oracle
(oracle/knx_oracle.py) or a float64 reference of the same op. Integer work (int8 quantisation, int32
accumulators) must be bit-exact; float work within the tolerance stated per test."""
import numpy as np
import pytest

from conftest import rel_err
from oracle import knx_oracle as ko

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

F32 = np.float32


@pytest.fixture(scope="module")
def kx(libkx):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from kernix_b200 import kx_abi
    return kx_abi


_KEEP = []  # device tensors passed by raw pointer must outlive the asynchronous launches that read them


@pytest.fixture(autouse=True)
def _release_after_test():
    yield
    torch.cuda.synchronize()
    _KEEP.clear()


def dev(a):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    _KEEP.append(t)
    return t


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def sp():
    return torch.cuda.current_stream().cuda_stream


def status():
    return torch.zeros(1, dtype=torch.int32, device="cuda")


def check_status(st):
    assert int(st.item()) == 0, "kernel reported a timeout"


# ------------------------------------------------------------------------------------------ int8
def _quant(kx, x, ldq):
    rows, k = x.shape
    dx = dev(x)
    xq = torch.full((rows, ldq), 99, dtype=torch.int8, device="cuda")
    sx = torch.empty(rows, dtype=torch.float32, device="cuda")
    kx.call("kx_quant_rows", dx.data_ptr(), k, rows, k, xq.data_ptr(), ldq, sx.data_ptr(), sp())
    return host(xq), host(sx)


@pytest.mark.parametrize("rows,k", [(7, 1024), (33, 55), (5, 4096), (3, 5000), (2, 16)])
def test_quant_rows_bitexact(kx, rows, k):
    rng = np.random.default_rng(rows * 1000 + k)
    x = (rng.standard_normal((rows, k)) * rng.uniform(0.01, 10, (rows, 1))).astype(F32)
    x[0, :] = 0.0                      # zero row: sx = 1, all zeros
    if rows > 2:
        x[1, k // 2] = np.nan          # NaN row
        x[2, 0] = np.inf               # infinite row
    # values exactly on rounding ties after scaling
    x[-1, : min(k, 8)] = np.array([0.5, -0.5, 1.5, -2.5, 127, -127, 63.5, 0.0], F32)[: min(k, 8)]
    ldq = (k + 15) // 16 * 16
    xq, sx = _quant(kx, x, ldq)
    wq, wsx, bad = ko.quantize_rows(x)
    assert np.array_equal(xq[~bad, :k], wq[~bad]), "int8 values differ"
    assert np.array_equal(sx[~bad].view(np.uint32), wsx[~bad].view(np.uint32)), "row scales differ"
    assert np.all(np.isnan(sx[bad]))
    assert np.all(xq[:, k:] == 0), "padding columns must be zero"


def _prep_i8(kx, q):
    k, n = q.shape
    ldw = (k + 15) // 16 * 16
    wq = torch.empty((n, ldw), dtype=torch.int8, device="cuda")
    kx.call("kx_prep_i8_weight", dev(q).data_ptr(), k, n, wq.data_ptr(), ldw, sp())
    return wq, ldw


@pytest.mark.parametrize("m,k,n", [(300, 1000, 520), (128, 256, 256), (5, 55, 31), (1, 16, 16), (130, 4096, 384),
                                   (2100, 1024, 4100), (1500, 4096, 4096)])
def test_gemm_i8_accumulators_bitexact(kx, m, k, n):
    """int32 sums bit-exact; N > 128 runs on CTA pairs (256 x 256 tiles): ragged pair tiles whose second CTA's rows
    or columns lie wholly outside the matrix, and several tiles per cluster (both accumulator buffers reused)."""
    rng = np.random.default_rng(m + k + n)
    xq = rng.integers(-127, 128, (m, k), dtype=np.int8)
    q = rng.integers(-127, 128, (k, n), dtype=np.int8)
    ldq = (k + 15) // 16 * 16
    xqp = np.zeros((m, ldq), np.int8)
    xqp[:, :k] = xq
    wq, ldw = _prep_i8(kx, q)
    acc = torch.zeros((m, n), dtype=torch.int32, device="cuda")
    st = status()
    kx.call("kx_gemm_i8_acc", dev(xqp).data_ptr(), ldq, wq.data_ptr(), ldw, acc.data_ptr(), n, m, n, k, st.data_ptr(), sp())
    got = host(acc)
    check_status(st)
    assert np.array_equal(got, ko.int8_acc(xq, q))


def test_gemm_i8_int32_overflow_edge(kx):
    """reference test/model_test.c:430-440: K = 131072, q = -128, x = 1 stays inside int32."""
    k, n = ko.INT8_MAX_K, 16
    xq = np.full((1, k), 127, np.int8)
    q = np.full((k, n), -128, np.int8)
    wq, ldw = _prep_i8(kx, q)
    acc = torch.zeros((1, n), dtype=torch.int32, device="cuda")
    kx.call("kx_gemm_i8_acc", dev(xq).data_ptr(), k, wq.data_ptr(), ldw, acc.data_ptr(), n, 1, n, k, None, sp())
    assert np.all(host(acc) == -128 * 127 * k)


@pytest.mark.parametrize("act", [ko.ACT_NONE, 0, 1])
@pytest.mark.parametrize("m,k,n,bias", [(257, 1024, 4096, True), (33, 55, 31, False), (3, 128, 1000, True)])
def test_gemm_i8_dequant_epilogue(kx, m, k, n, bias, act):
    """quantise + int8 GEMM + ((float)acc*sx)*scale + bias (+act) vs the oracle's kernix_qmatmul restatement."""
    rng = np.random.default_rng(m * n + k)
    x = rng.standard_normal((m, k)).astype(F32)
    x[0] = 0.0
    if m > 2:
        x[1, 3] = np.nan
    w = (rng.standard_normal((k, n)) * 0.02).astype(F32)
    from kernix_b200.knx_writer import quantize_int8
    scale, q = quantize_int8(w)
    b = rng.standard_normal(n).astype(F32) if bias else None
    ldq = (k + 15) // 16 * 16
    dx = dev(x)
    xq = torch.empty((m, ldq), dtype=torch.int8, device="cuda")
    sx = torch.empty(m, dtype=torch.float32, device="cuda")
    kx.call("kx_quant_rows", dx.data_ptr(), k, m, k, xq.data_ptr(), ldq, sx.data_ptr(), sp())
    wq, ldw = _prep_i8(kx, q)
    dscale = dev(scale)
    db = dev(b) if bias else None
    y = torch.empty((m, n), dtype=torch.float32, device="cuda")
    st = status()
    kx.call("kx_gemm_i8", xq.data_ptr(), ldq, sx.data_ptr(), wq.data_ptr(), ldw, dscale.data_ptr(),
            db.data_ptr() if bias else None, y.data_ptr(), n, m, n, k, act, 0.0, st.data_ptr(), sp())
    got = host(y)
    check_status(st)
    want = ko.act(ko.qlinear(x, q, scale, b), act)
    if act in (ko.ACT_NONE, 0):  # same IEEE operations in the same order: bit-exact
        assert np.array_equal(np.isnan(got), np.isnan(want))
        assert np.array_equal(np.nan_to_num(got), np.nan_to_num(want))
    else:  # GELU uses the device expf (a few ulp from glibc's)
        assert rel_err(got, want) <= 1e-6


@pytest.mark.parametrize("m,k,n,act", [(64, 1024, 4096, 1), (33, 55, 31, -1), (300, 4096, 1024, 0)])
def test_linear_i8_step(kx, m, k, n, act):
    """kx_linear_i8 (quantise + int8 GEMM, caller scratch) == the oracle's kernix_qmatmul + activation"""
    rng = np.random.default_rng(k + n)
    x = (rng.standard_normal((m, k)) * rng.uniform(0.1, 4, (m, 1))).astype(F32)
    from kernix_b200.knx_writer import quantize_int8
    scale, q = quantize_int8((rng.standard_normal((k, n)) * 0.02).astype(F32))
    b = rng.standard_normal(n).astype(F32)
    wq, ldw = _prep_i8(kx, q)
    ldq = (k + 15) // 16 * 16
    xq = torch.empty((m, ldq), dtype=torch.int8, device="cuda")
    sx = torch.empty(m, dtype=torch.float32, device="cuda")
    y = torch.empty((m, n), dtype=torch.float32, device="cuda")
    st = status()
    kx.call("kx_linear_i8", dev(x).data_ptr(), k, m, k, wq.data_ptr(), ldw, dev(scale).data_ptr(), dev(b).data_ptr(),
            y.data_ptr(), n, n, act, 0.0, xq.data_ptr(), sx.data_ptr(), st.data_ptr(), sp())
    got = host(y)
    check_status(st)
    want = ko.act(ko.qlinear(x, q, scale, b), act)
    if act == 1:
        assert rel_err(got, want) <= 1e-6
    else:
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


# ------------------------------------------------------------------------------------------ fp32
def _prep_f32(kx, w):
    k, n = w.shape
    ldw = (k + 31) // 32 * 32
    hi = torch.empty((n, ldw), dtype=torch.float32, device="cuda")
    lo = torch.empty((n, ldw), dtype=torch.float32, device="cuda")
    kx.call("kx_prep_f32_weight", dev(w).data_ptr(), k, n, hi.data_ptr(), lo.data_ptr(), ldw, sp())
    return hi, lo, ldw


def test_prep_f32_split_is_exact(kx):
    rng = np.random.default_rng(5)
    w = (rng.standard_normal((37, 19)) * 10.0 ** rng.integers(-8, 8, (37, 19))).astype(F32)
    hi, lo, ldw = _prep_f32(kx, w)
    h, lo_ = host(hi), host(lo)
    assert np.array_equal((h[:, :37] + lo_[:, :37]).T, w), "hi + lo must reproduce w exactly"
    assert np.all(h.view(np.uint32) & 0x1FFF == 0), "hi must be a tf32 value"
    assert np.all(h[:, 37:] == 0) and np.all(lo_[:, 37:] == 0)


@pytest.mark.parametrize("m,k,n", [(256, 784, 512), (300, 27, 64), (129, 250, 10), (1, 2048, 300), (512, 512, 1536),
                                   (256, 512, 1536), (256, 2048, 512), (64, 16384, 300), (130, 5000, 520), (300, 8192, 260)])
@pytest.mark.parametrize("act", [ko.ACT_NONE, 0])
def test_gemm_f32_3xtf32(kx, m, k, n, act):
    """3xTF32 GEMM + bias + act vs float64: max abs error <= 1e-5 x output scale (the dense-MLP bound). tcgen05's
    truncating fp32 accumulation adds ~2e-9 * (accumulation length): reductions longer than 2048 drain their
    partial sums every 256 and meet 1e-5 up to K = 16384."""
    rng = np.random.default_rng(m + 7 * k + n)
    x = rng.standard_normal((m, k)).astype(F32)
    w = (rng.standard_normal((k, n)) / np.sqrt(k)).astype(F32)
    b = rng.standard_normal(n).astype(F32)
    hi, lo, ldw = _prep_f32(kx, w)
    y = torch.empty((m, n), dtype=torch.float32, device="cuda")
    st = status()
    db = dev(b)
    kx.call("kx_gemm_f32", dev(x).data_ptr(), k, hi.data_ptr(), lo.data_ptr(), ldw, db.data_ptr(), y.data_ptr(), n, m, n, k,
            act, 0.0, st.data_ptr(), sp())
    got = host(y)
    check_status(st)
    ref = x.astype(np.float64) @ w.astype(np.float64) + b
    if act == 0:
        ref = np.maximum(ref, 0)
    assert rel_err(got, ref) <= 1e-5


@pytest.mark.parametrize("m,k,n,act,splits", [(64, 16384, 4096, 0, 4), (64, 16384, 8192, -1, 2), (128, 8192, 1024, 0, 4),
                                              (17, 5000, 520, 1, 4), (100, 2048, 300, -1, 2), (64, 3000, 260, 0, 3),
                                              (50, 2100, 130, 0, 4), (1, 4096, 64, -1, 4)])
def test_gemm_f32_split_k(kx, m, k, n, act, splits):
    """kx_gemm_f32_split: the reduction cut into `splits` ranges of whole 256-column chunks (ragged last range; fewer
    ranges than asked when K is short), each run by its own CTAs into a partial-sum plane, the planes then added in
    range order with bias and activation: within the same 1e-5 bound of float64 as the unsplit kernel, and the same
    bits on a second call (a fixed order of additions)."""
    rng = np.random.default_rng(m + 3 * k + n + splits)
    x = rng.standard_normal((m, k)).astype(F32)
    w = (rng.standard_normal((k, n)) / np.sqrt(k)).astype(F32)
    b = rng.standard_normal(n).astype(F32)
    hi, lo, ldw = _prep_f32(kx, w)
    part = torch.full((splits * m * n,), float("nan"), dtype=torch.float32, device="cuda")
    st = status()
    dx, db = dev(x), dev(b)
    outs = []
    for _ in range(2):
        y = torch.empty((m, n), dtype=torch.float32, device="cuda")
        kx.call("kx_gemm_f32_split", dx.data_ptr(), k, hi.data_ptr(), lo.data_ptr(), ldw, db.data_ptr(), y.data_ptr(), n, m,
                n, k, act, 0.0, splits, part.data_ptr(), st.data_ptr(), sp())
        outs.append(host(y))
    check_status(st)
    ref = ko.act((x.astype(np.float64) @ w.astype(np.float64) + b).astype(F32), act) if act == 1 else \
        x.astype(np.float64) @ w.astype(np.float64) + b
    if act == 0:
        ref = np.maximum(ref, 0)
    assert rel_err(outs[0], ref) <= 1e-5
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))


def test_gemm_f32_split_count(kx):
    """The split policy: only <= 128 rows and K >= 2048, only when the output tiles leave SMs idle, at most 4 ranges
    of at least 1024."""
    f = kx.lib().kx_gemm_f32_splits
    assert torch.cuda.get_device_properties(0).multi_processor_count == 148
    assert f(200, 4096, 16384) == 1 and f(64, 300, 1024) == 1 and f(64, 16384, 8192) == 1  # 128 tiles: no room
    assert f(64, 4096, 16384) == 4 and f(64, 8192, 16384) == 2  # 32 and 64 tiles of 128 columns
    assert f(1, 128, 2048) == 2 and f(128, 128, 3000) == 2  # ranges of at least 1024


@pytest.mark.parametrize("m,k,n", [(32, 1024, 4096), (32, 4096, 4096), (32, 4096, 1024), (1, 4096, 1024), (77, 2000, 520),
                                   (128, 4096, 300), (5, 96, 100)])
def test_gemm_i8_split_k_is_exact(kx, m, k, n):
    """Small-batch int8 layers with K split over the SMs: the int32 planes add up to kx_gemm_i8_acc's accumulators
    exactly; kx_i8_rows gives kx_gemm_i8's fp32 rows bit for bit (GELU and none), and its quantised rows and row scales
    are kx_quant_rows applied to those rows (as kx_gemm_i8_q's are): a zero row, a NaN row, an inf input included."""
    rng = np.random.default_rng(m + k + n)
    x = rng.standard_normal((m, k)).astype(F32)
    x[0] = 0.0
    if m > 2:
        x[1, 3] = np.nan
        x[2, 5] = np.inf
    from kernix_b200.knx_writer import quantize_int8
    scale, qw = quantize_int8((rng.standard_normal((k, n)) * 0.02).astype(F32))
    b = rng.standard_normal(n).astype(F32) * 0.1
    ldq, ldo = (k + 15) // 16 * 16, (n + 15) // 16 * 16
    xq = torch.empty((m, ldq), dtype=torch.int8, device="cuda")
    sx = torch.empty(m, dtype=torch.float32, device="cuda")
    kx.call("kx_quant_rows", dev(x).data_ptr(), k, m, k, xq.data_ptr(), ldq, sx.data_ptr(), sp())
    wq, ldw = _prep_i8(kx, qw)
    kbs = kx.lib().kx_i8_split_blocks(m, n, k)
    planes = ((k + 127) // 128 + kbs - 1) // kbs
    part = torch.empty((planes, m, n), dtype=torch.int32, device="cuda")
    st = status()
    kx.call("kx_gemm_i8_split_acc", xq.data_ptr(), ldq, wq.data_ptr(), ldw, m, n, k, kbs, part.data_ptr(), st.data_ptr(), sp())
    acc = torch.empty((m, n), dtype=torch.int32, device="cuda")
    kx.call("kx_gemm_i8_acc", xq.data_ptr(), ldq, wq.data_ptr(), ldw, acc.data_ptr(), n, m, n, k, st.data_ptr(), sp())
    check_status(st)
    assert np.array_equal(host(part).astype(np.int64).sum(0).astype(np.int32), host(acc))
    ds, db = dev(scale), dev(b)
    for act in (1, -1):
        want = torch.empty((m, n), dtype=torch.float32, device="cuda")
        kx.call("kx_gemm_i8", xq.data_ptr(), ldq, sx.data_ptr(), wq.data_ptr(), ldw, ds.data_ptr(), db.data_ptr(), want.data_ptr(),
                n, m, n, k, act, 0.0, st.data_ptr(), sp())
        got = torch.empty((m, n), dtype=torch.float32, device="cuda")
        kx.call("kx_i8_rows", part.data_ptr(), planes, m, n, sx.data_ptr(), ds.data_ptr(), db.data_ptr(), act, 0.0, got.data_ptr(),
                n, None, 0, None, sp())
        check_status(st)
        assert np.array_equal(host(got).view(np.uint32), host(want).view(np.uint32)), f"act {act}"
        q_got = torch.full((m, ldo), 7, dtype=torch.int8, device="cuda")
        s_got = torch.empty(m, dtype=torch.float32, device="cuda")
        kx.call("kx_i8_rows", part.data_ptr(), planes, m, n, sx.data_ptr(), ds.data_ptr(), db.data_ptr(), act, 0.0, None, 0,
                q_got.data_ptr(), ldo, s_got.data_ptr(), sp())
        q_want = torch.full((m, ldo), 9, dtype=torch.int8, device="cuda")
        s_want = torch.empty(m, dtype=torch.float32, device="cuda")
        kx.call("kx_quant_rows", want.data_ptr(), n, m, n, q_want.data_ptr(), ldo, s_want.data_ptr(), sp())
        assert np.array_equal(host(q_got), host(q_want)), f"act {act}: int8 rows differ"
        assert np.array_equal(host(s_got).view(np.uint32), host(s_want).view(np.uint32)), f"act {act}: row scales differ"


@pytest.mark.parametrize("m,k,n,act,inplace", [(100, 300, 200, 0, False), (300, 512, 512, -1, True), (4096, 512, 1536, 1, False),
                                               (700, 2500, 130, -1, False), (5000, 1000, 520, 0, True)])
def test_gemm_f32_residual_is_gemm_then_add(kx, m, k, n, act, inplace):
    """kx_gemm_f32_res (a LINEAR step and the ADD that consumes it, in one kernel) gives bitwise what kx_gemm_f32
    followed by the elementwise add gives, on every tile kind (one CTA, CTA pairs, persistent pairs, drained K),
    also in place (y = res)."""
    rng = np.random.default_rng(m + n)
    x = rng.standard_normal((m, k)).astype(F32)
    w = (rng.standard_normal((k, n)) / np.sqrt(k)).astype(F32)
    b = rng.standard_normal(n).astype(F32)
    r = rng.standard_normal((m, n)).astype(F32)
    hi, lo, ldw = _prep_f32(kx, w)
    st = status()
    dx, db = dev(x), dev(b)
    y0 = torch.empty((m, n), dtype=torch.float32, device="cuda")
    kx.call("kx_gemm_f32", dx.data_ptr(), k, hi.data_ptr(), lo.data_ptr(), ldw, db.data_ptr(), y0.data_ptr(), n, m, n, k, act,
            0.0, st.data_ptr(), sp())
    want = (host(y0) + r).astype(F32)
    dr = dev(r)
    y = dr if inplace else torch.empty((m, n), dtype=torch.float32, device="cuda")
    kx.call("kx_gemm_f32_res", dx.data_ptr(), k, hi.data_ptr(), lo.data_ptr(), ldw, db.data_ptr(), y.data_ptr(), n, m, n, k,
            act, 0.0, dr.data_ptr(), n, st.data_ptr(), sp())
    check_status(st)
    assert np.array_equal(host(y), want)


@pytest.mark.parametrize("m,k,n,act", [(4096, 512, 1536, 0), (5000, 1000, 2500, -1), (20000, 100, 1024, 0),
                                       (4352, 1024, 2304, -1)])
def test_gemm_f32_persistent_pairs(kx, m, k, n, act):
    """More 256 x 256 tiles than resident CTA pairs and K <= 1024: the persistent CTA-pair kernel (each cluster walks
    several tiles, a tile's epilogue overlapping the next tile's mainloop, ragged M, N and K), within the same 1e-5
    bound as the other 3xTF32 paths although its three products share one accumulator."""
    rng = np.random.default_rng(m + k + n)
    x = rng.standard_normal((m, k)).astype(F32)
    w = (rng.standard_normal((k, n)) / np.sqrt(k)).astype(F32)
    b = rng.standard_normal(n).astype(F32)
    hi, lo, ldw = _prep_f32(kx, w)
    y = torch.empty((m, n), dtype=torch.float32, device="cuda")
    st = status()
    db = dev(b)
    for _ in range(2):  # twice: the second call reuses the cached launch state
        kx.call("kx_gemm_f32", dev(x).data_ptr(), k, hi.data_ptr(), lo.data_ptr(), ldw, db.data_ptr(), y.data_ptr(), n, m, n,
                k, act, 0.0, st.data_ptr(), sp())
        got = host(y)
        check_status(st)
        ref = x.astype(np.float64) @ w.astype(np.float64) + b
        if act == 0:
            ref = np.maximum(ref, 0)
        assert rel_err(got, ref) <= 1e-5


@pytest.mark.parametrize("m,k,n,act", [(1, 8192, 16384, 0), (5, 1000, 300, -1), (16, 4096, 2050, 0), (3, 77, 9, -1),
                                      (9, 16384, 1024, 0), (8, 300, 4096, 4)])
def test_gemm_f32_skinny(kx, m, k, n, act):
    """Dense layer for <= 16 rows (weight streaming on the CUDA cores, K split over the SMs, partial sums added in
    slice order) vs float64: fp32 fma accumulation, within a few 1e-6 of the output scale."""
    rng = np.random.default_rng(m * 7 + k + n)
    x = rng.uniform(-1, 1, (m, k)).astype(F32)
    w = (rng.standard_normal((k, n)) * np.sqrt(2.0 / k)).astype(F32)
    b = rng.standard_normal(n).astype(F32) * 0.1
    S = kx.lib().kx_skinny_slices(n, k)
    part = torch.empty(S * 16 * n, dtype=torch.float32, device="cuda")
    y = torch.empty((m, n), dtype=torch.float32, device="cuda")
    db, dw = dev(b), dev(w)
    kx.call("kx_gemm_f32_skinny", dev(x).data_ptr(), k, dw.data_ptr(), db.data_ptr(), y.data_ptr(), n, m, n, k, act, 0.0,
            part.data_ptr(), part.numel(), sp())
    ref = ko.act((x.astype(np.float64) @ w.astype(np.float64) + b).astype(F32), act) if act == 4 else \
        x.astype(np.float64) @ w.astype(np.float64) + b
    if act == 0:
        ref = np.maximum(ref, 0)
    assert rel_err(host(y), ref) <= 3e-6  # fp32 fma over up to K / slices terms per thread, like a CPU sgemm


@pytest.mark.parametrize("cfg", [
    dict(B=2, H=8, W=8, C=3, Co=16, k=3, s=1, d=1, p=1, g=1),
    dict(B=3, H=9, W=7, C=64, Co=64, k=3, s=1, d=1, p=1, g=1),
    dict(B=2, H=10, W=10, C=32, Co=48, k=3, s=2, d=1, p=1, g=2),
    dict(B=1, H=12, W=12, C=16, Co=24, k=3, s=1, d=2, p=2, g=1),
    dict(B=2, H=6, W=5, C=8, Co=300, k=2, s=1, d=1, p=0, g=1),
    dict(B=3, H=16, W=16, C=64, Co=128, k=3, s=1, d=1, p=1, g=1),
    dict(B=2, H=8, W=8, C=128, Co=256, k=3, s=1, d=1, p=1, g=1),
    dict(B=5, H=8, W=8, C=128, Co=256, k=3, s=1, d=1, p=1, g=1),
    dict(B=4, H=12, W=12, C=32, Co=48, k=3, s=1, d=1, p=1, g=2),
    # channel-major tiles (at most 128 channels per group, more than 128 pixels, K <= 2048)
    dict(B=2, H=32, W=32, C=64, Co=64, k=3, s=1, d=1, p=1, g=1, a=1),
    dict(B=4, H=16, W=16, C=32, Co=100, k=3, s=1, d=1, p=1, g=1),
    dict(B=3, H=11, W=13, C=6, Co=64, k=3, s=1, d=1, p=1, g=1, a=-1),
    dict(B=2, H=20, W=20, C=64, Co=128, k=3, s=2, d=1, p=1, g=1),
    dict(B=2, H=16, W=16, C=64, Co=64, k=3, s=1, d=1, p=1, g=4, a=1),
    dict(B=2, H=16, W=16, C=128, Co=128, k=3, s=1, d=1, p=1, g=1),
    dict(B=1, H=30, W=30, C=16, Co=8, k=5, s=1, d=1, p=2, g=1),
    # K = 2304 > 2048 with 64 channels: drained CTA-pair tiles
    dict(B=3, H=8, W=8, C=256, Co=64, k=3, s=1, d=1, p=1, g=1),
    # direct CUDA-core convolution (K <= 32, <= 64 channels): ragged tiles, stride 2, GELU
    dict(B=3, H=13, W=11, C=3, Co=64, k=3, s=2, d=1, p=1, g=1),
    dict(B=4, H=7, W=9, C=2, Co=40, k=3, s=1, d=1, p=1, g=1, a=1),
    dict(B=7, H=32, W=32, C=3, Co=64, k=3, s=1, d=1, p=1, g=1),
    # planes + TMA boxes (kx_conv_f32_ws): several images per tile, no padding, dilation, groups of 32 channels
    dict(B=5, H=8, W=8, C=64, Co=64, k=3, s=1, d=1, p=1, g=1, a=1),
    dict(B=2, H=18, W=18, C=32, Co=64, k=3, s=1, d=1, p=0, g=1),
    dict(B=1, H=16, W=16, C=64, Co=48, k=3, s=1, d=2, p=2, g=1),
    dict(B=3, H=16, W=16, C=64, Co=64, k=3, s=1, d=1, p=1, g=2, a=-1),
])
def test_conv_implicit_gemm(kx, cfg):
    """implicit-GEMM conv (no im2col buffer) vs the oracle's im2col + sgemm restatement of kernix_conv_run."""
    rng = np.random.default_rng(cfg["C"] * cfg["Co"])
    B, H, W, C, Co, kk, s, d, p, g = (cfg[k] for k in ("B", "H", "W", "C", "Co", "k", "s", "d", "p", "g"))
    act = cfg.get("a", 0)
    Ho = (H + 2 * p - d * (kk - 1) - 1) // s + 1
    Wo = (W + 2 * p - d * (kk - 1) - 1) // s + 1
    x = rng.standard_normal((B * H * W, C)).astype(F32)
    K = kk * kk * (C // g)
    w = (rng.standard_normal((K, Co)) / np.sqrt(K)).astype(F32)
    b = rng.standard_normal(Co).astype(F32)
    hi, lo, ldw = _prep_f32(kx, w)
    y = torch.empty((B * Ho * Wo, Co), dtype=torch.float32, device="cuda")
    st = status()
    db = dev(b)
    kx.call("kx_conv_f32", dev(x).data_ptr(), hi.data_ptr(), lo.data_ptr(), ldw, db.data_ptr(), y.data_ptr(), B, H, W, C, Co,
            Ho, Wo, kk, kk, s, s, d, d, p, p, g, act, 0.0, st.data_ptr(), sp())
    got = host(y)
    check_status(st)
    step = dict(kind=ko.OP["CONV"], act=act, alpha=0.0, groups=g, kh=kk, kw=kk, sh=s, sw=s, dh=d, dw=d, pt=p, pb=p, pl=p, pr=p,
                w=("f32", w), bias=b)
    want = ko.conv(step, ko._val([H, W, C]), ko._val([Ho, Wo, Co]), x)
    assert rel_err(got, want) <= 1e-5
    # with scratch for the tf32 planes (TMA-fed tiles where the geometry allows, the same kernels otherwise)
    ws = torch.full((2 * B * H * W * C + 64,), float("nan"), dtype=torch.float32, device="cuda")
    y2 = torch.empty_like(y)
    kx.call("kx_conv_f32_ws", dev(x).data_ptr(), hi.data_ptr(), lo.data_ptr(), ldw, db.data_ptr(), y2.data_ptr(), B, H, W, C,
            Co, Ho, Wo, kk, kk, s, s, d, d, p, p, g, act, 0.0, ws.data_ptr(), ws.numel(), st.data_ptr(), sp())
    check_status(st)
    assert rel_err(host(y2), want) <= 1e-5


# ------------------------------------------------------------------------------------ memory-bound
@pytest.mark.parametrize("act", list(range(-1, 16)))
def test_bias_act_all_activations(kx, act):
    rng = np.random.default_rng(act + 10)
    x = (rng.standard_normal((37, 100)) * 4).astype(F32)
    x[0, :4] = [0.0, -0.0, 25.0, -25.0]
    b = rng.standard_normal(100).astype(F32)
    y = torch.empty_like(dev(x))
    kx.call("kx_bias_act", dev(x).data_ptr(), y.data_ptr(), 37, 100, dev(b).data_ptr(), act, 0.3, sp())
    want = ko.act((x + b).astype(F32), act, 0.3)
    assert rel_err(host(y), want) <= 2e-6


@pytest.mark.parametrize("rows,cols", [(256, 10), (64, 512), (7, 3000), (3, 1)])
def test_softmax_layernorm_rows(kx, rows, cols):
    rng = np.random.default_rng(rows + cols)
    x = (rng.standard_normal((rows, cols)) * 3).astype(F32)
    g = rng.standard_normal(cols).astype(F32)
    b = rng.standard_normal(cols).astype(F32)
    d = dev(x)
    y = torch.empty_like(d)
    kx.call("kx_softmax_rows", d.data_ptr(), y.data_ptr(), rows, cols, sp())
    assert rel_err(host(y), ko.softmax_rows(x)) <= 1e-6
    kx.call("kx_layernorm_rows", d.data_ptr(), d.data_ptr(), rows, cols, dev(g).data_ptr(), dev(b).data_ptr(), 1e-5, sp())
    assert rel_err(host(d), ko.layer_norm_rows(x, g, b, 1e-5)) <= 1e-5


def test_binary_broadcast_and_inplace(kx):
    rng = np.random.default_rng(3)
    a = rng.standard_normal((4 * 6, 5)).astype(F32)
    for (rb, cb) in [(6, 5), (1, 5), (6, 1), (1, 1)]:
        b = rng.standard_normal((4 * rb, cb)).astype(F32) + 3
        for op in range(6):
            y = torch.empty((24, 5), dtype=torch.float32, device="cuda")
            kx.call("kx_binary", dev(a).data_ptr(), 6, 5, dev(b).data_ptr(), rb, cb, y.data_ptr(), 4, 6, 5, op, sp())
            s = dict(bop=op)
            want = ko.binary(s, ko._val([6, 5]), a, ko._val([rb, cb]), b, ko._val([6, 5]))
            assert rel_err(host(y), want) <= 1e-7
    da = dev(a)
    kx.call("kx_binary", da.data_ptr(), 6, 5, da.data_ptr(), 6, 5, da.data_ptr(), 4, 6, 5, 0, sp())
    assert np.array_equal(host(da), a + a)


@pytest.mark.parametrize("C", [8, 64])
def test_pool2d_four_channels_at_a_time(kx, C):
    """Channel counts that are multiples of 4 take the float4 pooling path: same windows, same per-element
    combination as the reference (max keeps a NaN only where the reference's comparison does), with NaNs planted."""
    rng = np.random.default_rng(C)
    B, H, W = 3, 9, 10
    x = rng.standard_normal((B * H * W, C)).astype(F32)
    x[rng.integers(0, B * H * W, 7), rng.integers(0, C, 7)] = np.nan
    dx = dev(x)
    for ptype, k, s, p, cp in [(0, 2, 2, 0, 0), (1, 3, 2, 1, 0), (1, 3, 2, 1, 1), (0, 3, 1, 1, 0)]:
        Ho, Wo = (H + 2 * p - k) // s + 1, (W + 2 * p - k) // s + 1
        y = torch.empty((B * Ho * Wo, C), dtype=torch.float32, device="cuda")
        kx.call("kx_pool2d", dx.data_ptr(), y.data_ptr(), B, H, W, C, Ho, Wo, k, k, s, s, p, p, ptype, cp, sp())
        st = dict(ptype=ptype, kh=k, kw=k, sh=s, sw=s, pt=p, pb=p, pl=p, pr=p, count_pad=cp)
        assert rel_err(host(y), ko.pool(st, ko._val([H, W, C]), ko._val([Ho, Wo, C]), x)) <= 1e-6


def test_pool_gpool_permute_pad_upsample(kx):
    rng = np.random.default_rng(11)
    B, H, W, C = 2, 7, 6, 5
    x = rng.standard_normal((B * H * W, C)).astype(F32)
    dx = dev(x)
    for ptype, k, s, p, cp in [(0, 2, 2, 0, 0), (1, 3, 2, 1, 0), (1, 3, 2, 1, 1), (0, 3, 1, 1, 0)]:
        Ho, Wo = (H + 2 * p - k) // s + 1, (W + 2 * p - k) // s + 1
        y = torch.empty((B * Ho * Wo, C), dtype=torch.float32, device="cuda")
        kx.call("kx_pool2d", dx.data_ptr(), y.data_ptr(), B, H, W, C, Ho, Wo, k, k, s, s, p, p, ptype, cp, sp())
        st = dict(ptype=ptype, kh=k, kw=k, sh=s, sw=s, pt=p, pb=p, pl=p, pr=p, count_pad=cp)
        assert rel_err(host(y), ko.pool(st, ko._val([H, W, C]), ko._val([Ho, Wo, C]), x)) <= 1e-6
    for ptype in (0, 1):
        y = torch.empty((B, C), dtype=torch.float32, device="cuda")
        kx.call("kx_global_pool", dx.data_ptr(), y.data_ptr(), B, H * W, C, ptype, sp())
        assert rel_err(host(y), ko.global_pool(dict(ptype=ptype), ko._val([H, W, C]), x)) <= 1e-6
    import ctypes
    for perm in [(2, 0, 1), (1, 0, 2), (0, 2, 1)]:
        dims = (ctypes.c_int * 4)(H, W, C, 0)
        pm = (ctypes.c_int * 4)(*perm, 0)
        y = torch.empty_like(dx)
        kx.call("kx_permute", dx.data_ptr(), y.data_ptr(), B, 3, dims, pm, sp())
        assert np.array_equal(host(y).reshape(-1), ko.permute(dict(perm=list(perm)), ko._val([H, W, C]), x).reshape(-1))
    y = torch.empty((B * (H + 3) * (W + 2), C), dtype=torch.float32, device="cuda")
    kx.call("kx_pad2d", dx.data_ptr(), y.data_ptr(), B, H, W, C, H + 3, W + 2, 1, 2, sp())
    want = np.zeros((B, H + 3, W + 2, C), F32)
    want[:, 1:1 + H, 2:2 + W] = x.reshape(B, H, W, C)
    assert np.array_equal(host(y).reshape(want.shape), want)
    y = torch.empty((B * H * 2 * W * 3, C), dtype=torch.float32, device="cuda")
    kx.call("kx_upsample2d", dx.data_ptr(), y.data_ptr(), B, H, W, C, 2 * H, 3 * W, 2, 3, sp())
    want = x.reshape(B, H, W, C).repeat(2, axis=1).repeat(3, axis=2)
    assert np.array_equal(host(y).reshape(want.shape), want)


def test_depthwise_embedding_fma_relu(kx):
    rng = np.random.default_rng(12)
    B, H, W, C, mult = 2, 6, 5, 4, 2
    x = rng.standard_normal((B * H * W, C)).astype(F32)
    w = rng.standard_normal((9, C * mult)).astype(F32)
    b = rng.standard_normal(C * mult).astype(F32)
    y = torch.empty((B * H * W, C * mult), dtype=torch.float32, device="cuda")
    kx.call("kx_conv_depthwise", dev(x).data_ptr(), dev(w).data_ptr(), dev(b).data_ptr(), y.data_ptr(), B, H, W, C, C * mult,
            H, W, 3, 3, 1, 1, 1, 1, 1, 1, 0, 0.0, sp())
    st = dict(groups=C, kh=3, kw=3, sh=1, sw=1, dh=1, dw=1, pt=1, pb=1, pl=1, pr=1, w=("f32", w), bias=b, act=0, alpha=0.0)
    assert rel_err(host(y), ko.conv(st, ko._val([H, W, C]), ko._val([H, W, C * mult]), x)) <= 1e-6
    table = rng.standard_normal((10, 6)).astype(F32)
    ids = np.array([0, 3, 9, 10, -1, 2.5, 7], F32)
    y = torch.empty((7, 6), dtype=torch.float32, device="cuda")
    kx.call("kx_embedding", dev(ids).data_ptr(), 7, dev(table).data_ptr(), 10, 6, y.data_ptr(), sp())
    got = host(y)
    assert np.array_equal(got[[0, 1, 2, 6]], table[[0, 3, 9, 7]]) and np.all(np.isnan(got[[3, 4, 5]]))
    n = 1000003
    a, xx, bb = (rng.standard_normal(n).astype(F32) for _ in range(3))
    y = torch.empty(n, dtype=torch.float32, device="cuda")
    kx.call("kx_fma_relu", dev(a).data_ptr(), dev(xx).data_ptr(), dev(bb).data_ptr(), y.data_ptr(), n, sp())
    want = np.maximum((a.astype(np.float64) * xx + bb), 0).astype(F32)
    assert rel_err(host(y), want) <= 1e-7


@pytest.mark.parametrize("Rq,S,H,dk,dv,causal,packed", [(128, 128, 8, 64, 64, False, False), (10, 10, 4, 4, 4, True, False),
                                                        (5, 17, 2, 32, 48, False, False), (128, 128, 8, 64, 64, False, True),
                                                        (128, 96, 2, 60, 36, True, False), (128, 128, 3, 62, 30, False, True),
                                                        (128, 128, 1, 64, 64, True, True), (1, 1, 1, 8, 8, False, False),
                                                        (200, 200, 4, 64, 64, True, False), (256, 256, 2, 16, 64, False, True),
                                                        (70, 300, 2, 80, 96, True, False), (33, 257, 3, 64, 64, False, False)])
def test_attention_core(kx, Rq, S, H, dk, dv, causal, packed):
    """packed: Q, K, V are column blocks of one [Q | K | V] row buffer (the fused-projection layout). Rq, S <= 128 with
    head dims <= 64 run on the tensor cores (3xTF32: ragged rows and keys, head dims not multiples of 8, causal
    masks); S <= 256 with head dims <= 64 the register-tiled CUDA-core kernel; longer or wider heads the
    one-row-per-thread kernel."""
    rng = np.random.default_rng(Rq + S + dk)
    B = 3
    q = rng.standard_normal((B * Rq, H * dk)).astype(F32)
    k = rng.standard_normal((B * S, H * dk)).astype(F32)
    v = rng.standard_normal((B * S, H * dv)).astype(F32)
    ctx = torch.empty((B * Rq, H * dv), dtype=torch.float32, device="cuda")
    st = status()
    if packed:
        qkv = dev(np.concatenate([q, k, v], axis=1))
        ld = 2 * H * dk + H * dv
        base = qkv.data_ptr()
        kx.call("kx_attention", base, ld, base + 4 * H * dk, ld, base + 8 * H * dk, ld, ctx.data_ptr(), H * dv, B, Rq, S, H, dk,
                dv, int(causal), st.data_ptr(), sp())
    else:
        kx.call("kx_attention", dev(q).data_ptr(), H * dk, dev(k).data_ptr(), H * dk, dev(v).data_ptr(), H * dv,
                ctx.data_ptr(), H * dv, B, Rq, S, H, dk, dv, int(causal), st.data_ptr(), sp())
    Q = q.reshape(B, Rq, H, dk).transpose(0, 2, 1, 3).astype(np.float64)
    K = k.reshape(B, S, H, dk).transpose(0, 2, 1, 3).astype(np.float64)
    V = v.reshape(B, S, H, dv).transpose(0, 2, 1, 3).astype(np.float64)
    P = Q @ K.transpose(0, 1, 3, 2) / np.sqrt(dk)
    if causal:
        P = np.where(np.triu(np.ones((Rq, S), bool), 1), -np.inf, P)
    P = np.exp(P - P.max(-1, keepdims=True))
    P /= P.sum(-1, keepdims=True)
    want = (P @ V).transpose(0, 2, 1, 3).reshape(B * Rq, H * dv)
    check_status(st)
    assert rel_err(host(ctx), want) <= 1e-5


@pytest.mark.parametrize("arrive", [1, 0])
def test_bounded_wait_reports_timeout(libkx, arrive):
    """Failure detection without a fault: the bounded mbarrier wait every tcgen05 kernel here uses gives up after its
    limit and reports KX_STATUS_TIMEOUT through the status word (a barrier nothing arrives at, 20 ms limit), while a
    barrier that completes leaves the status alone; either way the launch ends and the context stays usable."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from kernix_b200 import kx_abi as kx
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    waited = torch.zeros(1, dtype=torch.int64, device="cuda")
    kx.call("kx_probe_bounded_wait", arrive, 20_000_000, status.data_ptr(), waited.data_ptr(), None)
    torch.cuda.synchronize()
    ns = int(waited.item())
    if arrive:
        assert int(status.item()) == 0 and ns < 20_000_000
    else:
        assert int(status.item()) == 1 and 20_000_000 <= ns < 1_000_000_000
    assert torch.ones(4, device="cuda").sum().item() == 4.0  # the context is still usable


@pytest.mark.parametrize("m,k,n,act", [(4096, 1024, 4096, 1), (300, 4096, 1024, -1), (333, 200, 1000, 0), (1, 64, 512, 1),
                                       (1500, 512, 2304, 1)])
def test_gemm_i8_quantised_output_equals_quantiser(kx, m, k, n, act):
    """A hidden int8 layer with its quantisation fused into the epilogue (kx_gemm_i8_q) gives bit for bit the int8
    rows and row scales that kx_quant_rows computes from kx_gemm_i8's fp32 output: the same max over the row (NaN
    and inf rows included), sx = m / 127, rint(y * (1 / sx)) clamped to +-127, zero padding up to ldq. Two launches
    in a row, the second's row maxima and counters cleared by the first (clear-ahead), the first's by torch."""
    from kernix_b200.knx_writer import quantize_int8
    rng = np.random.default_rng(m + k + n)
    scale, q = quantize_int8((rng.standard_normal((k, n)) * 0.05).astype(F32))
    wq, ldw = _prep_i8(kx, q)
    dscale, db = dev(scale), dev(rng.standard_normal(n).astype(F32) * 0.1)
    ldq, ldo = (k + 15) // 16 * 16, (n + 15) // 16 * 16
    words = m + (m + 127) // 128
    ctl = [torch.zeros(words, dtype=torch.int32, device="cuda") for _ in range(2)]
    for call in range(2):
        x = (rng.standard_normal((m, k)) * rng.uniform(0.1, 3, (m, 1))).astype(F32)
        if m > 4:
            x[1] = 0.0
            x[2, 5] = np.nan
            x[3] *= 1e37  # overflows to inf in the dequantisation: an inf row
        dx = dev(x)
        xq = torch.empty((m, ldq), dtype=torch.int8, device="cuda")
        sx = torch.empty(m, dtype=torch.float32, device="cuda")
        kx.call("kx_quant_rows", dx.data_ptr(), k, m, k, xq.data_ptr(), ldq, sx.data_ptr(), sp())
        y = torch.empty((m, n), dtype=torch.float32, device="cuda")
        st = status()
        kx.call("kx_gemm_i8", xq.data_ptr(), ldq, sx.data_ptr(), wq.data_ptr(), ldw, dscale.data_ptr(), db.data_ptr(),
                y.data_ptr(), n, m, n, k, act, 0.0, st.data_ptr(), sp())
        want_q = torch.full((m, ldo), 77, dtype=torch.int8, device="cuda")
        want_sx = torch.empty(m, dtype=torch.float32, device="cuda")
        kx.call("kx_quant_rows", y.data_ptr(), n, m, n, want_q.data_ptr(), ldo, want_sx.data_ptr(), sp())
        got_q = torch.full((m, ldo), 77, dtype=torch.int8, device="cuda")
        got_sx = torch.empty(m, dtype=torch.float32, device="cuda")
        kx.call("kx_gemm_i8_q", xq.data_ptr(), ldq, sx.data_ptr(), wq.data_ptr(), ldw, dscale.data_ptr(), db.data_ptr(),
                m, n, k, act, 0.0, got_q.data_ptr(), ldo, got_sx.data_ptr(), ctl[call].data_ptr(), ctl[1 - call].data_ptr(),
                words, st.data_ptr(), sp())
        torch.cuda.synchronize()
        check_status(st)
        assert np.array_equal(host(got_q), host(want_q)), f"call {call}: int8 rows differ"
        assert np.array_equal(host(got_sx).view(np.uint32), host(want_sx).view(np.uint32)), f"call {call}: row scales differ"
    assert not host(ctl[0]).any(), "the second launch clears the first's row maxima and counters"
