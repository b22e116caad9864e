"""GPU: kx_linear_i8_noalloc, the int8 LINEAR step for callers that cannot allocate device memory (its scratch is a
fixed array inside libkernix.so), must give exactly what kx_linear_i8 gives with caller-provided scratch, call after
call, and must refuse problems larger than its built-in scratch instead of allocating. This file sorts last so that a
run stopping at the first failure has already run every other test."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def test_noalloc_linear_matches_caller_scratch_twice(libkx):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from kernix_b200 import kx_abi as kx
    from kernix_b200.knx_writer import quantize_int8
    rng = np.random.default_rng(2024)
    m, k, n = 300, 1000, 520
    keep = []

    def dev(a):
        t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
        keep.append(t)
        return t

    scale, q = quantize_int8((rng.standard_normal((k, n)) * 0.02).astype(np.float32))
    ldw = (k + 15) // 16 * 16
    wq = torch.empty((n, ldw), dtype=torch.int8, device="cuda")
    kx.call("kx_prep_i8_weight", dev(q).data_ptr(), k, n, wq.data_ptr(), ldw, None)
    dscale = dev(scale)
    dbias = dev(rng.standard_normal(n).astype(np.float32))
    ldq = ldw
    xq = torch.empty((m, ldq), dtype=torch.int8, device="cuda")
    sx = torch.empty(m, dtype=torch.float32, device="cuda")
    status = torch.zeros(2, dtype=torch.int32, device="cuda")
    for call, act in enumerate((1, 0)):  # two calls in a row, different inputs and activations
        x = (rng.standard_normal((m, k)) * rng.uniform(0.1, 3, (m, 1))).astype(np.float32)
        x[0] = 0.0
        dx = dev(x)
        want = torch.empty((m, n), device="cuda")
        got = torch.empty((m, n), device="cuda")
        kx.call("kx_linear_i8", dx.data_ptr(), k, m, k, wq.data_ptr(), ldw, dscale.data_ptr(), dbias.data_ptr(),
                want.data_ptr(), n, n, act, 0.0, xq.data_ptr(), sx.data_ptr(), status.data_ptr(), None)
        kx.call("kx_linear_i8_noalloc", dx.data_ptr(), k, m, k, wq.data_ptr(), ldw, dscale.data_ptr(), dbias.data_ptr(),
                got.data_ptr(), n, n, act, 0.0, status.data_ptr() + 4, None)
        torch.cuda.synchronize()
        assert status.cpu().tolist() == [0, 0]
        g, w = got.cpu().numpy(), want.cpu().numpy()
        assert np.array_equal(g.view(np.uint32), w.view(np.uint32)), f"call {call}: outputs differ"


def test_noalloc_linear_rejects_oversize(libkx):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from kernix_b200 import kx_abi as kx
    lib = kx.lib()
    big_rows = 20000  # 20000 x 1024 bytes of int8 activations alone exceed the 16 MiB array
    rc = lib.kx_linear_i8_noalloc(None, 1024, big_rows, 1024, None, 1024, None, None, None, 1024, 1024, -1, 0.0, None, None)
    assert rc == -1
