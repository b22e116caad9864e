"""GPU: kx_linear_i8_noalloc, the int8 LINEAR step for callers that cannot allocate device memory (its scratch is a
fixed array inside libkernix.so), must give exactly what kx_linear_i8 gives with caller-provided scratch, call after
call, must take no device memory after its first call, and must refuse problems larger than its built-in scratch
instead of allocating. This file sorts last so that a run stopping at the first failure has already run every other
test."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def test_noalloc_linear_matches_caller_scratch(libkx):
    """Three calls in a row: the first two share a shape (different inputs and activations), the third has fewer
    rows and a shorter K with a different row pitch (968 -> 976), so any padding or row scale left over in the
    shared array from a larger call would show. Free device memory is read after each call: only the first call
    on a device may take any (it loads the module that holds the array)."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from kernix_b200 import kx_abi as kx
    from kernix_b200.knx_writer import quantize_int8
    rng = np.random.default_rng(2024)
    n = 520
    cases = [(300, 1000, 1), (300, 1000, 0), (77, 968, 1)]  # rows, k, activation (1 = GELU)
    prepared = []
    for m, k, act in cases:  # every device buffer is made before the first call
        scale, q = quantize_int8((rng.standard_normal((k, n)) * 0.02).astype(np.float32))
        ldw = (k + 15) // 16 * 16
        wq = torch.empty((n, ldw), dtype=torch.int8, device="cuda")
        kx.call("kx_prep_i8_weight", torch.from_numpy(q).cuda().data_ptr(), k, n, wq.data_ptr(), ldw, None)
        x = (rng.standard_normal((m, k)) * rng.uniform(0.1, 3, (m, 1))).astype(np.float32)
        x[0] = 0.0
        prepared.append(dict(
            m=m, k=k, act=act, ldw=ldw, wq=wq, x=torch.from_numpy(x).cuda(),
            scale=torch.from_numpy(scale).cuda(), bias=torch.from_numpy(rng.standard_normal(n).astype(np.float32)).cuda(),
            xq=torch.empty((m, ldw), dtype=torch.int8, device="cuda"), sx=torch.empty(m, dtype=torch.float32, device="cuda"),
            want=torch.empty((m, n), device="cuda"), got=torch.empty((m, n), device="cuda")))
    status = torch.zeros(2, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    free_after = []
    for call, c in enumerate(prepared):
        kx.call("kx_linear_i8", c["x"].data_ptr(), c["k"], c["m"], c["k"], c["wq"].data_ptr(), c["ldw"],
                c["scale"].data_ptr(), c["bias"].data_ptr(), c["want"].data_ptr(), n, n, c["act"], 0.0,
                c["xq"].data_ptr(), c["sx"].data_ptr(), status.data_ptr(), None)
        kx.call("kx_linear_i8_noalloc", c["x"].data_ptr(), c["k"], c["m"], c["k"], c["wq"].data_ptr(), c["ldw"],
                c["scale"].data_ptr(), c["bias"].data_ptr(), c["got"].data_ptr(), n, n, c["act"], 0.0,
                status.data_ptr() + 4, None)
        torch.cuda.synchronize()
        free_after.append(torch.cuda.mem_get_info()[0])
        assert status.cpu().tolist() == [0, 0]
        g, w = c["got"].cpu().numpy(), c["want"].cpu().numpy()
        assert np.array_equal(g.view(np.uint32), w.view(np.uint32)), f"call {call}: outputs differ"
    assert free_after[1] == free_after[0] and free_after[2] == free_after[0], free_after


def test_noalloc_linear_rejects_oversize(libkx):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from kernix_b200 import kx_abi as kx
    lib = kx.lib()
    big_rows = 20000  # 20000 x 1024 bytes of int8 activations alone exceed the 16 MiB array
    rc = lib.kx_linear_i8_noalloc(None, 1024, big_rows, 1024, None, 1024, None, None, None, 1024, 1024, -1, 0.0, None, None)
    assert rc == -1
