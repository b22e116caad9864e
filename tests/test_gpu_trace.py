"""GPU trace: every intermediate value of a forward (read back with the kx_model_debug_value hook) against the
oracle's value of the same graph edge, so a mismatch names the first step that goes wrong."""
import ctypes

import numpy as np
import pytest

from conftest import rel_err
from oracle import knx_oracle as ko

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def trace_compare(path, x, batch, tol):
    from kernix_b200 import Model, kx_abi
    L = kx_abi.lib()
    L.kx_model_forward_trace.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
    L.kx_model_forward_trace.restype = ctypes.c_int
    m = Model(path, workspace_mb=0)
    mod = ko.load(path)
    views = []
    ko.forward(mod, x, trace=views)
    last = {}
    for o, f in enumerate(mod["fused_map"]):
        last[f] = o
    n = mod["n_fused_steps"]
    outs = [np.empty(views[last[f]].size, np.float32) for f in range(1, n + 1)]
    ptrs = (ctypes.c_void_p * n)(*[o.ctypes.data for o in outs])
    xr = np.ascontiguousarray(x.reshape(-1, m.in_dim), np.float32)
    assert L.kx_model_forward_trace(m._h, xr.ctypes.data, xr.shape[0], ptrs) == 0
    report = []
    for f in range(1, n + 1):
        want = views[last[f]]
        e = rel_err(outs[f - 1].reshape(want.shape), want)
        kind, act = mod["fused_steps"][f - 1]
        report.append((f, ko.OP_NAMES[kind], act, e))
        if not e <= tol:
            pytest.fail(f"value {f} ({ko.OP_NAMES[kind]}, act {act}) differs: {e:.3e}; steps so far: {report}")
    return report


@pytest.mark.parametrize("cfg,batch,tol", [("c3", 3, 1e-4), ("c4", 2, 1e-4), ("c1", 5, 2e-5)])
def test_every_value_matches_oracle(libkx, model_dir, cfg, batch, tol):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from kernix_b200 import configs
    p = configs.model_path(cfg, model_dir)
    x = configs.inputs(cfg, batch)
    rep = trace_compare(p, x, batch, tol)
    print(cfg, [(f, k, round(e, 9)) for f, k, _, e in rep])


@pytest.mark.parametrize("cfg,batch", [("c4", 3), ("c4", 40)])
def test_fused_forward_equals_step_by_step(libkx, model_dir, monkeypatch, cfg, batch):
    """The forward runs a LINEAR / ATTENTION step and the ADD that consumes its output as one GEMM (the residual added
    in the epilogue); the trace hook runs every step on its own. With the same rows per GEMM (one piece) their final
    outputs are bitwise equal (c4 has one such pair per encoder block for the attention output and one for the
    feed-forward output; 40 x 128 rows take the persistent tiles)."""
    monkeypatch.setenv("KERNIX_PIPELINE", "1")
    from kernix_b200 import Model, configs, kx_abi
    L = kx_abi.lib()
    L.kx_model_forward_trace.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
    L.kx_model_forward_trace.restype = ctypes.c_int
    p = configs.model_path(cfg, model_dir)
    x = configs.inputs(cfg, batch)
    m = Model(p, workspace_mb=0)
    got = m(x)
    xr = np.ascontiguousarray(x.reshape(-1, m.in_dim), np.float32)
    mod = ko.load(p)
    n = mod["n_fused_steps"]
    last = np.empty(got.size, np.float32)
    ptrs = (ctypes.c_void_p * n)(*([None] * (n - 1) + [last.ctypes.data]))
    assert L.kx_model_forward_trace(m._h, xr.ctypes.data, xr.shape[0], ptrs) == 0
    m.close()
    assert np.array_equal(last.reshape(got.shape), got)
