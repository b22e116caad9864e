"""GPU: the reference's own Python binding (python/kernix.py) and verify tool (tools/verify.py), unchanged, run on this
library through $KERNIX_LIB -- the drop-in claim for existing users of the numpy/ctypes binding.

The two files are the reference's, staged byte for byte under oracle/_ref/ by oracle/ref/Makefile (untracked; they
travel with the tree). The tests are skipped where they were not staged. Also here: the public workspace fields
of a loaded model, whose default differs from the reference's by design (device memory instead of host memory)."""
import ctypes
import importlib.util
import os
import subprocess
import sys

import numpy as np
import pytest

from conftest import ROOT, rel_err
from oracle import knx_oracle as ko

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

REF_BINDING = os.path.join(ROOT, "oracle", "_ref", "python", "kernix.py")
REF_VERIFY = os.path.join(ROOT, "oracle", "_ref", "tools", "verify.py")
staged = pytest.mark.skipif(not os.path.exists(REF_BINDING), reason="reference binding not staged (make -C oracle/ref)")


@pytest.fixture(scope="module")
def ref_kernix(libkx):
    """The reference binding module, imported under its own name with KERNIX_LIB naming libkernix.so."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from kernix_b200 import build
    old = os.environ.get("KERNIX_LIB")
    os.environ["KERNIX_LIB"] = build.LIB
    try:
        spec = importlib.util.spec_from_file_location("reference_kernix_binding", REF_BINDING)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
    finally:
        if old is None:
            os.environ.pop("KERNIX_LIB", None)
        else:
            os.environ["KERNIX_LIB"] = old
    return mod


@staged
def test_reference_binding_runs_c1(ref_kernix, model_dir):
    from kernix_b200 import configs
    p = configs.model_path("c1", model_dir)
    m = ref_kernix.Model(p)
    assert (m.in_dim, m.out_dim, m.seq_len, m.in_shape, m.out_shape) == (784, 10, 1, (784,), (10,))
    x = configs.inputs("c1", 256)
    assert rel_err(m(x), ko.forward(ko.load(p), x)) <= 1e-5
    m.trim()
    assert rel_err(m(x[:7]), ko.forward(ko.load(p), x[:7])) <= 1e-5
    m.close()


@staged
def test_reference_binding_runs_channels_first_c3(ref_kernix, model_dir):
    """c3 is a PyTorch-layout model (layout 1): the binding takes (batch, 3, 32, 32) and moves the channel axis."""
    from kernix_b200 import configs
    p = configs.model_path("c3", model_dir)
    m = ref_kernix.Model(p, workspace_mb=0)
    assert m.channels_first and m.in_shape == (3, 32, 32) and m.out_shape == (10,)
    rows = configs.inputs("c3", 6)  # channels-last rows: 6 samples x 1024 pixels x 3 channels
    x_cf = np.ascontiguousarray(rows.reshape(6, 32, 32, 3).transpose(0, 3, 1, 2))
    got = m(x_cf)
    assert got.shape == (6, 10)
    assert rel_err(got, ko.forward(ko.load(p), rows)) <= 1e-4
    with pytest.raises(ValueError):
        m(x_cf[:, :2])
    m.close()


def _verify(pt, knx, *extra):
    from kernix_b200 import build
    env = dict(os.environ, KERNIX_LIB=build.LIB)
    return subprocess.run([sys.executable, REF_VERIFY, pt, knx, *extra], env=env, capture_output=True, text=True, timeout=600)


@pytest.mark.skipif(not os.path.exists(REF_VERIFY), reason="reference verify tool not staged (make -C oracle/ref)")
def test_reference_verify_tool(libkx, tmp_path):
    """tools/verify.py compares a PyTorch original with its .knx through the binding: exit 0 within the tolerance,
    exit 1 when the .knx's weights differ."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from kernix_b200 import knx_writer
    torch.manual_seed(0)
    model = torch.nn.Sequential(torch.nn.Linear(20, 64), torch.nn.ReLU(), torch.nn.Linear(64, 10), torch.nn.Tanh())
    pt = str(tmp_path / "model.pt")
    torch.save(model, pt)
    w = [(model[i].weight.detach().numpy().T.copy(), model[i].bias.detach().numpy()) for i in (0, 2)]

    def write(path, bump=0.0):
        knx_writer.Sequential().linear(w[0][0] + bump, w[0][1]).act("relu").linear(*w[1]).act("tanh").write(path)

    good, bad = str(tmp_path / "good.knx"), str(tmp_path / "bad.knx")
    write(good)
    write(bad, bump=0.01)
    r = _verify(pt, good, "--batch", "32")
    assert r.returncode == 0, r.stdout + r.stderr
    r = _verify(pt, bad, "--batch", "32")
    assert r.returncode == 1, r.stdout + r.stderr


class KernixModel(ctypes.Structure):
    _fields_ = [("n_steps", ctypes.c_int), ("in_dim", ctypes.c_int), ("out_dim", ctypes.c_int), ("seq_len", ctypes.c_int),
                ("batch", ctypes.c_int), ("ws_limit", ctypes.c_size_t), ("ws_per_sample", ctypes.c_size_t),
                ("ws_fixed", ctypes.c_size_t), ("in_nd", ctypes.c_int), ("in_shape", ctypes.c_int * 4),
                ("out_nd", ctypes.c_int), ("out_shape", ctypes.c_int * 4), ("layout", ctypes.c_int),
                ("impl", ctypes.c_void_p)]


def test_workspace_fields_by_design(libkx, model_dir):
    """The public workspace fields of c2 (include/kernix_model.h): the workspace is device memory, so the default
    bound is 4 GiB (the reference's is 64 MiB of host memory) and no batch-independent part exists (ws_fixed 0:
    int8 weights are never dequantised into the workspace). With the default bound a 4096-sample forward runs as
    one chunk (batch = 4096 rows); with the reference's 64 MiB bound the chunk is 64 MiB / (4 * ws_per_sample)
    samples. Results never depend on the chunk (tested elsewhere)."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from kernix_b200 import configs
    L = libkx
    L.kernix_model_load.restype = ctypes.c_void_p  # as every other caller in this process declares it
    L.kernix_model_load.argtypes = [ctypes.c_char_p]
    L.kernix_model_free.argtypes = [ctypes.c_void_p]
    L.kernix_model_set_workspace_limit.argtypes = [ctypes.c_void_p, ctypes.c_size_t]
    L.kernix_capi_forward.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
    L.kernix_capi_forward.restype = ctypes.c_int
    from kernix_b200 import kx_abi
    p = configs.model_path("c2", model_dir)
    storage_per_sample = kx_abi.inspect(p)["storage_per_sample"]
    h = L.kernix_model_load(p.encode())
    assert h
    mp = ctypes.cast(h, ctypes.POINTER(KernixModel))
    m = mp.contents
    assert m.ws_limit == 4 << 30 and m.ws_fixed == 0 and m.batch == -1
    # storage buffers + the input rows + the int8 step's scratch (activations: ldq bytes, + a row scale)
    assert m.ws_per_sample >= storage_per_sample + 1024
    x = configs.inputs("c2", 4096)
    out = np.empty((4096, 1024), np.float32)
    assert L.kernix_capi_forward(h, x.ctypes.data, 4096, out.ctypes.data) == 0
    assert mp.contents.batch == 4096
    L.kernix_model_set_workspace_limit(h, 64 << 20)
    assert L.kernix_capi_forward(h, x.ctypes.data, 4096, out.ctypes.data) == 0
    assert mp.contents.batch == (64 << 20) // (4 * m.ws_per_sample)
    L.kernix_model_free(h)
