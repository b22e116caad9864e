"""CPU: the C-ABI library builds, loads without a GPU, and exports every function include/*.h declares."""
import ctypes
import os
import re
import subprocess

from conftest import ROOT


def _declared():
    names = set()
    for h in os.listdir(os.path.join(ROOT, "include")):
        text = open(os.path.join(ROOT, "include", h)).read()
        names |= set(re.findall(r"KERNIX_API\s+[\w\s\*]+?\b(\w+)\s*\(", text))
    return names


def test_headers_declare_reference_boundary():
    names = _declared()
    capi = {"kernix_capi_load", "kernix_capi_free", "kernix_capi_trim", "kernix_capi_set_workspace_limit", "kernix_capi_dims",
            "kernix_capi_forward", "kernix_capi_set_ane", "kernix_capi_ane_info", "kernix_capi_ane_dump", "kernix_capi_shapes"}
    model = {"kernix_model_load", "kernix_model_forward", "kernix_model_free", "kernix_model_trim",
             "kernix_model_set_workspace_limit", "kernix_model_set_ane", "kernix_model_ane_info"}
    assert capi <= names and model <= names


def test_library_exports_every_declared_symbol(libkx):
    so = os.path.join(ROOT, "kernix_b200", "libkernix.so")
    out = subprocess.run(["nm", "-D", "--defined-only", so], capture_output=True, text=True, check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    missing = _declared() - exported
    assert not missing, f"declared but not exported: {sorted(missing)}"
    for name in _declared():
        assert getattr(libkx, name) is not None


def test_load_without_gpu_fails_cleanly(libkx, tmp_path):
    """With no CUDA device the loader returns NULL after parsing (no crash, no CPU fallback)."""
    import torch
    if torch.cuda.is_available():
        return
    from kernix_b200 import knx_writer
    import numpy as np
    p = str(tmp_path / "m.knx")
    knx_writer.Sequential().linear(np.ones((4, 3), np.float32), np.zeros(3, np.float32)).write(p)
    libkx.kernix_capi_load.restype = ctypes.c_void_p
    assert libkx.kernix_capi_load(p.encode()) is None
