"""ctypes access to the compiled KERNIX reference (oracle/_ref/libkernix_ref.so).

TEST INFRASTRUCTURE ONLY. Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load
this, as the checker or as the timed reference CPU implementation; the product never does. The
library is built by oracle/ref/Makefile from the reference sources (src/kernix_capi.c exports the
same kernix_capi_* ABI the product exports).
"""
import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_SO = os.path.join(HERE, "_ref", "libkernix_ref.so")

_lib = None


def available():
    return os.path.exists(REF_SO)


def lib():
    global _lib
    if _lib is None:
        if not available():
            raise FileNotFoundError(f"{REF_SO} is not built (make -C oracle/ref, needs the reference sources)")
        L = ctypes.CDLL(REF_SO)
        vp, ip = ctypes.c_void_p, ctypes.POINTER(ctypes.c_int)
        L.kernix_capi_load.argtypes = [ctypes.c_char_p]
        L.kernix_capi_load.restype = vp
        L.kernix_capi_free.argtypes = [vp]
        L.kernix_capi_free.restype = None
        L.kernix_capi_dims.argtypes = [vp, ip, ip, ip]
        L.kernix_capi_dims.restype = None
        L.kernix_capi_forward.argtypes = [vp, vp, ctypes.c_int, vp]
        L.kernix_capi_forward.restype = ctypes.c_int
        L.kernix_capi_set_workspace_limit.argtypes = [vp, ctypes.c_size_t]
        L.kernix_capi_set_workspace_limit.restype = None
        L.kernix_capi_shapes.argtypes = [vp, ip, ip, ip, ip, ip]
        L.kernix_capi_shapes.restype = None
        L.kx_ref_qmatmul.argtypes = [vp, ctypes.c_int, vp, vp, ctypes.c_int, ctypes.c_int, vp, ctypes.c_int, vp]
        L.kx_ref_qmatmul.restype = ctypes.c_int
        L.kx_ref_model_info.argtypes = [vp, ctypes.POINTER(ctypes.c_long)]
        L.kx_ref_model_info.restype = None
        L.kx_ref_model_steps.argtypes = [vp, ip, ip, ctypes.c_int]
        L.kx_ref_model_steps.restype = ctypes.c_int
        L.kx_ref_model_plan.argtypes = [vp, ip, ip, ctypes.c_int]
        L.kx_ref_model_plan.restype = ctypes.c_int
        _lib = L
    return _lib


class RefModel:
    """The reference runtime on one .knx file (kernix_model_load / kernix_model_forward via kernix_capi_*)."""

    def __init__(self, path, workspace_bytes=None):
        L = lib()
        self.h = L.kernix_capi_load(os.fsencode(path))
        if not self.h:
            raise ValueError(f"reference rejected {path}")
        if workspace_bytes is not None:
            L.kernix_capi_set_workspace_limit(self.h, int(workspace_bytes))
        d = [ctypes.c_int() for _ in range(3)]
        L.kernix_capi_dims(self.h, *[ctypes.byref(v) for v in d])
        self.in_dim, self.out_dim, self.seq_len = (v.value for v in d)

    def info(self):
        out = (ctypes.c_long * 9)()
        lib().kx_ref_model_info(self.h, out)
        keys = ("n_steps", "in_dim", "out_dim", "seq_len", "batch", "ws_limit", "ws_per_sample", "ws_fixed", "layout")
        return dict(zip(keys, list(out)))

    def steps(self):
        kind = (ctypes.c_int * 1024)()
        act = (ctypes.c_int * 1024)()
        n = lib().kx_ref_model_steps(self.h, kind, act, 1024)
        return list(zip(kind[:n], act[:n]))

    def plan(self):
        st = (ctypes.c_int * 2048)()
        last = (ctypes.c_int * 2048)()
        n = lib().kx_ref_model_plan(self.h, st, last, 2048)
        return list(st[:n]), list(last[:n])

    def set_workspace_limit(self, nbytes):
        lib().kernix_capi_set_workspace_limit(self.h, int(nbytes))

    def forward(self, x):
        """x: (rows, in_dim) float32 with rows a multiple of seq_len. Returns (rows/seq_len, out_dim)."""
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, self.in_dim)
        rows = x.shape[0]
        out = np.empty((rows // self.seq_len, self.out_dim), np.float32)
        if lib().kernix_capi_forward(self.h, x.ctypes.data, rows, out.ctypes.data) != 0:
            raise RuntimeError("reference forward failed")
        return out

    def close(self):
        if self.h:
            lib().kernix_capi_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def qmatmul(x, q, scale, bias=None, accumulate=False, y=None):
    """The reference int8 kernel (kernix_qmatmul) on x (rows x k) and q (k x n int8, in x out)."""
    x = np.ascontiguousarray(x, np.float32)
    q = np.ascontiguousarray(q, np.int8)
    scale = np.ascontiguousarray(scale, np.float32)
    rows, k = x.shape
    n = q.shape[1]
    y = np.zeros((rows, n), np.float32) if y is None else np.ascontiguousarray(y, np.float32).copy()
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    rc = lib().kx_ref_qmatmul(x.ctypes.data, rows, q.ctypes.data, scale.ctypes.data, k, n,
                              None if b is None else b.ctypes.data, int(bool(accumulate)), y.ctypes.data)
    if rc != 0:
        raise RuntimeError("reference qmatmul failed")
    return y
