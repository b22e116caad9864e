"""numpy/ctypes binding of the KERNIX-B200 runtime: the same `Model` interface as the reference's
python/kernix.py (constructor arguments, attributes, call convention, exceptions), backed by libkernix.so.

    from kernix_b200 import Model
    m = Model("model.knx")
    y = m(x)   # x: (batch, *m.in_shape) float32 -> (batch, *m.out_shape); PyTorch conv models take (batch, C, H, W)
               # (rows, in_dim) is accepted too (rows a multiple of seq_len)

One Model serialises its own calls (the library reuses per-model buffers); use one Model per thread for
concurrency. The library is $KERNIX_LIB if set, else kernix_b200/libkernix.so next to this file; the
reference's own binding also works unchanged against it (KERNIX_LIB=/path/to/libkernix.so).
"""
import ctypes
import os
import threading
import warnings

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("KERNIX_LIB", os.path.join(_HERE, "libkernix.so"))

_lib = None


def lib():
    """Load libkernix.so once (raises OSError if it is missing: there is no fallback implementation)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise OSError(f"{LIB_PATH} not found: build it with `python -m kernix_b200.build`")
        L = ctypes.CDLL(LIB_PATH)
        vp, ip = ctypes.c_void_p, ctypes.POINTER(ctypes.c_int)
        L.kernix_capi_load.argtypes = [ctypes.c_char_p]
        L.kernix_capi_load.restype = vp
        L.kernix_capi_free.argtypes = [vp]
        L.kernix_capi_free.restype = None
        L.kernix_capi_dims.argtypes = [vp, ip, ip, ip]
        L.kernix_capi_dims.restype = None
        L.kernix_capi_forward.argtypes = [vp, vp, ctypes.c_int, vp]
        L.kernix_capi_forward.restype = ctypes.c_int
        L.kernix_capi_trim.argtypes = [vp]
        L.kernix_capi_trim.restype = None
        L.kernix_capi_set_workspace_limit.argtypes = [vp, ctypes.c_size_t]
        L.kernix_capi_set_workspace_limit.restype = None
        L.kernix_capi_shapes.argtypes = [vp, ip, ip, ip, ip, ip]
        L.kernix_capi_shapes.restype = None
        L.kernix_capi_set_ane.argtypes = [vp, ctypes.c_int]
        L.kernix_capi_set_ane.restype = ctypes.c_int
        L.kernix_capi_ane_info.argtypes = [vp, ip]
        L.kernix_capi_ane_info.restype = None
        L.kernix_capi_ane_dump.argtypes = [vp, ctypes.c_int, ctypes.c_int, ctypes.c_char_p]
        L.kernix_capi_ane_dump.restype = ctypes.c_int
        L.kernix_model_load_sharded.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.c_int, vp, vp]
        L.kernix_model_load_sharded.restype = vp
        L.kernix_model_load_sharded_nccl.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.c_int, ctypes.c_char_p]
        L.kernix_model_load_sharded_nccl.restype = vp
        L.kernix_nccl_unique_id.argtypes = [ctypes.c_char_p]
        L.kernix_nccl_unique_id.restype = ctypes.c_int
        # device pointers are 64-bit: without these declarations ctypes would pass them as C ints
        L.kernix_model_forward_device.argtypes = [vp, vp, ctypes.c_int, vp, vp]
        L.kernix_model_forward_device.restype = ctypes.c_int
        L.kernix_model_check.argtypes = [vp]
        L.kernix_model_check.restype = ctypes.c_int
        _lib = L
    return _lib


# int gather(void* ctx, const float* send, float* recv, size_t count, void* stream)
GATHER_FN = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p)


class Model:
    def __init__(self, path, workspace_mb=None, ane=False, shard=None):
        """workspace_mb: bound of the forward workspace (device memory) in MB; larger batches run in chunks with
        identical results. None = library default, 0 = unlimited. ane: there is no Apple Neural Engine on a
        B200 host, so ane=True warns and runs on the GPU.
        shard: (rank, world, gather) to split the wide fp32 dense layers by output columns across `world`
        processes. gather is either the 128-byte NCCL unique id shared by all ranks (bytes, from
        kernix_b200.shard.nccl_unique_id() on one rank): the runtime then all-gathers with NCCL itself
        (kernix_model_load_sharded_nccl); or a callable gather(send_ptr, recv_ptr, count, stream) that all-gathers
        `count` device floats per rank on the CUDA stream (kernix_model_load_sharded; see
        kernix_b200.shard.torch_allgather)."""
        self._lock = threading.Lock()
        L = lib()
        self._free = L.kernix_capi_free  # held here: at interpreter exit the module globals may already be gone
        self._gather_cb = None
        if shard is None:
            self._h = L.kernix_capi_load(os.fsencode(path))
        elif isinstance(shard[2], (bytes, bytearray)):
            rank, world, nccl_id = shard
            if len(nccl_id) != 128:
                raise ValueError("an NCCL unique id has 128 bytes")
            self._h = L.kernix_model_load_sharded_nccl(os.fsencode(path), int(rank), int(world), bytes(nccl_id))
        else:
            rank, world, gather = shard

            def _cb(ctx, send, recv, count, stream):
                try:
                    gather(send or 0, recv or 0, int(count), stream or 0)
                    return 0
                except Exception as e:  # noqa: BLE001  (reported to the runtime as a failed step)
                    warnings.warn(f"KERNIX all-gather failed: {e!r}", RuntimeWarning, stacklevel=1)
                    return -1

            self._gather_cb = GATHER_FN(_cb)  # kept alive as long as the model
            self._h = L.kernix_model_load_sharded(os.fsencode(path), int(rank), int(world),
                                                  ctypes.cast(self._gather_cb, ctypes.c_void_p), None)
        if not self._h:
            raise ValueError(f"cannot load KERNIX model: {path}")
        if workspace_mb is not None:
            if workspace_mb < 0:
                raise ValueError("workspace_mb must be >= 0")
            L.kernix_capi_set_workspace_limit(self._h, int(workspace_mb * (1 << 20)))
        if ane and L.kernix_capi_set_ane(self._h, 1) != 0:
            warnings.warn("ANE assist is not available on this platform: running on the GPU", RuntimeWarning, stacklevel=2)
        d = [ctypes.c_int() for _ in range(3)]
        L.kernix_capi_dims(self._h, *[ctypes.byref(v) for v in d])
        self.in_dim, self.out_dim, self.seq_len = (v.value for v in d)
        in_nd, out_nd, layout = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        in_s, out_s = (ctypes.c_int * 4)(), (ctypes.c_int * 4)()
        L.kernix_capi_shapes(self._h, ctypes.byref(in_nd), in_s, ctypes.byref(out_nd), out_s, ctypes.byref(layout))
        self._in_cl, self._out_cl = tuple(in_s[:in_nd.value]), tuple(out_s[:out_nd.value])
        self.channels_first = layout.value == 1
        cf = lambda s: s[-1:] + s[:-1] if self.channels_first and len(s) >= 2 else s  # noqa: E731
        self.in_shape, self.out_shape = cf(self._in_cl), cf(self._out_cl)
        self._forward = L.kernix_capi_forward

    def __call__(self, x, out=None):
        """Forward pass. out: optional preallocated float32 C-contiguous (batch, *out_shape channels-last) array,
        e.g. in page-locked memory, written in place and returned."""
        x = np.asarray(x)
        if x.ndim >= 2 and tuple(x.shape[1:]) == self.in_shape:
            if self.channels_first and x.ndim >= 3:
                x = np.moveaxis(x, 1, -1)
        elif not (x.ndim == 2 and x.shape[1] == self.in_dim):
            raise ValueError(f"input shape {x.shape}: expected (batch, {', '.join(map(str, self.in_shape))}) or (rows, {self.in_dim})")
        x = np.ascontiguousarray(x, dtype=np.float32)
        rows = x.size // self.in_dim
        if rows == 0 or rows % self.seq_len:
            raise ValueError(f"input rows {rows} must be a positive multiple of seq_len {self.seq_len}")
        shape = (rows // self.seq_len,) + self._out_cl
        if out is None:
            out = np.empty(shape, np.float32)
        elif out.dtype != np.float32 or not out.flags.c_contiguous or out.size != int(np.prod(shape)):
            raise ValueError("out must be a C-contiguous float32 array of the output size")
        with self._lock:
            status = self._forward(self._h, x.ctypes.data, rows, out.ctypes.data)
        if status != 0:
            raise RuntimeError("KERNIX forward failed")
        out = out.reshape(shape)
        return np.moveaxis(out, -1, 1) if self.channels_first and out.ndim >= 3 else out

    def ane_info(self):
        out = (ctypes.c_int * 4)()
        with self._lock:
            lib().kernix_capi_ane_info(self._h, out)
        return dict(zip(("segments", "compiles", "ane_runs", "failures"), out))

    def trim(self):
        """Release the workspace (device arena); weights stay. The next call allocates again."""
        with self._lock:
            lib().kernix_capi_trim(self._h)

    def close(self):
        if getattr(self, "_h", None):
            with self._lock:
                self._free(self._h)
                self._h = None

    __del__ = close
