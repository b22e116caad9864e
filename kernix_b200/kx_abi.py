"""ctypes declarations of the kernel-level C ABI (include/kx_kernels.h) and the host-only inspector
(include/kx_inspect.h) of libkernix.so. Device pointers are passed as integers (e.g. torch's data_ptr()),
streams as integers (torch.cuda.current_stream().cuda_stream)."""
import ctypes

from .kernix import lib as _capi_lib

_vp, _i, _l, _f, _sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_long, ctypes.c_float, ctypes.c_size_t

SIGNATURES = {
    "kx_quant_rows": [_vp, _i, _i, _i, _vp, _i, _vp, _vp],
    "kx_gemm_i8": [_vp, _i, _vp, _vp, _i, _vp, _vp, _vp, _i, _i, _i, _i, _i, _f, _vp, _vp],
    "kx_linear_i8": [_vp, _i, _i, _i, _vp, _i, _vp, _vp, _vp, _i, _i, _i, _f, _vp, _vp, _vp, _vp],
    "kx_linear_i8_noalloc": [_vp, _i, _i, _i, _vp, _i, _vp, _vp, _vp, _i, _i, _i, _f, _vp, _vp],
    "kx_gemm_i8_acc": [_vp, _i, _vp, _i, _vp, _i, _i, _i, _i, _vp, _vp],
    "kx_probe_bounded_wait": [_i, ctypes.c_ulonglong, _vp, _vp, _vp],
    "kx_gemm_i8_q": [_vp, _i, _vp, _vp, _i, _vp, _vp, _i, _i, _i, _i, _f, _vp, _i, _vp, _vp, _vp, _i, _vp, _vp],
    "kx_quant_rows_z": [_vp, _i, _i, _i, _vp, _i, _vp, _vp, _i, _vp],
    "kx_i8_chain": [_i, _i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp],
    "kx_prep_i8_weight": [_vp, _i, _i, _vp, _i, _vp],
    "kx_gemm_f32": [_vp, _i, _vp, _vp, _i, _vp, _vp, _i, _i, _i, _i, _i, _f, _vp, _vp],
    "kx_gemm_f32_res": [_vp, _i, _vp, _vp, _i, _vp, _vp, _i, _i, _i, _i, _i, _f, _vp, _i, _vp, _vp],
    "kx_i8_split_blocks": [_i, _i, _i],
    "kx_gemm_i8_split_acc": [_vp, _i, _vp, _i, _i, _i, _i, _i, _vp, _vp, _vp],
    "kx_i8_rows": [_vp, _i, _i, _i, _vp, _vp, _vp, _i, _f, _vp, _i, _vp, _i, _vp, _vp],
    "kx_gemm_f32_split": [_vp, _i, _vp, _vp, _i, _vp, _vp, _i, _i, _i, _i, _i, _f, _i, _vp, _vp, _vp],
    "kx_gemm_f32_splits": [_i, _i, _i],
    "kx_add_planes": [_vp, _i, _i, _i, _vp, _i, _f, _vp, _i, _vp],
    "kx_prep_f32_weight": [_vp, _i, _i, _vp, _vp, _i, _vp],
    "kx_bias_act": [_vp, _vp, _l, _i, _vp, _i, _f, _vp],
    "kx_softmax_rows": [_vp, _vp, _l, _i, _vp],
    "kx_layernorm_rows": [_vp, _vp, _l, _i, _vp, _vp, _f, _vp],
    "kx_affine_rows": [_vp, _vp, _l, _i, _vp, _vp, _vp],
    "kx_add_const": [_vp, _vp, _l, _l, _vp, _vp],
    "kx_binary": [_vp, _i, _i, _vp, _i, _i, _vp, _l, _i, _i, _i, _vp],
    "kx_pool2d": [_vp, _vp] + [_i] * 14 + [_vp],
    "kx_global_pool": [_vp, _vp, _l, _i, _i, _i, _vp],
    "kx_permute": [_vp, _vp, _l, _i, _vp, _vp, _vp],
    "kx_copy_cols": [_vp, _l, _vp, _l, _l, _l, _l, _vp],
    "kx_pad2d": [_vp, _vp] + [_i] * 8 + [_vp],
    "kx_upsample2d": [_vp, _vp] + [_i] * 8 + [_vp],
    "kx_embedding": [_vp, _l, _vp, _i, _i, _vp, _vp],
    "kx_conv_depthwise": [_vp, _vp, _vp, _vp] + [_i] * 15 + [_i, _f, _vp],
    "kx_conv_f32": [_vp, _vp, _vp, _i, _vp, _vp] + [_i] * 16 + [_i, _f, _vp, _vp],
    "kx_conv_f32_ws": [_vp, _vp, _vp, _i, _vp, _vp] + [_i] * 16 + [_i, _f, _vp, _sz, _vp, _vp],
    "kx_attention": [_vp, _i, _vp, _i, _vp, _i, _vp, _i, _i, _i, _i, _i, _i, _i, _i, _vp, _vp],
    "kx_fma_relu": [_vp, _vp, _vp, _vp, _sz, _vp],
    "kx_unshard_cols": [_vp, _i, _l, _i, _vp, _i, _vp],
    "kx_rnn_step": [_i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _l, _i, _i, _i, _i, _i, _i, _i, _i, _f, _vp],
    "kx_rnn_merge": [_vp, _vp, _l, _i, _vp],
    "kx_skinny_slices": [_i, _i],
    "kx_gemm_f32_skinny": [_vp, _i, _vp, _vp, _vp, _i, _i, _i, _i, _i, _f, _vp, _sz, _vp],
    "kx_knx_plan": [ctypes.c_char_p, ctypes.POINTER(_i), ctypes.POINTER(_i), _i],
    "kx_knx_inspect": [ctypes.c_char_p, ctypes.POINTER(_l), ctypes.POINTER(_i), ctypes.POINTER(_i), ctypes.POINTER(_i), _i,
                       ctypes.c_char_p, _i],
}

_done = False


def lib():
    global _done
    L = _capi_lib()
    if not _done:
        for name, args in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = ctypes.c_int
        _done = True
    return L


def call(name, *args):
    """Call a kx_* entry point; raises RuntimeError when it rejects the arguments or the launch fails."""
    rc = getattr(lib(), name)(*args)
    if rc != 0:
        raise RuntimeError(f"{name} returned {rc}")


def inspect(path):
    """Host-only parse of a .knx file with the runtime's own loader. Returns a dict, or raises ValueError(reason)."""
    info = (ctypes.c_long * 12)()
    shapes = (ctypes.c_int * 8)()
    kinds = (ctypes.c_int * 1024)()
    acts = (ctypes.c_int * 1024)()
    err = ctypes.create_string_buffer(256)
    rc = lib().kx_knx_inspect(path.encode() if isinstance(path, str) else path, info, shapes, kinds, acts, 1024, err, 256)
    if rc != 0:
        raise ValueError(err.value.decode())
    n = info[0]
    return dict(n_steps=n, in_dim=info[1], out_dim=info[2], seq_len=info[3], layout=info[4],
                in_shape=list(shapes[:info[5]]), out_shape=list(shapes[4:4 + info[6]]), n_storage=info[7],
                version=info[8], storage_per_sample=info[9], steps=list(zip(kinds[:n], acts[:n])))


def plan(path):
    """(storage id per value, last reader per value) of the runtime's storage plan."""
    st = (ctypes.c_int * 2048)()
    last = (ctypes.c_int * 2048)()
    n = lib().kx_knx_plan(path.encode() if isinstance(path, str) else path, st, last, 2048)
    if n < 0:
        raise ValueError("rejected")
    return list(st[:n]), list(last[:n])
