"""ctypes binding of libb2.so (the C ABI declared in include/b2.h).

The library is built in-tree by ``csrc/build.py``.  There is no fallback:
if the library or a GPU is missing, every op raises.
"""
import ctypes

import torch
import os

from .errors import B2Error, raise_for_status

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libb2.so")

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_f32 = ctypes.c_float
_pi64 = ctypes.POINTER(ctypes.c_int64)

# name -> (restype, argtypes); must match include/b2.h exactly.
SIGNATURES = {
    "b2_version": (_i32, []),
    "b2_last_error": (ctypes.c_char_p, []),
    "b2_device_error": (_i32, [_vp, ctypes.POINTER(ctypes.c_uint)]),
    "b2_int4_matmul": (_i32, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i32, _vp]),
    "b2_int4_matmul_ref": (_i32, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i32, _vp]),
    "b2_int8_matmul": (_i32, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i32, _vp]),
    "b2_gemm_bf16": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "b2_int4_dequant": (_i32, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i32, _vp]),
    "b2_int4_repack_ref_to_gptq": (_i32, [_vp, _vp, _i64, _i64, _vp]),
    "b2_w4_gemv_plan": (_i32, [_i64, _i64, _i64, _i64, _i32, _i32, _pi64]),
    "b2_flash_attn_fwd": (_i32, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64,
                                 _pi64, _pi64, _pi64, _pi64, _f32, _i32, _i32, _vp]),
    "b2_flash_attn_fwd_window": (_i32, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _pi64, _pi64, _pi64,
                                        _pi64, _f32, _i64, _i32, _vp]),
    "b2_decode_attn_workspace_size": (ctypes.c_size_t, [_i64, _i64, _i64, _i64, _i64]),
    "b2_decode_attn": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                              _pi64, _pi64, _vp, _i64, _vp, _f32, _i32, _i32, _vp]),
    "b2_repeat_kv": (_i32, [_vp, _vp, _i64, _i64, _i64, _i64, _i64, _vp]),
    "b2_kda_workspace_size": (ctypes.c_size_t, [_i64, _i64, _i64, _i64, _i64, _i64]),
    "b2_kda_fwd_noalloc": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                  _i64, _i64, _i64, _i64, _i64, _i64, _f32, _i32, _vp]),
    "b2_kda_fwd": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                          _i64, _i64, _i64, _i64, _i64, _i64, _f32, _i32, _vp]),
}

_lib = None


def load():
    """Load libb2.so once and bind every symbol of include/b2.h."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise B2Error(f"libb2.so not built at {LIB_PATH}: run csrc/build.py")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)  # AttributeError if the symbol is missing
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


_fns = {}


def call(name, *args):
    """Invoke an int-returning entry point and raise on a non-zero status."""
    fn = _fns.get(name)
    if fn is None:
        fn = _fns[name] = getattr(load(), name)
    status = fn(*args)
    if status != 0:
        raise_for_status(status, name, load().b2_last_error().decode())
    return status


def fn(name):
    """The bound ctypes function of an entry point (for hot paths that check
    the status themselves with ``check``)."""
    f = _fns.get(name)
    if f is None:
        f = _fns[name] = getattr(load(), name)
    return f


def check(status, name):
    if status != 0:
        raise_for_status(status, name, load().b2_last_error().decode())


def check_out(out, shape, dtype, name, contiguous=True):
    """A caller-supplied output must be a CUDA tensor of the op's shape and
    dtype (and, where the kernel writes it densely, contiguous): the kernel
    writes through its raw pointer."""
    from .errors import B2ShapeError
    if not out.is_cuda or out.dtype != dtype or tuple(out.shape) != tuple(shape) or \
            (contiguous and not out.is_contiguous()):
        raise B2ShapeError(f"{name}: out must be a {'contiguous ' if contiguous else ''}CUDA {dtype} tensor of "
                           f"shape {tuple(shape)}, got {out.dtype} {tuple(out.shape)} on {out.device}")
    return out


def strides_arg(t):
    return (ctypes.c_int64 * 3)(*t)


_fast = False  # not looked up yet


def fast():
    """The _b2fast binding (C++ argument handling of the per-layer decode
    call, built by csrc/build.py next to libb2.so and linked against it), or
    None when it is not built or libb2.so was loaded from another path."""
    global _fast
    if _fast is False:
        _fast = None
        if os.path.dirname(os.path.abspath(LIB_PATH)) == _HERE:
            load()
            try:
                from . import _b2fast
                _fast = _b2fast
            except ImportError:
                pass
    return _fast


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def current_stream():
    """cudaStream_t of the caller's current stream on the current device."""
    if _raw_stream is not None:
        return _raw_stream(torch.cuda.current_device())
    return torch.cuda.current_stream().cuda_stream
