"""The C-ABI library loads and exports every entry point include/b2.h
declares, with the status codes the Python side maps (no GPU needed)."""
import ctypes
import os
import re

from conftest import REPO, PKG_ROOT

HEADER = os.path.join(REPO, "include", "b2.h")


def _declared():
    src = open(HEADER).read()
    return set(re.findall(r"^B2_API\s+[\w\s\*]+?\b(b2_\w+)\s*\(", src, flags=re.M))


def test_header_declares_entry_points():
    names = _declared()
    assert {"b2_int4_matmul", "b2_int8_matmul", "b2_flash_attn_fwd", "b2_kda_fwd"} <= names


def test_library_exports_every_declared_symbol():
    from b200kern import _lib
    lib = ctypes.CDLL(_lib.LIB_PATH)
    for name in _declared():
        assert hasattr(lib, name), f"{name} declared in b2.h but not exported"
    assert _declared() == set(_lib.SIGNATURES), "ctypes signatures out of sync with b2.h"


def test_load_and_version():
    from b200kern import _lib
    lib = _lib.load()
    assert lib.b2_version() >= 10000
    assert isinstance(lib.b2_last_error(), bytes)


def test_status_codes_match_header():
    from b200kern import errors
    src = open(HEADER).read()
    codes = {m[0]: int(m[1]) for m in re.findall(r"#define (B2_(?:OK|ERR_\w+))\s+\(?(-?\d+)\)?", src)}
    assert codes["B2_OK"] == errors.OK
    for k, v in codes.items():
        if k != "B2_OK":
            assert getattr(errors, k[3:]) == v


def test_host_validation_without_gpu():
    """Shape checks run on the host before any launch (null stream, no GPU)."""
    from b200kern import _lib, errors
    lib = _lib.load()
    # K not a multiple of the group size -> invalid, no device work
    st = lib.b2_int4_matmul(1, 1, 1, 1, None, 1, 32, 200, 128, 0, None)
    assert st == errors.ERR_INVALID
    assert b"group_size" in lib.b2_last_error()
    st = lib.b2_int4_matmul(1, 1, 1, 1, None, 1, 32, 128, 128, 7, None)
    assert st == errors.ERR_DTYPE
    st = lib.b2_int8_matmul(None, 1, 1, 1, None, 1, 32, 128, 0, None)
    assert st == errors.ERR_INVALID


def test_caller_output_must_be_a_device_tensor_of_the_right_shape():
    """A caller-supplied ``out`` is written through its raw pointer, so a host
    tensor, a wrong dtype or a wrong shape is refused before any launch."""
    import pytest
    import torch
    from b200kern import _lib, errors
    with pytest.raises(errors.B2ShapeError):
        _lib.check_out(torch.empty(2, 3), (2, 3), torch.float32, "op")  # host memory
    with pytest.raises(errors.B2ShapeError):
        _lib.check_out(torch.empty(2, 3, device="meta"), (2, 4), torch.float32, "op")


def test_fast_binding_is_built_and_declines_host_tensors():
    """_b2fast (the C++ argument handling of the per-layer int4 call) loads on
    a machine without a GPU and hands every case it does not take (here:
    host tensors) back to the Python operator by returning None."""
    import torch
    from b200kern import _lib
    fast = _lib.fast()
    assert fast is not None
    x = torch.zeros(1, 64, dtype=torch.float16)
    w = torch.zeros(8, 32, dtype=torch.int32)
    s = torch.zeros(1, 32, dtype=torch.float16)
    assert fast.int4_matmul(x, w, s, 64, None) is None
    assert fast.int4_matmul(x.float(), w, s, 64) is None


def test_fast_binding_status_raises_the_typed_error(monkeypatch):
    """A nonzero b2 status from the binding raises the same typed error as the
    ctypes path (status -> B2Error subclass)."""
    import pytest
    import torch
    import b200kern as bk
    from b200kern import _lib, errors

    class _Fake:
        @staticmethod
        def int4_matmul(*args):
            return errors.ERR_UNSUPPORTED

    monkeypatch.setattr(_lib, "_fast", _Fake())
    x = torch.zeros(1, 64, dtype=torch.float16)
    with pytest.raises(errors.B2UnsupportedError):
        bk.int4_matmul(x, torch.zeros(8, 32, dtype=torch.int32), torch.zeros(1, 32, dtype=torch.float16),
                       group_size=64)
