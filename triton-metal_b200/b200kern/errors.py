"""Typed errors mapped from the C ABI status codes (include/b2.h).

The reference raises RuntimeError on a failed Metal command buffer
(triton_metal/backend/driver.py:220-225) and has typed compile/launch
errors (triton_metal/errors.py:13-103); these are the CUDA-side analogues.
"""

OK = 0
ERR_INVALID = -1
ERR_DTYPE = -2
ERR_ALIGN = -3
ERR_UNSUPPORTED = -4
ERR_LAUNCH = -5
ERR_TIMEOUT = -6


class B2Error(RuntimeError):
    """Base error of the b200kern ops."""


class B2ShapeError(B2Error, ValueError):
    pass


class B2DtypeError(B2Error, TypeError):
    pass


class B2AlignmentError(B2Error, ValueError):
    pass


class B2UnsupportedError(B2Error, NotImplementedError):
    pass


class B2LaunchError(B2Error):
    pass


class B2TimeoutError(B2Error, TimeoutError):
    pass


_BY_CODE = {
    ERR_INVALID: B2ShapeError,
    ERR_DTYPE: B2DtypeError,
    ERR_ALIGN: B2AlignmentError,
    ERR_UNSUPPORTED: B2UnsupportedError,
    ERR_LAUNCH: B2LaunchError,
    ERR_TIMEOUT: B2TimeoutError,
}


def raise_for_status(status, where, message):
    cls = _BY_CODE.get(status, B2Error)
    raise cls(f"{where} failed (status {status}): {message}")
