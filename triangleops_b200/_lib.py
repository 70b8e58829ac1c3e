"""ctypes binding of the C-ABI library ``libtriangleops_b200.so``.

Every entry point of ``include/triangleops_b200.h`` returns an ``int`` status.
:func:`check` maps it onto the exception types the reference raises for the same
condition: ``AssertionError`` for shape / alignment mismatches (the reference's
``assert`` statements, e.g. ``triangle_attn/kernel.py:273-277``) and
``ValueError`` for an unsupported dtype (``_common/dtype.py:19``) or an unknown
direction (``triangle_mul/module.py:76``).

There is no CPU fallback: if the library is missing or no CUDA device is
present, every op raises.
"""

from __future__ import annotations

import ctypes
import os

import torch

from . import _build

OK = 0
ERR_SHAPE = -1
ERR_DTYPE = -2
ERR_ARG = -3
ERR_ALIGN = -4
ERR_TMAP = -5
ERR_CUDA = -6
ERR_TIMEOUT = -7
ERR_CAPACITY = -8

F16, BF16, F32 = 0, 1, 2
_DTYPE_CODE = {torch.float16: F16, torch.bfloat16: BF16, torch.float32: F32}

_LIB = None

_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_F = ctypes.c_float

# name -> argtypes (restype is always int unless listed in _RESTYPE)
_SIGS: dict[str, list] = {
    "tops_version": [],
    "tops_status_string": [_I],
    "tops_device_error": [_P, ctypes.POINTER(_I)],
    "tops_selftest_umma": [_I, _P, _P, _P, _P],
}
_RESTYPE = {"tops_status_string": ctypes.c_char_p}


def register(name: str, argtypes: list, restype=ctypes.c_int) -> None:
    """Declare the ctypes signature of an entry point (used by the op modules)."""
    _SIGS[name] = argtypes
    if restype is not ctypes.c_int:
        _RESTYPE[name] = restype
    if _LIB is not None:
        _bind(_LIB, name)


def _bind(lib, name):
    fn = getattr(lib, name)
    fn.argtypes = _SIGS[name]
    fn.restype = _RESTYPE.get(name, ctypes.c_int)


def lib():
    """Load (building first if the sources are newer) and return the CDLL."""
    global _LIB
    if _LIB is None:
        path = _build.LIB_PATH
        if _build.needs_build():
            _build.build()
        if not os.path.exists(path):
            raise RuntimeError(f"triangleops_b200 native library not found at {path}")
        _LIB = ctypes.CDLL(path)
        for name in _SIGS:
            _bind(_LIB, name)
    return _LIB


def status_string(code: int) -> str:
    return lib().tops_status_string(code).decode()


def check(code: int, what: str) -> None:
    if code == OK:
        return
    msg = f"{what}: {status_string(code)} (status {code})"
    if code in (ERR_SHAPE, ERR_ALIGN):
        raise AssertionError(msg)
    if code in (ERR_DTYPE, ERR_ARG):
        raise ValueError(msg)
    raise RuntimeError(msg)


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args), name)


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPE_CODE[dtype]
    except KeyError as e:
        raise ValueError(f"unsupported IO dtype {dtype}; expected one of {list(_DTYPE_CODE)}") from e


def require_cuda(*tensors: torch.Tensor) -> None:
    """The product path has no CPU fallback: every tensor must live on a CUDA device."""
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError(
                "triangleops_b200 runs only on CUDA (sm_100a) tensors; got a tensor on "
                f"{t.device}. There is no CPU fallback."
            )


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def device_error(stream: int | None = None) -> tuple[int, int]:
    """Return (status, site) of the device-side error word and clear it."""
    site = ctypes.c_int(0)
    st = lib().tops_device_error(stream if stream is not None else stream_ptr(), ctypes.byref(site))
    return st, site.value
