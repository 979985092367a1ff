"""ctypes binding of the CUDA library ``_lib/libsilkern_b200.so``.

The library exports the C ABI declared in ``include/silkern_b200.h``. Loading
fails loudly: there is no CPU or Triton fallback behind these entry points.
"""

from __future__ import annotations

import ctypes
import os
import threading

from silkern_b200.errors import LocalizationError

LIB_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib")
LIB_PATH = os.path.join(LIB_DIR, "libsilkern_b200.so")
ABI_VERSION = 1

_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_u32 = ctypes.c_uint32
_ptr = ctypes.c_void_p

#: name -> (restype, argtypes) for every symbol the header declares.
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "silkern_localize_rowwise_v1": (
        _i32,
        [_ptr, _ptr, _i64, _i64, _ptr, _ptr, _ptr, _i64, _i64, _i32, _i32, _i32, _i32, _i32,
         _ptr, _ptr],
    ),
    "silkern_localize_hierarchical_v1": (
        _i32,
        [_ptr, _ptr, _i64, _i64, _ptr, _ptr, _ptr, _ptr, _ptr, _ptr, _ptr, _i64, _i64, _i32,
         _i32, _i32, _i32, _i32, _i32, _ptr, _ptr],
    ),
    "silkern_workspace_shapes_v1": (_i32, [_i64, _i64, _i32, ctypes.POINTER(_i64)]),
    "silkern_localize_hierarchical_noalloc_v1": (
        _i32,
        [_ptr, _ptr, _i64, _i64, _ptr, _ptr, _ptr, _i64, _i64, _i32, _i32, _i32, _i32, _i32, _i32,
         _ptr, _ptr],
    ),
    "silkern_localize_explicit_v1": (
        _i32,
        [_ptr, _ptr, _i64, _i64, _ptr, _ptr, _ptr, _ptr, _ptr, _i64, _i64, _i32, _i32, _i32,
         _i32, _i32, _i32, _i32, _i32, _i32, _i32, _ptr, _ptr],
    ),
    "silkern_count_mismatches_v1": (_i32, [_ptr, _ptr, _i64, _ptr, _ptr]),
    "silkern_count_segment_mismatches_v1": (_i32, [_ptr, _ptr, _i64, _i64, _ptr, _ptr]),
    "silkern_copy_floor_v1": (_i32, [_ptr, _ptr, _i64, _i32, _i32, _i32, _ptr]),
    "silkern_atomic_baseline_v1": (
        _i32,
        [_ptr, _ptr, _i64, _i64, _ptr, _ptr, _ptr, _ptr, _i64, _i64, _i32, _i32, _i32, _i32, _ptr],
    ),
    "silkern_topk_localize_v1": (
        _i32,
        [_ptr, _i64, _i64, _ptr, _ptr, _ptr, _i64, _i64, _ptr, _ptr, _ptr, _i64, _i32, _i32, _i32,
         _i32, _i32, _i32, _ptr, _ptr],
    ),
    "silkern_topk_localize_explicit_v1": (
        _i32,
        [_ptr, _i64, _i64, _ptr, _ptr, _ptr, _i64, _i64, _ptr, _ptr, _ptr, _i64, _i32, _i32, _i32,
         _i32, _i32, _i32, _i32, _i32, _ptr, _ptr],
    ),
    "silkern_topk_localize_explicit_v2": (
        _i32,
        [_ptr, _i64, _i64, _ptr, _ptr, _ptr, _i64, _i64, _ptr, _ptr, _ptr, _i64, _i32, _i32, _i32,
         _i32, _i32, _i32, _i32, _i32, _i32, _ptr, _ptr],
    ),
    "silkern_status_string_v1": (ctypes.c_char_p, [ctypes.c_int]),
    "silkern_abi_version_v1": (ctypes.c_int, []),
    "silkern_fastdiv_selftest_v1": (_i64, [_u32, _u32, _u32]),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Load the library once and attach the C signatures."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise LocalizationError(
                f"the silkern_b200 CUDA library is not built ({LIB_PATH} is missing); "
                "run `python -m silkern_b200.build`"
            )
        lib = ctypes.CDLL(LIB_PATH)
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        version = lib.silkern_abi_version_v1()
        if version != ABI_VERSION:
            raise LocalizationError(
                f"silkern_b200 library ABI {version} does not match the Python layer ({ABI_VERSION})"
            )
        _lib = lib
        return lib


def status_string(code: int) -> str:
    return load().silkern_status_string_v1(int(code)).decode()


def check(code: int, what: str) -> None:
    """Raise for a non-zero C ABI return code."""
    if code == 0:
        return
    message = status_string(code)
    if code > 0:
        raise LocalizationError(f"{what} rejected by the CUDA library: {message}")
    raise RuntimeError(f"{what} launch failed: CUDA error {-code} ({message})")
