"""ctypes binding of libgollama_cuda.so (the C ABI declared in include/gollama_cuda.h).

The library is loaded from the package directory.  There is no fallback: if the
shared object is missing or cannot be loaded, importing this module raises.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libgollama_cuda.so"

GLC_OK = 0
ERRORS = {
    -1: "GLC_ERR_INVALID",
    -2: "GLC_ERR_CUDA",
    -3: "GLC_ERR_DEVICE",
    -4: "GLC_ERR_NOMEM",
    -5: "GLC_ERR_NCCL",
    -6: "GLC_ERR_UNSUPPORTED",
}

_p = C.c_void_p
_i = C.c_int
_f = C.c_float
_d = C.c_double
_sz = C.c_size_t
_u64 = C.c_uint64
_i64 = C.c_int64

# name -> argtypes (every function returns int)
SIGNATURES: dict[str, list] = {
    "glc_init": [_i, C.POINTER(_p)],
    "glc_destroy": [_p],
    "glc_last_error": [_p, C.c_char_p, _sz],
    "glc_device_name": [_p, C.c_char_p, _sz],
    "glc_sync": [_p],
    "glc_launch_count": [_p, C.POINTER(_u64)],
    "glc_malloc": [_p, _sz, C.POINTER(_p)],
    "glc_free": [_p, _p],
    "glc_memcpy_h2d": [_p, _p, _p, _sz],
    "glc_memcpy_d2h": [_p, _p, _p, _sz],
    "glc_memcpy_d2d": [_p, _p, _p, _sz],
    "glc_memset": [_p, _p, _i, _sz],
    "glc_host_alloc": [_p, _sz, C.POINTER(_p)],
    "glc_host_free": [_p, _p],
    "glc_memcpy_h2d_async": [_p, _p, _p, _sz],
    "glc_memcpy_d2h_async": [_p, _p, _p, _sz],
    "glc_timer_start": [_p],
    "glc_timer_stop": [_p, C.POINTER(_f)],
    "glc_linear_fwd": [_p, _p, _p, _p, _i, _i, _i, _p],
    "glc_linear_bwd_dx": [_p, _p, _p, _p, _i, _i, _i, _i],
    "glc_linear_bwd_dw": [_p, _p, _p, _p, _i, _i, _i, _i],
    "glc_gemm_tf32": [_p, _p, _i, _i, _p, _i, _i, _p, _i, _i, _i, _i, _i, _p, _i, _i],
}


def load(path: Path | str = LIB_PATH) -> C.CDLL:
    path = Path(path)
    if not path.exists():
        raise ImportError(
            f"{path} is missing: build it with `python -m gollama_b200.build` "
            "(the CUDA path has no CPU fallback)"
        )
    lib = C.CDLL(str(path))
    for name, argtypes in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = C.c_int
    return lib


_LIB: C.CDLL | None = None


def lib() -> C.CDLL:
    global _LIB
    if _LIB is None:
        _LIB = load()
    return _LIB
