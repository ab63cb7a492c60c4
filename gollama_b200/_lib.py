"""ctypes binding of libgollama_cuda.so.

Argument types are derived from the C declarations in include/gollama_cuda.h,
so the binding cannot drift from the C ABI.  The library is loaded from the
package directory.  There is no fallback: if the shared object is missing or
cannot be loaded, loading raises.
"""
from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libgollama_cuda.so"
HEADER = PKG.parent / "include" / "gollama_cuda.h"

ERRORS = {
    -1: "GLC_ERR_INVALID",
    -2: "GLC_ERR_CUDA",
    -3: "GLC_ERR_DEVICE",
    -4: "GLC_ERR_NOMEM",
    -5: "GLC_ERR_NCCL",
    -6: "GLC_ERR_UNSUPPORTED",
    -7: "GLC_ERR_IO",
}

_SCALARS = {
    "int": C.c_int,
    "float": C.c_float,
    "double": C.c_double,
    "size_t": C.c_size_t,
    "int64_t": C.c_int64,
    "uint64_t": C.c_uint64,
}


def _ctype(decl: str):
    decl = decl.strip()
    if "*" in decl or "[" in decl:
        return C.c_void_p
    words = [w for w in re.split(r"\s+", decl) if w not in ("const", "unsigned")]
    # drop the parameter name
    base = words[0] if len(words) == 1 else " ".join(words[:-1])
    if base not in _SCALARS:
        raise ValueError(f"unsupported C type in header: {decl!r}")
    return _SCALARS[base]


def parse_header(path: Path = HEADER) -> dict[str, list]:
    """name -> argtypes for every `GLC_API int glc_*(...)` declaration."""
    text = path.read_text()
    text = re.sub(r"/\*.*?\*/", " ", text, flags=re.S)
    out: dict[str, list] = {}
    for m in re.finditer(r"GLC_API\s+int\s+(glc_\w+)\s*\(([^)]*)\)\s*;", text, flags=re.S):
        name, args = m.group(1), m.group(2).strip()
        if args in ("", "void"):
            out[name] = []
        else:
            out[name] = [_ctype(a) for a in args.split(",")]
    return out


SIGNATURES = parse_header()


class TrainConfigC(C.Structure):
    """glc_train_config (include/gollama_cuda.h)."""

    _fields_ = [
        ("vocab_size", C.c_int),
        ("hidden_size", C.c_int),
        ("num_layers", C.c_int),
        ("num_heads", C.c_int),
        ("intermediate_size", C.c_int),
        ("max_seq_len", C.c_int),
        ("batch_size", C.c_int),
        ("block_size", C.c_int),
        ("learning_rate", C.c_float),
        ("weight_decay", C.c_float),
        ("warmup_steps", C.c_int),
        ("max_steps", C.c_int),
        ("grad_clip_norm", C.c_float),
        ("beta1", C.c_float),
        ("beta2", C.c_float),
        ("epsilon", C.c_float),
        ("num_kv_heads", C.c_int),
        ("semantics", C.c_int),
        ("norm_eps", C.c_float),
        ("rope_theta", C.c_float),
        ("init_std", C.c_float),
        ("seed", C.c_uint64),
        ("world_size", C.c_int),
    ]


def _nccl_hint() -> None:
    """Point the library at the NCCL that PyTorch bundles, when installed, so
    one process never holds two NCCL builds under the same soname."""
    import importlib.util
    import os

    if "GLC_NCCL_LIB" in os.environ:
        return
    spec = importlib.util.find_spec("nvidia")
    for base in (spec.submodule_search_locations or []) if spec else []:
        cand = Path(base) / "nccl" / "lib" / "libnccl.so.2"
        if cand.exists():
            os.environ["GLC_NCCL_LIB"] = str(cand)
            return


def load(path: Path | str = LIB_PATH) -> C.CDLL:
    _nccl_hint()
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
