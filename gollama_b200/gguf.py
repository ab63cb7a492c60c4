"""GGUF files through libgollama_cuda (host parser in csrc/gguf.cpp).

Mirrors gguf.Reader (pkg/gguf/reader.go) and gguf.TensorInfo
(pkg/gguf/format.go:152-186) with the Go names: Open, Close, Header,
Metadata, GetMetadata, GetString, GetUint32, GetUint64, GetFloat32,
GetInt32, GetStringArray, GetFloat32Array, GetInt32Array, Tensors,
GetTensorInfo, GetTensorData, Architecture.  The typed getters return
(value, ok) and succeed only when the stored value has exactly that type,
like Go's type assertions.  Metadata values keep their GGUF type: numpy
scalars for the sized numeric types, bool, str, and lists for arrays.

Two device calls sit beside them: UploadTensor puts a tensor's stored bytes
(quantized blocks as they are) in device memory, the weight operand of
glc_linear_bwd_dx_q, and LoadTensor is loadTensor
(pkg/model/transformer.go:285-303) with the dequantization on the device.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np

from . import _lib
from .device import GlcError

# metadata value types (pkg/gguf/format.go:20-34)
TypeUint8, TypeInt8, TypeUint16, TypeInt16, TypeUint32, TypeInt32, TypeFloat32, TypeBool, TypeString, TypeArray, \
    TypeUint64, TypeInt64, TypeFloat64 = range(13)
_NUMPY = {TypeUint8: np.uint8, TypeInt8: np.int8, TypeUint16: np.uint16, TypeInt16: np.int16, TypeUint32: np.uint32,
          TypeInt32: np.int32, TypeFloat32: np.float32, TypeUint64: np.uint64, TypeInt64: np.int64,
          TypeFloat64: np.float64}
_SIGNED = {TypeInt8, TypeInt16, TypeInt32, TypeInt64}
_FLOAT = {TypeFloat32, TypeFloat64}

# GGMLType.String (format.go:70-103)
TYPE_NAMES = {0: "F32", 1: "F16", 2: "Q4_0", 3: "Q4_1", 6: "Q5_0", 7: "Q5_1", 8: "Q8_0", 9: "Q8_1", 10: "Q2_K",
              11: "Q3_K", 12: "Q4_K", 13: "Q5_K", 14: "Q6_K", 15: "Q8_K", 30: "BF16"}
# GetTypeInfo (format.go:117-149): (elements per block, bytes per block)
TYPE_INFO = {0: (1, 4), 1: (1, 2), 2: (32, 18), 3: (32, 20), 6: (32, 22), 7: (32, 24), 8: (32, 34), 9: (32, 36),
             10: (256, 84), 11: (256, 110), 12: (256, 144), 13: (256, 176), 14: (256, 210), 15: (256, 292),
             30: (1, 2)}


def _check(rc: int, where: str) -> None:
    if rc != 0:
        buf = C.create_string_buffer(1024)
        _lib.lib().glc_last_error(None, buf, 1024)
        raise GlcError(rc, where, buf.value.decode(errors="replace"))


@dataclass
class Header:
    Magic: int
    Version: int
    TensorCount: int
    MetadataKVCount: int


@dataclass
class TensorInfo:
    Name: str
    NDims: int
    Dimensions: list = field(default_factory=list)  # GGUF order: innermost first
    Type: int = 0
    Offset: int = 0
    _index: int = -1

    def NumElements(self) -> int:
        if not self.Dimensions:
            return 0
        n = 1
        for d in self.Dimensions:
            n *= d
        return n

    def SizeBytes(self) -> int:
        block, size = TYPE_INFO.get(self.Type, (1, 4))
        return (self.NumElements() + block - 1) // block * size

    def Shape(self) -> list:
        """Logical order (format.go:181-188): the GGUF dimensions reversed."""
        return [int(d) for d in reversed(self.Dimensions)]

    def TypeName(self) -> str:
        return TYPE_NAMES.get(self.Type, "UNKNOWN")


class Reader:
    """gguf.Reader: a read-only mapping of one GGUF file."""

    def __init__(self, path):
        self._lib = _lib.lib()
        h = C.c_void_p()
        _check(self._lib.glc_gguf_open(str(path).encode(), C.byref(h)), "glc_gguf_open")
        self.h = h
        ver, nt, nkv, off = C.c_uint32(), C.c_uint64(), C.c_uint64(), C.c_uint64()
        _check(self._lib.glc_gguf_header(h, C.byref(ver), C.byref(nt), C.byref(nkv), C.byref(off)), "glc_gguf_header")
        self._header = Header(0x46554747, ver.value, nt.value, nkv.value)
        self.data_offset = off.value
        self._meta = {}
        self._types = {}
        for i in range(nkv.value):
            key = self._string(self._lib.glc_gguf_meta_key, i)
            self._meta[key], self._types[key] = self._value(i)
        self._tensors = [self._tensor(i) for i in range(nt.value)]
        self._by_name = {t.Name: t for t in self._tensors}  # a later duplicate wins, like the reference's map

    # -- helpers
    def _string(self, fn, *args) -> str:
        n = C.c_size_t()
        _check(fn(self.h, *args, None, 0, C.byref(n)), fn.__name__)
        buf = C.create_string_buffer(n.value + 1)
        _check(fn(self.h, *args, buf, n.value + 1, C.byref(n)), fn.__name__)
        return buf.raw[: n.value].decode("utf-8", errors="surrogateescape")

    def _scalar(self, i: int, t: int, elem: int):
        if t == TypeString:
            return self._string(self._lib.glc_gguf_meta_string, i, C.c_uint64(elem))
        si, ui, fd = C.c_int64(), C.c_uint64(), C.c_double()
        _check(self._lib.glc_gguf_meta_number(self.h, i, C.c_uint64(elem), C.byref(si), C.byref(ui), C.byref(fd)),
               "glc_gguf_meta_number")
        if t == TypeBool:
            return bool(ui.value)
        if t in _FLOAT:
            return _NUMPY[t](fd.value)
        return _NUMPY[t](si.value if t in _SIGNED else ui.value)

    def _value(self, i: int):
        t, et, n = C.c_int(), C.c_int(), C.c_uint64()
        _check(self._lib.glc_gguf_meta_type(self.h, i, C.byref(t), C.byref(et), C.byref(n)), "glc_gguf_meta_type")
        if t.value != TypeArray:
            return self._scalar(i, t.value, 0), (t.value, None)
        if et.value == TypeArray:  # nested arrays: only their count is exposed
            return [None] * n.value, (TypeArray, TypeArray)
        return [self._scalar(i, et.value, k) for k in range(n.value)], (TypeArray, et.value)

    def _tensor(self, i: int) -> TensorInfo:
        n = C.c_size_t()
        t, nd, off, nb = C.c_int(), C.c_int(), C.c_uint64(), C.c_uint64()
        _check(self._lib.glc_gguf_tensor_info(self.h, i, None, 0, C.byref(n), C.byref(t), C.byref(nd), None, 0,
                                              C.byref(off), C.byref(nb)), "glc_gguf_tensor_info")
        buf = C.create_string_buffer(n.value + 1)
        dims = (C.c_uint64 * max(nd.value, 1))()
        _check(self._lib.glc_gguf_tensor_info(self.h, i, buf, n.value + 1, C.byref(n), C.byref(t), C.byref(nd), dims,
                                              nd.value, C.byref(off), C.byref(nb)), "glc_gguf_tensor_info")
        name = buf.raw[: n.value].decode("utf-8", errors="surrogateescape")
        return TensorInfo(name, nd.value, [int(dims[k]) for k in range(nd.value)], t.value, off.value, i)

    # -- reader.go API
    def Close(self) -> None:
        if getattr(self, "h", None):
            self._lib.glc_gguf_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.Close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.Close()

    def Header(self) -> Header:
        return self._header

    def Metadata(self) -> dict:
        return dict(self._meta)

    def GetMetadata(self, key):
        return (self._meta[key], True) if key in self._meta else (None, False)

    def _typed(self, key, want):
        if key not in self._meta or self._types[key] != (want, None):
            return None, False
        return self._meta[key], True

    def GetString(self, key):
        v, ok = self._typed(key, TypeString)
        return (v, True) if ok else ("", False)

    def GetUint32(self, key):
        v, ok = self._typed(key, TypeUint32)
        return (v, True) if ok else (0, False)

    def GetUint64(self, key):
        v, ok = self._typed(key, TypeUint64)
        return (v, True) if ok else (0, False)

    def GetFloat32(self, key):
        v, ok = self._typed(key, TypeFloat32)
        return (v, True) if ok else (0.0, False)

    def GetInt32(self, key):
        v, ok = self._typed(key, TypeInt32)
        return (v, True) if ok else (0, False)

    def _array(self, key, want):
        if key not in self._meta or self._types[key] != (TypeArray, want):
            return None, False
        return list(self._meta[key]), True

    def GetStringArray(self, key):
        return self._array(key, TypeString)

    def GetFloat32Array(self, key):
        return self._array(key, TypeFloat32)

    def GetInt32Array(self, key):
        return self._array(key, TypeInt32)

    def Tensors(self) -> list:
        return list(self._tensors)

    def GetTensorInfo(self, name):
        t = self._by_name.get(name)
        return (t, t is not None)

    def _index(self, name) -> int:
        t = self._by_name.get(name)
        if t is None:
            raise KeyError(f"tensor not found: {name}")
        return t._index

    def GetTensorData(self, name) -> bytes:
        p, n = C.c_void_p(), C.c_uint64()
        _check(self._lib.glc_gguf_tensor_data(self.h, self._index(name), C.byref(p), C.byref(n)),
               "glc_gguf_tensor_data")
        return C.string_at(p, n.value) if n.value else b""

    def Architecture(self) -> str:
        return self.GetString("general.architecture")[0]

    # -- device
    def UploadTensor(self, ctx, name):
        """The stored bytes of `name` in a device uint8 array."""
        t = self._by_name[name]
        buf = ctx.empty((t.SizeBytes(),), np.uint8)
        ctx.check(self._lib.glc_gguf_tensor_upload(ctx.h, self.h, t._index, buf.ptr, buf.nbytes),
                  "glc_gguf_tensor_upload")
        return buf

    def LoadTensor(self, ctx, name):
        """loadTensor on the device: a float32 device array of the tensor's
        logical shape, dequantized bit-exactly."""
        t = self._by_name[name]
        out = ctx.empty(tuple(t.Shape()) or (0,), np.float32)
        ctx.check(self._lib.glc_gguf_tensor_load(ctx.h, self.h, t._index, out.ptr, t.NumElements()),
                  "glc_gguf_tensor_load")
        return out


def Open(path) -> Reader:
    """gguf.Open (reader.go:22-49)."""
    return Reader(path)


__all__ = ["Open", "Reader", "Header", "TensorInfo", "TYPE_NAMES", "TYPE_INFO"]
