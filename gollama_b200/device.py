"""Host-side handles over the C ABI: a device context and device-resident arrays."""
from __future__ import annotations

import ctypes as C
import weakref

import numpy as np

from . import _lib


class GlcError(RuntimeError):
    """A non-zero status returned by libgollama_cuda."""

    def __init__(self, code: int, where: str, message: str):
        self.code = code
        super().__init__(f"{where}: {_lib.ERRORS.get(code, code)}: {message}")


class Context:
    """One device context (glc_ctx): a CUDA device, its compute stream and error word."""

    def __init__(self, device: int = 0):
        self.lib = _lib.lib()
        h = C.c_void_p()
        rc = self.lib.glc_init(device, C.byref(h))
        if rc != 0:
            raise GlcError(rc, "glc_init", f"cannot open device {device} (sm_100a required)")
        self.h = h
        self.device = device
        # objects holding resources of this context, closed before it (order:
        # trainers, then models); weak, so they may also go first on their own
        self._owned: list[tuple[int, weakref.ref]] = []

    def adopt(self, obj, order: int) -> None:
        """Close obj (obj.close()) before this context is destroyed, lower order first."""
        self._owned.append((order, weakref.ref(obj)))

    def check(self, rc: int, where: str) -> None:
        if rc != 0:
            buf = C.create_string_buffer(1024)
            self.lib.glc_last_error(self.h, buf, 1024)
            raise GlcError(rc, where, buf.value.decode(errors="replace"))

    def call(self, name: str, *args) -> None:
        self.check(getattr(self.lib, name)(self.h, *args), name)

    def sync(self) -> None:
        self.call("glc_sync")

    def launches(self) -> int:
        v = C.c_uint64()
        self.call("glc_launch_count", C.byref(v))
        return v.value

    def name(self) -> str:
        buf = C.create_string_buffer(256)
        self.call("glc_device_name", buf, 256)
        return buf.value.decode()

    def close(self) -> None:
        if getattr(self, "h", None):
            # the library's models and trainers refer to the context: they go first
            for _, ref in sorted(getattr(self, "_owned", []), key=lambda e: e[0]):
                obj = ref()
                if obj is not None:
                    obj.close()
            self._owned = []
            self.lib.glc_destroy(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # -- arrays
    def empty(self, shape, dtype=np.float32) -> "DeviceArray":
        return DeviceArray(self, shape, dtype)

    def zeros(self, shape, dtype=np.float32) -> "DeviceArray":
        a = DeviceArray(self, shape, dtype)
        a.zero()
        return a

    def from_numpy(self, x: np.ndarray) -> "DeviceArray":
        x = np.ascontiguousarray(x)
        a = DeviceArray(self, x.shape, x.dtype)
        if x.nbytes:
            self.call("glc_memcpy_h2d", a.ptr, x.ctypes.data_as(C.c_void_p), x.nbytes)
        return a


class DeviceArray:
    """A contiguous device buffer with a numpy shape/dtype (owned; freed on close/GC)."""

    def __init__(self, ctx: Context, shape, dtype=np.float32):
        self.ctx = ctx
        self.shape = tuple(int(s) for s in (shape if isinstance(shape, (tuple, list)) else (shape,)))
        self.dtype = np.dtype(dtype)
        self.nbytes = int(np.prod(self.shape, dtype=np.int64)) * self.dtype.itemsize
        p = C.c_void_p()
        ctx.call("glc_malloc", self.nbytes, C.byref(p))
        self._p = p

    @property
    def ptr(self) -> C.c_void_p:
        return self._p

    @property
    def addr(self) -> int:
        return self._p.value or 0

    def zero(self) -> "DeviceArray":
        if self.nbytes:
            self.ctx.call("glc_memset", self._p, 0, self.nbytes)
        return self

    def numpy(self) -> np.ndarray:
        out = np.empty(self.shape, self.dtype)
        if self.nbytes:
            self.ctx.call("glc_memcpy_d2h", out.ctypes.data_as(C.c_void_p), self._p, self.nbytes)
        return out

    def upload(self, x: np.ndarray) -> None:
        x = np.ascontiguousarray(x, dtype=self.dtype)
        assert x.nbytes == self.nbytes
        if self.nbytes:
            self.ctx.call("glc_memcpy_h2d", self._p, x.ctypes.data_as(C.c_void_p), self.nbytes)

    def free(self) -> None:
        if self._p and self._p.value and self.ctx.h:
            self.ctx.lib.glc_free(self.ctx.h, self._p)
        self._p = C.c_void_p()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass
