"""Checkpoint files through libgollama_cuda's host-only entry points.

The text format is the one Trainer.SaveCheckpoint writes
(pkg/train/trainer.go:554-584): a `GOLLAMA_CKPT` header with the step and
the model dimensions, a `WEIGHTS` line, then one line per parameter in
Params() order with each float32 printed as Go's `%v` prints it and followed
by a space.  The binary state file adds what the text format lacks (AdamW's
m, v and step, the scheduler's step).  These functions touch no device; the
trainer's own save/load methods (gollama_b200.train) move the device arenas.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib
from .device import GlcError


def _check(rc: int, where: str) -> None:
    if rc != 0:
        buf = C.create_string_buffer(1024)
        _lib.lib().glc_last_error(None, buf, 1024)
        raise GlcError(rc, where, buf.value.decode(errors="replace"))


def _path(p) -> bytes:
    return str(p).encode()


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def param_count(cfg) -> int:
    """Parameter count of a TrainConfig's model (Params() of NewTrainableModel):
    the end of the last gradient bucket, which closes the arena."""
    n = C.c_int()
    c = cfg.to_c()
    _check(_lib.lib().glc_dp_bucket_plan(C.byref(c), None, None, 0, C.byref(n)), "glc_dp_bucket_plan")
    begin = (C.c_int64 * n.value)()
    end = (C.c_int64 * n.value)()
    _check(_lib.lib().glc_dp_bucket_plan(C.byref(c), begin, end, n.value, C.byref(n)), "glc_dp_bucket_plan")
    return int(end[n.value - 1])


def write_checkpoint(path, step: int, cfg, params: np.ndarray) -> None:
    """Writes `params` (the flat Params() arena) in SaveCheckpoint's text format."""
    flat = np.ascontiguousarray(params, np.float32).reshape(-1)
    c = cfg.to_c()
    _check(_lib.lib().glc_checkpoint_write(_path(path), step, C.byref(c), _ptr(flat), flat.size),
           "glc_checkpoint_write")


def read_checkpoint(path, cfg) -> tuple[int, np.ndarray]:
    """Reads a SaveCheckpoint text file of `cfg`'s model: (step, flat parameters)."""
    flat = np.empty(param_count(cfg), np.float32)
    step = C.c_int()
    c = cfg.to_c()
    _check(_lib.lib().glc_checkpoint_read(_path(path), C.byref(c), C.byref(step), _ptr(flat), flat.size),
           "glc_checkpoint_read")
    return step.value, flat


def write_state(path, cfg, step: int, adam_step: int, params: np.ndarray, m: np.ndarray, v: np.ndarray) -> None:
    arrs = [np.ascontiguousarray(a, np.float32).reshape(-1) for a in (params, m, v)]
    if len({a.size for a in arrs}) != 1:
        raise ValueError("params, m and v must have the same size")
    c = cfg.to_c()
    _check(_lib.lib().glc_state_write(_path(path), C.byref(c), step, adam_step, *(_ptr(a) for a in arrs),
                                      arrs[0].size), "glc_state_write")


def read_state(path, cfg) -> tuple[int, int, np.ndarray, np.ndarray, np.ndarray]:
    """(step, adam_step, params, m, v) of a binary state file of `cfg`'s model."""
    n = param_count(cfg)
    arrs = [np.empty(n, np.float32) for _ in range(3)]
    step, adam_step = C.c_int(), C.c_int()
    c = cfg.to_c()
    _check(_lib.lib().glc_state_read(_path(path), C.byref(c), C.byref(step), C.byref(adam_step),
                                     *(_ptr(a) for a in arrs), n), "glc_state_read")
    return step.value, adam_step.value, *arrs


__all__ = ["param_count", "write_checkpoint", "read_checkpoint", "write_state", "read_state"]
