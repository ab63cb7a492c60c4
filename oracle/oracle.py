"""ctypes wrapper of the CPU oracle (oracle/liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, by __graft_entry__.smoke() and by
bench.py's CPU-baseline leg, always as the checker, never as the thing measured
or shipped.  Parity status: UNPINNED (see oracle.h).
"""
from __future__ import annotations

import ctypes as C
import subprocess
from dataclasses import dataclass
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"

MODE_REFERENCE = 0
MODE_LLAMA = 1


def build() -> Path:
    r = subprocess.run(["make", "-C", str(HERE)], capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{r.stdout}\n{r.stderr}")
    return LIB_PATH


class Config(C.Structure):
    _fields_ = [
        ("vocab", C.c_int),
        ("hidden", C.c_int),
        ("layers", C.c_int),
        ("heads", C.c_int),
        ("kv_heads", C.c_int),
        ("inter", C.c_int),
        ("max_seq", C.c_int),
        ("norm_eps", C.c_float),
        ("rope_theta", C.c_float),
        ("mode", C.c_int),
    ]


class OptimState(C.Structure):
    _fields_ = [
        ("lr", C.c_float),
        ("beta1", C.c_float),
        ("beta2", C.c_float),
        ("eps", C.c_float),
        ("weight_decay", C.c_float),
        ("adam_step", C.c_int),
        ("initial_lr", C.c_float),
        ("warmup_steps", C.c_int),
        ("total_steps", C.c_int),
        ("grad_clip", C.c_float),
        ("trainer_step", C.c_int),
    ]


SCALAR_LIB_PATH = HERE / "liboracle_scalar.so"
_libs: dict = {}


def lib(scalar: bool = False) -> C.CDLL:
    """The oracle library: the test build, or (scalar=True) the build compiled
    like Go's amd64 code, which the CPU baseline times."""
    path = SCALAR_LIB_PATH if scalar else LIB_PATH
    if path not in _libs:
        if not path.exists():
            build()
        L = C.CDLL(str(path))
        for pre in ("orc_", "orcd_"):
            for name in ("exp32", "log32"):
                getattr(L, pre + name).restype = C.c_float
                getattr(L, pre + name).argtypes = [C.c_float]
            for name in ("go_exp", "go_log"):
                getattr(L, pre + name).restype = C.c_double
                getattr(L, pre + name).argtypes = [C.c_double]
            getattr(L, pre + "param_total").restype = C.c_int64
            getattr(L, pre + "get_lr").restype = C.c_float
            getattr(L, pre + "grad_clip").restype = C.c_double
        L.orc_softmax_ce.restype = C.c_float
        L.orcd_softmax_ce.restype = C.c_double
        L.orc_forward_backward.restype = C.c_float
        L.orcd_forward_backward.restype = C.c_double
        L.orc_train_step.restype = C.c_float
        L.orcd_train_step.restype = C.c_double
        _libs[path] = L
    return _libs[path]


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


class Oracle:
    """Typed access to one precision of the oracle (float32: orc_, float64: orcd_)."""

    def __init__(self, double: bool = False, threads: int = 1, literal: bool = False, scalar: bool = False):
        self.L = lib(scalar)
        self.pre = "orcd_" if double else "orc_"
        self.dtype = np.float64 if double else np.float32
        self.fn("set_threads")(int(threads), int(bool(literal)))

    def fn(self, name):
        return getattr(self.L, self.pre + name)

    def set_threads(self, threads: int, literal: bool = False):
        self.fn("set_threads")(int(threads), int(bool(literal)))

    def arr(self, x) -> np.ndarray:
        return np.ascontiguousarray(x, dtype=self.dtype)

    # -- model layout
    def param_layout(self, cfg: Config):
        n = self.fn("num_params")(C.byref(cfg))
        out = []
        for i in range(n):
            off, r, c = C.c_int64(), C.c_int64(), C.c_int64()
            self.fn("param_info")(C.byref(cfg), i, C.byref(off), C.byref(r), C.byref(c))
            out.append((off.value, r.value, c.value))
        return out

    def param_total(self, cfg: Config) -> int:
        return int(self.fn("param_total")(C.byref(cfg)))

    # -- ops
    def matmul_transpose_b(self, a, b):
        a, b = self.arr(a), self.arr(b)
        M, K = a.shape
        N = b.shape[0]
        out = np.zeros((M, N), self.dtype)
        self.fn("matmul_transpose_b")(_p(a), _p(b), _p(out), M, K, N)
        return out

    def matmul_grad_da(self, dc, b, da=None):
        dc, b = self.arr(dc), self.arr(b)
        M, N = dc.shape
        K = b.shape[1]
        da = np.zeros((M, K), self.dtype) if da is None else da
        self.fn("matmul_grad_da")(_p(dc), _p(b), _p(da), M, K, N)
        return da

    def matmul_grad_db(self, dc, a, db=None):
        dc, a = self.arr(dc), self.arr(a)
        M, N = dc.shape
        K = a.shape[1]
        db = np.zeros((N, K), self.dtype) if db is None else db
        self.fn("matmul_grad_db")(_p(dc), _p(a), _p(db), M, K, N)
        return db

    def rmsnorm_fwd(self, x, w, eps=1e-5):
        x, w = self.arr(x), self.arr(w)
        rows, cols = x.shape
        out = np.zeros_like(x)
        rms = np.zeros(rows, self.dtype)
        self.fn("rmsnorm_fwd")(_p(x), _p(w), _p(out), _p(rms), rows, cols, C.c_float(eps))
        return out, rms

    def rmsnorm_bwd(self, x, w, rms, dout, full, dx=None, dw=None):
        x, w, rms, dout = self.arr(x), self.arr(w), self.arr(rms), self.arr(dout)
        rows, cols = x.shape
        dx = np.zeros_like(x) if dx is None else dx
        dw = np.zeros_like(w) if dw is None else dw
        self.fn("rmsnorm_bwd")(_p(x), _p(w), _p(rms), _p(dout), _p(dx), _p(dw), rows, cols, int(full))
        return dx, dw

    def silu_fwd(self, x):
        x = self.arr(x)
        out, sig = np.zeros_like(x), np.zeros_like(x)
        self.fn("silu_fwd")(_p(x), _p(out), _p(sig), C.c_int64(x.size))
        return out, sig

    def silu_bwd(self, x, sig, dout, dx=None):
        x, sig, dout = self.arr(x), self.arr(sig), self.arr(dout)
        dx = np.zeros_like(x) if dx is None else dx
        self.fn("silu_bwd")(_p(x), _p(sig), _p(dout), _p(dx), C.c_int64(x.size))
        return dx

    def softmax_ce(self, logits, targets, want_probs=False):
        logits = self.arr(logits)
        t = np.ascontiguousarray(targets, np.int64)
        rows, V = logits.shape
        probs = np.zeros_like(logits) if want_probs else None
        loss = self.fn("softmax_ce")(_p(logits), _p(t), rows, V, _p(probs))
        return (float(loss), probs) if want_probs else float(loss)

    def softmax_ce_grad(self, probs, targets, dlogits=None):
        probs = self.arr(probs)
        t = np.ascontiguousarray(targets, np.int64)
        rows, V = probs.shape
        dl = np.zeros_like(probs) if dlogits is None else dlogits
        self.fn("softmax_ce_grad")(_p(probs), _p(t), rows, V, _p(dl))
        return dl

    def rope_table(self, hd, max_seq, theta):
        cos_t = np.zeros((max_seq, hd // 2), self.dtype)
        sin_t = np.zeros((max_seq, hd // 2), self.dtype)
        self.fn("rope_table")(hd, max_seq, C.c_float(theta), _p(cos_t), _p(sin_t))
        return cos_t, sin_t

    def rope_apply(self, x, S, nh, hd, cos_t, sin_t, inverse=False):
        x = self.arr(x).copy()
        T = x.shape[0]
        self.fn("rope_apply")(_p(x), T, S, nh, hd, _p(self.arr(cos_t)), _p(self.arr(sin_t)), int(inverse))
        return x

    def attention_fwd(self, q, k, v, S, H, Hkv, hd):
        q, k, v = self.arr(q), self.arr(k), self.arr(v)
        T = q.shape[0]
        out = np.zeros((T, H * hd), self.dtype)
        self.fn("attention_fwd")(_p(q), _p(k), _p(v), _p(out), T, S, H, Hkv, hd)
        return out

    def attention_bwd(self, q, k, v, dout, S, H, Hkv, hd):
        q, k, v, dout = self.arr(q), self.arr(k), self.arr(v), self.arr(dout)
        T = q.shape[0]
        dq, dk, dv = np.zeros_like(q), np.zeros_like(k), np.zeros_like(v)
        self.fn("attention_bwd")(_p(q), _p(k), _p(v), _p(dout), _p(dq), _p(dk), _p(dv), T, S, H, Hkv, hd)
        return dq, dk, dv

    def exp32(self, x: float) -> float:
        return float(self.L.orc_exp32(C.c_float(x)))

    def log32(self, x: float) -> float:
        return float(self.L.orc_log32(C.c_float(x)))

    def get_lr(self, st: OptimState, step: int) -> float:
        return float(self.fn("get_lr")(C.byref(st), int(step)))

    # -- whole model
    def forward_backward(self, cfg: Config, params, inputs, targets, backward=True):
        params = self.arr(params)
        B, S = inputs.shape
        grads = np.zeros_like(params)
        has = np.zeros(self.fn("num_params")(C.byref(cfg)), np.uint8)
        inp = np.ascontiguousarray(inputs, np.int64)
        tgt = np.ascontiguousarray(targets, np.int64)
        loss = self.fn("forward_backward")(
            C.byref(cfg), _p(params), _p(grads), _p(has), _p(inp), _p(tgt), B, S, int(backward)
        )
        return float(loss), grads, has.astype(bool)

    def train_step(self, cfg: Config, state: "TrainState", inputs, targets):
        B, S = inputs.shape
        inp = np.ascontiguousarray(inputs, np.int64)
        tgt = np.ascontiguousarray(targets, np.int64)
        norm = C.c_double()
        loss = self.fn("train_step")(
            C.byref(cfg), _p(state.params), _p(state.grads), _p(state.has_grad), _p(state.m), _p(state.v),
            C.byref(state.opt), _p(inp), _p(tgt), B, S, C.byref(norm),
        )
        return float(loss), float(norm.value)


@dataclass
class TrainState:
    """Mutable training state of the oracle: params, grads (+ which exist), AdamW m/v."""

    params: np.ndarray
    grads: np.ndarray
    has_grad: np.ndarray
    m: np.ndarray
    v: np.ndarray
    opt: OptimState

    @classmethod
    def create(cls, params: np.ndarray, n_params: int, opt: OptimState, dtype=np.float32):
        p = np.ascontiguousarray(params, dtype).copy()
        return cls(p, np.zeros_like(p), np.zeros(n_params, np.uint8), np.zeros_like(p), np.zeros_like(p), opt)
