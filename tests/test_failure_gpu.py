"""Failure handling without a GPU fault.

* A bounded device wait: the library's mbarrier wait (gollama_b200/csrc/
  sm100.cuh), built with a 200 ms limit into a test-only kernel
  (tests/native/selftest.cu), waits on a barrier nothing arrives on.  Every
  thread gives up, records the error code and returns; the context stays
  usable for the library's own kernels afterwards.
* A data-parallel rank that never joins: rank 0 of a world of 2 calls
  glc_dp_init and nobody else does.  The non-blocking communicator is polled
  against the caller's deadline, aborted, and glc_dp_init returns
  GLC_ERR_NCCL instead of hanging (pkg/train has no distributed code; the
  reference's only failure path is the SIGINT checkpoint handler,
  cmd/gollama/main.go:850-859).  NVLS is off in the child process."""
import ctypes as C
import multiprocessing as mp
import os
import time

import numpy as np
import pytest

from tests.helpers import rel_fro

pytestmark = pytest.mark.gpu

GLC_ERR_NCCL = -5
TIMEOUT_EPILOGUE = 104  # glc_dev_error code of the waiting role


def _selftest_lib():
    from gollama_b200 import build

    lib = C.CDLL(str(build.SELFTEST_LIB))
    lib.glc_selftest_bounded_wait.argtypes = [C.c_int, C.c_void_p]
    lib.glc_selftest_bounded_wait.restype = C.c_int
    return lib


def _rmsnorm_still_works(ctx):
    x = np.random.default_rng(0).standard_normal((64, 128), dtype=np.float32)
    w = np.ones(128, np.float32)
    bx, bw, by, br = ctx.from_numpy(x), ctx.from_numpy(w), ctx.empty((64, 128)), ctx.empty((64,))
    ctx.call("glc_rmsnorm_fwd", bx.ptr, bw.ptr, by.ptr, br.ptr, 64, 128, C.c_float(1e-5), 0)
    ctx.sync()
    ref = x / np.sqrt((x.astype(np.float64) ** 2).mean(1, keepdims=True) + 1e-5)
    return rel_fro(by.numpy(), ref) < 1e-6


def test_bounded_device_wait_gives_up_and_context_survives(ctx):
    lib = _selftest_lib()
    out = (C.c_longlong * 3)()
    assert lib.glc_selftest_bounded_wait(128, out) == 0
    code, gave_up, ns = out[0], out[1], out[2]
    assert code == TIMEOUT_EPILOGUE
    assert gave_up == 128
    assert 0.19e9 <= ns < 3e9, ns
    assert _rmsnorm_still_works(ctx)


def _never_joined_child(q):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    from gollama_b200.device import Context

    try:
        with Context(0) as ctx:
            uid = (C.c_ubyte * 128)()
            assert ctx.lib.glc_dp_unique_id(uid) == 0
            t0 = time.monotonic()
            rc = ctx.lib.glc_dp_init(ctx.h, 0, 2, uid, 3000)
            elapsed = time.monotonic() - t0
            buf = C.create_string_buffer(512)
            ctx.lib.glc_last_error(ctx.h, buf, 512)
            q.put((rc, elapsed, buf.value.decode(errors="replace"), _rmsnorm_still_works(ctx)))
    except Exception as e:  # report instead of hanging the parent
        q.put(("exception", repr(e), "", False))


def test_dp_init_fails_when_a_rank_never_joins():
    ctx_mp = mp.get_context("spawn")
    q = ctx_mp.Queue()
    p = ctx_mp.Process(target=_never_joined_child, args=(q,))
    p.start()
    try:
        rc, elapsed, msg, usable = q.get(timeout=240)
    finally:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert rc == GLC_ERR_NCCL, (rc, elapsed, msg)
    assert 2.5 <= elapsed < 60, elapsed
    assert "timed out" in msg or "ncclCommInitRankConfig" in msg, msg
    assert usable
