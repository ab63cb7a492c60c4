"""glc_attention_bwd_noalloc: the attention backward for callers that cannot
allocate device memory during a call (their memory is reserved by their own
allocator, or a call must never synchronise the device, as growing the
library's workspace does).  Its scratch is a fixed device array inside the
library.  Checked through the C ABI against glc_attention_bwd on two calls in a
row; this file is collected last so a failure here stops nothing else."""
import gc
import os

import numpy as np
import pytest

from gollama_b200.device import Context, GlcError
from oracle.oracle import Oracle
from tests.helpers import FP32_RTOL, rel_fro, threads
from tests.test_ops_gpu import ATTN_TOL, tf32

pytestmark = pytest.mark.gpu


def _run(ctx, B, S, H, Hkv, hd, seed, round_dv):
    T = B * S
    r = np.random.default_rng(seed)
    q = r.standard_normal((T, H * hd), dtype=np.float32)
    k = r.standard_normal((T, Hkv * hd), dtype=np.float32)
    v = r.standard_normal((T, Hkv * hd), dtype=np.float32)
    dO = r.standard_normal((T, H * hd), dtype=np.float32)
    bq, bk, bv, bdo = ctx.from_numpy(q), ctx.from_numpy(k), ctx.from_numpy(v), ctx.from_numpy(dO)
    bo, blse = ctx.empty((T, H * hd)), ctx.empty((B, H, S))
    ctx.call("glc_attention_fwd", bq.ptr, bk.ptr, bv.ptr, bo.ptr, blse.ptr, B, S, H, Hkv, hd, 0)
    outs = []
    for name in ("glc_attention_bwd", "glc_attention_bwd_noalloc"):
        dq, dk, dv = ctx.empty(q.shape), ctx.empty(k.shape), ctx.empty(v.shape)
        ctx.call(name, bq.ptr, bk.ptr, bv.ptr, bo.ptr, blse.ptr, bdo.ptr, dq.ptr, dk.ptr, dv.ptr, B, S, H, Hkv, hd,
                 round_dv)
        ctx.sync()
        outs.append((dq.numpy(), dk.numpy(), dv.numpy()))
    return outs


@pytest.mark.parametrize("round_dv", [0, 1])
def test_noalloc_matches_allocating_entry_point_twice(ctx, round_dv):
    # two calls in a row with different shapes and data: the shared scratch
    # keeps the first call's contents, which must not leak into the second.
    # The two entry points sum a KV head's query-head group in different fp32
    # orders (one accumulator across the group here, per-head partials summed
    # afterwards there), so fp32 outputs agree to rounding; with round_dv the
    # TF32 rounding of dV can turn that into one TF32 unit (2^-11 relative).
    tol = FP32_RTOL if round_dv == 0 else 2.0**-11
    for seed, (B, S, H, Hkv, hd) in enumerate([(2, 256, 8, 4, 64), (1, 130, 4, 2, 32)]):
        ref, got = _run(ctx, B, S, H, Hkv, hd, seed, round_dv)
        for a, b in zip(got, ref):
            assert rel_fro(a, b) < tol


def _buffers(c, B, S, H, Hkv, hd, seed):
    """Inputs (with the forward's o and lse) and outputs of one attention
    backward on context c; returns the argument list of the entry points."""
    T = B * S
    r = np.random.default_rng(seed)
    q, dO = (r.standard_normal((T, H * hd), dtype=np.float32) for _ in range(2))
    k, v = (r.standard_normal((T, Hkv * hd), dtype=np.float32) for _ in range(2))
    bq, bk, bv, bdo = c.from_numpy(q), c.from_numpy(k), c.from_numpy(v), c.from_numpy(dO)
    bo, blse = c.empty((T, H * hd)), c.empty((B, H, S))
    c.call("glc_attention_fwd", bq.ptr, bk.ptr, bv.ptr, bo.ptr, blse.ptr, B, S, H, Hkv, hd, 0)
    dq, dk, dv = c.empty(q.shape), c.empty(k.shape), c.empty(v.shape)
    keep = (bq, bk, bv, bdo, bo, blse, dq, dk, dv)
    return keep, [bq.ptr, bk.ptr, bv.ptr, bo.ptr, blse.ptr, bdo.ptr, dq.ptr, dk.ptr, dv.ptr, B, S, H, Hkv, hd, 0]


def test_noalloc_call_allocates_nothing(ctx):
    """The entry point's promise: on a fresh context (no workspace yet), after
    one call, a call with eight times the rows (B*H*S) leaves the device's
    free memory as it was, where glc_attention_bwd would allocate the
    context's workspace.  The kernels of both shapes are loaded first, so no
    lazy module load counts here."""
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device visible to torch")
    dev = int(os.environ.get("GLC_TEST_DEVICE", "0"))
    small, large = (1, 256, 8, 2, 64), (2, 1024, 8, 2, 64)
    keep0, args = _buffers(ctx, *large, 7)
    ctx.call("glc_attention_bwd_noalloc", *args)
    ctx.call("glc_attention_bwd", *args)
    ctx.sync()
    c = Context(dev)
    try:
        keep_s, args_s = _buffers(c, *small, 8)
        keep_l, args_l = _buffers(c, *large, 9)
        c.call("glc_attention_bwd_noalloc", *args_s)
        c.sync()
        # no buffer of an earlier test may be freed by the collector in between
        gc.collect()
        gc.disable()
        try:
            free0 = torch.cuda.mem_get_info(dev)[0]
            c.call("glc_attention_bwd_noalloc", *args_l)
            c.sync()
            free1 = torch.cuda.mem_get_info(dev)[0]
        finally:
            gc.enable()
        assert free1 == free0, (free0, free1)
    finally:
        c.close()


def test_noalloc_rejects_sizes_beyond_its_scratch(ctx):
    B, S, H, Hkv, hd = 1, 1 << 16, 32, 4, 64  # B*H*S = 2^21 rows > 2^20
    with pytest.raises(GlcError) as e:
        ctx.call("glc_attention_bwd_noalloc", None, None, None, None, None, None, None, None, None,
                 B, S, H, Hkv, hd, 0)
    assert e.value.code == -1
    assert "exceeds the fixed scratch" in str(e.value)


def test_noalloc_matches_oracle(ctx):
    """One causal attention backward with a KV head shared by four query heads
    over a 1024-token sequence, against the oracle's restatement of the
    trainer's attention (pkg/train/trainer.go:323-389, head map of
    pkg/model/attention.go:118,149), within the bar of the other attention tests."""
    B, S, H, Hkv, hd = 1, 1024, 4, 1, 64
    T = B * S
    r = np.random.default_rng(1024)
    q = tf32(r.standard_normal((T, H * hd), dtype=np.float32))
    k = tf32(r.standard_normal((T, Hkv * hd), dtype=np.float32))
    v = tf32(r.standard_normal((T, Hkv * hd), dtype=np.float32))
    dO = tf32(r.standard_normal((T, H * hd), dtype=np.float32))
    bq, bk, bv, bdo = ctx.from_numpy(q), ctx.from_numpy(k), ctx.from_numpy(v), ctx.from_numpy(dO)
    bo, blse = ctx.empty((T, H * hd)), ctx.empty((B, H, S))
    ctx.call("glc_attention_fwd", bq.ptr, bk.ptr, bv.ptr, bo.ptr, blse.ptr, B, S, H, Hkv, hd, 0)
    dq, dk, dv = ctx.empty(q.shape), ctx.empty(k.shape), ctx.empty(v.shape)
    ctx.call("glc_attention_bwd_noalloc", bq.ptr, bk.ptr, bv.ptr, bo.ptr, blse.ptr, bdo.ptr, dq.ptr, dk.ptr, dv.ptr,
             B, S, H, Hkv, hd, 0)
    ctx.sync()
    ref = Oracle(threads=threads()).attention_bwd(q, k, v, dO, S, H, Hkv, hd)
    errs = [rel_fro(a.numpy(), b) for a, b in zip((dq, dk, dv), ref)]
    assert max(errs) < ATTN_TOL, errs
