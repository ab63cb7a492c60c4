"""Out-of-bounds writes, caught without a sanitizer: every output of the ops
below lies inside a larger allocation whose guard regions (before, after,
and between the rows of strided outputs) hold a sentinel NaN pattern, and
after the op the guards must still hold it.  Shapes are ragged on purpose
(rows and columns that are not multiples of the kernels' tiles, sequences
that end inside a tile).  Inputs are ordinary in-bounds buffers."""
import ctypes as C

import numpy as np
import pytest

from tests.test_quant import Q4_K, sane_format_weight

pytestmark = pytest.mark.gpu

GUARD = 256  # floats on each side: keeps 16-byte (and 1 KB) alignment
SENT = np.uint32(0x7FBADBAD)


class Guarded:
    """A device array of n floats (or int64-free float payload) between two
    guard regions; rows of a strided [rows][cols] view with row stride ld keep
    their padding columns as guards too."""

    def __init__(self, ctx, n, init=None, rows=None, cols=None, ld=None):
        self.n, self.rows, self.cols, self.ld = n, rows, cols, ld
        host = np.full(n + 2 * GUARD, SENT, np.uint32).view(np.float32)
        if init is not None:
            body = host[GUARD:GUARD + n]
            if ld is not None:
                body.reshape(rows, ld)[:, :cols] = np.asarray(init, np.float32).reshape(rows, cols)
            else:
                body[:] = np.asarray(init, np.float32).reshape(-1)
        self.buf = ctx.from_numpy(host)
        self.ptr = C.c_void_p(self.buf.addr + GUARD * 4)

    def check(self, what):
        h = self.buf.numpy().view(np.uint32)
        assert np.all(h[:GUARD] == SENT), f"{what}: write before the buffer"
        assert np.all(h[GUARD + self.n:] == SENT), f"{what}: write past the buffer"
        if self.ld is not None and self.ld > self.cols:
            pad = h[GUARD:GUARD + self.n].reshape(self.rows, self.ld)[:, self.cols:]
            assert np.all(pad == SENT), f"{what}: write into the row padding"


def rnd(shape, seed, scale=1.0):
    return (np.random.default_rng(seed).standard_normal(shape) * scale).astype(np.float32)


@pytest.mark.parametrize("M,K,N", [(300, 100, 196), (129, 36, 260), (5, 2048, 12)])
def test_linear_ops(ctx, M, K, N):
    x, w, dy = ctx.from_numpy(rnd((M, K), 1)), ctx.from_numpy(rnd((N, K), 2)), ctx.from_numpy(rnd((M, N), 3))
    y = Guarded(ctx, M * N)
    ctx.call("glc_linear_fwd", x.ptr, w.ptr, y.ptr, M, K, N, None)
    dx = Guarded(ctx, M * K, init=rnd((M, K), 4))
    ctx.call("glc_linear_bwd_dx", dy.ptr, w.ptr, dx.ptr, M, K, N, 1)
    dw = Guarded(ctx, N * K, init=rnd((N, K), 5))
    ctx.call("glc_linear_bwd_dw", dy.ptr, x.ptr, dw.ptr, M, K, N, 1)
    ctx.sync()
    for g, name in ((y, "linear_fwd"), (dx, "linear_bwd_dx"), (dw, "linear_bwd_dw")):
        g.check(name)


@pytest.mark.parametrize("M,N,K,ldc", [(300, 196, 100, 212), (257, 260, 64, 264)])
def test_gemm_strided_output(ctx, M, N, K, ldc):
    a, b = ctx.from_numpy(rnd((M, K), 6)), ctx.from_numpy(rnd((N, K), 7))
    c = Guarded(ctx, M * ldc, init=rnd((M, N), 8), rows=M, cols=N, ld=ldc)
    ctx.call("glc_gemm_tf32", a.ptr, K, 0, b.ptr, K, 0, c.ptr, ldc, M, N, K, 1, None, 0, 0)
    ctx.sync()
    c.check("gemm_tf32 (ldc > N)")


@pytest.mark.parametrize("rows,cols", [(333, 2048), (77, 516), (3, 8192)])
def test_rmsnorm(ctx, rows, cols):
    x, w = ctx.from_numpy(rnd((rows, cols), 9)), ctx.from_numpy(1 + rnd(cols, 10, 0.1))
    y, rms = Guarded(ctx, rows * cols), Guarded(ctx, rows)
    ctx.call("glc_rmsnorm_fwd", x.ptr, w.ptr, y.ptr, rms.ptr, rows, cols, C.c_float(1e-5), 1)
    g = ctx.from_numpy(rnd((rows, cols), 11))
    dx, dxr, dw = Guarded(ctx, rows * cols, init=rnd((rows, cols), 12)), Guarded(ctx, rows * cols), \
        Guarded(ctx, cols, init=rnd(cols, 13))
    ctx.call("glc_rmsnorm_bwd", x.ptr, w.ptr, rms.ptr, g.ptr, dx.ptr, dxr.ptr, dw.ptr, rows, cols, 1, 1, 1)
    ctx.sync()
    for a, name in ((y, "rmsnorm y"), (rms, "rmsnorm rms"), (dx, "rmsnorm dx"), (dxr, "rmsnorm dx_round"),
                    (dw, "rmsnorm dw")):
        a.check(name)


def test_swiglu(ctx):
    n = 4 * 250001
    gt, up, dh = ctx.from_numpy(rnd(n, 14, 3)), ctx.from_numpy(rnd(n, 15)), ctx.from_numpy(rnd(n, 16))
    h = Guarded(ctx, n)
    ctx.call("glc_swiglu_fwd", gt.ptr, up.ptr, h.ptr, n, 1)
    dg, du = Guarded(ctx, n, init=rnd(n, 17)), Guarded(ctx, n, init=rnd(n, 18))
    ctx.call("glc_swiglu_bwd", gt.ptr, up.ptr, dh.ptr, dg.ptr, du.ptr, n, 1, 1)
    ctx.sync()
    for a, name in ((h, "swiglu h"), (dg, "swiglu dgate"), (du, "swiglu dup")):
        a.check(name)


@pytest.mark.parametrize("rows,V", [(37, 40000), (33, 1000), (5, 8196), (37, 32000), (7, 16388)])
@pytest.mark.parametrize("fn,variant", [("glc_softmax_ce", 0), ("glc_softmax_ce", 2), ("glc_softmax_ce_llama", 0),
                                        ("glc_softmax_ce_llama", 1)])
def test_softmax_ce_in_place(ctx, rows, V, fn, variant):
    logits = Guarded(ctx, rows * V, init=rnd((rows, V), 19, 2.0))
    tg = ctx.from_numpy(np.random.default_rng(20).integers(-1, V + 1, rows).astype(np.int64))
    logp, loss = Guarded(ctx, rows), Guarded(ctx, 1)
    try:
        ctx.call("glc_set_ce_variant", variant)
        ctx.call(fn, logits.ptr, tg.ptr, rows, V, C.c_float(1.0 / rows), logp.ptr, loss.ptr, 1, 1)
        ctx.sync()
    finally:
        ctx.call("glc_set_ce_variant", 0)
    for a, name in ((logits, "ce dlogits"), (logp, "ce row_logp"), (loss, "ce loss")):
        a.check(name)


@pytest.mark.parametrize("B,S,H,Hkv,hd", [(2, 257, 4, 2, 64), (1, 130, 3, 3, 32)])
def test_attention(ctx, B, S, H, Hkv, hd):
    T = B * S
    q, k, v = (ctx.from_numpy(np.float32(0.5) * rnd((T, n * hd), s)) for s, n in ((21, H), (22, Hkv), (23, Hkv)))
    o, lse = Guarded(ctx, T * H * hd), Guarded(ctx, B * H * S)
    ctx.call("glc_attention_fwd", q.ptr, k.ptr, v.ptr, o.ptr, lse.ptr, B, S, H, Hkv, hd, 1)
    dO = ctx.from_numpy(rnd((T, H * hd), 24))
    dq, dk, dv = Guarded(ctx, T * H * hd), Guarded(ctx, T * Hkv * hd), Guarded(ctx, T * Hkv * hd)
    ctx.call("glc_attention_bwd", q.ptr, k.ptr, v.ptr, o.ptr, lse.ptr, dO.ptr, dq.ptr, dk.ptr, dv.ptr, B, S, H, Hkv,
             hd, 1)
    ctx.sync()
    for a, name in ((o, "attention o"), (lse, "attention lse"), (dq, "attention dq"), (dk, "attention dk"),
                    (dv, "attention dv")):
        a.check(name)


def test_embedding_and_rope(ctx):
    T, S, d, V = 300, 100, 132, 50
    tok = np.random.default_rng(25).integers(-2, V + 2, T).astype(np.int64)
    d_tok, E, P = ctx.from_numpy(tok), ctx.from_numpy(rnd((V, d), 26)), ctx.from_numpy(rnd((S, d), 27))
    out = Guarded(ctx, T * d)
    ctx.call("glc_embed_fwd", d_tok.ptr, E.ptr, P.ptr, out.ptr, T, S, d, V)
    dE = Guarded(ctx, V * d, init=rnd((V, d), 28))
    dh = ctx.from_numpy(rnd((T, d), 29))
    ctx.call("glc_embed_bwd", tok.ctypes.data_as(C.c_void_p), T, dh.ptr, dE.ptr, d, V)
    nh, hd = 3, 44
    cos_h, sin_h = np.empty((S, hd // 2), np.float32), np.empty((S, hd // 2), np.float32)
    assert ctx.lib.glc_rope_table(hd, S, C.c_float(10000.0), cos_h.ctypes.data_as(C.c_void_p),
                                  sin_h.ctypes.data_as(C.c_void_p)) == 0
    cs, sn = ctx.from_numpy(cos_h), ctx.from_numpy(sin_h)
    x = Guarded(ctx, T * nh * hd, init=rnd((T, nh * hd), 30))
    ctx.call("glc_rope", x.ptr, T, S, nh, hd, cs.ptr, sn.ptr, 0, 1)
    ctx.sync()
    for a, name in ((out, "embed_fwd"), (dE, "embed_bwd"), (x, "rope")):
        a.check(name)


def test_dequantize_and_optimizer_segments(ctx):
    n = 256 * 5
    wq = ctx.from_numpy(np.frombuffer(sane_format_weight(Q4_K, 5, 256, 31), np.uint8).copy())
    dst = Guarded(ctx, n)
    ctx.call("glc_dequantize", Q4_K, wq.ptr, dst.ptr, n)
    # AdamW over two segments of a 4096-float arena: everything outside them stays as it was
    N = 4096
    segs = np.array([128, 1000, 2048, 512], np.int64)
    inside = np.zeros(N, bool)
    inside[128:1128] = inside[2048:2560] = True
    body = [np.where(inside, rnd(N, 32 + i, 0.02), np.float32(i + 1)) for i in range(5)]
    body[3] = np.abs(body[3])  # the second moment is non-negative
    arenas = [Guarded(ctx, N, init=b) for b in body]
    p, g, m, v, sh = arenas
    ctx.call("glc_adamw_step", p.ptr, g.ptr, m.ptr, v.ptr, sh.ptr, segs.ctypes.data_as(C.c_void_p), 2, None,
             C.c_float(3e-4), C.c_float(0.9), C.c_float(0.95), C.c_float(1e-8), C.c_float(0.1), 1)
    ctx.sync()
    dst.check("dequantize")
    for i, a in enumerate(arenas):
        a.check(f"adamw arena {i}")
        body = a.buf.numpy()[GUARD:GUARD + N]
        assert np.all(body[~inside] == np.float32(i + 1)), f"adamw arena {i}: write outside the segments"
